#!/usr/bin/env python3
"""Decode-step ASTC-KV attention benchmark (B200, sm_100a).

Metric: decode-attention KV tokens/s, and the fraction of HBM
peak over the compressed bytes read, at 1/2/4/8 GPUs.

Workloads (``--workload``; the default is the benchmark line):
  c2      Llama-3-8B-shaped batched GQA decode: batch 32, Hq 32 /
          Hkv 8, head_dim 128, T = 32768, bf16 q, FP16 K, scalar ASTC 6x6 V
          with a per-block fp16 affine map. The V blocks are real astcenc
          5.7.0 6x6 blocks from the reference's golden corpus
          (tests/golden/block_geometry_identity.npz) tiled to size, as the
          reference's own traffic fixtures do (scripts/make_traffic_fixture.py).
          Sharded one set of KV heads per GPU (8/N heads each; strong scaling).
  c2fp16  The same shape with FP16 K and FP16 V: the FP16 control the
          reference compares ASTC against (its own FP16 kernel,
          metal/probe_gqa_v10.mm:669), sharded the same way.
  c1      SmolLM2-shaped, 30 layers in one launch, T = 8192, split 64 x 128,
          FP16 K + RGBA ASTC 4x4 V (this library's encoder; astcenc is
          absent). Too small to shard: replicas at N > 1 (weak scaling).
  c3      Llama-3-70B-shaped: ASTC 4x4 K + 2-channel FP16 side plane, ASTC 8x8
          V, batch 8, T = 131072. Sharded by sequence (8/N each; strong).
  c4      Ragged paged atlas: 64 sequences of U[1024, 65536] tokens, 256-token
          pages of a shared 4x4 V atlas, permuted pages, int32 block table.
          Sharded by sequence, greedily balanced on tokens (strong).
  decode4 / decode6 / decode8
          The config-4 standalone decode microbench: 1 GiB of random legal
          ASTC blocks of one footprint decoded to UNORM8 RGBA (replicas).

Every unit of work (a KV head of c2, a sequence of c3/c4, a layer of c1) is
drawn from its own seeded generator, so a rank's shard holds the same values
whatever the number of GPUs, and the CPU reference path times exactly the
data the GPU arm sees. A step is one decode-attention pass over every
sequence of the job.

Multi-GPU: one process per GPU (torchrun). Shards are independent, so no
collective runs on the data path; timing is bracketed by barriers and the
reported time is the max over ranks.

``--impl reference`` times the reference's CPU path on the host cores: the
ASTC decode the reference runs through astcenc (absent here, so the C oracle
port of it) plus NumPy restore and attention (astc_kv/codec.py:198-208,
:253-267), on a bounded sample of the same workload's data.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "astc-kv_b200"))

METRIC = "decode-attn KV tokens/s per GPU & % HBM peak (compressed bytes), 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


# --------------------------------------------------------------------------- setup

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reduce(values: list[float], world: int, device=None, op: str = "max") -> list[float]:
    """Element-wise max (timing: the slowest rank defines a step) or sum over ranks."""
    if world <= 1:
        return list(values)
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.tolist()


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(workload: str) -> tuple[float | None, str | None]:
    """Per-launch DRAM traffic of the split kernel for a full launch, read from
    the workload's committed ncu summary (profiles/*_<workload>.md, line
    ``traffic_bytes_per_full_launch: N``; or any summary covering several
    workloads, line ``traffic_bytes_per_full_launch[<workload>]: N``). None
    when no summary carries it."""
    for f in sorted((ROOT / "profiles").glob(f"*_{workload}.md")):
        m = re.search(r"^traffic_bytes_per_full_launch:\s*([0-9.eE+]+)", f.read_text(), re.M)
        if m:
            return float(m.group(1)), f.name
    for f in sorted((ROOT / "profiles").glob("*.md")):
        m = re.search(r"^traffic_bytes_per_full_launch\[" + re.escape(workload) + r"\]:\s*([0-9.eE+]+)",
                      f.read_text(), re.M)
        if m:
            return float(m.group(1)), f.name
    return None, None


class ClockSampler:
    """NVML samples of SM clock and throttle reasons while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clocks_setting"}

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((sm, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "source": "nvml unavailable"}
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit and name not in ("gpu_idle",):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml"}


# ------------------------------------------------------------------ sharding

def shard_range(n: int, rank: int, world: int) -> list[int]:
    """Units [lo, hi) of rank `rank` when n units are split into `world`
    contiguous parts whose sizes differ by at most one."""
    lo = n * rank // world
    hi = n * (rank + 1) // world
    return list(range(lo, hi))


def balance(lens: list[int], world: int) -> list[list[int]]:
    """Greedy longest-first assignment of sequences to ranks on their token
    counts (equal bytes per GPU is what keeps the scaling linear)."""
    order = sorted(range(len(lens)), key=lambda i: (-lens[i], i))
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        out[r].append(i)
        load[r] += lens[i]
    return [sorted(x) for x in out]


def c4_lengths() -> list[int]:
    """Config 4's 64 sequence lengths, uniform in [1024, 65536] (seed 20261029)."""
    return [int(x) for x in np.random.default_rng(20261029).integers(1024, 65537, 64)]


def unit_gen(device, config: int, unit: int):
    """The generator of one unit of work (a KV head, a sequence or a layer)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(20261028 + 1_000_003 * config + 7919 * unit)
    return g


# ----------------------------------------------------------------------- workloads

def golden_pool_6x6() -> np.ndarray:
    """Real astcenc 6x6 block rows: [rows, 11, 16] (11 blocks = 66 texels)."""
    with np.load(ROOT / "tests" / "golden" / "block_geometry_identity.npz") as z:
        b = z["blocks"]  # [pairs, 1584, 16] = pairs x (3 heads x 48 rows x 11 cols)
    return b.reshape(-1, 11, 16)


_POOLS: dict = {}


def encoder_pool(block: int, layout: str, D: int, rows: int, seed: int, norm: str = "block_affine") -> np.ndarray:
    """Block rows from this library's CPU encoder on the configs' value
    distribution (N(0,1) x lognormal(0, 0.5) channel scale): [rows, cols, 16]."""
    key = (block, layout, D, rows, seed, norm)
    if key not in _POOLS:
        import astc_kv_cuda as A
        rng = np.random.default_rng(seed)
        T = rows * block
        x = rng.standard_normal((1, T, D)).astype(np.float32) * rng.lognormal(0, 0.5, (1, 1, D)).astype(np.float32)
        P = 16 if norm == "page_channel" else block
        while T % P:
            P += block
        e = A.encode_tensor(x, {"block": block, "layout": layout, "normalization": norm}, page_tokens=P, quality=60)
        _POOLS[key] = e.blocks_array()[0]
    return _POOLS[key]


# Pools of block rows each workload tiles its planes from (key -> builder args).
POOL_ARGS = {"c1v": (4, "rgba", 64, 2048, 1, "page_channel"), "c3k": (4, "scalar", 128, 4096, 2),
             "c3v": (8, "scalar", 128, 2048, 3), "c4v": (4, "scalar", 128, 4096, 4)}


def pool(name: str) -> np.ndarray:
    return golden_pool_6x6() if name == "c2v" else encoder_pool(*POOL_ARGS[name])


SPEC = {
    "c2": {"workload": "config2_llama3_8b_gqa", "batch": 32, "q_heads": 32, "kv_heads": 8, "head_dim": 128,
           "tokens": 32768, "q_dtype": "bf16", "k": "fp16", "v": "astc 6x6 scalar block_affine",
           "v_blocks": "astcenc 5.7.0 golden 6x6 blocks (reference corpus) tiled", "page_tokens": 96},
    "c2fp16": {"workload": "config2_llama3_8b_gqa_fp16_control", "batch": 32, "q_heads": 32, "kv_heads": 8,
               "head_dim": 128, "tokens": 32768, "q_dtype": "bf16", "k": "fp16", "v": "fp16", "page_tokens": 96},
    "c1": {"workload": "config1_smollm2_30_layers", "layers": 30, "q_heads": 9, "kv_heads": 3, "head_dim": 64,
           "tokens": 8192, "k": "fp16", "v": "astc 4x4 rgba page_channel(16)",
           "v_blocks": "this library's encoder (astcenc absent)", "split": "64 x 128"},
    "c3": {"workload": "config3_llama3_70b", "batch": 8, "q_heads": 64, "kv_heads": 8, "head_dim": 128,
           "tokens": 131072, "q_dtype": "bf16", "k": "astc 4x4 scalar block_affine + 2-channel fp16 side plane",
           "v": "astc 8x8 scalar block_affine", "blocks": "this library's encoder (astcenc absent)", "page_tokens": 64},
    "c4": {"workload": "config4_ragged_paged_atlas", "sequences": 64, "q_heads": 32, "kv_heads": 8, "head_dim": 128,
           "page_tokens": 256, "k": "fp16 pages", "v": "astc 4x4 scalar block_affine atlas",
           "blocks": "this library's encoder (astcenc absent)", "lengths": "U[1024, 65536], seed 20261029"},
}

SHARD = {"c2": "kv_head", "c2fp16": "kv_head", "c3": "sequence", "c4": "sequence", "c1": "replica"}


def job_bytes(name: str) -> int:
    """Algorithmic bytes one step of the whole job reads (every rank together):
    compressed blocks + K + fp16 metadata + side plane + q + block table."""
    s = SPEC[name]
    if name in ("c2", "c2fp16"):
        B, Hkv, Hq, D, T = s["batch"], s["kv_heads"], s["q_heads"], s["head_dim"], s["tokens"]
        v = T * D * 2 if name == "c2fp16" else math.ceil(T / 6) * 22 * (16 + 4)
        return B * Hkv * (T * D * 2 + v) + B * Hq * D * 2 + B * 4
    if name == "c1":
        L, Hkv, Hq, D, T = s["layers"], s["kv_heads"], s["q_heads"], s["head_dim"], s["tokens"]
        return L * Hkv * (T * D * 2 + (T // 4) * 4 * 16 + (T // 16) * D * 4) + L * Hq * D * 4
    if name == "c3":
        B, Hkv, Hq, D, T = s["batch"], s["kv_heads"], s["q_heads"], s["head_dim"], s["tokens"]
        return B * Hkv * (T // 4 * 32 * 20 + T * 2 * 2 + T // 8 * 16 * 20) + B * Hq * D * 2
    if name == "c4":
        lens = c4_lengths()
        Hkv, Hq, D = s["kv_heads"], s["q_heads"], s["head_dim"]
        return Hkv * sum(n * D * 2 + math.ceil(n / 4) * 32 * 20 for n in lens) + len(lens) * Hq * D * 2 + \
            len(lens) * max(math.ceil(n / 256) for n in lens) * 4
    raise KeyError(name)


def job_tokens(name: str) -> int:
    s = SPEC[name]
    if name in ("c2", "c2fp16", "c3"):
        return s["batch"] * s["tokens"]
    if name == "c1":
        return s["layers"] * s["tokens"]
    return sum(c4_lengths())


def line_config(name: str, world: int, shard: str) -> dict:
    """The `config` object of a bench line (identical in both arms)."""
    cfg = dict(SPEC[name])
    cfg["bytes_per_step"] = job_bytes(name)
    cfg["l2"] = "inputs larger than L2 (no flush needed)" if name != "c1" else \
        "30 layers = 118 MB, about the size of L2; one launch reads each byte once"
    if shard == "replica":
        cfg["global_batch"] = (SPEC[name].get("layers") or SPEC[name].get("batch")) * world
        cfg["parallelism"] = f"replicas x{world} (no shard: too small to split), no collective"
    else:
        cfg["global_batch"] = SPEC[name].get("batch") or SPEC[name].get("sequences")
        how = {"kv_head": "kv heads", "sequence": "sequences (token-balanced)" if name == "c4" else "sequences"}[shard]
        cfg["parallelism"] = f"sharded by {how} over {world} GPU(s), no collective"
    return cfg


class Workload:
    """Device-resident inputs of one rank (its shard of the job) plus the
    prepared attention call. `units` selects the shard: KV heads (c2),
    sequences (c3, c4) or layers (c1); None = the whole job."""

    def __init__(self, name: str, device, units: list[int] | None = None, batch: int = 0, split_tokens: int = 0,
                 lens: list[int] | None = None, prepare: bool = True):
        import torch
        from astc_kv_cuda.ops import (Attention, contiguous_astc_plane, contiguous_fp16_plane, paged_astc_plane,
                                      paged_fp16_plane)
        self.name = name
        s = SPEC[name]
        f16 = torch.float16
        self.seq_lens = None
        self.table = None
        self.host = {}  # what the CPU reference path needs to rebuild the values
        num_pages = 0
        split = 0
        if name in ("c2", "c2fp16"):
            B, Hq, Hkv, D, T, P, bs = batch or s["batch"], s["q_heads"], s["kv_heads"], s["head_dim"], s["tokens"], 96, 6
            G = Hq // Hkv
            heads = list(range(Hkv)) if units is None else list(units)
            cap = math.ceil(T / P) * P
            rows, cols = cap // bs, 22
            pl = torch.from_numpy(pool("c2v")).to(device)
            ks, qs, vb, vo, vs, vf = [], [], [], [], [], []
            idx = []
            for h in heads:
                g = unit_gen(device, 2, h)
                left = torch.randint(0, pl.shape[0], (B, rows), generator=g, device=device)
                right = torch.randint(0, pl.shape[0], (B, rows), generator=g, device=device)
                off = (torch.randn(B, rows, cols, generator=g, device=device) * 0.5).to(f16)
                scl = (torch.rand(B, rows, cols, generator=g, device=device) * 3 + 0.25).to(f16)
                ks.append(torch.randn(B, cap, D, generator=g, device=device, dtype=f16))
                qs.append(torch.randn(B, G, D, generator=g, device=device).to(torch.bfloat16))
                if name == "c2":
                    vb.append(torch.cat([pl[left], pl[right]], dim=2))
                    vo.append(off)
                    vs.append(scl)
                    idx.append(torch.stack([left, right], -1))
                else:
                    vf.append(torch.randn(B, cap, D, generator=g, device=device, dtype=f16))
            k = torch.stack(ks, 1).contiguous()
            del ks
            self.kp = contiguous_fp16_plane(k, P)
            if name == "c2":
                self.vp = contiguous_astc_plane(torch.stack(vb, 1).contiguous(), torch.stack(vo, 1).contiguous(),
                                                torch.stack(vs, 1).contiguous(), block=bs, layout="scalar",
                                                normalization="block_affine", head_dim=D, page_tokens=P)
                self.host = {"pool": "c2v", "idx": torch.stack(idx, 1)}
            else:
                self.vp = contiguous_fp16_plane(torch.stack(vf, 1).contiguous(), P)
            del vb, vf
            q = torch.cat(qs, 1).contiguous()
            self.seq_lens = torch.full((B,), T, dtype=torch.int32, device=device)
            self.lens = [T] * B
            H = len(heads)
            vbytes = T * D * 2 if name == "c2fp16" else math.ceil(T / bs) * cols * (16 + 4)
            self.bytes = B * H * (T * D * 2 + vbytes) + q.numel() * 2 + B * 4
            self.job_units = B * T * H / Hkv  # tokens-equivalent of this shard (all heads = whole tokens)
            max_tokens = T
        elif name == "c1":
            L, Hq, Hkv, D, T, P, bs = s["layers"], s["q_heads"], s["kv_heads"], s["head_dim"], s["tokens"], 16, 4
            layers = list(range(L)) if units is None else list(units)
            cols, rows, pages = 4, T // bs, T // P
            pl = torch.from_numpy(pool("c1v")).to(device)
            vb, vo, vs, ks, qs, idx = [], [], [], [], [], []
            for l in layers:
                g = unit_gen(device, 1, l)
                ix = torch.randint(0, pl.shape[0], (Hkv, rows), generator=g, device=device)
                vb.append(pl[ix])
                idx.append(ix)
                vo.append((torch.randn(Hkv, pages, D, generator=g, device=device) * 0.5).to(f16))
                vs.append((torch.rand(Hkv, pages, D, generator=g, device=device) * 3 + 0.25).to(f16))
                ks.append(torch.randn(Hkv, T, D, generator=g, device=device, dtype=f16))
                qs.append(torch.randn(Hq, D, generator=g, device=device))
            self.kp = contiguous_fp16_plane(torch.stack(ks).contiguous(), P)
            self.vp = contiguous_astc_plane(torch.stack(vb).contiguous(), torch.stack(vo).contiguous(),
                                            torch.stack(vs).contiguous(), block=bs, layout="rgba",
                                            normalization="page_channel", head_dim=D, page_tokens=P)
            self.host = {"pool": "c1v", "idx": torch.stack(idx)}
            q = torch.stack(qs).contiguous()
            B = len(layers)
            self.lens = [T] * B
            self.bytes = B * Hkv * (T * D * 2 + rows * cols * 16 + pages * D * 4) + q.numel() * 4
            self.job_units = B * T
            split = 128
            max_tokens = T
        elif name == "c3":
            B, Hq, Hkv, D, T, P = batch or s["batch"], s["q_heads"], s["kv_heads"], s["head_dim"], s["tokens"], 64
            seqs = list(range(B)) if units is None else list(units)
            kcols, vcols = 32, 16
            kpl = torch.from_numpy(pool("c3k")).to(device)
            vpl = torch.from_numpy(pool("c3v")).to(device)
            g0 = unit_gen(device, 3, 1_000_000)
            ch = torch.stack([torch.randperm(D, generator=g0, device=device)[:2] for _ in range(Hkv)]).to(torch.int32)
            kb, ko, kss, vb, vo, vs, sd, qs, kidx, vidx = [], [], [], [], [], [], [], [], [], []
            for b in seqs:
                g = unit_gen(device, 3, b)
                ki = torch.randint(0, kpl.shape[0], (Hkv, T // 4), generator=g, device=device)
                vi = torch.randint(0, vpl.shape[0], (Hkv, T // 8), generator=g, device=device)
                kb.append(kpl[ki])
                vb.append(vpl[vi])
                kidx.append(ki)
                vidx.append(vi)
                ko.append((torch.randn(Hkv, T // 4, kcols, generator=g, device=device) * 0.5).to(f16))
                kss.append((torch.rand(Hkv, T // 4, kcols, generator=g, device=device) * 3 + 0.25).to(f16))
                vo.append((torch.randn(Hkv, T // 8, vcols, generator=g, device=device) * 0.5).to(f16))
                vs.append((torch.rand(Hkv, T // 8, vcols, generator=g, device=device) * 3 + 0.25).to(f16))
                sd.append(torch.randn(Hkv, T, 2, generator=g, device=device, dtype=f16) * 8)
                qs.append(torch.randn(Hq, D, generator=g, device=device).to(torch.bfloat16))
            st = lambda xs: torch.stack(xs).contiguous()  # noqa: E731
            self.kp = contiguous_astc_plane(st(kb), st(ko), st(kss), block=4, layout="scalar",
                                            normalization="block_affine", head_dim=D, page_tokens=P, side=st(sd),
                                            side_channels=ch)
            self.vp = contiguous_astc_plane(st(vb), st(vo), st(vs), block=8, layout="scalar",
                                            normalization="block_affine", head_dim=D, page_tokens=P)
            self.host = {"kpool": "c3k", "vpool": "c3v", "kidx": st(kidx), "vidx": st(vidx), "side_channels": ch}
            q = st(qs)
            B = len(seqs)
            self.lens = [T] * B
            self.bytes = B * Hkv * (T // 4 * kcols * 20 + T * 2 * 2 + T // 8 * vcols * 20) + q.numel() * 2
            self.job_units = B * T
            max_tokens = T
        elif name == "c4":
            Hq, Hkv, D, P, bs = s["q_heads"], s["kv_heads"], s["head_dim"], s["page_tokens"], 4
            all_lens = c4_lengths() if lens is None else list(lens)
            seqs = list(range(len(all_lens))) if units is None else list(units)
            self.lens = [all_lens[i] for i in seqs]
            pps = [math.ceil(n / P) for n in self.lens]
            num_pages = sum(pps)
            maxp = max(pps)
            cols, prow = 32, P // bs
            pl = torch.from_numpy(pool("c4v")).to(device)
            vb, vo, vs, kpg, qs, vidx = [], [], [], [], [], []
            for i in seqs:
                g = unit_gen(device, 4, i)
                npg = math.ceil(all_lens[i] / P)
                vi = torch.randint(0, pl.shape[0], (npg, Hkv, prow), generator=g, device=device)
                vb.append(pl[vi])
                vidx.append(vi)
                vo.append((torch.randn(npg, Hkv, prow, cols, generator=g, device=device) * 0.5).to(f16))
                vs.append((torch.rand(npg, Hkv, prow, cols, generator=g, device=device) * 3 + 0.25).to(f16))
                kpg.append(torch.randn(npg, Hkv, P, D, generator=g, device=device, dtype=f16))
                qs.append(torch.randn(Hq, D, generator=g, device=device).to(torch.bfloat16))
            # The shard's pages in one atlas, at randomly permuted positions.
            perm = np.random.default_rng(20261029 + sum(seqs) + 65537 * len(seqs)).permutation(num_pages)
            table = np.zeros((len(seqs), maxp), np.int32)
            o = 0
            for j, n in enumerate(pps):
                table[j, :n] = perm[o:o + n]
                o += n
            where = torch.from_numpy(np.argsort(perm)).to(device)  # atlas slot -> page in sequence order

            def atlas(xs):
                return torch.cat(xs)[where].contiguous()
            self.kp = paged_fp16_plane(atlas(kpg))
            self.vp = paged_astc_plane(atlas(vb), atlas(vo), atlas(vs), block=bs, layout="scalar",
                                       normalization="block_affine", head_dim=D, page_tokens=P)
            self.table = torch.from_numpy(table).to(device)
            self.seq_lens = torch.tensor(self.lens, dtype=torch.int32, device=device)
            self.host = {"pool": "c4v", "idx": atlas(vidx)}
            q = torch.stack(qs).contiguous()
            tok = sum(self.lens)
            self.bytes = Hkv * (tok * D * 2 + sum(math.ceil(n / bs) for n in self.lens) * cols * 20) + \
                q.numel() * 2 + table.nbytes
            B = len(seqs)
            self.job_units = tok
            max_tokens = maxp * P
        else:
            raise SystemExit(f"unknown workload {name}")
        self.q = q
        self.B = B
        self.tokens = int(sum(self.lens))
        if split_tokens:
            split = split_tokens  # explicit split (profiling a small case with the full run's splits)
        self.max_tokens, self.num_pages, self.split = max_tokens, num_pages, split
        if not prepare:  # inputs only (the CPU reference arm)
            self.attn = None
            return
        self.attn = Attention(q, self.kp, self.vp, page_tokens=self.kp_page(name), max_tokens=max_tokens,
                              seq_lens=self.seq_lens, block_table=self.table, num_pages=num_pages, split_tokens=split)

    @staticmethod
    def kp_page(name: str) -> int:
        return {"c2": 96, "c2fp16": 96, "c1": 16, "c3": 64, "c4": 256}[name]


# ------------------------------------------------------------- CPU reference path

def host_sample(wl: Workload, seq: int = 0, heads: int | None = None) -> dict:
    """The host copy of what the reference path needs for `heads` KV heads of
    sequence (or layer) `seq` of a built workload: compressed blocks (or FP16
    values), fp16 metadata, K and the query rows of those heads."""
    import torch
    name = wl.name
    Hkv = SPEC[name]["kv_heads"]
    heads = Hkv if heads is None else heads
    G = SPEC[name]["q_heads"] // Hkv
    out = {"name": name, "heads": heads, "G": G, "q": wl.q[seq, :heads * G].float().cpu().numpy()}
    T = wl.lens[seq]
    out["T"] = T
    if name in ("c2", "c2fp16", "c1"):
        out["k"] = wl.kp.data[seq, :heads].cpu().numpy()
        if name == "c2fp16":
            out["v"] = wl.vp.data[seq, :heads].cpu().numpy()
        else:
            out["vblocks"] = wl.vp.data[seq, :heads].cpu().numpy()
            out["voff"] = wl.vp.offsets[seq, :heads].cpu().numpy()
            out["vscl"] = wl.vp.scales[seq, :heads].cpu().numpy()
    elif name == "c3":
        out["kblocks"] = wl.kp.data[seq, :heads].cpu().numpy()
        out["koff"] = wl.kp.offsets[seq, :heads].cpu().numpy()
        out["kscl"] = wl.kp.scales[seq, :heads].cpu().numpy()
        out["side"] = wl.kp.side[seq, :heads].cpu().numpy()
        out["side_channels"] = wl.kp.side_channels[:heads].cpu().numpy()
        out["vblocks"] = wl.vp.data[seq, :heads].cpu().numpy()
        out["voff"] = wl.vp.offsets[seq, :heads].cpu().numpy()
        out["vscl"] = wl.vp.scales[seq, :heads].cpu().numpy()
    elif name == "c4":
        P = 256
        pages = wl.table[seq, :math.ceil(T / P)].long()
        out["k"] = wl.kp.data[pages][:, :heads].transpose(0, 1).reshape(heads, -1, wl.kp.data.shape[-1]).cpu().numpy()
        vb = wl.vp.data[pages][:, :heads]  # [pages, heads, prow, cols, 16]
        out["vblocks"] = vb.transpose(0, 1).reshape(heads, -1, vb.shape[3], 16).cpu().numpy()
        for key, t in (("voff", wl.vp.offsets), ("vscl", wl.vp.scales)):
            m = t[pages][:, :heads]
            out[key] = m.transpose(0, 1).reshape(heads, -1, m.shape[3]).cpu().numpy()
    torch.cuda.synchronize()
    return out


def _unit(blocks: np.ndarray, bs: int, layout: str, D: int, threads: int) -> np.ndarray:
    """Oracle decode (fp16 view, as astcenc's F32 LDR output) of blocks
    [H, rows, cols, 16] -> u [H, rows*bs, D] float32."""
    from oracle import oracle as O
    H, rows, cols, _ = blocks.shape
    tex = O.decode_blocks(blocks.reshape(-1, 16), bs, O.OUT_FP16, threads=threads).astype(np.float32)
    tex = tex.reshape(H, rows, cols, bs, bs, 4).transpose(0, 1, 3, 2, 4, 5)  # [H, rows, y, cols, x, 4]
    if layout == "scalar":
        return tex[..., 0].reshape(H, rows * bs, cols * bs)[:, :, :D]
    return tex.reshape(H, rows * bs, cols * bs * 4)[:, :, :D]


def _block_affine(u: np.ndarray, off: np.ndarray, scl: np.ndarray, bs: int) -> np.ndarray:
    """fp32 restore with one (offset, scale) per block (unfused mul + add, codec.py:206)."""
    H, T, D = u.shape
    s = np.repeat(np.repeat(scl.astype(np.float32), bs, 1), bs, 2)[:, :T, :D]
    o = np.repeat(np.repeat(off.astype(np.float32), bs, 1), bs, 2)[:, :T, :D]
    return u * s + o


def cpu_reference_step(sm: dict, threads: int) -> np.ndarray:
    """The reference's CPU path on one host sample: ASTC decode (the C oracle,
    astcenc's decode restated, on `threads` threads) -> fp32 restore
    (codec.py:198-208) -> NumPy GQA attention (codec.py:253-267)."""
    from oracle import oracle as O
    name, T, H = sm["name"], sm["T"], sm["heads"]
    D = sm["q"].shape[-1]
    if name == "c2fp16":
        k, v = sm["k"][:, :T].astype(np.float32), sm["v"][:, :T].astype(np.float32)
    elif name == "c2":
        k = sm["k"][:, :T].astype(np.float32)
        v = _block_affine(_unit(sm["vblocks"], 6, "scalar", D, threads), sm["voff"], sm["vscl"], 6)[:, :T]
    elif name == "c1":
        k = sm["k"][:, :T].astype(np.float32)
        u = _unit(sm["vblocks"], 4, "rgba", D, threads)
        pages = T // 16
        v = (u.reshape(H, pages, 16, D) * sm["vscl"][:, :, None, :].astype(np.float32)
             + sm["voff"][:, :, None, :].astype(np.float32)).reshape(H, T, D)
    elif name == "c3":
        k = _block_affine(_unit(sm["kblocks"], 4, "scalar", D, threads), sm["koff"], sm["kscl"], 4)[:, :T]
        for h in range(H):
            k[h][:, sm["side_channels"][h]] = sm["side"][h].astype(np.float32)
        v = _block_affine(_unit(sm["vblocks"], 8, "scalar", D, threads), sm["voff"], sm["vscl"], 8)[:, :T]
    elif name == "c4":
        k = sm["k"][:, :T].astype(np.float32)
        v = _block_affine(_unit(sm["vblocks"], 4, "scalar", D, threads), sm["voff"], sm["vscl"], 4)[:, :T]
    else:
        raise KeyError(name)
    out, _ = O.attention(sm["q"][:, None, :], np.ascontiguousarray(k), np.ascontiguousarray(v), np.array([T - 1]))
    return out


def time_reference(wl: Workload, steps: int, warmup: int, budget_s: float, threads: int) -> dict:
    """Time the reference path on samples of `wl`: per step one sequence (c1:
    one layer) with as many of its KV heads as fit `budget_s` per step."""
    Hkv = SPEC[wl.name]["kv_heads"]
    full = host_sample(wl, 0)
    t0 = time.perf_counter()
    cpu_reference_step(full, threads)
    per_full = time.perf_counter() - t0
    heads = max(1, min(Hkv, int(Hkv * budget_s / max(per_full, 1e-9))))
    sm = full if heads == Hkv else host_sample(wl, 0, heads)
    for _ in range(warmup):
        cpu_reference_step(sm, threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_reference_step(sm, threads)
    dt = time.perf_counter() - t0
    tokens = sm["T"] * heads / Hkv  # tokens-equivalent: a token counts once all its KV heads are done
    what = "layer" if wl.name == "c1" else "sequence"
    return {"value": steps * tokens / dt, "seconds": dt, "steps": steps, "heads": heads,
            "sample": f"per step {heads}/{Hkv} kv heads of {what} 0 of the same data ({sm['T']} tokens): "
                      f"C oracle ASTC decode on {threads} threads + NumPy fp32 restore and attention"}


# ------------------------------------------------------------------------ our arm

def init_dist(world: int, dev):
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)


def rank_units(name: str, rank: int, world: int, shard: str) -> list[int] | None:
    if shard == "replica" or world == 1:
        return None
    s = SPEC[name]
    if shard == "kv_head":
        return shard_range(s["kv_heads"], rank, world)
    if name == "c4":
        return balance(c4_lengths(), world)[rank]
    return shard_range(s["batch"], rank, world)


def run_ours(args) -> dict | None:
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(world, dev)
    import torch.distributed as dist
    import astc_kv_cuda as A
    A.init(local)
    shard = "replica" if args.shard == "replica" or args.batch else SHARD[args.workload]
    units = rank_units(args.workload, rank, world, shard)
    if args.shard_of > 1 and world == 1 and shard != "replica":
        # Rank 0's share of an N-GPU job on one GPU (profiling the per-rank work).
        units = rank_units(args.workload, 0, args.shard_of, shard)
    wl = Workload(args.workload, dev, units=units, batch=args.batch, split_tokens=args.split_tokens)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        wl.attn.run_phase(1)
        wl.attn.run_phase(2)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            ev_s[i].record(stream)
            wl.attn.run_phase(1)
            ev_e[i].record(stream)
            wl.attn.run_phase(2)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = start.elapsed_time(end)
    split_ms = statistics.mean(ev_s[i].elapsed_time(ev_e[i]) for i in range(args.steps))
    # e2e: the public call with the step's inputs and result in pinned host memory.
    qh = wl.q.cpu().pin_memory()
    outh = torch.empty(wl.attn.out.shape, dtype=torch.float32).pin_memory()
    for _ in range(max(1, args.warmup)):
        wl.q.copy_(qh, non_blocking=True)
        wl.attn.run()
        outh.copy_(wl.attn.out, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        wl.q.copy_(qh, non_blocking=True)
        wl.attn.run()
        outh.copy_(wl.attn.out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    h2d, d2h = wl.q.numel() * wl.q.element_size(), wl.attn.out.numel() * 4
    total_ms, e2e_ms, split_ms_max = reduce([total_ms, e2e_ms, split_ms], world, dev, "max")
    job_units, h2d, d2h = reduce([wl.job_units, h2d, d2h], world, dev, "sum")
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    hbm, hbm_src = peaks()
    achieved = wl.bytes / (split_ms * 1e-3) / 1e9
    toks = job_units * args.steps
    traffic, traffic_src = profile_traffic(args.workload)
    if traffic is not None:
        # The committed figure is for the whole job on one GPU; a rank's shard
        # (or a smaller profiling case) moves its share of it.
        traffic = traffic * wl.bytes / job_bytes(args.workload)
    cfg = line_config(args.workload, world, shard)
    if args.batch:
        cfg["batch_override"] = args.batch
    if args.split_tokens:
        cfg["split_tokens"] = args.split_tokens
    if args.shard_of > 1 and world == 1:
        cfg["shard_of"] = f"rank 0's share of a {args.shard_of}-GPU job"
    line = {
        "metric": METRIC, "value": toks / (total_ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak" if shard == "replica" else "strong", "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded per unit); V 6x6 blocks are real astcenc blocks from the reference corpus"
        if args.workload == "c2" else "synthetic (seeded per unit)",
        "config": cfg,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": hbm_src + " (MEASURED_PEAKS.json hbm_gbs)" if hbm_src == "measured" else hbm_src,
                     "kernel": wl.attn.plan()["kernel"], "kernel_ms": split_ms,
                     "kernel_ms_max_over_ranks": split_ms_max, "bytes_per_launch": wl.bytes,
                     "traffic": traffic, "traffic_source": traffic_src and f"profiles/{traffic_src}"},
        "e2e": {"value": toks / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "api": "astc_kv_cuda.ops.Attention.run (akv_cuda_decode_attention)",
                "note": "the compressed KV cache is resident in HBM; per step the query goes up and the output comes back"},
        "clocks": clk.summary(),
        "gpu_launches": 2 * args.steps,
        "split_plan": wl.attn.plan(),
    }
    if world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT))
        from oracle import oracle as O
        threads = O.cpu_threads()
        r = time_reference(wl, 3, 1, args.cpu_seconds / 3, threads)
        line["cpu_baseline"] = {"value": r["value"], "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": r["sample"], "seconds": r["seconds"]}
    return line


# ------------------------------------------------------- per-layer model step

def run_c1_layers(args) -> dict | None:
    """Config 1 as a model decode step issues it: one attention call per layer
    (30 launches of split + merge, each timed with CUDA events), the same 30
    calls replayed from one CUDA graph, and the single 30-layer launch, on the
    same data. The reference never measured attention's share of a decode
    step (docs/research_v4_report.md:85); this gives the per-layer figure."""
    import torch
    from astc_kv_cuda.ops import Attention, contiguous_astc_plane, contiguous_fp16_plane
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import astc_kv_cuda as A
    A.init(local)
    wl = Workload("c1", dev)
    L, T, P = SPEC["c1"]["layers"], SPEC["c1"]["tokens"], 16
    layers = []
    for l in range(L):
        kp = contiguous_fp16_plane(wl.kp.data[l:l + 1], P)
        vp = contiguous_astc_plane(wl.vp.data[l:l + 1], wl.vp.offsets[l:l + 1], wl.vp.scales[l:l + 1], block=4,
                                   layout="rgba", normalization="page_channel", head_dim=64, page_tokens=P)
        layers.append(Attention(wl.q[l:l + 1], kp, vp, page_tokens=P, max_tokens=T, split_tokens=128))
    stream = torch.cuda.current_stream()

    def step_layers():
        for a in layers:
            a.run()

    for _ in range(args.warmup):
        step_layers()
        wl.attn.run()
    torch.cuda.synchronize()
    # (1) per-layer launches with an event between layers.
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(L + 1)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            evs[i][0].record(stream)
            for l, a in enumerate(layers):
                a.run()
                evs[i][l + 1].record(stream)
        torch.cuda.synchronize()
    per_layer = [statistics.median(evs[i][l].elapsed_time(evs[i][l + 1]) for i in range(args.steps)) for l in range(L)]
    step_ms = statistics.median(evs[i][0].elapsed_time(evs[i][L]) for i in range(args.steps))
    # (2) the 30 calls as one CUDA graph.
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step_layers()
    stream.wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step_layers()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    g1.record(stream)
    torch.cuda.synchronize()
    graph_ms = g0.elapsed_time(g1) / args.steps
    # (3) the single 30-layer launch.
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        wl.attn.run()
    s1.record(stream)
    torch.cuda.synchronize()
    single_ms = s0.elapsed_time(s1) / args.steps
    del graph
    hbm, src = peaks()
    tokens = L * T
    return {"metric": METRIC + " [config 1 per-layer decode step]", "value": tokens / (graph_ms * 1e-3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": graph_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded per unit)",
            "config": {**line_config("c1", 1, "replica"), "step": "30 attention calls (one per layer), CUDA graph"},
            "per_layer": {"layer_us_median": [round(x * 1e3, 2) for x in per_layer],
                          "layer_us_mean": sum(per_layer) / L * 1e3,
                          "eager_30_launches_ms": step_ms, "graph_30_launches_ms": graph_ms,
                          "single_30_layer_launch_ms": single_ms,
                          "roofline_frac_graph": job_bytes("c1") / (graph_ms * 1e-3) / 1e9 / hbm,
                          "roofline_frac_single": job_bytes("c1") / (single_ms * 1e-3) / 1e9 / hbm},
            "clocks": clk.summary(), "gpu_launches": 2 * L * args.steps}


# ----------------------------------------------------------------- decode bench

class DecodeWorkload:
    """Config-4 decode microbench: 1 GiB of random legal blocks -> UNORM8."""

    def __init__(self, name: str, device, blocks_total: int = 1 << 26):
        import torch
        import astc_kv_cuda as A
        self.name = name
        self.block = int(name[-1])
        # A pool of distinct random legal blocks, tiled to 1 GiB on the device.
        pool = torch.from_numpy(A.random_blocks(1 << 20, self.block, seed=20261029)).to(device)
        reps = blocks_total // pool.shape[0]
        self.blocks = pool.repeat(reps, 1).contiguous()
        self.n = self.blocks.shape[0]
        tex = self.block * self.block
        self.out = torch.empty(self.n, self.block, self.block, 4, dtype=torch.uint8, device=device)
        self.bytes = self.n * 16 + self.n * tex * 4
        self.sample = pool[:1 << 16].cpu().numpy()
        self.desc = {"workload": f"config4_decode_microbench_{self.block}x{self.block}", "blocks": self.n,
                     "block_bytes": self.n * 16, "output": "UNORM8 RGBA", "output_bytes": self.n * tex * 4,
                     "blocks_source": "random legal LDR blocks (1 Mi distinct, tiled)",
                     "l2": "inputs larger than L2 (no flush needed)"}

    def run(self):
        from astc_kv_cuda.ops import decode_blocks
        decode_blocks(self.blocks, self.block, "unorm8", out=self.out)


def decode_reference(sample: np.ndarray, block: int, seconds: float, threads: int) -> tuple[float, str, float]:
    from oracle import oracle as O
    O.decode_blocks(sample[:1024], block, O.OUT_UNORM8, threads=threads)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        O.decode_blocks(sample, block, O.OUT_UNORM8, threads=threads)
        done += sample.shape[0]
    dt = time.perf_counter() - t0
    return done / dt, f"{done} random legal blocks (the GPU arm's pool) decoded to UNORM8 by the C oracle on {threads} threads", dt


def run_decode(args) -> dict | None:
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(world, dev)
    import torch.distributed as dist
    import astc_kv_cuda as A
    A.init(local)
    wl = DecodeWorkload(args.workload, dev, args.decode_blocks)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        wl.run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record(stream)
        for _ in range(args.steps):
            wl.run()
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = start.elapsed_time(end)
    # e2e: blocks up from pinned host memory, UNORM8 texels back, per step
    # (a 1/16 slice of the job per step keeps the host buffers modest).
    n_e2e = wl.n // 16
    hb = wl.blocks[:n_e2e].cpu().pin_memory()
    ho = torch.empty(n_e2e, wl.block, wl.block, 4, dtype=torch.uint8).pin_memory()
    from astc_kv_cuda.ops import decode_blocks
    db, do = wl.blocks[:n_e2e], wl.out[:n_e2e]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        db.copy_(hb, non_blocking=True)
        decode_blocks(db, wl.block, "unorm8", out=do)
        ho.copy_(do, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    (total_ms, e2e_ms) = reduce([total_ms, e2e_ms], world, dev, "max")
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    hbm, src = peaks()
    per = total_ms / args.steps
    achieved = wl.bytes / (per * 1e-3) / 1e9
    # The committed figure is for a launch of the default 2^26 blocks.
    traffic, traffic_src = profile_traffic(args.workload)
    if traffic is not None:
        traffic = traffic * wl.n / float(1 << 26)
    line = {"metric": METRIC + " [decode microbench: blocks/s]", "value": wl.n * world * args.steps / (total_ms * 1e-3),
            "unit": "blocks/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic random legal blocks",
            "config": {**wl.desc, "parallelism": f"replicas x{world}, no collective"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": src, "kernel": "decode_blocks_kernel", "kernel_ms": per,
                         "traffic": traffic, "traffic_source": traffic_src and f"profiles/{traffic_src}",
                         "bytes": "16 B read + texels*4 B written per block"},
            "e2e": {"value": n_e2e * world * args.steps / (e2e_ms * 1e-3), "unit": "blocks/s",
                    "h2d_bytes_per_step": n_e2e * 16, "d2h_bytes_per_step": n_e2e * wl.block * wl.block * 4,
                    "api": "astc_kv_cuda.ops.decode_blocks (akv_cuda_decode_blocks)",
                    "note": "per step 1/16 of the job's blocks go up and their texels come back"},
            "clocks": clk.summary(), "gpu_launches": args.steps}
    if world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT))
        from oracle import oracle as O
        threads = O.cpu_threads()
        v, sample, dt = decode_reference(wl.sample, wl.block, args.cpu_seconds, threads)
        line["cpu_baseline"] = {"value": v, "unit": "blocks/s", "cores": threads, "kind": "port", "sample": sample,
                                "seconds": dt}
    return line


# ------------------------------------------------------------------- reference arm

def run_reference(args) -> dict | None:
    """The reference's CPU path (oracle port) on rank 0, on the host cores.
    Inputs are synthesised exactly as the GPU arm synthesises them (the same
    per-unit generators, on the device, outside the timed region), then the
    sample is copied to the host; nothing of this library runs on the path."""
    world, rank, local = dist_env()
    if rank != 0:
        return None
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    threads = O.cpu_threads()
    try:
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device to synthesise the GPU arm's inputs")
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    except Exception as e:  # pragma: no cover - GPU box only
        return {"impl": "reference", "unavailable": f"input synthesis needs the GPU arm's generators: {e}"}
    base = {"impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "vs_baseline": None}
    if args.workload.startswith("decode"):
        import astc_kv_cuda as A
        block = int(args.workload[-1])
        sample = A.random_blocks(1 << 20, block, seed=20261029)[:1 << 16]
        per_step = max(0.5, 120.0 / (args.steps + args.warmup))
        decode_reference(sample, block, min(1.0, per_step) * args.warmup, threads)
        v, what, dt = decode_reference(sample, block, per_step * args.steps, threads)
        return {**base, "metric": METRIC + " [decode microbench: blocks/s]", "value": v, "unit": "blocks/s",
                "ms_per_step": dt / args.steps * 1e3, "scaling": "weak", "dtype": "u8",
                "data": "synthetic random legal blocks",
                "config": {"workload": f"config4_decode_microbench_{block}x{block}"},
                "cpu_baseline": {"value": v, "unit": "blocks/s", "cores": threads, "kind": "port", "sample": what},
                "e2e": {"value": v, "unit": "blocks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    name = args.workload
    shard = SHARD[name]
    # Only the sampled unit's data is needed: unit 0 (c2: all heads of the
    # first sequences come from per-head generators, so build every head).
    units = None if name in ("c2", "c2fp16") else [0]
    wl = Workload(name, dev, units=units, prepare=False)
    budget = 120.0 / max(1, args.steps + args.warmup)
    r = time_reference(wl, args.steps, args.warmup, budget, threads)
    del wl
    torch.cuda.empty_cache()
    return {**base, "metric": METRIC, "value": r["value"], "unit": "tokens/s",
            "ms_per_step": r["seconds"] / args.steps * 1e3,
            "scaling": "weak" if shard == "replica" else "strong", "dtype": "fp32",
            "data": "synthetic (seeded per unit); V 6x6 blocks are real astcenc blocks from the reference corpus"
            if name == "c2" else "synthetic (seeded per unit)",
            "config": line_config(name, world, shard),
            "cpu_baseline": {"value": r["value"], "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": r["sample"]},
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c1", "c2", "c2fp16", "c3", "c4", "decode4", "decode6", "decode8"],
                    default="c2")
    ap.add_argument("--shard", choices=["auto", "replica"], default="auto",
                    help="auto: the workload's partition (c2 by kv head, c3/c4 by sequence); replica: every rank "
                         "runs the whole job (weak scaling)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling of small cases)")
    ap.add_argument("--split-tokens", type=int, default=0,
                    help="tokens per split (0: the library's automatic choice; set it to profile a small batch "
                         "with the full run's split structure)")
    ap.add_argument("--decode-blocks", type=int, default=1 << 26,
                    help="blocks per step of the decode microbench (a multiple of 2^20; smaller for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="on one GPU, run only rank 0's shard of an N-GPU job (profiling the per-rank work)")
    ap.add_argument("--per-layer", action="store_true",
                    help="c1 only: time one attention call per layer (eager and as one CUDA graph) next to the "
                         "single 30-layer launch")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        line = run_reference(args)
    elif args.workload.startswith("decode"):
        line = run_decode(args)
    elif args.per_layer:
        if args.workload != "c1":
            raise SystemExit("--per-layer is for the c1 workload")
        line = run_c1_layers(args)
    else:
        line = run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
