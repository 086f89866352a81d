#!/usr/bin/env python3
"""Decode-step ASTC-KV attention benchmark (B200, sm_100a).

Metric: decode-attention KV tokens/s, and the fraction of HBM
peak over the compressed bytes read, at 1/2/4/8 GPUs.

Workloads (``--workload``; the default is the benchmark line):
  c2      Llama-3-8B-shaped batched GQA decode: batch 32 per GPU,
          Hq 32 / Hkv 8, head_dim 128, T = 32768, bf16 q, FP16 K, scalar ASTC
          6x6 V with a per-block fp16 affine map. The V blocks are real astcenc
          5.7.0 6x6 blocks from the reference's golden corpus
          (tests/golden/block_geometry_identity.npz) tiled to size, as the
          reference's own traffic fixtures do (scripts/make_traffic_fixture.py).
  c1      SmolLM2-shaped, 30 layers in one launch, T = 8192, split 64 x 128,
          FP16 K + RGBA ASTC 4x4 V (this library's encoder; astcenc is absent).
  c3      Llama-3-70B-shaped: ASTC 4x4 K + 2-channel FP16 side plane, ASTC 8x8 V.
  c4      Ragged paged atlas: 64 sequences of U[1024, 65536] tokens, 256-token
          pages of a shared 4x4 V atlas, permuted pages, int32 block table.
  decode4 / decode6 / decode8
          The config-4 standalone decode microbench: 1 GiB of random legal
          ASTC blocks of one footprint (every block mode, 1-4 partitions,
          dual plane, void extent) decoded to UNORM8 RGBA; the CPU baseline
          decodes a sample of the same blocks with the C oracle on all cores.
A step is one decode-attention pass over every sequence of the batch.

Multi-GPU: one process per GPU (torchrun). Sequences are independent, so each
rank runs its own batch (weak scaling, sharded by sequence batch) with no
collective on the data path; timing is bracketed by barriers and the reported
time is the max over ranks.

``--impl reference`` times the reference's CPU path on the host cores: the
ASTC decode the reference runs through astcenc (absent here, so the C oracle
port of it) plus NumPy restore and attention (astc_kv/codec.py:198-208,
:253-267), on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
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


def reduce_max(values: list[float], world: int, device=None) -> list[float]:
    """Element-wise max over ranks (timing: the slowest rank defines a step)."""
    if world <= 1:
        return list(values)
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


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


# ----------------------------------------------------------------------- workloads

def golden_pool_6x6() -> np.ndarray:
    """Real astcenc 6x6 block rows: [rows, 11, 16] (11 blocks = 66 texels)."""
    with np.load(ROOT / "tests" / "golden" / "block_geometry_identity.npz") as z:
        b = z["blocks"]  # [pairs, 1584, 16] = pairs x (3 heads x 48 rows x 11 cols)
    return b.reshape(-1, 11, 16)


def encoder_pool(block: int, layout: str, D: int, rows: int, seed: int, norm: str = "block_affine") -> np.ndarray:
    """Block rows from this library's CPU encoder on the configs' value
    distribution (N(0,1) x lognormal(0, 0.5) channel scale): [rows, cols, 16]."""
    import astc_kv_cuda as A
    rng = np.random.default_rng(seed)
    T = rows * block
    x = rng.standard_normal((1, T, D)).astype(np.float32) * rng.lognormal(0, 0.5, (1, 1, D)).astype(np.float32)
    P = 16 if norm == "page_channel" else block
    while T % P:
        P += block
    e = A.encode_tensor(x, {"block": block, "layout": layout, "normalization": norm}, page_tokens=P, quality=60)
    return e.blocks_array()[0]


class DecodeWorkload:
    """Config-4 decode microbench: 1 GiB of random legal blocks -> UNORM8."""

    def __init__(self, name: str, rank: int, device, blocks_total: int = 1 << 26):
        import torch
        import astc_kv_cuda as A
        self.name = name
        self.block = int(name[-1])
        # A pool of distinct random legal blocks, tiled to 1 GiB on the device.
        pool = torch.from_numpy(A.random_blocks(1 << 20, self.block, seed=20261029 + rank)).to(device)
        reps = blocks_total // pool.shape[0]
        self.blocks = pool.repeat(reps, 1).contiguous()
        self.n = self.blocks.shape[0]
        tex = self.block * self.block
        self.out = torch.empty(self.n, self.block, self.block, 4, dtype=torch.uint8, device=device)
        self.bytes = self.n * 16 + self.n * tex * 4
        self.tokens = self.n  # units: blocks
        self.sample = pool[:1 << 16].cpu().numpy()
        self.desc = {"workload": f"config4_decode_microbench_{self.block}x{self.block}", "blocks": self.n,
                     "block_bytes": self.n * 16, "output": "UNORM8 RGBA", "output_bytes": self.n * tex * 4,
                     "blocks_source": "random legal LDR blocks (1 Mi distinct, tiled)"}

    def run(self):
        from astc_kv_cuda.ops import decode_blocks
        decode_blocks(self.blocks, self.block, "unorm8", out=self.out)


def run_decode(args) -> dict | None:
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    import astc_kv_cuda as A
    A.init(local)
    wl = DecodeWorkload(args.workload, rank, dev, args.decode_blocks)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        wl.run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(local) as clk:
        ev[0].record(stream)
        for i in range(args.steps):
            wl.run()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = ev[0].elapsed_time(ev[-1])
    (total_ms,) = reduce_max([total_ms], world, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    hbm, src = peaks()
    per = total_ms / args.steps
    achieved = wl.bytes / (per * 1e-3) / 1e9
    line = {"metric": METRIC + " [decode microbench: blocks/s]", "value": wl.n * world * args.steps / (total_ms * 1e-3),
            "unit": "blocks/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic random legal blocks", "config": {**wl.desc, "l2": "inputs larger than L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": src, "kernel": "decode_blocks_kernel", "kernel_ms": per,
                         "traffic": None, "bytes": "16 B read + texels*4 B written per block"},
            "clocks": clk.summary(), "gpu_launches": args.steps}
    if world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT))
        from oracle import oracle as O
        threads = O.cpu_threads()
        O.decode_blocks(wl.sample[:1024], wl.block, O.OUT_UNORM8, threads=threads)
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < args.cpu_seconds:
            O.decode_blocks(wl.sample, wl.block, O.OUT_UNORM8, threads=threads)
            done += wl.sample.shape[0]
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": done / dt, "unit": "blocks/s", "cores": threads, "kind": "port",
                                "sample": f"{done} random legal blocks decoded to UNORM8 by the C oracle on {threads} threads"}
    return line


class Workload:
    """Device-resident inputs of one rank plus the prepared attention call."""

    def __init__(self, name: str, rank: int, device, batch: int = 0, split_tokens: int = 0):
        import torch
        from astc_kv_cuda.ops import (Attention, contiguous_astc_plane, contiguous_fp16_plane, paged_astc_plane,
                                      paged_fp16_plane)
        self.name = name
        g = torch.Generator(device=device)
        g.manual_seed(20261028 + 7919 * rank)
        rng = np.random.default_rng(20261028 + rank)
        f16 = torch.float16
        self.seq_lens = None
        self.table = None
        num_pages = 0
        if name == "c2":
            B, Hq, Hkv, D, T, P, bs = batch or 32, 32, 8, 128, 32768, 96, 6
            cap = math.ceil(T / P) * P
            rows, cols = cap // bs, 22
            pool = torch.from_numpy(golden_pool_6x6()).to(device)
            left = torch.randint(0, pool.shape[0], (B, Hkv, rows), generator=g, device=device)
            right = torch.randint(0, pool.shape[0], (B, Hkv, rows), generator=g, device=device)
            vblk = torch.cat([pool[left], pool[right]], dim=3).contiguous()  # [B,H,rows,22,16]
            voff = (torch.randn(B, Hkv, rows, cols, generator=g, device=device) * 0.5).to(f16)
            vscl = (torch.rand(B, Hkv, rows, cols, generator=g, device=device) * 3 + 0.25).to(f16)
            k = torch.randn(B, Hkv, cap, D, generator=g, device=device, dtype=f16)
            self.kp = contiguous_fp16_plane(k, P)
            self.vp = contiguous_astc_plane(vblk, voff, vscl, block=bs, layout="scalar", normalization="block_affine",
                                            head_dim=D, page_tokens=P)
            q = torch.randn(B, Hq, D, generator=g, device=device).to(torch.bfloat16)
            self.seq_lens = torch.full((B,), T, dtype=torch.int32, device=device)
            self.lens = [T] * B
            vrows_read = math.ceil(T / bs)
            self.bytes = (B * Hkv * T * D * 2 + B * Hkv * vrows_read * cols * (16 + 4) + q.numel() * 2 + B * 4)
            self.desc = {"workload": "config2_llama3_8b_gqa", "batch_per_gpu": B, "q_heads": Hq, "kv_heads": Hkv,
                         "head_dim": D, "tokens": T, "q_dtype": "bf16", "k": "fp16", "v": "astc 6x6 scalar block_affine",
                         "v_blocks": "astcenc 5.7.0 golden 6x6 blocks (reference corpus) tiled", "page_tokens": P}
            split = 0
        elif name == "c1":
            L, Hq, Hkv, D, T, P, bs = 30, 9, 3, 64, 8192, 16, 4
            cols = 4
            rows = T // bs
            pool = torch.from_numpy(encoder_pool(bs, "rgba", D, 2048, 1, "page_channel")).to(device)
            idx = torch.randint(0, pool.shape[0], (L, Hkv, rows), generator=g, device=device)
            vblk = pool[idx].contiguous()
            pages = T // P
            voff = (torch.randn(L, Hkv, pages, D, generator=g, device=device) * 0.5).to(f16)
            vscl = (torch.rand(L, Hkv, pages, D, generator=g, device=device) * 3 + 0.25).to(f16)
            k = torch.randn(L, Hkv, T, D, generator=g, device=device, dtype=f16)
            self.kp = contiguous_fp16_plane(k, P)
            self.vp = contiguous_astc_plane(vblk, voff, vscl, block=bs, layout="rgba", normalization="page_channel",
                                            head_dim=D, page_tokens=P)
            q = torch.randn(L, Hq, D, generator=g, device=device)
            self.lens = [T] * L
            self.bytes = L * Hkv * (T * D * 2 + rows * cols * 16 + pages * D * 4) + q.numel() * 4
            B = L
            self.desc = {"workload": "config1_smollm2_30_layers", "layers": L, "q_heads": Hq, "kv_heads": Hkv,
                         "head_dim": D, "tokens": T, "k": "fp16", "v": "astc 4x4 rgba page_channel(16)",
                         "v_blocks": "this library's encoder (astcenc absent)", "split": "64 x 128"}
            split = 128
        elif name == "c3":
            B, Hq, Hkv, D, T, P = batch or 8, 64, 8, 128, 131072, 64
            kcols, vcols = 32, 16
            kpool = torch.from_numpy(encoder_pool(4, "scalar", D, 4096, 2)).to(device)
            vpool = torch.from_numpy(encoder_pool(8, "scalar", D, 2048, 3)).to(device)
            kblk = kpool[torch.randint(0, kpool.shape[0], (B, Hkv, T // 4), generator=g, device=device)].contiguous()
            vblk = vpool[torch.randint(0, vpool.shape[0], (B, Hkv, T // 8), generator=g, device=device)].contiguous()

            def meta(rows, cols):
                return ((torch.randn(B, Hkv, rows, cols, generator=g, device=device) * 0.5).to(f16),
                        (torch.rand(B, Hkv, rows, cols, generator=g, device=device) * 3 + 0.25).to(f16))
            koff, kscl = meta(T // 4, kcols)
            voff, vscl = meta(T // 8, vcols)
            side = torch.randn(B, Hkv, T, 2, generator=g, device=device, dtype=f16) * 8
            ch = torch.stack([torch.randperm(D, generator=g, device=device)[:2] for _ in range(Hkv)]).to(torch.int32)
            self.kp = contiguous_astc_plane(kblk, koff, kscl, block=4, layout="scalar", normalization="block_affine",
                                            head_dim=D, page_tokens=P, side=side, side_channels=ch)
            self.vp = contiguous_astc_plane(vblk, voff, vscl, block=8, layout="scalar", normalization="block_affine",
                                            head_dim=D, page_tokens=P)
            q = torch.randn(B, Hq, D, generator=g, device=device).to(torch.bfloat16)
            self.lens = [T] * B
            self.bytes = B * Hkv * (T // 4 * kcols * 20 + T * 2 * 2 + T // 8 * vcols * 20) + q.numel() * 2
            self.desc = {"workload": "config3_llama3_70b", "batch_per_gpu": B, "q_heads": Hq, "kv_heads": Hkv,
                         "head_dim": D, "tokens": T, "k": "astc 4x4 scalar block_affine + 2-channel fp16 side plane",
                         "v": "astc 8x8 scalar block_affine", "blocks": "this library's encoder (astcenc absent)"}
            split = 0
        elif name == "c4":
            S, Hq, Hkv, D, P, bs = 64, 32, 8, 128, 256, 4
            lens = np.random.default_rng(20261029).integers(1024, 65537, S)
            self.lens = [int(x) for x in lens]
            pps = [math.ceil(n / P) for n in self.lens]
            num_pages = sum(pps)
            maxp = max(pps)
            perm = rng.permutation(num_pages)
            table = np.zeros((S, maxp), np.int32)
            o = 0
            for s in range(S):
                table[s, :pps[s]] = perm[o:o + pps[s]]
                o += pps[s]
            cols = 32
            pool = torch.from_numpy(encoder_pool(bs, "scalar", D, 4096, 4)).to(device)
            prow = P // bs
            atlas = pool[torch.randint(0, pool.shape[0], (num_pages, Hkv, prow), generator=g, device=device)].contiguous()
            voff = (torch.randn(num_pages, Hkv, prow, cols, generator=g, device=device) * 0.5).to(f16)
            vscl = (torch.rand(num_pages, Hkv, prow, cols, generator=g, device=device) * 3 + 0.25).to(f16)
            kpages = torch.randn(num_pages, Hkv, P, D, generator=g, device=device, dtype=f16)
            self.kp = paged_fp16_plane(kpages)
            self.vp = paged_astc_plane(atlas, voff, vscl, block=bs, layout="scalar", normalization="block_affine",
                                       head_dim=D, page_tokens=P)
            self.table = torch.from_numpy(table).to(device)
            self.seq_lens = torch.from_numpy(lens.astype(np.int32)).to(device)
            q = torch.randn(S, Hq, D, generator=g, device=device).to(torch.bfloat16)
            tok = int(lens.sum())
            self.bytes = Hkv * (tok * D * 2 + sum(math.ceil(n / bs) for n in self.lens) * cols * 20) + q.numel() * 2 + table.nbytes
            T = maxp * P
            B = S
            self.desc = {"workload": "config4_ragged_paged_atlas", "sequences": S, "tokens_total": tok, "pages": num_pages,
                         "q_heads": Hq, "kv_heads": Hkv, "head_dim": D, "page_tokens": P, "k": "fp16 pages",
                         "v": "astc 4x4 scalar block_affine atlas", "blocks": "this library's encoder (astcenc absent)"}
            split = 0
        else:
            raise SystemExit(f"unknown workload {name}")
        self.q = q
        self.tokens = int(sum(self.lens))
        if split_tokens:
            split = split_tokens  # explicit split (profiling a small case with the full run's splits)
        self.attn = Attention(q, self.kp, self.vp, page_tokens=P, max_tokens=T, seq_lens=self.seq_lens,
                              block_table=self.table, num_pages=num_pages, split_tokens=split)
        self.B = B


# ------------------------------------------------------------------------ our arm

def run_ours(args) -> dict | None:
    import torch
    import torch.distributed as dist
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    import astc_kv_cuda as A
    A.init(local)
    wl = Workload(args.workload, rank, dev, args.batch, args.split_tokens)
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
    total_ms, e2e_ms, split_ms = reduce_max([total_ms, e2e_ms, split_ms], world, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    hbm, hbm_src = peaks()
    achieved = wl.bytes / (split_ms * 1e-3) / 1e9
    toks = wl.tokens * world * args.steps
    line = {
        "metric": METRIC, "value": toks / (total_ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded); V 6x6 blocks are real astcenc blocks from the reference corpus" if args.workload == "c2" else "synthetic (seeded)",
        "config": {**wl.desc, "global_batch": wl.B * world, "parallelism": f"sequence-batch shard x{world}, no collective",
                   "l2": "inputs larger than L2 (no flush needed)", "bytes_per_step_per_gpu": wl.bytes},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": hbm_src + " (MEASURED_PEAKS.json hbm_gbs)" if hbm_src == "measured" else hbm_src,
                     "kernel": wl.attn.plan()["kernel"], "kernel_ms": split_ms,
                     "traffic": TRAFFIC.get(args.workload)},
        "e2e": {"value": toks / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": wl.q.numel() * wl.q.element_size(),
                "d2h_bytes_per_step": wl.attn.out.numel() * 4,
                "api": "astc_kv_cuda.ops.Attention.run (akv_cuda_decode_attention)",
                "note": "the compressed KV cache is resident in HBM; per step the query goes up and the output comes back"},
        "clocks": clk.summary(),
        "gpu_launches": 2 * args.steps,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
    return line


# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of
# the split kernel from the committed ncu captures (profiles/), bytes: c2 was
# captured at batch 4 with the full run's splits (353.1 MB) and scaled by the 8x units of the batch-32
# launch, c3 at batch 1 (220.3 MB) and scaled by the 8x units of the batch-8
# launch (traffic grows with the batch).
TRAFFIC: dict[str, float | None] = {"c2": 353.055e6 * 8, "c3": 220.313e6 * 8}


# ------------------------------------------------------------- CPU reference path

def cpu_unit_inputs(wl_name: str, n_seq: int, rank_seed: int = 0):
    """Host inputs for `n_seq` sequences of the workload (c2 only for now)."""
    rng = np.random.default_rng(99)
    if wl_name != "c2":
        raise SystemExit("the CPU reference arm is implemented for the c2 workload")
    Hq, Hkv, D, T, bs, cols = 32, 8, 128, 32768, 6, 22
    rows = math.ceil(T / bs)
    pool = golden_pool_6x6()
    seqs = []
    for _ in range(n_seq):
        left = rng.integers(0, pool.shape[0], (Hkv, rows))
        right = rng.integers(0, pool.shape[0], (Hkv, rows))
        blocks = np.concatenate([pool[left], pool[right]], axis=2)
        off = (rng.standard_normal((Hkv, rows, cols)) * 0.5).astype(np.float16)
        scl = (rng.random((Hkv, rows, cols)) * 3 + 0.25).astype(np.float16)
        k = rng.standard_normal((Hkv, T, D)).astype(np.float16)
        q = rng.standard_normal((Hq, D)).astype(np.float32)
        seqs.append((blocks, off, scl, k, q))
    return seqs, (Hq, Hkv, D, T, bs, cols)


def cpu_reference_step(seq, shape, threads):
    """Reference CPU path for one sequence: ASTC decode (oracle port of astcenc's
    decode, all threads) -> fp32 restore -> NumPy GQA attention (codec.py)."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    Hq, Hkv, D, T, bs, cols = shape
    blocks, off, scl, k, q = seq
    rows = blocks.shape[1]
    tex = O.decode_blocks(blocks.reshape(-1, 16), bs, O.OUT_FP16, threads=threads)
    u = tex[..., 0].astype(np.float32).reshape(Hkv, rows, cols, bs, bs).transpose(0, 1, 3, 2, 4).reshape(Hkv, rows * bs, cols * bs)
    s = np.repeat(np.repeat(scl.astype(np.float32), bs, 1), bs, 2)
    o = np.repeat(np.repeat(off.astype(np.float32), bs, 1), bs, 2)
    v = (u * s + o)[:, :T, :D]
    out, _ = O.attention(q[:, None, :], k.astype(np.float32), v, np.array([T - 1]))
    return out


def cpu_baseline(wl, seconds: float) -> dict:
    """Rank 0, N=1: the reference CPU path on a bounded sample of the workload."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    threads = O.cpu_threads()
    if wl.name != "c2":
        return {"value": None, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": "not implemented for " + wl.name}
    seqs, shape = cpu_unit_inputs("c2", 1)
    cpu_reference_step(seqs[0], shape, threads)  # warm
    done, t0 = 0, time.perf_counter()
    while True:
        cpu_reference_step(seqs[0], shape, threads)
        done += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": done * shape[3] / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{done} sequence(s) of the c2 workload (8 kv heads x 32768 tokens, 32 query heads): "
                      "C oracle ASTC decode on all threads + NumPy fp32 restore and attention",
            "seconds": dt}


def run_reference(args) -> dict | None:
    world, rank, local = dist_env()
    if rank != 0:
        return None
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    threads = O.cpu_threads()
    if args.workload != "c2":
        return {"impl": "reference", "unavailable": f"CPU reference arm implemented for the c2 workload, not {args.workload}"}
    seqs, shape = cpu_unit_inputs("c2", 1)
    t0 = time.perf_counter()
    cpu_reference_step(seqs[0], shape, threads)
    per_seq = time.perf_counter() - t0
    # One step = a bounded sample: whole sequences if they fit ~120 s overall,
    # else a fraction measured in kv heads (value counts tokens x heads / Hkv).
    budget = 120.0 / max(1, args.steps + args.warmup)
    Hq, Hkv, D, T, bs, cols = shape
    heads = max(1, min(Hkv, int(Hkv * budget / max(per_seq, 1e-9))))
    blocks, off, scl, k, q = seqs[0]
    g = Hq // Hkv
    sub = (blocks[:heads], off[:heads], scl[:heads], k[:heads], q[: heads * g])
    sub_shape = (heads * g, heads, D, T, bs, cols)
    for _ in range(args.warmup):
        cpu_reference_step(sub, sub_shape, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(sub, sub_shape, threads)
    dt = time.perf_counter() - t0
    value = args.steps * T * heads / Hkv / dt
    sample = (f"per step {heads}/{Hkv} kv heads of one c2 sequence (32768 tokens): C oracle ASTC decode on "
              f"{threads} threads + NumPy fp32 restore and attention")
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded)",
            "config": {"workload": "config2_llama3_8b_gqa", "q_heads": Hq, "kv_heads": Hkv, "head_dim": D, "tokens": T,
                       "v": "astc 6x6 scalar block_affine (astcenc golden blocks tiled)", "k": "fp16"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c1", "c2", "c3", "c4", "decode4", "decode6", "decode8"], default="c2")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling of small cases)")
    ap.add_argument("--split-tokens", type=int, default=0,
                    help="tokens per split (0: the library's automatic choice; set it to profile a small batch "
                         "with the full run's split structure)")
    ap.add_argument("--decode-blocks", type=int, default=1 << 26,
                    help="blocks per step of the decode microbench (a multiple of 2^20; smaller for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        line = run_reference(args)
    elif args.workload.startswith("decode"):
        line = run_decode(args)
    else:
        line = run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
