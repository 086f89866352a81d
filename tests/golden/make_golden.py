#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ from the reference tree.

Run here (where the reference is mounted); the GPU box only reads the
committed .npz files. Sources, all encoded by Arm astcenc 5.7.0 at quality 98,
6x6 LDR, scalar layout:

* results/metal_fixtures/story_l17_v_token6 — V ASTC (token normalisation),
  FP16 K, the query, and the reference restore `v_decoded.f32`.
* results/metal_fixtures/story_l17_kv_page6 — K and V ASTC (page_channel).
* results/block_geometry_v2/<capture>_l<layer>/identity.bin + identity.npy +
  fixed_input.npz — 24 capture/layer pairs (token normalisation, 288 tokens).
* metrics_golden.npz — the reference's `errors` / `attention_metrics`
  (codec.py:270-283) evaluated on seeded inputs.

Attention goldens come from importing the reference's own
astc_kv/codec.py `attention` (codec.py:253-267) on the reference restores.
Large restores are stored as SHA-256 digests of their float32 bytes.

Usage: python tests/golden/make_golden.py --reference /path/to/reference
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def read_astc(path: Path) -> tuple[int, int, int, np.ndarray]:
    raw = path.read_bytes()
    assert int.from_bytes(raw[:4], "little") == 0x5CA1AB13
    b = raw[4]
    w = int.from_bytes(raw[7:10], "little")
    h = int.from_bytes(raw[10:13], "little")
    return b, w, h, np.frombuffer(raw[16:], np.uint8).reshape(h // b, (w + b - 1) // b, 16)


def metrics_golden(ref: Path) -> None:
    """The reference's own `errors` / `attention_metrics` (codec.py:270-283) on
    seeded inputs: one attention output pair and one probability pair, with
    the values the reference returns."""
    from astc_kv.codec import attention_metrics, errors
    rng = np.random.default_rng(20261030)
    a = rng.standard_normal((9, 3, 64)).astype(np.float32)
    b = (a + rng.standard_normal(a.shape) * 1e-3).astype(np.float32)
    s1 = rng.standard_normal((9, 3, 384))
    s2 = s1 + rng.standard_normal(s1.shape) * 0.05
    pa = np.exp(s1 - s1.max(-1, keepdims=True))
    pa = (pa / pa.sum(-1, keepdims=True)).astype(np.float32)
    pb = np.exp(s2 - s2.max(-1, keepdims=True))
    pb = (pb / pb.sum(-1, keepdims=True)).astype(np.float32)
    e = errors(a, b)
    m = attention_metrics(a, b, pa, pb)
    keys_e, keys_m = sorted(e), sorted(m)
    np.savez_compressed(HERE / "metrics_golden.npz", a=a, b=b, pa=pa, pb=pb,
                        errors_keys=np.array(keys_e), errors_values=np.array([e[k] for k in keys_e]),
                        metrics_keys=np.array(keys_m), metrics_values=np.array([m[k] for k in keys_m]))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, required=True,
                    help="checkout of the reference project (BoyJayy/ASTC-KV)")
    ap.add_argument("--only", choices=["all", "metrics"], default="all",
                    help="metrics: write only metrics_golden.npz (the other fixtures stay as they are)")
    args = ap.parse_args()
    ref = args.reference
    sys.path.insert(0, str(ref))
    from astc_kv.codec import attention  # the reference implementation

    metrics_golden(ref)
    if args.only == "metrics":
        return

    # 1. V-only token fixture.
    d = ref / "results/metal_fixtures/story_l17_v_token6"
    m = json.loads((d / "manifest.json").read_text())
    T, Hq, Hkv, D = m["tokens"], m["query_heads"], m["kv_heads"], m["head_dim"]
    vb = np.stack([read_astc(d / f)[3] for f in m["v_files"]])
    q = np.fromfile(d / "q.f32", "<f4").reshape(Hq, D)
    k16 = np.fromfile(d / "k.f16", "<f2").reshape(Hkv, T, D)
    kd = np.fromfile(d / "k_decoded.f32", "<f4").reshape(Hkv, T, D)
    vd = np.fromfile(d / "v_decoded.f32", "<f4").reshape(Hkv, T, D)
    out, _ = attention(q[:, None, :], kd, vd, np.array([T - 1]))
    np.savez_compressed(HERE / "story_l17_v_token6.npz", v_blocks=vb,
                        v_offset=np.fromfile(d / "v_offset.f16", "<f2").reshape(Hkv, T, 1),
                        v_scale=np.fromfile(d / "v_scale.f16", "<f2").reshape(Hkv, T, 1),
                        v_decoded=vd, q=q, k=k16, attn_out=out[:, 0], page_tokens=m["page_tokens"])

    # 2. K+V page_channel fixture.
    d = ref / "results/metal_fixtures/story_l17_kv_page6"
    m = json.loads((d / "manifest.json").read_text())
    T, Hq, Hkv, D, P = m["tokens"], m["query_heads"], m["kv_heads"], m["head_dim"], m["page_tokens"]
    kb = np.stack([read_astc(d / f)[3] for f in m["k_files"]])
    vb = np.stack([read_astc(d / f)[3] for f in m["v_files"]])
    q = np.fromfile(d / "q.f32", "<f4").reshape(Hq, D)
    kd = np.fromfile(d / "k_decoded.f32", "<f4").reshape(Hkv, T, D)
    vd = np.fromfile(d / "v_decoded.f32", "<f4").reshape(Hkv, T, D)
    positions = np.array([T - 1, 200, 95, 0])
    out, _ = attention(np.repeat(q[:, None, :], len(positions), 1), kd, vd, positions)
    fields = {}
    for side, blocks in (("k", kb), ("v", vb)):
        fields[side + "_blocks"] = blocks
        for part in ("offset", "scale"):
            fields[f"{side}_{part}"] = np.fromfile(d / f"{side}_{part}.f16", "<f2").reshape(Hkv, T // P, D)
    np.savez_compressed(HERE / "story_l17_kv_page6.npz", q=q, positions=positions, attn_out=out,
                        k_decoded_sha256=sha(kd), v_decoded_sha256=sha(vd),
                        k_decoded_head0=kd[0], v_decoded_head0=vd[0], page_tokens=P, **fields)

    # 3. Block-geometry identity encodings (24 capture/layer pairs).
    base = ref / "results/block_geometry_v2"
    names, blocks, offs, scls, digests = [], [], [], [], []
    for pair in sorted(p for p in base.iterdir() if p.is_dir() and (p / "identity.bin").exists()):
        fi = np.load(pair / "fixed_input.npz")
        names.append(pair.name)
        blocks.append(np.fromfile(pair / "identity.bin", np.uint8).reshape(-1, 16))
        offs.append(fi["fp16_offsets"][..., 0])
        scls.append(fi["fp16_scales"][..., 0])
        digests.append(sha(np.load(pair / "identity.npy").astype("<f4")))
    np.savez_compressed(HERE / "block_geometry_identity.npz", names=np.array(names), blocks=np.stack(blocks),
                        offsets=np.stack(offs), scales=np.stack(scls), decoded_sha256=np.array(digests),
                        heads=3, tokens=288, dim=64, block=6, cols=11)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
