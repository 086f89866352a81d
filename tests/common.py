"""Shared helpers for the tests: golden loaders, synthetic caches, oracle views."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"

# Tolerances of the attention parity gate (north star): max-abs 2e-3 and
# relative 1e-3 against the NumPy reference on the same decoded values, plus
# the reference probe's own gate, relative L2 <= 1e-4 (probe_gqa_v10.mm:722).
ATOL, RTOL, REL_L2 = 2e-3, 1e-3, 1e-4


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def oracle_u(blocks: np.ndarray, block: int, layout: str, dim: int) -> np.ndarray:
    """Oracle fp16 view of a plane: blocks [H, rows, cols, 16] -> u [H, T, D] (float32)."""
    H, rows, cols, _ = blocks.shape
    tex = O.decode_blocks(blocks.reshape(-1, 16), block, O.OUT_FP16, threads=O.cpu_threads()).astype(np.float32)
    out = []
    for h in range(H):
        img = O.blocks_to_image(tex[h * rows * cols:(h + 1) * rows * cols], cols, rows)
        out.append(img[:, :dim, 0] if layout == "scalar" else img[:, : dim // 4, :].reshape(rows * block, dim))
    return np.stack(out)


def oracle_restore(blocks, offsets, scales, normalization, block, layout, dim, page_tokens):
    """Oracle decode + unfused fp32 restore (codec.py:198-208) of [H, rows, cols, 16]."""
    u = oracle_u(blocks, block, layout, dim)
    H, T = u.shape[:2]
    if normalization == "token":
        return (u * scales.reshape(H, T, 1).astype(np.float32) + offsets.reshape(H, T, 1).astype(np.float32)).astype(np.float32)
    if normalization == "page_channel":
        pages = T // page_tokens
        r = u.reshape(H, pages, page_tokens, dim) * scales.reshape(H, pages, 1, dim).astype(np.float32) \
            + offsets.reshape(H, pages, 1, dim).astype(np.float32)
        return r.reshape(H, T, dim).astype(np.float32)
    if normalization == "block_affine":
        bw = block * (4 if layout == "rgba" else 1)  # channels one block spans
        s = np.repeat(np.repeat(scales.astype(np.float32), block, 1), bw, 2)[:, :T, :dim]
        o = np.repeat(np.repeat(offsets.astype(np.float32), block, 1), bw, 2)[:, :T, :dim]
        return (u * s + o).astype(np.float32)
    raise ValueError(normalization)


def kv_values(rng: np.random.Generator, B: int, H: int, T: int, D: int, outliers: int = 0):
    """x [B, H, T, D] ~ N(0,1) x per-channel lognormal(0, 0.5) scale, with
    `outliers` channels per kv head scaled x8 (the value distribution the
    benchmark configurations name). Returns (x, outlier_channels [H, outliers])."""
    x = rng.standard_normal((B, H, T, D)).astype(np.float32)
    x *= rng.lognormal(0.0, 0.5, size=(1, H, 1, D)).astype(np.float32)
    ch = np.stack([np.sort(rng.choice(D, outliers, replace=False)) for _ in range(H)]).astype(np.int32) \
        if outliers else np.zeros((H, 0), np.int32)
    for h in range(H):
        x[:, h][..., ch[h]] *= 8
    return x, ch


def make_astc_plane(x: np.ndarray, *, block: int, layout: str, normalization: str, page_tokens: int,
                    side_channels: np.ndarray | None = None, effort: int = 0) -> dict:
    """Encode x [B, H, T, D] per batch element with the package's CPU encoder.

    Returns numpy blocks [B, H, rows, cols, 16], offsets/scales with a batch
    dimension, the oracle restore [B, H, T, D] of exactly those blocks, and
    the side plane [B, H, T, S] when `side_channels` is given (those channels
    are zeroed before encoding and restored from the fp16 side values)."""
    from astc_kv_cuda.codec import encode_tensor
    B, H, T, D = x.shape
    quality = {0: 10, 1: 60, 2: 98}[effort]
    enc_in = x.copy()
    side = None
    if side_channels is not None and side_channels.shape[1]:
        side = np.stack([np.stack([x[b, h][:, side_channels[h]] for h in range(H)]) for b in range(B)]).astype(np.float16)
        for h in range(H):
            enc_in[:, h][..., side_channels[h]] = 0.0
    blocks, offs, scls, rec = [], [], [], []
    for b in range(B):
        e = encode_tensor(enc_in[b], {"block": block, "layout": layout, "normalization": normalization},
                          page_tokens=page_tokens, quality=quality)
        bl = e.blocks_array()
        blocks.append(bl)
        offs.append(e.offsets)
        scls.append(e.scales)
        rec.append(oracle_restore(bl, e.offsets, e.scales, normalization, block, layout, D, page_tokens))
    out = {"blocks": np.stack(blocks), "offsets": np.stack(offs), "scales": np.stack(scls), "restored": np.stack(rec)}
    if side is not None:
        r = out["restored"]
        for h in range(H):
            r[:, h][..., side_channels[h]] = side[:, h].astype(np.float32)
        out["side"] = side
        out["side_channels"] = side_channels
    return out


def device_astc_plane(p: dict, *, block: int, layout: str, normalization: str, page_tokens: int, dim: int):
    import torch
    from astc_kv_cuda.ops import contiguous_astc_plane

    def f16(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float16).view(np.int16)).view(torch.float16).cuda()
    side = f16(p["side"]) if "side" in p else None
    ch = torch.from_numpy(np.ascontiguousarray(p["side_channels"], np.int32)).cuda() if "side" in p else None
    plane = contiguous_astc_plane(torch.from_numpy(p["blocks"]).cuda(), f16(p["offsets"]), f16(p["scales"]),
                                  block=block, layout=layout, normalization=normalization, head_dim=dim,
                                  page_tokens=page_tokens, side=side, side_channels=ch)
    plane.keepalive.append((side, ch))
    return plane


def assert_attention_close(got, ref, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL, err_msg=what)
    rel = np.linalg.norm((got - ref).ravel()) / max(np.linalg.norm(ref.ravel()), 1e-30)
    assert rel <= REL_L2, f"{what}: relative L2 {rel:.3e} > {REL_L2}"
