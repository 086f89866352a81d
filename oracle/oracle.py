"""TEST INFRASTRUCTURE ONLY — the CPU oracle for the ASTC-KV decode-attention path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module. It is the checker, never the shipped path.

Two halves:

* ``decode_blocks`` / ``decode_image_f32`` wrap ``astc_oracle.c`` (a plain-C
  restatement of the Khronos ASTC LDR decode that astcenc 5.7.0 implements for
  the reference's ``akv_decode``, astc_kv/bridge.cpp:27-35).
* ``restore``, ``attention``, ``errors`` and ``attention_metrics`` restate the
  NumPy numerics of astc_kv/codec.py: the fp32 affine restore
  (codec.py:198-208, unfused ``rec*scale + offset``), GQA causal attention
  (codec.py:253-267) and the error metrics (codec.py:270-283).
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libastc_oracle.so"

OUT_UNORM8, OUT_FP16, OUT_UNORM16 = 0, 1, 2

_lib = None


def build() -> Path:
    """Compile the C oracle with its Makefile (gcc only; no GPU)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ct.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        l = ct.CDLL(str(LIB_PATH))
        l.astc_oracle_decode_blocks.argtypes = [ct.c_void_p, ct.c_int64, ct.c_int, ct.c_int, ct.c_int, ct.c_void_p, ct.c_int]
        l.astc_oracle_decode_blocks.restype = ct.c_int
        l.astc_oracle_decode_image_f32.argtypes = [ct.c_void_p, ct.c_size_t, ct.c_int, ct.c_int, ct.c_void_p, ct.c_uint, ct.c_uint]
        l.astc_oracle_decode_image_f32.restype = ct.c_int
        l.astc_oracle_block_info.argtypes = [ct.c_void_p, ct.c_int, ct.c_int, ct.c_void_p]
        l.astc_oracle_unorm16_to_half.argtypes = [ct.c_uint16]
        l.astc_oracle_unorm16_to_half.restype = ct.c_uint16
        for name in ("astc_oracle_unquant_color", "astc_oracle_unquant_weight", "astc_oracle_bise_bits"):
            getattr(l, name).argtypes = [ct.c_int, ct.c_int]
        l.astc_oracle_partition.argtypes = [ct.c_int] * 5
        _lib = l
    return _lib


def decode_blocks(blocks: np.ndarray, block: int, mode: int = OUT_UNORM8, threads: int = 1) -> np.ndarray:
    """Decode uint8[n,16] blocks of a square footprint -> [n, block, block, 4]
    (uint8 / fp16 / uint16 per ``mode``)."""
    bx = by = block
    blocks = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 16)
    n = blocks.shape[0]
    dtype = {OUT_UNORM8: np.uint8, OUT_FP16: np.float16, OUT_UNORM16: np.uint16}[mode]
    out = np.empty((n, by, bx, 4), dtype)
    rc = lib().astc_oracle_decode_blocks(blocks.ctypes.data, n, bx, by, mode, out.ctypes.data, threads)
    if rc:
        raise ValueError("oracle decode rejected its arguments")
    return out


def decode_image_f32(payload: bytes | np.ndarray, block: int, width: int, height: int) -> np.ndarray:
    """Same contract as the reference's ``akv_decode`` (bridge.cpp:27-35): float32 [h, w, 4]."""
    buf = np.frombuffer(bytes(payload), np.uint8) if not isinstance(payload, np.ndarray) else np.ascontiguousarray(payload, np.uint8)
    out = np.empty((height, width, 4), np.float32)
    rc = lib().astc_oracle_decode_image_f32(buf.ctypes.data, buf.size, block, block, out.ctypes.data, width, height)
    if rc:
        raise ValueError("payload size does not match the image")
    return out


def block_info(block16: np.ndarray, block: int) -> dict:
    bx = by = block
    info = np.zeros(8, np.int32)
    b = np.ascontiguousarray(block16, np.uint8)
    lib().astc_oracle_block_info(b.ctypes.data, bx, by, info.ctypes.data)
    keys = ("partitions", "dual", "wx", "wy", "wq", "cq", "cem0", "kind")
    return dict(zip(keys, map(int, info)))


def blocks_to_image(texels: np.ndarray, cols: int, rows: int) -> np.ndarray:
    """[rows*cols, by, bx, C] per-block texels -> [rows*by, cols*bx, C] image."""
    n, by, bx, c = texels.shape
    assert n == rows * cols
    return texels.reshape(rows, cols, by, bx, c).transpose(0, 2, 1, 3, 4).reshape(rows * by, cols * bx, c)


def image_to_blocks(image: np.ndarray, bx: int, by: int) -> np.ndarray:
    """Inverse of ``blocks_to_image`` for images whose sides are block multiples."""
    h, w = image.shape[:2]
    rest = image.shape[2:]
    return image.reshape(h // by, by, w // bx, bx, *rest).swapaxes(1, 2).reshape(-1, by, bx, *rest)


# ---------------------------------------------------------------------------
# NumPy numerics restated from astc_kv/codec.py
# ---------------------------------------------------------------------------

def restore(u: np.ndarray, offsets: np.ndarray, scales: np.ndarray | None, normalization: str,
            page_tokens: int, dim: int, layout: str = "scalar", block: int | None = None) -> np.ndarray:
    """Affine restore of normalised decoded values, codec.py:198-208.

    ``u`` is the per-head decoded plane: scalar layout ``[H, T, W]`` (channel R),
    rgba ``[H, T, W, 4]``. Computation is fp32 ``rec*scale + offset`` (unfused),
    which reproduces the golden ``*_decoded.f32`` files bit for bit.
    ``block_affine`` (one (offset, scale) pair per ASTC block) is the
    per-block extension used by the larger configurations.
    """
    u = np.asarray(u, np.float32)
    heads, tokens = u.shape[0], u.shape[1]
    rec = u if layout == "scalar" else u[:, :, : dim // 4, :].reshape(heads, tokens, dim)
    rec = rec[:, :, :dim] if layout == "scalar" else rec
    if normalization == "page_channel":
        pages = tokens // page_tokens
        r = rec.reshape(heads, pages, page_tokens, dim) * scales[:, :, None, :].astype(np.float32) + offsets[:, :, None, :].astype(np.float32)
        return r.reshape(heads, tokens, dim)
    if normalization == "token":
        return rec * scales.astype(np.float32) + offsets.astype(np.float32)
    if normalization == "block_affine":
        s = np.repeat(np.repeat(scales.astype(np.float32), block, 1), block, 2)[:, :tokens, :dim]
        o = np.repeat(np.repeat(offsets.astype(np.float32), block, 1), block, 2)[:, :tokens, :dim]
        return rec * s + o
    raise ValueError("Unknown normalization")


def attention(q, k, v, positions):
    """GQA causal attention, codec.py:253-267 (fp32 NumPy)."""
    hq, n, d = q.shape
    hk, t, kd = k.shape
    if v.shape != k.shape or kd != d or hq % hk:
        raise ValueError("Incompatible attention shapes")
    qq = q.reshape(hk, hq // hk, n, d)
    scores = np.matmul(qq, k[:, None].swapaxes(-1, -2)) * np.float32(d ** -0.5)
    mask = np.arange(t)[None, :] <= np.asarray(positions)[:, None]
    scores = np.where(mask[None, None], scores, np.float32(-np.inf))
    scores -= scores.max(-1, keepdims=True)
    p = np.exp(scores)
    p /= p.sum(-1, keepdims=True)
    out = np.matmul(p, v[:, None]).reshape(hq, n, d)
    return out, p.reshape(hq, n, t)


def attention_f64(q, k, v, lengths=None):
    """Decode-step attention in float64 for every (batch, kv-head) group.

    q ``[B, Hq, D]``, k/v ``[B, Hkv, T, D]``; ``lengths[b]`` tokens are visible
    (all T when None). Same math as codec.py:253-267 with the query at the
    last visible position.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    b, hq, d = q.shape
    hk, t = k.shape[1], k.shape[2]
    out = np.zeros((b, hq, d))
    for i in range(b):
        n = t if lengths is None else int(lengths[i])
        if n == 0:
            continue  # empty sequence: the GPU path defines the output as 0
        qq = q[i].reshape(hk, hq // hk, d)
        s = np.einsum("hgd,htd->hgt", qq, k[i, :, :n]) * d ** -0.5
        s -= s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[i] = np.einsum("hgt,htd->hgd", p, v[i, :, :n]).reshape(hq, d)
    return out


def errors(reference, estimate):
    """codec.py:270-274."""
    a, b = np.asarray(reference, np.float64), np.asarray(estimate, np.float64)
    err = b - a
    return {"mse": float(np.mean(err * err)),
            "relative_l2": float(np.linalg.norm(err.ravel()) / max(np.linalg.norm(a.ravel()), 1e-30)),
            "max_abs": float(np.max(np.abs(err))),
            "cosine": float(np.sum(a * b) / max(np.linalg.norm(a.ravel()) * np.linalg.norm(b.ravel()), 1e-30))}


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
