""".astc files and the ``astc-kv-probe-v1`` manifest (reference interchange).

File format (astc_kv/codec.py:110-113; metal/probe_gqa_v10.mm:120-134):
magic 0x5CA1AB13 (LE u32), block x/y/z (u8 each), width/height/depth (LE u24
each), then row-major 16-byte blocks. Manifest fields: docs/metal_path.md:50-73.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

MAGIC = 0x5CA1AB13


def read_astc(raw: bytes) -> tuple[int, int, int, bytes]:
    """-> (block, width, height, payload). 2D, square footprints only."""
    if len(raw) < 16 or struct.unpack("<I", raw[:4])[0] != MAGIC:
        raise ValueError("not an .astc file (bad magic)")
    bx, by, bz = raw[4], raw[5], raw[6]
    w = int.from_bytes(raw[7:10], "little")
    h = int.from_bytes(raw[10:13], "little")
    d = int.from_bytes(raw[13:16], "little")
    if bz != 1 or d != 1 or bx != by or bx not in (4, 6, 8):
        raise ValueError("only 2D square 4x4/6x6/8x8 .astc files are supported")
    n = ((w + bx - 1) // bx) * ((h + by - 1) // by) * 16
    if len(raw) - 16 != n:
        raise ValueError("payload size does not match the header")
    return bx, w, h, raw[16:]


def write_astc(block: int, width: int, height: int, payload: bytes) -> bytes:
    def u24(v):
        return bytes((v & 255, (v >> 8) & 255, (v >> 16) & 255))
    return struct.pack("<I", MAGIC) + bytes((block, block, 1)) + u24(width) + u24(height) + u24(1) + payload


def load_manifest(directory: str | Path) -> dict:
    """Read an astc-kv-probe-v1 fixture into NumPy arrays.

    Returns q [Hq, D] and, per side 'k'/'v', either {'fp16': [Hkv, T, D]} or
    {'blocks': uint8 [Hkv, rows, cols, 16], 'block', 'normalization',
    'offsets', 'scales'} plus the optional '*_decoded' reference restore.
    """
    root = Path(directory)
    m = json.loads((root / "manifest.json").read_text())
    if m.get("format") != "astc-kv-probe-v1" or m.get("metadata_dtype") != "float16_le":
        raise ValueError("not an astc-kv-probe-v1 manifest")
    T, Hq, Hkv, D, P = m["tokens"], m["query_heads"], m["kv_heads"], m["head_dim"], m["page_tokens"]
    out = {"manifest": m, "q": np.fromfile(root / m["query_file"], "<f4").reshape(Hq, D)}
    for side in ("k", "v"):
        storage = m.get(side + "_storage", "astc")
        entry: dict = {"storage": storage}
        if storage == "fp16":
            entry["fp16"] = np.fromfile(root / m[side + "_file"], "<f2").reshape(Hkv, T, D)
        else:
            blocks = []
            for name in m[side + "_files"]:
                b, w, h, payload = read_astc((root / name).read_bytes())
                blocks.append(np.frombuffer(payload, np.uint8).reshape(h // b, w // b, 16))
                entry.update(block=b, width=w, height=h)
            entry["blocks"] = np.stack(blocks)
            norm = m.get(side + "_normalization", "page_channel")
            entry["normalization"] = norm
            shape = (Hkv, T, 1) if norm == "token" else (Hkv, -1, D)
            entry["offsets"] = np.fromfile(root / m[side + "_offset_file"], "<f2").reshape(shape)
            entry["scales"] = np.fromfile(root / m[side + "_scale_file"], "<f2").reshape(shape)
        if m.get(side + "_decoded_file"):
            entry["decoded"] = np.fromfile(root / m[side + "_decoded_file"], "<f4").reshape(Hkv, T, D)
        out[side] = entry
    return out
