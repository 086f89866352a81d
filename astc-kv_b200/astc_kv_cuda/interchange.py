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


def write_manifest(directory: str | Path, q: np.ndarray, k, v, *, page_tokens: int, layout: str = "scalar",
                   tokens: int | None = None, extra: dict | None = None, with_decoded: bool = True) -> dict:
    """Write an astc-kv-probe-v1 fixture (the reader above loads it back).

    `q` is float32 [Hq, D]; `k` / `v` are each either an ``EncodedTensor``
    (written as one ``.astc`` file per head plus fp16 offsets / scales and the
    fp32 restore) or a float array [Hkv, T, D] (written as FP16). Field names,
    file naming and byte accounting follow the reference's exporter
    (scripts/export_metal_fixture.py:31-63, docs/metal_path.md:50-73):
    ``logical_cache_bytes`` per ASTC side equals the tensor's ``byte_counts``
    (blocks with edge padding, fp16 offsets, fp16 scales). Token-normalised
    metadata is cut to the real tokens. ``with_decoded=False`` leaves out the
    optional ``*_decoded.f32`` restores (an ASTC side's restore runs on the
    GPU). Returns the manifest.
    """
    from .codec import EncodedTensor
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=True)
    q = np.asarray(q, np.float32)
    hq, dim = q.shape
    sides = {"k": k, "v": v}
    kvh = {s: (x.heads if isinstance(x, EncodedTensor) else np.asarray(x).shape[0]) for s, x in sides.items()}
    if kvh["k"] != kvh["v"]:
        raise ValueError("K and V must have the same kv heads")
    t_all = {s: (x.tokens if isinstance(x, EncodedTensor) else np.asarray(x).shape[1]) for s, x in sides.items()}
    t = tokens if tokens is not None else min(t_all.values())
    if all(not isinstance(x, EncodedTensor) for x in sides.values()):
        raise ValueError("At least one side must use ASTC for this probe")
    q.astype("<f4").tofile(root / "q.f32")
    m = {"format": "astc-kv-probe-v1", "tokens": int(t), "query_heads": int(hq), "kv_heads": int(kvh["k"]),
         "head_dim": int(dim), "page_tokens": int(page_tokens), "layout": layout, "metadata_dtype": "float16_le",
         "query_file": "q.f32", "logical_cache_bytes": {}, "file_header_bytes": 0, **(extra or {})}
    for name, x in sides.items():
        if isinstance(x, EncodedTensor):
            m[name + "_storage"] = "astc"
            files = []
            for h in range(x.heads):
                fn = f"{name}-h{h:03d}.astc"
                (root / fn).write_bytes(x.astc_file(h))
                files.append(fn)
            m[name + "_files"] = files
            m[name + "_normalization"] = x.normalization
            off, scl = x.offsets, x.scales
            if x.normalization == "token":
                off, scl = off[:, :t], scl[:, :t]
            for suffix, a in (("offset", off), ("scale", scl)):
                fn = f"{name}_{suffix}.f16"
                np.asarray(a, "<f2").tofile(root / fn)
                m[f"{name}_{suffix}_file"] = fn
            decoded = np.asarray(x.decoded, np.float32)[:, :t] if with_decoded else None
            m["logical_cache_bytes"][name] = {"astc_blocks_with_padding": int(sum(map(len, x.payloads))),
                                              "fp16_offsets": int(np.asarray(off).nbytes),
                                              "fp16_scales": int(np.asarray(scl).nbytes)}
            m["file_header_bytes"] += 16 * x.heads
        else:
            xa = np.asarray(x, np.float32)[:, :t]
            fn = name + ".f16"
            xa.astype("<f2").tofile(root / fn)
            m[name + "_storage"] = "fp16"
            m[name + "_file"] = fn
            decoded = xa.astype(np.float16).astype(np.float32)
            m["logical_cache_bytes"][name] = {"fp16_payload": int(xa.size * 2)}
        if with_decoded:
            fn = name + "_decoded.f32"
            decoded.astype("<f4").tofile(root / fn)
            m[name + "_decoded_file"] = fn
    scalars = 2 * kvh["k"] * t * dim
    m["logical_bits_per_original_kv_scalar"] = sum(sum(b.values()) for b in m["logical_cache_bytes"].values()) * 8 / scalars
    (root / "manifest.json").write_text(json.dumps(m, indent=2) + "\n")
    return m
