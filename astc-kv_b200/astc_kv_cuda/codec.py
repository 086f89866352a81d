"""Drop-in mirror of the reference's ``astc_kv/codec.py`` call surface, with the
decode + restore + attention half on the B200.

Same names, arguments and errors as the reference module:

* ``encode_tensor`` (codec.py:116-215) normalises on the CPU exactly as the
  reference does and encodes with ``AstcEncoder``; ``EncodedTensor.decoded``
  is restored on the GPU (akv_cuda_restore_plane) instead of by astcenc's
  CPU decode (codec.py:56, :198-208).
* ``attention`` (codec.py:253-267) runs the fused split-K kernel when K/V are
  ``EncodedTensor``s (or fp16 arrays) and returns ``(out, None)``: the
  flash-decoding kernel never materialises the probability matrix.
* ``fp16_floor`` / ``fp16_ceil`` / ``align`` / ``errors`` / ``attention_metrics``
  are the same host helpers (codec.py:18-19, :70-81, :270-283).

Extension: ``normalization='block_affine'`` (one fp16 (offset, scale) per ASTC
block, LDR) generalises the reference's HDR-only ``block_min`` (codec.py:167-172)
to the per-block affine map the benchmark configurations use.

``AstcEncoder`` uses the reference's astcenc bridge (``libakv_astc.so``, built
from astc_kv/bridge.cpp against astcenc 5.7.0) when ``AKV_ASTCENC_BRIDGE`` names
one; otherwise this library's own CPU encoder (include/akv_host.h), which
writes legal ASTC but does not reproduce astcenc's block choices.
"""
from __future__ import annotations

import ctypes as ct
import math
import os
import struct
import time
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L


def align(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def fp16_floor(x):
    """Largest fp16 <= x (codec.py:70-74)."""
    x = np.asarray(x, np.float32)
    h = x.astype(np.float16)
    return np.where(h.astype(np.float32) > x, np.nextafter(h, np.float16(-np.inf)), h).astype(np.float16)


def fp16_ceil(x):
    """Smallest fp16 >= x (codec.py:77-81)."""
    x = np.asarray(x, np.float32)
    h = x.astype(np.float16)
    return np.where(h.astype(np.float32) < x, np.nextafter(h, np.float16(np.inf)), h).astype(np.float16)


class AstcEncoder:
    """CPU ASTC encoder with the reference class's interface (codec.py:22-67)."""

    def __init__(self, block: int, quality: float = 98, hdr: bool = False):
        if block not in (4, 6, 8):
            raise ValueError("block must be 4, 6 or 8")
        self.block = block
        self.quality = quality
        self.hdr = hdr
        self.ctx = None
        self.bridge = None
        path = os.environ.get("AKV_ASTCENC_BRIDGE")
        if path:
            lib = ct.CDLL(path)
            lib.akv_create.argtypes = [ct.c_uint, ct.c_uint, ct.c_float, ct.c_int, ct.POINTER(ct.c_int)]
            lib.akv_create.restype = ct.c_void_p
            lib.akv_destroy.argtypes = [ct.c_void_p]
            lib.akv_error.argtypes = [ct.c_int]
            lib.akv_error.restype = ct.c_char_p
            lib.akv_encode.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_uint, ct.c_uint, ct.c_void_p, ct.c_size_t]
            err = ct.c_int()
            self.ctx = lib.akv_create(block, block, quality, int(hdr), ct.byref(err))
            if err.value:
                raise RuntimeError(lib.akv_error(err.value).decode())
            if not self.ctx:
                raise RuntimeError("astcenc context allocation failed")
            self.bridge = lib
        elif hdr:
            raise ValueError("HDR encoding needs the astcenc bridge (AKV_ASTCENC_BRIDGE)")
        self.name = "astcenc-bridge" if self.bridge else "akv-host-encoder"

    def encode(self, image: np.ndarray, layout: str = "scalar") -> tuple[bytes, float]:
        image = np.ascontiguousarray(image, dtype=np.float32)
        h, w, components = image.shape
        if components != 4 or not np.all(np.isfinite(image)):
            raise ValueError("Expected finite HxWx4 input")
        n = math.ceil(w / self.block) * math.ceil(h / self.block) * 16
        t0 = time.perf_counter()
        if self.bridge:
            payload = np.empty(n, np.uint8)
            code = self.bridge.akv_encode(self.ctx, image.ctypes.data, w, h, payload.ctypes.data, n)
            if code:
                raise RuntimeError(self.bridge.akv_error(code).decode())
            out = payload.tobytes()
        else:
            effort = 0 if self.quality < 40 else (1 if self.quality < 90 else 2)
            from .ops import host_encode
            out = host_encode(image, self.block, layout, effort)
        return out, time.perf_counter() - t0

    def roundtrip(self, image: np.ndarray, layout: str = "scalar") -> tuple[bytes, np.ndarray, float]:
        """Encode on the CPU, decode on the GPU (float32 [h, w, 4], the fp16 view)."""
        import torch
        from .ops import decode_image
        payload, seconds = self.encode(image, layout)
        h, w, _ = image.shape
        dev = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
        dec = decode_image(dev, self.block, w, h).cpu().numpy()
        if not np.all(np.isfinite(dec)):
            raise ValueError("Non-finite ASTC reconstruction")
        return payload, dec, seconds

    def close(self):
        if self.bridge is not None and self.ctx:
            self.bridge.akv_destroy(self.ctx)
        self.ctx = None

    def __del__(self):
        self.close()


@dataclass
class EncodedTensor:
    """Same fields as codec.py:84-113. ``decoded`` is restored on the GPU on
    first access when the encoder did not provide it."""
    _decoded: np.ndarray | None
    payloads: list[bytes]
    width: int
    height: int
    block: int
    layout: str
    profile: str
    normalization: str
    offsets: np.ndarray
    scales: np.ndarray | None
    page_tokens: int
    byte_counts: dict[str, int]
    encode_cpu_s: float
    permutation: str | None = None
    metadata: dict = field(default_factory=dict)
    p_tokens: np.ndarray | None = None
    p_channels: np.ndarray | None = None

    @property
    def heads(self) -> int:
        return len(self.payloads)

    @property
    def dim(self) -> int:
        return int(self.metadata["dim"])

    @property
    def tokens(self) -> int:
        return self.height

    @property
    def decoded(self) -> np.ndarray:
        if self._decoded is None:
            self._decoded = self.restore_gpu().cpu().numpy()
        return self._decoded

    @property
    def logical_bytes(self):
        return sum(self.byte_counts.values())

    @property
    def bits_per_scalar(self):
        return self.logical_bytes * 8 / (self.heads * self.tokens * self.dim)

    def astc_file(self, head: int) -> bytes:
        """16-byte .astc header + blocks (codec.py:110-113)."""
        def u24(v):
            return bytes((v & 255, (v >> 8) & 255, (v >> 16) & 255))
        return struct.pack("<I", 0x5CA1AB13) + bytes((self.block, self.block, 1)) + u24(self.width) + u24(self.height) + u24(1) + self.payloads[head]

    # ---- device forms -------------------------------------------------
    def blocks_array(self) -> np.ndarray:
        """uint8 [H, rows, cols, 16]."""
        rows, cols = self.height // self.block, self.width // self.block
        return np.stack([np.frombuffer(p, np.uint8).reshape(rows, cols, 16) for p in self.payloads])

    def device_plane(self, device=None):
        """`DevicePlane` (batch 1) holding this tensor's blocks and metadata."""
        import torch
        from .ops import contiguous_astc_plane
        if self.permutation is not None:
            raise ValueError("permuted encodings have no direct device plane")
        dev = torch.device("cuda") if device is None else device
        blocks = torch.from_numpy(self.blocks_array()[None].copy()).to(dev)
        off = torch.from_numpy(np.ascontiguousarray(self.offsets).view(np.int16).copy()).view(torch.float16).to(dev)
        scl = torch.from_numpy(np.ascontiguousarray(self.scales).view(np.int16).copy()).view(torch.float16).to(dev)
        return contiguous_astc_plane(blocks, off.reshape(1, *off.shape), scl.reshape(1, *scl.shape), block=self.block,
                                     layout=self.layout, normalization=self.normalization, head_dim=self.dim,
                                     page_tokens=self.page_tokens)

    def restore_gpu(self):
        """fp32 [H, T, D] torch tensor on the GPU: decode + restore (+ inverse permutation)."""
        from .ops import restore_plane
        import torch
        perm = self.permutation
        self.permutation = None
        try:
            plane = self.device_plane()
        finally:
            self.permutation = perm
        rec = restore_plane(plane, batch=1, kv_heads=self.heads, max_tokens=self.height, head_dim=self.dim,
                            page_tokens=self.page_tokens)[0]
        if self.p_tokens is not None:
            inv_t = torch.from_numpy(np.argsort(self.p_tokens)).to(rec.device)
            inv_c = torch.from_numpy(np.argsort(self.p_channels)).to(rec.device)
            rec = rec[:, inv_t][:, :, inv_c]
        return rec.contiguous()


def encode_tensor(x: np.ndarray, config: dict, page_tokens: int = 96, quality: float = 98,
                  seed: int = 20261028) -> EncodedTensor:
    """Encode [H,T,D]. Call only on already completed historical pages.

    Validation, normalisation and byte accounting follow codec.py:116-215.
    """
    x = np.asarray(x, np.float32)
    if x.ndim != 3 or not np.all(np.isfinite(x)):
        raise ValueError("Expected finite [H,T,D]")
    heads, tokens, dim = x.shape
    block = int(config["block"])
    layout = config["layout"]
    profile = config.get("profile", "ldr")
    normalization = config["normalization"]
    permutation = config.get("permutation")
    if page_tokens % block:
        raise ValueError("Page boundary must align to ASTC block rows")
    if layout not in ("scalar", "rgba") or (layout == "rgba" and dim % 4):
        raise ValueError("Unsupported scalar/component layout")
    if tokens % page_tokens:
        raise ValueError("Only completed pages enter encoder; keep incomplete page in tail")
    if profile == "hdr" and (layout != "scalar" or normalization != "block_min"):
        raise ValueError("HDR pilot supports scalar block-min only")
    if normalization == "block_affine" and (layout != "scalar" or profile != "ldr"):
        raise ValueError("block_affine is a scalar LDR normalisation")
    comp = 1 if layout == "scalar" else 4
    width, height = align(dim // comp, block), tokens
    work = x.copy()
    rng = np.random.default_rng(seed)
    p_tokens = np.arange(tokens)
    p_channels = np.arange(dim)
    map_bytes = 0
    if permutation == "tokens_within_page":
        perm = rng.permutation(page_tokens)
        p_tokens = (np.arange(tokens // page_tokens)[:, None] * page_tokens + perm[None]).ravel()
        work = work[:, p_tokens, :]
        map_bytes = page_tokens * 2
    elif permutation == "channels":
        p_channels = rng.permutation(dim)
        work = work[:, :, p_channels]
        map_bytes = dim * 2
    elif permutation is not None:
        raise ValueError("Unknown permutation")
    pages = tokens // page_tokens
    if normalization == "page_channel":
        view = work.reshape(heads, pages, page_tokens, dim)
        lo = view.min(axis=2)
        hi = view.max(axis=2)
        offset = fp16_floor(lo)
        scale = fp16_ceil(np.maximum(hi - offset.astype(np.float32), np.float32(2 ** -24)))
        normalized = ((view - offset[:, :, None, :].astype(np.float32)) / scale[:, :, None, :].astype(np.float32)).reshape(work.shape)
    elif normalization == "token":
        lo, hi = work.min(-1, keepdims=True), work.max(-1, keepdims=True)
        offset = fp16_floor(lo)
        scale = fp16_ceil(np.maximum(hi - offset.astype(np.float32), np.float32(2 ** -24)))
        normalized = (work - offset.astype(np.float32)) / scale.astype(np.float32)
    elif normalization == "block_affine":
        padded = np.pad(work, ((0, 0), (0, 0), (0, width - dim)), mode="edge")
        view = padded.reshape(heads, height // block, block, width // block, block)
        offset = fp16_floor(view.min(axis=(2, 4)))
        scale = fp16_ceil(np.maximum(view.max(axis=(2, 4)) - offset.astype(np.float32), np.float32(2 ** -24)))
        normalized = ((view - offset[:, :, None, :, None].astype(np.float32)) /
                      scale[:, :, None, :, None].astype(np.float32)).reshape(heads, height, width)
    elif normalization == "block_min":
        raise ValueError("block_min is the reference's HDR normalisation; it needs the astcenc bridge and has no GPU path")
    else:
        raise ValueError("Unknown normalization")
    if not np.all(np.isfinite(offset)) or (scale is not None and not np.all(np.isfinite(scale))):
        raise ValueError("FP16 metadata overflow")
    if normalized.min() < -1e-5 or normalized.max() > 1 + 1e-5:
        raise AssertionError("FP16 rounded metadata fails range coverage")
    normalized = np.clip(normalized, 0, 1)
    if layout == "scalar":
        scalar = np.pad(normalized, ((0, 0), (0, 0), (0, width - normalized.shape[-1])), mode="edge")
        images = np.ones((heads, height, width, 4), np.float32)
        images[..., :3] = scalar[..., None]
    else:
        rgba = normalized.reshape(heads, tokens, dim // 4, 4)
        images = np.pad(rgba, ((0, 0), (0, 0), (0, width - dim // 4), (0, 0)), mode="edge")
    encoder = AstcEncoder(block, quality, profile == "hdr")
    payloads, elapsed = [], 0.0
    try:
        for im in images:
            payload, seconds = encoder.encode(im, layout)
            payloads.append(payload)
            elapsed += seconds
    finally:
        encoder.close()
    counts = {"astc_blocks_including_edge_padding": sum(map(len, payloads)),
              "fp16_offsets": offset.nbytes, "fp16_scales": 0 if scale is None else scale.nbytes,
              "permutation_map": map_bytes}
    return EncodedTensor(None, payloads, width, height, block, layout, profile, normalization, offset, scale,
                         page_tokens, counts, elapsed, permutation,
                         {"quality": quality, "original_scalars": x.size, "file_header_bytes": 16 * heads,
                          "logical_bytes_scope": "blocks+metadata+fixed_permutation; no allocation/staging/tail",
                          "encoder": encoder.name, "dim": dim},
                         p_tokens if permutation else None, p_channels if permutation else None)


def attention(q, k, v, positions, k_tail=None, v_tail=None):
    """GQA causal attention with the reference's signature (codec.py:253-267).

    ``k`` and ``v`` are ``EncodedTensor`` (ASTC planes read directly by the
    kernel) or fp16-representable arrays ``[Hkv, T, D]`` (fp16 planes). Query
    i attends tokens t <= positions[i]. Returns ``(out [Hq, N, D], None)``.

    ``k_tail`` / ``v_tail`` (optional, arrays ``[Hkv, n, D]``, kept in FP16):
    the newest tokens that do not fill a page yet, positions T .. T + n - 1 of
    the same sequence, attended in the same softmax (the reference's encoder
    rejects incomplete pages, codec.py:132-133).
    """
    import torch
    from .ops import Attention, contiguous_fp16_plane
    q = np.asarray(q, np.float32)
    hq, n, d = q.shape

    def plane(x):
        if isinstance(x, EncodedTensor):
            if x.dim != d:
                raise ValueError("Incompatible attention shapes")
            p = x.device_plane()
            return p, x.heads, x.height, x.page_tokens
        a = np.asarray(x, np.float32)
        if a.ndim != 3 or a.shape[-1] != d:
            raise ValueError("Incompatible attention shapes")
        t = torch.from_numpy(a.astype(np.float16))[None].cuda().contiguous()
        return contiguous_fp16_plane(t, a.shape[1]), a.shape[0], a.shape[1], a.shape[1]

    kp, hk, tk, pk = plane(k)
    vp, hv, tv, pv = plane(v)
    if (hk, tk) != (hv, tv) or hq % hk:
        raise ValueError("Incompatible attention shapes")
    page = math.lcm(pk, pv)
    if tk % page:
        page = tk
    # Every query shares the same cache: batch stride 0.
    for p in (kp, vp):
        p.stride_batch = 0
        p.meta_stride_batch = 0
        p.side_stride_batch = 0
    qd = torch.from_numpy(np.ascontiguousarray(q.transpose(1, 0, 2))).cuda()
    pos1 = np.asarray(positions, np.int64) + 1
    lens = torch.from_numpy(pos1).clamp(0, tk).to(torch.int32).cuda()
    tail = {}
    if (k_tail is None) != (v_tail is None):
        raise ValueError("k_tail and v_tail go together")
    if k_tail is not None:
        tkp, htk, ntk, _ = plane(k_tail)
        tvp, htv, ntv, _ = plane(v_tail)
        if (htk, ntk) != (htv, ntv) or htk != hk:
            raise ValueError("Incompatible attention shapes")
        for p in (tkp, tvp):
            p.stride_batch = 0
        tail = {"tail_k": tkp, "tail_v": tvp, "tail_tokens": ntk,
                "tail_lens": torch.from_numpy(pos1 - tk).clamp(0, ntk).to(torch.int32).cuda()}
    out = Attention(qd, kp, vp, page_tokens=page, max_tokens=tk, seq_lens=lens, **tail).run()
    return out.cpu().numpy().transpose(1, 0, 2).copy(), None


def errors(reference, estimate):
    """codec.py:270-274."""
    a, b = np.asarray(reference, np.float64), np.asarray(estimate, np.float64)
    err = b - a
    return {"mse": float(np.mean(err * err)),
            "relative_l2": float(np.linalg.norm(err.ravel()) / max(np.linalg.norm(a.ravel()), 1e-30)),
            "max_abs": float(np.max(np.abs(err))),
            "cosine": float(np.sum(a * b) / max(np.linalg.norm(a.ravel()) * np.linalg.norm(b.ravel()), 1e-30))}


def attention_metrics(reference, estimate, reference_probs, estimate_probs):
    """codec.py:277-283."""
    metrics = errors(reference, estimate)
    a, b = reference_probs.astype(np.float64), estimate_probs.astype(np.float64)
    kl = np.sum(a * (np.log(np.maximum(a, 1e-300)) - np.log(np.maximum(b, 1e-300))), axis=-1)
    metrics.update(mean_kl_nats=float(np.mean(kl)), p95_kl_nats=float(np.percentile(kl, 95)),
                   mean_total_variation=float(np.mean(np.abs(a - b).sum(-1) * 0.5)))
    return metrics
