"""Device-resident ASTC KV planes and the GPU entry points.

This is the torch-facing layer over the C ABI: torch provides device memory
and streams; every computation below runs in libakv_cuda.so.

A `DevicePlane` is the HBM twin of one K or V side of a KV cache:

* ASTC storage: ``blocks`` uint8, one 16-byte block per ASTC block, laid out so
  that the page of (batch b, head h, physical page p) starts at
  ``b*stride_batch + h*stride_head + p*stride_page`` bytes and holds
  ``page_tokens/block`` block rows of ``ceil(width/block)`` blocks
  (the reference's per-head payload order, row-major blocks,
  metal/probe_gqa_v10.mm:235-236 / astc_kv/codec.py:110-113).
* fp16 offsets/scales with the same addressing in elements.
* FP16 storage: ``[.., page_tokens, head_dim]`` fp16 rows.
"""
from __future__ import annotations

import ctypes as ct
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(stream: torch.cuda.Stream | None) -> int | None:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("expected a CUDA tensor")


@dataclass
class DevicePlane:
    storage: str                      # "astc" | "fp16"
    data: torch.Tensor
    stride_batch: int
    stride_head: int
    stride_page: int
    block: int = 0
    layout: str = "scalar"
    normalization: str = "token"
    offsets: torch.Tensor | None = None
    scales: torch.Tensor | None = None
    meta_stride_batch: int = 0
    meta_stride_head: int = 0
    meta_stride_page: int = 0
    side: torch.Tensor | None = None
    side_channels: torch.Tensor | None = None
    side_stride_batch: int = 0
    side_stride_head: int = 0
    side_stride_page: int = 0
    kv_heads: int = 0
    capacity_tokens: int = 0          # tokens per sequence a contiguous plane holds (0 = paged)
    keepalive: list = field(default_factory=list)

    def to_c(self) -> L.AkvPlane:
        p = L.AkvPlane()
        p.storage = L.AKV_STORAGE_ASTC if self.storage == "astc" else L.AKV_STORAGE_FP16
        p.block = self.block
        p.layout = L.LAYOUTS[self.layout]
        p.normalization = L.NORMS[self.normalization]
        p.data = _ptr(self.data)
        p.stride_batch, p.stride_head, p.stride_page = self.stride_batch, self.stride_head, self.stride_page
        p.offsets, p.scales = _ptr(self.offsets), _ptr(self.scales)
        p.meta_stride_batch, p.meta_stride_head, p.meta_stride_page = (
            self.meta_stride_batch, self.meta_stride_head, self.meta_stride_page)
        p.side, p.side_channels_dev = _ptr(self.side), _ptr(self.side_channels)
        p.side_count = 0 if self.side_channels is None else int(self.side_channels.shape[-1])
        p.side_stride_batch, p.side_stride_head, p.side_stride_page = (
            self.side_stride_batch, self.side_stride_head, self.side_stride_page)
        return p

    @property
    def nbytes(self) -> int:
        """Resident bytes: payload + metadata + side plane."""
        n = self.data.numel() * self.data.element_size()
        for t in (self.offsets, self.scales, self.side, self.side_channels):
            if t is not None:
                n += t.numel() * t.element_size()
        return n


def astc_width(head_dim: int, layout: str, block: int) -> int:
    comp = 1 if layout == "scalar" else 4
    return (head_dim // comp + block - 1) // block * block


def _check_meta(offsets: torch.Tensor, scales: torch.Tensor) -> None:
    """Plane metadata must be finite fp16 (a NaN/inf scale or offset would
    poison every attention output that reads the block); checked once when
    the plane is built, not per step."""
    if offsets.dtype != torch.float16 or scales.dtype != torch.float16:
        raise ValueError("plane metadata must be fp16")
    if not bool(torch.isfinite(offsets).all()) or not bool(torch.isfinite(scales).all()):
        raise ValueError("non-finite plane metadata (offsets / scales)")


def contiguous_astc_plane(blocks: torch.Tensor, offsets: torch.Tensor, scales: torch.Tensor, *, block: int,
                          layout: str, normalization: str, head_dim: int, page_tokens: int,
                          side: torch.Tensor | None = None, side_channels: torch.Tensor | None = None) -> DevicePlane:
    """Plane over a contiguous cache: blocks [B, H, rows, cols, 16] with rows =
    tokens/block; metadata per ``normalization``:
    page_channel [B, H, pages, D], token [B, H, T], block_affine [B, H, rows, cols].
    Optional side plane [B, H, T, S] fp16 with channel ids [H, S] int32."""
    B, H, rows, cols, sixteen = blocks.shape
    assert sixteen == 16 and blocks.dtype == torch.uint8
    _check_meta(offsets, scales)
    T = rows * block
    if T % page_tokens or page_tokens % block:
        raise ValueError("tokens must be whole pages and pages whole block rows")
    page_bytes = (page_tokens // block) * cols * 16
    pages = T // page_tokens
    if normalization == "page_channel":
        mp = head_dim
    elif normalization == "token":
        mp = page_tokens
    elif normalization == "block_affine":
        mp = (page_tokens // block) * cols
    else:
        raise ValueError("Unknown normalization")
    plane = DevicePlane("astc", blocks, H * T // block * cols * 16, T // block * cols * 16, page_bytes, block=block,
                        layout=layout, normalization=normalization, offsets=offsets, scales=scales,
                        meta_stride_batch=H * pages * mp, meta_stride_head=pages * mp, meta_stride_page=mp,
                        kv_heads=H, capacity_tokens=T)
    if side is not None:
        S = side.shape[-1]
        plane.side, plane.side_channels = side, side_channels
        plane.side_stride_batch = H * T * S * 2
        plane.side_stride_head = T * S * 2
        plane.side_stride_page = page_tokens * S * 2
    return plane


def contiguous_fp16_plane(x: torch.Tensor, page_tokens: int) -> DevicePlane:
    """Plane over an fp16 cache [B, H, T, D] (T a multiple of page_tokens)."""
    B, H, T, D = x.shape
    assert x.dtype == torch.float16 and x.is_contiguous()
    if T % page_tokens:
        raise ValueError("tokens must be whole pages")
    return DevicePlane("fp16", x, H * T * D * 2, T * D * 2, page_tokens * D * 2, kv_heads=H, capacity_tokens=T)


def paged_astc_plane(atlas: torch.Tensor, offsets: torch.Tensor, scales: torch.Tensor, *, block: int, layout: str,
                     normalization: str, head_dim: int, page_tokens: int) -> DevicePlane:
    """Plane over a shared paged atlas: blocks [num_pages, H, page_tokens/block,
    cols, 16]; metadata [num_pages, H, per-page]. Pages are found through the
    block table passed to `decode_attention`."""
    P, H, prow, cols, sixteen = atlas.shape
    assert sixteen == 16 and prow * block == page_tokens
    _check_meta(offsets, scales)
    page_bytes = prow * cols * 16
    mp = offsets[0, 0].numel()
    return DevicePlane("astc", atlas, 0, page_bytes, H * page_bytes, block=block, layout=layout,
                       normalization=normalization, offsets=offsets, scales=scales,
                       meta_stride_batch=0, meta_stride_head=mp, meta_stride_page=H * mp, kv_heads=H)


def paged_fp16_plane(pages: torch.Tensor) -> DevicePlane:
    """Plane over fp16 pages [num_pages, H, page_tokens, D]."""
    P, H, pt, D = pages.shape
    return DevicePlane("fp16", pages, 0, pt * D * 2, H * pt * D * 2, kv_heads=H)


_Q_DTYPES = {torch.float32: L.AKV_Q_F32, torch.bfloat16: L.AKV_Q_BF16, torch.float16: L.AKV_Q_F16}


def _segment_desc(q: torch.Tensor, k: DevicePlane, v: DevicePlane, max_tokens: int, page_tokens: int,
                  seq_lens: torch.Tensor | None, block_table: torch.Tensor | None, num_pages: int,
                  split_tokens: int, keep: list) -> L.AkvAttnDesc:
    """Descriptor of one KV segment for query q [B, Hq, D] (no io pointers)."""
    B, Hq, D = q.shape
    d = L.AkvAttnDesc()
    d.batch, d.q_heads, d.head_dim = B, Hq, D
    d.kv_heads = Attention._kv_heads(k, v, Hq)
    for pl in (k, v):
        if block_table is None and pl.capacity_tokens and max_tokens > pl.capacity_tokens:
            raise ValueError("max_tokens exceeds the tokens the contiguous plane holds")
        if block_table is None and not pl.capacity_tokens:
            raise ValueError("a paged plane needs a block table")
        if block_table is not None and pl.capacity_tokens and pl.stride_batch:
            raise ValueError("a contiguous plane cannot be addressed through a block table")
    d.max_tokens, d.page_tokens, d.split_tokens = max_tokens, page_tokens, split_tokens
    lens = seq_lens.to(torch.int32).contiguous() if seq_lens is not None else None
    table = block_table.to(torch.int32).contiguous() if block_table is not None else None
    keep += [lens, table]
    d.seq_lens_dev = _ptr(lens)
    d.block_table_dev = _ptr(table)
    if table is not None:
        d.pages_per_seq = int(table.shape[1])
        d.num_pages = int(num_pages)
    d.k, d.v = k.to_c(), v.to_c()
    return d


class Attention:
    """A prepared decode-attention call (descriptor, workspace, output).

    Building the descriptor once and re-issuing `run()` keeps the per-step
    host cost to one C call; `run()` is what the benchmark times.

    An optional second KV segment (`tail_k`, `tail_v`: planes of, e.g., the
    exact FP16 tokens of each sequence's incomplete last page, `tail_lens`
    tokens per sequence out of `tail_tokens`) is attended in the same softmax
    through akv_cuda_decode_attention_tail.
    """

    def __init__(self, q: torch.Tensor, k: DevicePlane, v: DevicePlane, *, page_tokens: int, max_tokens: int,
                 seq_lens: torch.Tensor | None = None, block_table: torch.Tensor | None = None,
                 num_pages: int = 0, split_tokens: int = 0, scale: float = 0.0, out: torch.Tensor | None = None,
                 status: torch.Tensor | None = None, tail_k: DevicePlane | None = None,
                 tail_v: DevicePlane | None = None, tail_lens: torch.Tensor | None = None, tail_tokens: int = 0):
        _require_cuda(q, k.data, v.data, seq_lens, block_table)
        B, Hq, D = q.shape
        self.q, self.k, self.v = q, k, v
        self._keep: list = []
        d = _segment_desc(q, k, v, max_tokens, page_tokens, seq_lens, block_table, num_pages, split_tokens, self._keep)
        self.seq_lens, self.block_table = self._keep[0], self._keep[1]
        if q.dtype not in _Q_DTYPES or not q.is_contiguous():
            raise ValueError("q must be contiguous fp32/bf16/fp16 [B, Hq, D]")
        d.q_dtype = _Q_DTYPES[q.dtype]
        d.q_dev = q.data_ptr()
        d.scale = scale
        self.tail = None
        if (tail_k is None) != (tail_v is None):
            raise ValueError("a tail needs both K and V planes")
        if tail_k is not None:
            _require_cuda(tail_k.data, tail_v.data, tail_lens)
            if tail_tokens <= 0:
                raise ValueError("tail_tokens must be positive")
            self.tail = _segment_desc(q, tail_k, tail_v, tail_tokens, tail_tokens, tail_lens, None, 0, 0, self._keep)
            self._tref = ct.byref(self.tail)
            ws = L.lib().akv_cuda_attention_tail_workspace(ct.byref(d), self._tref)
        else:
            ws = L.lib().akv_cuda_attention_workspace(ct.byref(d))
        if ws == 0:
            # Surface the precise validation error.
            d.workspace_dev, d.workspace_bytes = None, 0
            if self.tail is not None:
                L.check(L.lib().akv_cuda_decode_attention_tail(ct.byref(d), self._tref, None), "decode_attention_tail")
            L.check(L.lib().akv_cuda_decode_attention(ct.byref(d), None), "decode_attention")
        self.workspace = torch.empty(ws // 4 + 4, dtype=torch.float32, device=q.device)
        d.workspace_dev, d.workspace_bytes = self.workspace.data_ptr(), ws
        self.out = out if out is not None else torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
        if self.out.shape != (B, Hq, D) or self.out.dtype != torch.float32 or not self.out.is_contiguous():
            raise ValueError("out must be contiguous fp32 [B, Hq, D]")
        d.out_dev = self.out.data_ptr()
        self.status = status
        d.status_dev = _ptr(status)
        self.desc = d
        self._dref = ct.byref(d)

    @staticmethod
    def _kv_heads(k: DevicePlane, v: DevicePlane, Hq: int) -> int:
        if not k.kv_heads or k.kv_heads != v.kv_heads or Hq % k.kv_heads:
            raise ValueError("K and V planes must agree on kv_heads, which must divide the query heads")
        return int(k.kv_heads)

    def run(self, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        if self.tail is not None:
            L.check(L.lib().akv_cuda_decode_attention_tail(self._dref, self._tref, _stream_handle(stream)),
                    "decode_attention_tail")
        else:
            L.check(L.lib().akv_cuda_decode_attention(self._dref, _stream_handle(stream)), "decode_attention")
        return self.out

    def plan(self) -> dict:
        """The launch plan (akv_cuda_attention_plan): kernel name, split size, splits."""
        k, sp, ns = ct.c_int(), ct.c_int(), ct.c_int()
        L.check(L.lib().akv_cuda_attention_plan(self._dref, ct.byref(k), ct.byref(sp), ct.byref(ns)), "attention_plan")
        names = {L.AKV_KERNEL_FAST: "attn_fast_kernel", L.AKV_KERNEL_FP16: "attn_fp16_kernel"}
        return {"kernel": names.get(k.value, "attn_split_kernel"),
                "split_tokens": sp.value, "nsplits": ns.value}

    def run_phase(self, phase: int, stream: torch.cuda.Stream | None = None) -> None:
        """Issue only the split (1) or merge (2) launch; see akv_cuda_decode_attention_phase."""
        if self.tail is not None:
            raise ValueError("phase-by-phase launches are not available with a tail segment")
        L.check(L.lib().akv_cuda_decode_attention_phase(self._dref, phase, _stream_handle(stream)), "decode_attention")


def decode_attention(q: torch.Tensor, k: DevicePlane, v: DevicePlane, **kw) -> torch.Tensor:
    """One decode step: out[b, hq] = softmax(scale q.K^T) V over the first
    seq_lens[b] tokens (all max_tokens when None). See `Attention`."""
    return Attention(q, k, v, **kw).run()


def decode_blocks(blocks: torch.Tensor, block: int, mode: str = "unorm8", out: torch.Tensor | None = None,
                  stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """uint8 [n, 16] device blocks -> [n, block, block, 4] texels.
    mode: 'unorm8' (uint8), 'fp16' (float16), 'unorm16' (int16 holding uint16 bits)."""
    _require_cuda(blocks)
    b = blocks.reshape(-1, 16)
    n = b.shape[0]
    codes = {"unorm8": (L.AKV_OUT_UNORM8, torch.uint8), "fp16": (L.AKV_OUT_FP16, torch.float16),
             "unorm16": (L.AKV_OUT_UNORM16, torch.int16)}
    m, dt = codes[mode]
    if out is None:
        out = torch.empty(n, block, block, 4, dtype=dt, device=blocks.device)
    L.check(L.lib().akv_cuda_decode_blocks(b.data_ptr(), n, block, m, out.data_ptr(), _stream_handle(stream)),
            "decode_blocks")
    return out


def decode_image(blocks: torch.Tensor, block: int, width: int, height: int,
                 stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Device twin of the reference's `akv_decode` (bridge.cpp:27-35): float32 [h, w, 4]."""
    _require_cuda(blocks)
    out = torch.empty(height, width, 4, dtype=torch.float32, device=blocks.device)
    L.check(L.lib().akv_cuda_decode_image(blocks.data_ptr(), blocks.numel(), block, out.data_ptr(), width, height,
                                          _stream_handle(stream)), "decode_image")
    return out


def restore_plane(plane: DevicePlane, *, batch: int, kv_heads: int, max_tokens: int, head_dim: int,
                  page_tokens: int, block_table: torch.Tensor | None = None, num_pages: int = 0,
                  status: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Decode + affine restore of a whole plane -> fp32 [B, H, T, D] (bit-exact
    with the reference's NumPy restore, codec.py:198-208)."""
    _require_cuda(plane.data, block_table)
    if block_table is None and (not plane.capacity_tokens or max_tokens > plane.capacity_tokens):
        raise ValueError("max_tokens exceeds the tokens the contiguous plane holds")
    out = torch.empty(batch, kv_heads, max_tokens, head_dim, dtype=torch.float32, device=plane.data.device)
    p = plane.to_c()
    bt = block_table.to(torch.int32).contiguous() if block_table is not None else None
    L.check(L.lib().akv_cuda_restore_plane(ct.byref(p), batch, kv_heads, max_tokens, head_dim, page_tokens, _ptr(bt),
                                           0 if bt is None else int(bt.shape[1]), int(num_pages), out.data_ptr(),
                                           _ptr(status), _stream_handle(stream)), "restore_plane")
    return out


def init(device: int | None = None) -> None:
    """Fill the decode tables on `device` (call before any CUDA-graph capture)."""
    dev = torch.cuda.current_device() if device is None else device
    L.check(L.lib().akv_cuda_init(dev), "init")


def host_tables() -> bytes:
    n = L.lib().akv_cuda_host_tables(None, 0)
    buf = (ct.c_uint8 * n)()
    L.lib().akv_cuda_host_tables(buf, n)
    return bytes(buf)


def host_encode(image: np.ndarray, block: int, layout: str = "scalar", effort: int = 1, threads: int = 0) -> bytes:
    """CPU ASTC encode of a float RGBA image [h, w, 4] in [0, 1] with this
    library's encoder (not astcenc; see include/akv_host.h)."""
    import os
    im = np.ascontiguousarray(image, np.float32)
    h, w, c = im.shape
    if c != 4 or not np.all(np.isfinite(im)):
        raise ValueError("Expected finite HxWx4 input")
    n = ((w + block - 1) // block) * ((h + block - 1) // block) * 16
    out = np.zeros(n, np.uint8)
    thr = threads or len(os.sched_getaffinity(0))
    rc = L.lib().akv_host_encode(im.ctypes.data, w, h, block, L.LAYOUTS[layout], effort, out.ctypes.data, n, thr)
    if rc:
        raise ValueError("akv_host_encode rejected the image (sides must be block multiples)")
    return out.tobytes()


def random_blocks(n: int, block: int, seed: int = 0, threads: int = 0) -> np.ndarray:
    """n random legal LDR blocks (uint8 [n, 16]) for decode benchmarks."""
    import os
    out = np.empty((n, 16), np.uint8)
    rc = L.lib().akv_host_random_blocks(n, block, seed, out.ctypes.data, threads or len(os.sched_getaffinity(0)))
    if rc:
        raise ValueError("akv_host_random_blocks rejected its arguments")
    return out
