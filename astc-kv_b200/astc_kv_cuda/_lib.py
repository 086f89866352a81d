"""ctypes binding of libakv_cuda.so (the C ABI in include/akv_cuda.h).

The library is the product path: nothing here falls back to CPU code. If the
shared object is missing or fails to load, `lib()` raises.
"""
from __future__ import annotations

import ctypes as ct
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libakv_cuda.so"

AKV_OK = 0
AKV_OUT_UNORM8, AKV_OUT_FP16, AKV_OUT_UNORM16 = 0, 1, 2
AKV_STORAGE_FP16, AKV_STORAGE_ASTC = 0, 1
AKV_LAYOUT_SCALAR, AKV_LAYOUT_RGBA = 0, 1
AKV_NORM_PAGE_CHANNEL, AKV_NORM_TOKEN, AKV_NORM_BLOCK_AFFINE = 0, 1, 2
AKV_Q_F32, AKV_Q_BF16, AKV_Q_F16 = 0, 1, 2
AKV_PHASE_SPLIT, AKV_PHASE_MERGE = 1, 2
AKV_KERNEL_GENERIC, AKV_KERNEL_FAST, AKV_KERNEL_FP16 = 0, 1, 2
AKV_ERR_STATIC_WORKSPACE = 8
AKV_STATIC_WORKSPACE_BYTES = 8 << 20

LAYOUTS = {"scalar": AKV_LAYOUT_SCALAR, "rgba": AKV_LAYOUT_RGBA}
NORMS = {"page_channel": AKV_NORM_PAGE_CHANNEL, "token": AKV_NORM_TOKEN, "block_affine": AKV_NORM_BLOCK_AFFINE}


class AkvPlane(ct.Structure):
    _fields_ = [
        ("storage", ct.c_int32), ("block", ct.c_int32), ("layout", ct.c_int32), ("normalization", ct.c_int32),
        ("data", ct.c_void_p),
        ("stride_batch", ct.c_int64), ("stride_head", ct.c_int64), ("stride_page", ct.c_int64),
        ("offsets", ct.c_void_p), ("scales", ct.c_void_p),
        ("meta_stride_batch", ct.c_int64), ("meta_stride_head", ct.c_int64), ("meta_stride_page", ct.c_int64),
        ("side", ct.c_void_p), ("side_channels_dev", ct.c_void_p), ("side_count", ct.c_int32), ("reserved0", ct.c_int32),
        ("side_stride_batch", ct.c_int64), ("side_stride_head", ct.c_int64), ("side_stride_page", ct.c_int64),
    ]


class AkvAttnDesc(ct.Structure):
    _fields_ = [
        ("batch", ct.c_int32), ("q_heads", ct.c_int32), ("kv_heads", ct.c_int32), ("head_dim", ct.c_int32),
        ("max_tokens", ct.c_int32), ("page_tokens", ct.c_int32), ("split_tokens", ct.c_int32), ("q_dtype", ct.c_int32),
        ("q_dev", ct.c_void_p), ("seq_lens_dev", ct.c_void_p), ("block_table_dev", ct.c_void_p),
        ("pages_per_seq", ct.c_int32), ("num_pages", ct.c_int32),
        ("k", AkvPlane), ("v", AkvPlane),
        ("scale", ct.c_float), ("reserved0", ct.c_int32),
        ("workspace_dev", ct.c_void_p), ("workspace_bytes", ct.c_size_t),
        ("out_dev", ct.c_void_p), ("status_dev", ct.c_void_p),
    ]


# Every symbol include/akv_cuda.h and include/akv_host.h declare.
EXPORTS = (
    "akv_cuda_error", "akv_cuda_abi_version", "akv_cuda_init", "akv_cuda_decode_blocks", "akv_cuda_decode_image",
    "akv_cuda_attention_workspace", "akv_cuda_attention_plan", "akv_cuda_attention_tail_workspace",
    "akv_cuda_decode_attention_tail", "akv_cuda_decode_attention",
    "akv_cuda_decode_attention_phase",
    "akv_cuda_decode_attention_noalloc", "akv_cuda_restore_plane", "akv_cuda_struct_size",
    "akv_cuda_host_tables", "akv_host_encode", "akv_host_random_blocks",
)

_lib = None
_lock = threading.Lock()


class AkvError(RuntimeError):
    """A non-zero status from the C ABI (mirrors codec.py:41-43 `_check`)."""

    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = lib().akv_cuda_error(code).decode()
        super().__init__(f"{what}: {msg} (status {code})" if what else f"{msg} (status {code})")


def lib() -> ct.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with astc_kv_cuda.build.build() "
                               "(nvcc, sm_100a); there is no CPU fallback")
        l = ct.CDLL(str(LIB_PATH))
        vp, i32, i64, sz = ct.c_void_p, ct.c_int32, ct.c_int64, ct.c_size_t
        l.akv_cuda_error.argtypes = [ct.c_int]
        l.akv_cuda_error.restype = ct.c_char_p
        l.akv_cuda_abi_version.restype = ct.c_int
        l.akv_cuda_init.argtypes = [ct.c_int]
        l.akv_cuda_decode_blocks.argtypes = [vp, i64, ct.c_int, ct.c_int, vp, vp]
        l.akv_cuda_decode_image.argtypes = [vp, sz, ct.c_int, vp, ct.c_uint, ct.c_uint, vp]
        l.akv_cuda_attention_workspace.argtypes = [ct.POINTER(AkvAttnDesc)]
        l.akv_cuda_attention_workspace.restype = sz
        ip = ct.POINTER(ct.c_int)
        l.akv_cuda_attention_plan.argtypes = [ct.POINTER(AkvAttnDesc), ip, ip, ip]
        l.akv_cuda_attention_tail_workspace.argtypes = [ct.POINTER(AkvAttnDesc), ct.POINTER(AkvAttnDesc)]
        l.akv_cuda_attention_tail_workspace.restype = sz
        l.akv_cuda_decode_attention_tail.argtypes = [ct.POINTER(AkvAttnDesc), ct.POINTER(AkvAttnDesc), vp]
        l.akv_cuda_decode_attention.argtypes = [ct.POINTER(AkvAttnDesc), vp]
        l.akv_cuda_decode_attention_phase.argtypes = [ct.POINTER(AkvAttnDesc), ct.c_int, vp]
        l.akv_cuda_decode_attention_noalloc.argtypes = [ct.POINTER(AkvAttnDesc), vp]
        l.akv_cuda_restore_plane.argtypes = [ct.POINTER(AkvPlane), i32, i32, i32, i32, i32, vp, i32, i32, vp, vp, vp]
        l.akv_cuda_struct_size.argtypes = [ct.c_int]
        l.akv_cuda_struct_size.restype = sz
        l.akv_cuda_host_tables.argtypes = [vp, sz]
        l.akv_cuda_host_tables.restype = sz
        l.akv_host_encode.argtypes = [vp, ct.c_uint, ct.c_uint, ct.c_int, ct.c_int, ct.c_int, vp, sz, ct.c_int]
        l.akv_host_random_blocks.argtypes = [i64, ct.c_int, ct.c_uint64, vp, ct.c_int]
        for name in EXPORTS:
            f = getattr(l, name)
            if f.restype is ct.c_int or name in ("akv_cuda_init", "akv_cuda_decode_blocks", "akv_cuda_decode_image",
                                                  "akv_cuda_decode_attention", "akv_cuda_restore_plane",
                                                  "akv_cuda_decode_attention_phase", "akv_cuda_decode_attention_noalloc",
                                                  "akv_host_encode", "akv_host_random_blocks"):
                f.restype = ct.c_int
        if l.akv_cuda_struct_size(0) != ct.sizeof(AkvPlane) or l.akv_cuda_struct_size(1) != ct.sizeof(AkvAttnDesc):
            raise RuntimeError("libakv_cuda.so struct layout does not match this binding")
        _lib = l
    return _lib


def check(code: int, what: str = "") -> None:
    if code:
        raise AkvError(code, what)
