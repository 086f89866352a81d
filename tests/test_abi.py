"""The C ABI library: loads, exports every declared symbol, matching struct
layouts, and argument validation that returns status codes (no GPU needed:
these calls fail validation before touching CUDA)."""
import ctypes as ct
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(akv_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_exports_every_declared_symbol():
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    names = declared_symbols()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
    assert names == set(L.EXPORTS)


def test_struct_layouts_and_version():
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    assert lib.akv_cuda_abi_version() == 1
    assert lib.akv_cuda_struct_size(0) == ct.sizeof(L.AkvPlane)
    assert lib.akv_cuda_struct_size(1) == ct.sizeof(L.AkvAttnDesc)
    assert lib.akv_cuda_struct_size(7) == 0


def test_error_strings():
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    for code in range(7):
        assert lib.akv_cuda_error(code)
    assert b"unknown" in lib.akv_cuda_error(1234)


@pytest.mark.parametrize("args", [
    (None, 10, 6, 0, None),       # null pointers
    (16, -1, 6, 0, 16),           # negative count
    (16, 10, 5, 0, 16),           # unsupported footprint
    (16, 10, 6, 9, 16),           # bad output mode
    (8, 10, 6, 0, 16),            # misaligned blocks
])
def test_decode_blocks_rejects_bad_arguments(args):
    from astc_kv_cuda import _lib as L
    assert L.lib().akv_cuda_decode_blocks(args[0], args[1], args[2], args[3], args[4], None) == 1


def test_decode_image_rejects_size_mismatch():
    from astc_kv_cuda import _lib as L
    assert L.lib().akv_cuda_decode_image(16, 100, 6, 16, 66, 384, None) == 1


def test_attention_descriptor_validation():
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    d = L.AkvAttnDesc()
    assert lib.akv_cuda_attention_workspace(ct.byref(d)) == 0
    assert lib.akv_cuda_decode_attention(ct.byref(d), None) == 1
    d.batch, d.q_heads, d.kv_heads, d.head_dim, d.max_tokens, d.page_tokens = 1, 9, 3, 64, 384, 96
    d.k.storage = L.AKV_STORAGE_FP16
    d.k.data = 4096
    d.v.storage = L.AKV_STORAGE_ASTC
    d.v.block, d.v.layout, d.v.normalization = 6, L.AKV_LAYOUT_SCALAR, L.AKV_NORM_TOKEN
    d.v.data, d.v.offsets, d.v.scales = 8192, 8192, 8192
    ws = lib.akv_cuda_attention_workspace(ct.byref(d))
    assert ws > 0
    kern, split, nsplits = ct.c_int(-1), ct.c_int(0), ct.c_int(0)
    assert lib.akv_cuda_attention_plan(ct.byref(d), ct.byref(kern), ct.byref(split), ct.byref(nsplits)) == 0
    assert kern.value in (L.AKV_KERNEL_GENERIC, L.AKV_KERNEL_FAST)
    assert split.value % 6 == 0 and nsplits.value == -(-384 // split.value)
    # Missing workspace -> AKV_ERR_WORKSPACE before any launch.
    d.q_dev, d.out_dev = 4096, 4096
    assert lib.akv_cuda_decode_attention(ct.byref(d), None) == 6
    # A group size that is not compiled in -> AKV_ERR_UNSUPPORTED.
    d.q_heads = 15
    assert lib.akv_cuda_decode_attention(ct.byref(d), None) == 2
    # Page size that does not hold whole block rows.
    d.q_heads, d.page_tokens = 9, 100
    assert lib.akv_cuda_decode_attention(ct.byref(d), None) == 1
    # Bad phase.
    d.page_tokens = 96
    assert lib.akv_cuda_decode_attention_phase(ct.byref(d), 7, None) == 1


def test_tail_descriptor_validation():
    """The two-segment entry point validates before touching the GPU."""
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    d = L.AkvAttnDesc()
    d.batch, d.q_heads, d.kv_heads, d.head_dim, d.max_tokens, d.page_tokens = 1, 9, 3, 64, 384, 96
    d.k.storage = d.v.storage = L.AKV_STORAGE_FP16
    d.k.data = d.v.data = 4096
    t = L.AkvAttnDesc.from_buffer_copy(d)
    t.max_tokens = t.page_tokens = 32
    assert lib.akv_cuda_attention_tail_workspace(ct.byref(d), None) == 0
    assert lib.akv_cuda_decode_attention_tail(ct.byref(d), None, None) == 1
    ws = lib.akv_cuda_attention_tail_workspace(ct.byref(d), ct.byref(t))
    assert ws == lib.akv_cuda_attention_workspace(ct.byref(d)) + lib.akv_cuda_attention_workspace(ct.byref(t))
    t.kv_heads = 1  # a tail must describe the same heads
    assert lib.akv_cuda_attention_tail_workspace(ct.byref(d), ct.byref(t)) == 0
    assert lib.akv_cuda_decode_attention_tail(ct.byref(d), ct.byref(t), None) == 1


def test_restore_plane_validation():
    from astc_kv_cuda import _lib as L
    p = L.AkvPlane()
    assert L.lib().akv_cuda_restore_plane(ct.byref(p), 1, 1, 96, 64, 96, None, 0, 0, 4096, None, None) == 1
