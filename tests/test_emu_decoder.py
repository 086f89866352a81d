"""The product's device decoder (compiled for the host by tests/emu) against
the oracle, bit for bit on the 16-bit interpolation result C."""
import ctypes as ct
from pathlib import Path

import numpy as np
import pytest

from common import golden
from oracle import oracle as O

EMU = Path(__file__).resolve().parent / "emu" / "_build" / "libakv_emu.so"


def emu_decode(blocks, bs):
    lib = ct.CDLL(str(EMU))
    lib.emu_decode_blocks_u16.argtypes = [ct.c_void_p, ct.c_int64, ct.c_int, ct.c_void_p]
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 16)
    out = np.empty((b.shape[0], bs, bs, 4), np.uint16)
    assert lib.emu_decode_blocks_u16(b.ctypes.data, b.shape[0], bs, out.ctypes.data) == 0
    return out


def test_golden_blocks():
    g = golden("block_geometry_identity")
    blocks = g["blocks"].reshape(-1, 16)
    np.testing.assert_array_equal(emu_decode(blocks, 6), O.decode_blocks(blocks, 6, O.OUT_UNORM16, threads=4))


@pytest.mark.parametrize("bs", [4, 6, 8])
def test_random_legal_blocks(bs):
    from astc_kv_cuda.ops import random_blocks
    blocks = random_blocks(20000, bs, seed=1000 + bs)
    np.testing.assert_array_equal(emu_decode(blocks, bs), O.decode_blocks(blocks, bs, O.OUT_UNORM16, threads=4))


@pytest.mark.parametrize("bs", [4, 6, 8])
def test_random_bytes_including_illegal_encodings(bs):
    blocks = np.random.default_rng(bs).integers(0, 256, (20000, 16), dtype=np.uint8)
    np.testing.assert_array_equal(emu_decode(blocks, bs), O.decode_blocks(blocks, bs, O.OUT_UNORM16, threads=4))


def emu_decode_rows(blocks, bs):
    lib = ct.CDLL(str(EMU))
    lib.emu_decode_rows_u16.argtypes = [ct.c_void_p, ct.c_int64, ct.c_int, ct.c_void_p]
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 16)
    out = np.empty((b.shape[0], bs, bs, 4), np.uint16)
    assert lib.emu_decode_rows_u16(b.ctypes.data, b.shape[0], bs, out.ctypes.data) == 0
    return out


@pytest.mark.parametrize("bs", [4, 6, 8])
def test_row_stage_matches_oracle(bs):
    """The standalone decoder's row-wise texel stage: random legal blocks
    (every mode: reduced grids, dual plane, 1-4 partitions, void extent),
    random bytes (illegal encodings -> error colour) and, for 6x6, the
    reference's astcenc goldens."""
    from astc_kv_cuda.ops import random_blocks
    sets = [random_blocks(20000, bs, seed=2000 + bs),
            np.random.default_rng(50 + bs).integers(0, 256, (20000, 16), dtype=np.uint8)]
    if bs == 6:
        sets.append(golden("block_geometry_identity")["blocks"].reshape(-1, 16))
    for blocks in sets:
        np.testing.assert_array_equal(emu_decode_rows(blocks, bs), O.decode_blocks(blocks, bs, O.OUT_UNORM16, threads=4))


def test_fp16_view_conversion_exhaustive():
    lib = ct.CDLL(str(EMU))
    lib.emu_unit.argtypes = [ct.c_uint32]
    lib.emu_unit.restype = ct.c_float
    L = O.lib()
    for c in list(range(0, 70000, 7)) + [65535, 65534, 4, 3, 2047, 2048]:
        c = min(c, 65535)
        h = np.array([L.astc_oracle_unorm16_to_half(c)], np.uint16).view(np.float16)[0]
        assert np.float32(h) == np.float32(lib.emu_unit(c)), c


def emu_fast_r(blocks, bs):
    lib = ct.CDLL(str(EMU))
    lib.emu_decode_fast_r.argtypes = [ct.c_void_p, ct.c_int64, ct.c_int, ct.c_void_p, ct.c_void_p]
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 16)
    out = np.empty((b.shape[0], bs * bs), np.float32)
    cls = np.empty(b.shape[0], np.int32)
    assert lib.emu_decode_fast_r(b.ctypes.data, b.shape[0], bs, out.ctypes.data, cls.ctypes.data) == 0
    return out, cls


@pytest.mark.parametrize("source", ["golden", "random", "garbage", "encoder"])
@pytest.mark.parametrize("bs", [4, 6, 8])
def test_fast_table_decode_matches_oracle(source, bs):
    """The attention kernel's block decode against the oracle's fp16 view:
    table blocks (single weight plane, full-resolution grid, luminance-direct
    endpoints), descriptor blocks (the same with a reduced grid or a large
    table, evaluated per texel through the infill taps), constant blocks (void
    extent, illegal encodings) and generic blocks (other endpoint modes, dual
    plane: generic header decode, then the per-texel evaluator phase 1b
    picks)."""
    from astc_kv_cuda.ops import host_encode, random_blocks
    if source == "golden":
        if bs != 6:
            pytest.skip("the reference's goldens are 6x6")
        blocks = golden("block_geometry_identity")["blocks"].reshape(-1, 16)
    elif source == "random":
        blocks = random_blocks(20000, bs, seed=50 + bs)
    elif source == "garbage":
        blocks = np.random.default_rng(60 + bs).integers(0, 256, (20000, 16), dtype=np.uint8)
    else:
        x = np.random.default_rng(bs).random((bs * 20, bs * 22), np.float32)
        x = np.repeat(x[..., None], 4, -1)
        x[..., 3] = 1
        blocks = np.frombuffer(host_encode(x, bs, "scalar", 1), np.uint8).reshape(-1, 16)
    got, cls = emu_fast_r(blocks, bs)
    ref = O.decode_blocks(blocks, bs, O.OUT_FP16, threads=4)[..., 0].reshape(len(got), bs * bs).astype(np.float32)
    # Uniformly random bytes almost never form a luminance block (valid mode
    # and all-zero endpoint-mode fields); they exercise constants and the
    # generic kind (kKindGeneric = 2).
    assert (cls <= 1).any() if source != "garbage" else ((cls == 3).any() and (cls == 2).any())
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("source", ["random", "garbage", "encoder"])
def test_rgba4_fast_decode_matches_oracle(source):
    """The attention kernel's RGBA 4x4 path (fast blocks: one plane, full
    grid, <= 2 partitions, RGBA-direct endpoints; constants; generic
    fallback) against the oracle's fp16 view of all four channels."""
    from astc_kv_cuda.ops import host_encode, random_blocks
    if source == "random":
        blocks = random_blocks(20000, 4, seed=91)
    elif source == "garbage":
        blocks = np.random.default_rng(92).integers(0, 256, (20000, 16), dtype=np.uint8)
    else:
        x = np.random.default_rng(93).random((4 * 20, 4 * 22, 4), np.float32)
        blocks = np.frombuffer(host_encode(x, 4, "rgba", 1), np.uint8).reshape(-1, 16)
    lib = ct.CDLL(str(EMU))
    lib.emu_decode_rgba4.argtypes = [ct.c_void_p, ct.c_int64, ct.c_void_p, ct.c_void_p]
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 16)
    got = np.empty((b.shape[0], 16, 4), np.float32)
    cls = np.empty(b.shape[0], np.int32)
    assert lib.emu_decode_rgba4(b.ctypes.data, b.shape[0], got.ctypes.data, cls.ctypes.data) == 0
    ref = O.decode_blocks(b, 4, O.OUT_FP16, threads=4).reshape(b.shape[0], 16, 4).astype(np.float32)
    if source == "encoder":
        assert (cls == 0).mean() > 0.9  # the encoder's RGBA blocks take the fast path
    np.testing.assert_array_equal(got, ref)
