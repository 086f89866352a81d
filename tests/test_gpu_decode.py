"""GPU parity of the standalone decoder and the plane restore, through the C ABI.

Bit-exact against the CPU oracle (UNORM8, fp16 and UNORM16 views) on the
reference's astcenc golden blocks, random legal blocks of every footprint and
random bytes (illegal encodings -> error colour), and bit-exact against the
reference's golden restores.
"""
import numpy as np
import pytest
import torch

from common import golden, sha
from oracle import oracle as O

pytestmark = pytest.mark.gpu

MODES = [("unorm8", O.OUT_UNORM8, np.uint8), ("fp16", O.OUT_FP16, np.float16), ("unorm16", O.OUT_UNORM16, np.uint16)]


def gpu_decode(blocks, bs, mode):
    from astc_kv_cuda.ops import decode_blocks
    t = torch.from_numpy(np.ascontiguousarray(blocks, np.uint8).reshape(-1, 16)).cuda()
    out = decode_blocks(t, bs, mode)
    torch.cuda.synchronize()
    a = out.cpu().numpy()
    return a.view(np.uint16) if mode == "unorm16" else a


@pytest.mark.parametrize("mode,omode,dt", MODES)
def test_golden_blocks_all_views(cuda, mode, omode, dt):
    g = golden("block_geometry_identity")
    blocks = g["blocks"].reshape(-1, 16)
    got = gpu_decode(blocks, 6, mode)
    ref = O.decode_blocks(blocks, 6, omode, threads=O.cpu_threads())
    np.testing.assert_array_equal(got.view(np.uint16) if dt is np.float16 else got,
                                  ref.view(np.uint16) if dt is np.float16 else ref)


@pytest.mark.parametrize("bs", [4, 6, 8])
@pytest.mark.parametrize("mode,omode,dt", MODES)
def test_random_legal_blocks(cuda, bs, mode, omode, dt):
    from astc_kv_cuda.ops import random_blocks
    blocks = random_blocks(50000 + 37, bs, seed=7 * bs)
    got = gpu_decode(blocks, bs, mode)
    ref = O.decode_blocks(blocks, bs, omode, threads=O.cpu_threads())
    np.testing.assert_array_equal(got.view(np.uint16) if dt is np.float16 else got,
                                  ref.view(np.uint16) if dt is np.float16 else ref)


@pytest.mark.parametrize("bs", [4, 6, 8])
def test_block_order_does_not_change_any_block(cuda, bs):
    # The kernel reorders each group of 256 blocks by header class before the
    # header stage. A block's texels must not depend on its neighbours: a
    # permutation of the input permutes the output, for a random order, for
    # an input already grouped into long runs of one partition count, and
    # with a ragged last group.
    from astc_kv_cuda.ops import random_blocks
    blocks = random_blocks(4 * 256 + 77, bs, seed=11 * bs)
    base = gpu_decode(blocks, bs, "unorm16")
    np.testing.assert_array_equal(base, O.decode_blocks(blocks, bs, O.OUT_UNORM16, threads=4))
    perm = np.random.default_rng(5).permutation(len(blocks))
    np.testing.assert_array_equal(gpu_decode(blocks[perm], bs, "unorm16"), base[perm])
    parts = (blocks[:, 1] >> 3) & 3  # header bits 11-12: partition count - 1
    grouped = np.argsort(parts, kind="stable")
    np.testing.assert_array_equal(gpu_decode(blocks[grouped], bs, "unorm16"), base[grouped])


@pytest.mark.parametrize("bs", [4, 6, 8])
def test_random_bytes_error_colour(cuda, bs):
    blocks = np.random.default_rng(99 + bs).integers(0, 256, (30011, 16), dtype=np.uint8)
    np.testing.assert_array_equal(gpu_decode(blocks, bs, "unorm16"), O.decode_blocks(blocks, bs, O.OUT_UNORM16, threads=4))


@pytest.mark.parametrize("n", [0, 1, 127, 128, 129])
def test_ragged_block_counts(cuda, n):
    g = golden("block_geometry_identity")
    blocks = g["blocks"].reshape(-1, 16)[:max(n, 1)][:n] if n else np.zeros((0, 16), np.uint8)
    if n == 0:
        from astc_kv_cuda.ops import decode_blocks
        out = decode_blocks(torch.zeros(0, 16, dtype=torch.uint8, device="cuda"), 6)
        assert out.shape == (0, 6, 6, 4)
        return
    np.testing.assert_array_equal(gpu_decode(blocks, 6, "unorm8"), O.decode_blocks(blocks, 6, O.OUT_UNORM8))


def test_decode_image_contract(cuda):
    from astc_kv_cuda.ops import decode_image
    g = golden("story_l17_v_token6")
    for h in range(3):
        payload = g["v_blocks"][h].tobytes()
        img = decode_image(torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda(), 6, 66, 384).cpu().numpy()
        np.testing.assert_array_equal(img, O.decode_image_f32(payload, 6, 66, 384))
        rec = img[:, :64, 0] * g["v_scale"][h].astype(np.float32) + g["v_offset"][h].astype(np.float32)
        np.testing.assert_array_equal(rec, g["v_decoded"][h])
    # Non-multiple image sides crop the last block row/column.
    payload = g["v_blocks"][0][:2, :3].tobytes()
    img = decode_image(torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda(), 6, 17, 11).cpu().numpy()
    np.testing.assert_array_equal(img, O.decode_image_f32(payload, 6, 17, 11))


def _restore(blocks, off, scl, norm, P, T):
    from astc_kv_cuda.ops import contiguous_astc_plane, restore_plane

    def f16(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float16).view(np.int16)).view(torch.float16).cuda()
    plane = contiguous_astc_plane(torch.from_numpy(np.ascontiguousarray(blocks[None])).cuda(), f16(off[None]), f16(scl[None]),
                                  block=6, layout="scalar", normalization=norm, head_dim=64, page_tokens=P)
    out = restore_plane(plane, batch=1, kv_heads=blocks.shape[0], max_tokens=T, head_dim=64, page_tokens=P)
    torch.cuda.synchronize()
    return out[0].cpu().numpy()


def test_restore_plane_bit_exact_token_fixture(cuda):
    g = golden("story_l17_v_token6")
    rec = _restore(g["v_blocks"], g["v_offset"][..., 0], g["v_scale"][..., 0], "token", int(g["page_tokens"]), 384)
    np.testing.assert_array_equal(rec, g["v_decoded"])


def test_restore_plane_bit_exact_page_channel_fixture(cuda):
    g = golden("story_l17_kv_page6")
    for side in ("k", "v"):
        rec = _restore(g[side + "_blocks"], g[side + "_offset"], g[side + "_scale"], "page_channel", int(g["page_tokens"]), 384)
        assert sha(rec) == str(g[side + "_decoded_sha256"])


def test_restore_plane_bit_exact_block_geometry(cuda):
    g = golden("block_geometry_identity")
    for i in range(len(g["names"])):
        rec = _restore(g["blocks"][i].reshape(3, 48, 11, 16), g["offsets"][i], g["scales"][i], "token", 96, 288)
        assert sha(rec) == str(g["decoded_sha256"][i]), str(g["names"][i])


@pytest.mark.parametrize("bs", [4, 6, 8])
@pytest.mark.parametrize("mode,offset", [("unorm8", 4), ("unorm8", 12), ("fp16", 8), ("unorm16", 8)])
def test_output_not_16_byte_aligned(cuda, bs, mode, offset):
    """Outputs that are only 4- (UNORM8) or 8-byte aligned take the decoder's
    word-store instance; results equal the aligned (vector-store) decode."""
    from astc_kv_cuda.ops import decode_blocks, random_blocks
    blocks = torch.from_numpy(random_blocks(4099, bs, seed=31 * bs)).cuda()
    ref = decode_blocks(blocks, bs, mode)
    nbytes = ref.numel() * ref.element_size()
    buf = torch.zeros(nbytes + 32, dtype=torch.uint8, device="cuda")
    assert buf.data_ptr() % 16 == 0
    out = buf[offset:offset + nbytes].view(ref.dtype).view(ref.shape)
    decode_blocks(blocks, bs, mode, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.uint8), ref.view(torch.uint8))
    assert not buf[:offset].any() and not buf[offset + nbytes:].any()  # nothing written outside
