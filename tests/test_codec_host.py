"""Host-side logic of the codec mirror (encode_tensor normalisation, checks and
byte accounting, .astc interchange) — the CPU half that stays on the CPU in
the reference too (astc_kv/codec.py:116-215). Ports of tests/test_numeric.py."""
import numpy as np
import pytest

import astc_kv_cuda as A
from astc_kv_cuda import interchange as I
from common import golden
from oracle import oracle as O


def test_payload_and_metadata_padding():
    """tests/test_numeric.py:29-38."""
    x = np.zeros((3, 288, 64), np.float32)
    p = A.encode_tensor(x, dict(layout="scalar", block=6, normalization="page_channel"))
    assert p.width == 66
    assert p.byte_counts["astc_blocks_including_edge_padding"] == 3 * 48 * 11 * 16
    assert p.logical_bytes == 3 * 288 * 64 * 4 // 8
    assert len(p.astc_file(0)) == 16 + 48 * 11 * 16
    t = A.encode_tensor(x, dict(layout="scalar", block=6, normalization="token"))
    assert t.bits_per_scalar == pytest.approx(4 + 1 / 6)


def test_no_future_in_incomplete_page():
    """tests/test_numeric.py:40-42."""
    with pytest.raises(ValueError):
        A.encode_tensor(np.zeros((1, 97, 64), "f4"), dict(layout="scalar", block=6, normalization="token"))


@pytest.mark.parametrize("bad", [
    dict(layout="scalar", block=6, normalization="token", permutation="bogus"),
    dict(layout="rgba", block=4, normalization="token", dim=62),
    dict(layout="scalar", block=6, normalization="nope"),
])
def test_rejections(bad):
    dim = bad.pop("dim", 64)
    with pytest.raises(ValueError):
        A.encode_tensor(np.zeros((1, 96, dim), "f4"), bad)


def test_page_must_align_to_block_rows():
    with pytest.raises(ValueError):
        A.encode_tensor(np.zeros((1, 100, 64), "f4"), dict(layout="scalar", block=8, normalization="token"), page_tokens=100)


def test_metadata_bounds():
    """tests/test_numeric.py:44-47."""
    x = np.concatenate([np.linspace(-500, 500, 10001), [0, 2 ** -27, -2 ** -27, 1.0004]]).astype("f4")
    assert np.all(A.fp16_floor(x).astype("f4") <= x)
    assert np.all(A.fp16_ceil(x).astype("f4") >= x)


@pytest.mark.parametrize("cfg,P", [
    ({"block": 6, "layout": "scalar", "normalization": "token"}, 96),
    ({"block": 4, "layout": "rgba", "normalization": "page_channel"}, 16),
    ({"block": 8, "layout": "scalar", "normalization": "block_affine"}, 64),
])
def test_encoder_output_decodes_close_to_input(cfg, P):
    """The package encoder writes legal blocks: the oracle decodes them without
    error colours and close to the normalised input."""
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((2, 192, 64)) * rng.lognormal(0, 0.5, (1, 1, 64))).astype(np.float32)
    e = A.encode_tensor(x, cfg, page_tokens=P, quality=60)
    blocks = e.blocks_array().reshape(-1, 16)
    kinds = {O.block_info(b, cfg["block"])["kind"] for b in blocks[::13]}
    assert 1 not in kinds
    from common import oracle_restore
    rec = oracle_restore(e.blocks_array(), e.offsets, e.scales, cfg["normalization"], cfg["block"], cfg["layout"], 64, P)
    rel = np.linalg.norm(rec - x) / np.linalg.norm(x)
    # A legality/sanity bound, not a quality claim. The values are i.i.d.
    # across channels and tokens: RGBA packs four independent channels behind
    # one weight per texel and an 8x8 block holds 64 independent values in
    # 128 bits, both poor fits for ASTC's endpoint/weight model (the reference
    # notes the RGBA risk too).
    bound = 0.4 if (cfg["layout"] == "scalar" and cfg["block"] < 8) else 0.95
    assert rel < bound, rel


def test_astc_file_roundtrip_and_reader():
    g = golden("story_l17_v_token6")
    payload = g["v_blocks"][1].tobytes()
    raw = I.write_astc(6, 66, 384, payload)
    assert I.read_astc(raw) == (6, 66, 384, payload)
    with pytest.raises(ValueError):
        I.read_astc(b"\x00" * 32)
    with pytest.raises(ValueError):
        I.read_astc(raw[:-16])


def test_random_blocks_are_legal_and_cover_modes():
    blocks = A.random_blocks(3000, 6, seed=3)
    infos = [O.block_info(b, 6) for b in blocks]
    assert all(i["kind"] != 1 for i in infos)
    assert {i["partitions"] for i in infos if i["kind"] == 0} == {1, 2, 3, 4}
    assert any(i["dual"] for i in infos)
    assert any(i["kind"] == 2 for i in infos)


def test_non_finite_plane_metadata_is_rejected():
    """Failure detection on the host: NaN / inf scales or offsets are refused
    when a device plane is built (before any launch)."""
    import torch
    from astc_kv_cuda.ops import contiguous_astc_plane, paged_astc_plane
    blocks = torch.zeros((1, 1, 16, 22, 16), dtype=torch.uint8)
    good = torch.ones((1, 1, 16, 22), dtype=torch.float16)
    for bad_value in (float("nan"), float("inf")):
        bad = good.clone()
        bad[0, 0, 3, 5] = bad_value
        for off, scl in ((bad, good), (good, bad)):
            with pytest.raises(ValueError, match="non-finite"):
                contiguous_astc_plane(blocks, off, scl, block=6, layout="scalar", normalization="block_affine",
                                      head_dim=128, page_tokens=96)
            with pytest.raises(ValueError, match="non-finite"):
                paged_astc_plane(blocks[0][:, None], off[0][:, None], scl[0][:, None], block=6, layout="scalar",
                                 normalization="block_affine", head_dim=128, page_tokens=96)
