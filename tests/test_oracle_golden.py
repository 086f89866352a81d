"""The CPU oracle against the reference's astcenc golden vectors (6x6 LDR, scalar).

Pins the oracle before anything trusts it: decode + unfused fp32 restore must
reproduce the reference's `*_decoded.f32` / `identity.npy` restores bit for
bit, and the restated NumPy attention must match the reference's own
`codec.attention` output on those values.
"""
import numpy as np

from common import golden, oracle_restore, sha
from oracle import oracle as O


def test_v_token_fixture_bit_exact():
    g = golden("story_l17_v_token6")
    rec = oracle_restore(g["v_blocks"], g["v_offset"], g["v_scale"], "token", 6, "scalar", 64, int(g["page_tokens"]))
    assert rec.dtype == np.float32
    np.testing.assert_array_equal(rec, g["v_decoded"])


def test_kv_page_channel_fixture_bit_exact():
    g = golden("story_l17_kv_page6")
    P = int(g["page_tokens"])
    for side in ("k", "v"):
        rec = oracle_restore(g[side + "_blocks"], g[side + "_offset"], g[side + "_scale"], "page_channel", 6, "scalar", 64, P)
        np.testing.assert_array_equal(rec[0], g[side + "_decoded_head0"])
        assert sha(rec) == str(g[side + "_decoded_sha256"])


def test_block_geometry_identity_sets_bit_exact():
    g = golden("block_geometry_identity")
    for i, name in enumerate(g["names"]):
        blocks = g["blocks"][i].reshape(3, 48, 11, 16)
        rec = oracle_restore(blocks, g["offsets"][i], g["scales"][i], "token", 6, "scalar", 64, 96)
        assert sha(rec) == str(g["decoded_sha256"][i]), f"{name}: restore differs from astcenc"


def test_image_decode_matches_akv_decode_contract():
    g = golden("story_l17_v_token6")
    payload = g["v_blocks"][0].tobytes()
    img = O.decode_image_f32(payload, 6, 66, 384)
    rec = img[:, :64, 0] * g["v_scale"][0].astype(np.float32) + g["v_offset"][0].astype(np.float32)
    np.testing.assert_array_equal(rec, g["v_decoded"][0])
    assert np.all(img[..., 3] == 1.0)  # rrr1 scalar layout keeps alpha at one


def test_oracle_attention_matches_reference_output():
    g = golden("story_l17_v_token6")
    k = g["k"].astype(np.float32)
    out, p = O.attention(g["q"][:, None, :], k, g["v_decoded"], np.array([383]))
    np.testing.assert_allclose(out[:, 0], g["attn_out"], rtol=1e-5, atol=1e-6)
    ref64 = O.attention_f64(g["q"][None], k[None], g["v_decoded"][None])[0]
    np.testing.assert_allclose(ref64, g["attn_out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(p.sum(-1), 1.0, rtol=1e-5)


def test_oracle_attention_positions_page_fixture():
    g = golden("story_l17_kv_page6")
    P = int(g["page_tokens"])
    k = oracle_restore(g["k_blocks"], g["k_offset"], g["k_scale"], "page_channel", 6, "scalar", 64, P)
    v = oracle_restore(g["v_blocks"], g["v_offset"], g["v_scale"], "page_channel", 6, "scalar", 64, P)
    q = np.repeat(g["q"][:, None, :], len(g["positions"]), 1)
    out, _ = O.attention(q, k, v, g["positions"])
    np.testing.assert_allclose(out, g["attn_out"], rtol=1e-5, atol=1e-6)


def test_unorm8_view_is_recoverable_from_golden_fp16():
    """The fp16 view astcenc emits pins C >> 8 exactly: floor(u * 256), u == 1 -> 255."""
    g = golden("block_geometry_identity")
    blocks = g["blocks"][0]
    u16 = O.decode_blocks(blocks, 6, O.OUT_UNORM16)
    f16 = O.decode_blocks(blocks, 6, O.OUT_FP16).astype(np.float64)
    u8 = O.decode_blocks(blocks, 6, O.OUT_UNORM8)
    np.testing.assert_array_equal(u8, (u16 >> 8).astype(np.uint8))
    np.testing.assert_array_equal(u8, np.minimum(np.floor(f16 * 256), 255).astype(np.uint8))
