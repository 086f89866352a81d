"""GPU parity of the codec.py mirror: encode_tensor -> GPU restore -> attention."""
import numpy as np
import pytest

from common import assert_attention_close, kv_values, oracle_restore
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", [
    {"block": 6, "layout": "scalar", "normalization": "token"},
    {"block": 4, "layout": "rgba", "normalization": "page_channel"},
    {"block": 8, "layout": "scalar", "normalization": "page_channel"},
    {"block": 6, "layout": "scalar", "normalization": "block_affine"},
    {"block": 6, "layout": "scalar", "normalization": "page_channel", "permutation": "channels"},
])
def test_encode_tensor_decoded_is_oracle_restore(cuda, cfg):
    import astc_kv_cuda as A
    x, _ = kv_values(np.random.default_rng(11), 1, 3, 192, 64)
    e = A.encode_tensor(x[0], cfg, page_tokens=96 if cfg["block"] == 6 else 64, quality=60)
    if cfg.get("permutation"):
        dec = e.decoded
        assert dec.shape == (3, 192, 64)
        assert np.abs(dec - x[0]).max() < np.abs(x[0]).max()  # restored to original channel order
        return
    ref = oracle_restore(e.blocks_array(), e.offsets, e.scales, e.normalization, e.block, e.layout, 64, e.page_tokens)
    np.testing.assert_array_equal(e.decoded, ref)
    rel = np.linalg.norm(e.decoded - x[0]) / np.linalg.norm(x[0])
    # A working encoder, not a quality claim: i.i.d. per-channel values are a
    # poor fit for ASTC's endpoint/weight model, worst for RGBA (four
    # independent channels per weight) and 8x8 (64 values in 128 bits);
    # astcenc 5.7.0 at quality 98 reaches ~0.18 relative L2 on the reference's
    # 6x6 scalar captures.
    bound = 0.4 if (cfg["layout"] == "scalar" and cfg["block"] < 8) else 0.95
    assert rel < bound, rel


def test_codec_attention_mirror_positions(cuda):
    import astc_kv_cuda as A
    rng = np.random.default_rng(12)
    k, _ = kv_values(rng, 1, 3, 192, 64)
    v, _ = kv_values(rng, 1, 3, 192, 64)
    ek = A.encode_tensor(k[0], {"block": 6, "layout": "scalar", "normalization": "page_channel"}, quality=60)
    ev = A.encode_tensor(v[0], {"block": 6, "layout": "scalar", "normalization": "token"}, quality=60)
    q = rng.standard_normal((9, 3, 64)).astype(np.float32)
    pos = np.array([191, 50, 0])
    got, probs = A.attention(q, ek, ev, pos)
    assert probs is None
    ref, _ = O.attention(q, ek.decoded, ev.decoded, pos)
    assert_attention_close(got, ref, "codec.attention mirror")
    # fp16 arrays as K/V planes
    got16, _ = A.attention(q, k[0].astype(np.float16), ev, pos)
    ref16, _ = O.attention(q, k[0].astype(np.float16).astype(np.float32), ev.decoded, pos)
    assert_attention_close(got16, ref16, "fp16 K plane")


def test_codec_attention_mirror_fresh_tail(cuda):
    """codec.attention with an FP16 tail: positions past the encoded pages
    attend the tail tokens in the same softmax."""
    import astc_kv_cuda as A
    rng = np.random.default_rng(13)
    k, _ = kv_values(rng, 1, 3, 192, 64)
    v, _ = kv_values(rng, 1, 3, 192, 64)
    kt, _ = kv_values(rng, 1, 3, 40, 64)
    vt, _ = kv_values(rng, 1, 3, 40, 64)
    ek = A.encode_tensor(k[0], {"block": 6, "layout": "scalar", "normalization": "page_channel"}, quality=60)
    ev = A.encode_tensor(v[0], {"block": 6, "layout": "scalar", "normalization": "token"}, quality=60)
    q = rng.standard_normal((9, 4, 64)).astype(np.float32)
    pos = np.array([231, 200, 191, 10])
    kt16, vt16 = kt[0].astype(np.float16), vt[0].astype(np.float16)
    got, _ = A.attention(q, ek, ev, pos, k_tail=kt16, v_tail=vt16)
    kall = np.concatenate([ek.decoded, kt16.astype(np.float32)], axis=1)
    vall = np.concatenate([ev.decoded, vt16.astype(np.float32)], axis=1)
    ref, _ = O.attention(q, kall, vall, pos)
    assert_attention_close(got, ref, "codec.attention mirror with FP16 tail")


def test_probe_fixture_through_the_gpu_attention(cuda, tmp_path):
    """A fixture written in the reference's astc-kv-probe-v1 format (the
    reference's own story_l17_v_token6 data), read back by load_manifest and
    attended on the GPU, reproduces the reference's codec.attention output."""
    import torch
    from astc_kv_cuda import interchange as I
    from astc_kv_cuda.codec import EncodedTensor
    from astc_kv_cuda.ops import Attention, contiguous_astc_plane, contiguous_fp16_plane
    from common import assert_attention_close, golden
    g = golden("story_l17_v_token6")
    H, T, D = g["k"].shape
    enc = EncodedTensor(g["v_decoded"], [g["v_blocks"][h].tobytes() for h in range(H)], 66, 384, 6, "scalar", "ldr",
                        "token", g["v_offset"], g["v_scale"], 96, {}, 0.0, metadata={"dim": D})
    I.write_manifest(tmp_path, g["q"], g["k"].astype(np.float32), enc, page_tokens=96)
    fx = I.load_manifest(tmp_path)
    m = fx["manifest"]
    P = m["page_tokens"]

    def f16(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()
    k = contiguous_fp16_plane(f16(fx["k"]["fp16"][None]), P)
    v = contiguous_astc_plane(torch.from_numpy(fx["v"]["blocks"][None].copy()).cuda(), f16(fx["v"]["offsets"][None, ..., 0]),
                              f16(fx["v"]["scales"][None, ..., 0]), block=fx["v"]["block"], layout=m["layout"],
                              normalization=fx["v"]["normalization"], head_dim=D, page_tokens=P)
    out = Attention(torch.from_numpy(fx["q"][None]).cuda(), k, v, page_tokens=P, max_tokens=m["tokens"]).run()
    torch.cuda.synchronize()
    assert_attention_close(out.cpu().numpy()[0], g["attn_out"], "probe-v1 fixture vs reference codec.attention")
