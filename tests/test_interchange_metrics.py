"""Host-side parity of the reference's interchange and metric helpers.

* `errors` / `attention_metrics` (codec.py:270-283) against the values the
  reference's own functions return on seeded inputs (tests/golden/
  metrics_golden.npz, written by make_golden.py from the reference module).
* The astc-kv-probe-v1 fixture format (docs/metal_path.md:50-73, writer
  scripts/export_metal_fixture.py:31-63): `write_manifest` then
  `load_manifest` gives back the same blocks, metadata, query and FP16 side
  bit for bit, and the manifest's byte accounting equals the encoded
  tensor's `byte_counts` (codec.py:209-215).
"""
import json

import numpy as np
import pytest

import astc_kv_cuda as A
from astc_kv_cuda import interchange as I
from common import golden


def test_errors_and_attention_metrics_match_the_reference_values():
    g = golden("metrics_golden")
    e = A.errors(g["a"], g["b"])
    for k, v in zip(g["errors_keys"], g["errors_values"]):
        assert e[str(k)] == pytest.approx(float(v), rel=1e-12, abs=1e-300), k
    m = A.attention_metrics(g["a"], g["b"], g["pa"], g["pb"])
    assert sorted(m) == sorted(map(str, g["metrics_keys"]))
    for k, v in zip(g["metrics_keys"], g["metrics_values"]):
        assert m[str(k)] == pytest.approx(float(v), rel=1e-12, abs=1e-300), k


def test_metrics_known_answers():
    a = np.array([[3.0, 4.0]])
    assert A.errors(a, a) == {"mse": 0.0, "relative_l2": 0.0, "max_abs": 0.0, "cosine": pytest.approx(1.0)}
    e = A.errors(a, np.array([[3.0, 5.0]]))
    assert e["mse"] == pytest.approx(0.5) and e["max_abs"] == 1.0 and e["relative_l2"] == pytest.approx(0.2)
    p = np.array([[0.5, 0.5]])
    r = np.array([[0.25, 0.75]])
    m = A.attention_metrics(a, a, p, r)
    assert m["mean_total_variation"] == pytest.approx(0.25)
    assert m["mean_kl_nats"] == pytest.approx(0.5 * np.log(2.0) + 0.5 * np.log(0.5 / 0.75))


@pytest.mark.parametrize("norm", ["token", "page_channel"])
def test_probe_manifest_roundtrip_and_byte_accounting(tmp_path, norm):
    rng = np.random.default_rng(11)
    H, Hq, T, D, P = 3, 9, 192, 64, 96
    x = (rng.standard_normal((H, T, D)) * rng.lognormal(0, 0.5, (1, 1, D))).astype(np.float32)
    kf = rng.standard_normal((H, T, D)).astype(np.float32)
    q = rng.standard_normal((Hq, D)).astype(np.float32)
    enc = A.encode_tensor(x, {"block": 6, "layout": "scalar", "normalization": norm}, page_tokens=P, quality=10)
    m = I.write_manifest(tmp_path, q, kf, enc, page_tokens=P, with_decoded=False)
    assert json.loads((tmp_path / "manifest.json").read_text()) == m
    lc = m["logical_cache_bytes"]
    counts = enc.byte_counts
    assert lc["v"] == {"astc_blocks_with_padding": counts["astc_blocks_including_edge_padding"],
                       "fp16_offsets": counts["fp16_offsets"], "fp16_scales": counts["fp16_scales"]}
    assert counts["permutation_map"] == 0 and sum(lc["v"].values()) == enc.logical_bytes
    assert lc["k"] == {"fp16_payload": H * T * D * 2}
    back = I.load_manifest(tmp_path)
    assert np.array_equal(back["q"], q)
    assert back["k"]["storage"] == "fp16" and np.array_equal(back["k"]["fp16"], kf.astype(np.float16))
    v = back["v"]
    assert v["storage"] == "astc" and v["block"] == 6 and v["normalization"] == norm
    assert np.array_equal(v["blocks"], enc.blocks_array())
    assert np.array_equal(v["offsets"].reshape(enc.offsets.shape), enc.offsets)
    assert np.array_equal(v["scales"].reshape(enc.scales.shape), enc.scales)
    for h in range(H):
        assert (tmp_path / f"v-h{h:03d}.astc").read_bytes() == enc.astc_file(h)


def test_probe_manifest_of_the_reference_fixture_layout(tmp_path):
    """The reference fixture story_l17_v_token6 (astcenc blocks, token
    metadata, FP16 K) written in the probe format and read back unchanged."""
    from astc_kv_cuda.codec import EncodedTensor
    g = golden("story_l17_v_token6")
    H, T, D = g["k"].shape
    enc = EncodedTensor(g["v_decoded"], [g["v_blocks"][h].tobytes() for h in range(H)], 66, 384, 6, "scalar", "ldr",
                        "token", g["v_offset"], g["v_scale"], int(g["page_tokens"]),
                        {"astc_blocks_including_edge_padding": g["v_blocks"].nbytes, "fp16_offsets": g["v_offset"].nbytes,
                         "fp16_scales": g["v_scale"].nbytes, "permutation_map": 0}, 0.0, metadata={"dim": D})
    I.write_manifest(tmp_path, g["q"], g["k"].astype(np.float32), enc, page_tokens=96)
    back = I.load_manifest(tmp_path)
    assert np.array_equal(back["v"]["blocks"], g["v_blocks"])
    assert np.array_equal(back["v"]["offsets"], g["v_offset"]) and np.array_equal(back["v"]["scales"], g["v_scale"])
    assert np.array_equal(back["v"]["decoded"], g["v_decoded"])
    assert np.array_equal(back["k"]["fp16"], g["k"])
    with pytest.raises(ValueError):
        I.write_manifest(tmp_path / "x", g["q"], g["k"], g["k"], page_tokens=96)
