"""Ports of the reference's numeric unit tests (tests/test_gqa_states_v10.py,
tests/test_factored_v.py, tests/test_numeric.py:49-61) run against the
oracle's restatement, plus the split-state algebra the CUDA kernel uses
(base-2 online softmax with a log-sum-exp merge)."""
import numpy as np
import pytest

from oracle import oracle as O


def merge_states(states):
    """The merge kernel's algebra: out = sum 2^(m_s-M) acc_s / sum 2^(m_s-M) l_s."""
    M = max(m for m, _, _ in states)
    num = sum(np.exp2(m - M) * a for m, _, a in states)
    den = sum(np.exp2(m - M) * l for m, l, _ in states)
    return num / den


def split_states(scores_log2, values, tile):
    """Per-split (m, l, acc) in base 2, as attn_split_kernel computes them."""
    states = []
    for start in range(0, len(scores_log2), tile):
        s = scores_log2[start:start + tile]
        m = s.max()
        w = np.exp2(s - m)
        states.append((m, w.sum(), w @ values[start:start + tile]))
    return states


def test_gqa_states_against_dense_oracle():
    """tests/test_gqa_states_v10.py:7-47 with the kernel's base-2 states."""
    rng = np.random.default_rng(20261102)
    for tokens, tile in ((1, 1), (7, 1), (31, 7), (31, 13), (391, 13), (391, 256)):
        for magnitude in (1, 1000):
            q = rng.normal(size=(9, 64)) * magnitude
            k = rng.normal(size=(3, tokens, 64))
            u = rng.random((3, tokens, 64))
            scale = np.exp(rng.normal(size=(3, tokens)))
            offset = rng.normal(size=(3, tokens)) * 5
            v = scale[:, :, None] * u + offset[:, :, None]
            expected = O.attention_f64(q[None], k[None], v[None])[0]
            for h in range(9):
                kh = h // 3
                s2 = (k[kh] @ q[h]) / 8 * np.log2(np.e)
                got = merge_states(split_states(s2, v[kh], tile))
                np.testing.assert_allclose(got, expected[h], atol=2e-11, rtol=2e-11)


@pytest.mark.parametrize("case", ["constant", "extreme", "nonuniform"])
def test_factored_v_affine(case):
    """tests/test_factored_v.py: sum p (s u + o) = sum (p s) u + sum p o across splits."""
    rng = np.random.default_rng({"constant": 1, "extreme": 42, "nonuniform": 20261028}[case])
    if case == "constant":
        scores, u, scale, offset = np.linspace(-12, 12, 23), np.ones((23, 64)), np.zeros(23), np.linspace(-2, 3, 23)
    elif case == "extreme":
        scores, u, scale, offset = np.linspace(-1000, 1000, 31), rng.random((31, 64)), rng.random(31) * 10, rng.normal(size=31) * 5
    else:
        scores, u, scale, offset = rng.normal(size=67) * 3, rng.random((67, 64)), np.exp(rng.normal(size=67) * 2), rng.normal(size=67) * 10
    w = np.exp(scores - scores.max())
    expected = w @ (u * scale[:, None] + offset[:, None]) / w.sum()
    states = []
    for start in range(0, len(scores), 7):
        s = scores[start:start + 7] * np.log2(np.e)
        m = s.max()
        ww = np.exp2(s - m)
        acc = (ww * scale[start:start + 7]) @ u[start:start + 7] + (ww @ offset[start:start + 7])
        states.append((m, ww.sum(), acc))
    np.testing.assert_allclose(merge_states(states), expected, rtol=2e-12, atol=2e-12)


def test_gqa_causal_against_scalar_oracle():
    """tests/test_numeric.py:49-61 against oracle.attention."""
    rng = np.random.default_rng(17)
    q = rng.normal(size=(6, 2, 8)).astype("f4")
    k = rng.normal(size=(2, 7, 8)).astype("f4")
    v = rng.normal(size=k.shape).astype("f4")
    positions = np.array([3, 6])
    got, p = O.attention(q, k, v, positions)
    ref = np.zeros_like(got)
    for h in range(6):
        for i, t in enumerate(positions):
            scores = k[h // 3, :t + 1].astype("f8") @ q[h, i].astype("f8") / np.sqrt(8)
            weights = np.exp(scores - scores.max())
            weights /= weights.sum()
            ref[h, i] = weights @ v[h // 3, :t + 1]
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=2e-6)
    assert np.all(p[:, 0, 4:] == 0)


def test_mask_and_gqa_with_irrelevant_future_key():
    """tests/test_error_diagnostic.py:35-42: future keys never leak."""
    q = np.ones((4, 1, 2), np.float32)
    k = np.zeros((2, 4, 2), np.float32)
    k[:, -1] = 1000
    v = np.array([[[2., 3.]] * 4, [[5., 7.]] * 4], np.float32)
    out, p = O.attention(q, k, v, np.array([1]))
    np.testing.assert_array_equal(p[:, :, 2:], 0)
    np.testing.assert_allclose(out[:, 0], [[2, 3], [2, 3], [5, 7], [5, 7]])
