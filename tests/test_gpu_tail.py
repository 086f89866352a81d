"""Fresh-tail decode attention: compressed complete pages plus an exact FP16
tail (the incomplete last page) in one softmax (akv_cuda_decode_attention_tail).

The reference's encoder only accepts whole pages (astc_kv/codec.py:132-133);
its pilot keeps the newest tokens in FP16 (scripts/run_pilot.py:70-75). Here the
two segments are attended together and compared with float64 NumPy attention
over the concatenation [decoded pages; tail] per sequence.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from common import O, assert_attention_close, device_astc_plane, kv_values, make_astc_plane

pytestmark = pytest.mark.gpu


def f16t(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()


def _case(B, Hq, Hkv, D, T, P, tail_cap, lens, tail_lens, *, vfmt, seed):
    from astc_kv_cuda.ops import Attention, contiguous_fp16_plane
    rng = np.random.default_rng(seed)
    xk, _ = kv_values(rng, B, Hkv, T, D, outliers=2)
    xv, _ = kv_values(rng, B, Hkv, T, D)
    tk, _ = kv_values(rng, B, Hkv, tail_cap, D, outliers=2)
    tv, _ = kv_values(rng, B, Hkv, tail_cap, D)
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    block, layout, norm = vfmt
    pv = make_astc_plane(xv, block=block, layout=layout, normalization=norm, page_tokens=P)
    k16, tk16, tv16 = xk.astype(np.float16), tk.astype(np.float16), tv.astype(np.float16)
    kp = contiguous_fp16_plane(f16t(k16), P)
    vp = device_astc_plane(pv, block=block, layout=layout, normalization=norm, page_tokens=P, dim=D)
    tkp = contiguous_fp16_plane(f16t(tk16), tail_cap)
    tvp = contiguous_fp16_plane(f16t(tv16), tail_cap)
    attn = Attention(torch.from_numpy(q).cuda(), kp, vp, page_tokens=P, max_tokens=T,
                     seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"), tail_k=tkp, tail_v=tvp,
                     tail_lens=torch.tensor(tail_lens, dtype=torch.int32, device="cuda"), tail_tokens=tail_cap)
    got = attn.run().cpu().numpy()
    # Reference: per sequence, the first lens[b] decoded tokens then the first
    # tail_lens[b] tail tokens.
    n = T + tail_cap
    kc = np.zeros((B, Hkv, n, D), np.float32)
    vc = np.zeros((B, Hkv, n, D), np.float32)
    tot = []
    for b in range(B):
        a, t = lens[b], tail_lens[b]
        kc[b, :, :a] = k16[b, :, :a].astype(np.float32)
        vc[b, :, :a] = pv["restored"][b, :, :a]
        kc[b, :, a:a + t] = tk16[b, :, :t].astype(np.float32)
        vc[b, :, a:a + t] = tv16[b, :, :t].astype(np.float32)
        tot.append(a + t)
    ref = O.attention_f64(q, kc, vc, tot)
    for b, m in enumerate(tot):
        if m == 0:
            ref[b] = 0.0
    return got, ref, attn


@pytest.mark.parametrize("vfmt", [(6, "scalar", "block_affine"), (4, "scalar", "token")])
def test_tail_segment_in_one_softmax(cuda, vfmt):
    P = 96 if vfmt[0] == 6 else 64
    T = 4 * P
    lens = [T, P, 0, 2 * P + 13, 0]
    tail_lens = [17, 0, 5, P - 1, 0]
    got, ref, attn = _case(5, 9, 3, 64, T, P, P, lens, tail_lens, vfmt=vfmt, seed=41)
    assert_attention_close(got, ref, f"tail {vfmt}")
    assert np.all(got[4] == 0.0)  # nothing to attend: zeros, as the single-segment call gives


def test_tail_matches_single_segment_when_empty(cuda):
    """An all-empty tail leaves the result of the ordinary call unchanged."""
    P, T = 96, 384
    got, ref, attn = _case(3, 9, 3, 64, T, P, 32, [T, 150, 7], [0, 0, 0], vfmt=(6, "scalar", "token"), seed=5)
    assert_attention_close(got, ref, "empty tail")
    from astc_kv_cuda import _lib as L
    plain = L.AkvAttnDesc.from_buffer_copy(attn.desc)
    ws = torch.empty(L.lib().akv_cuda_attention_workspace(ct.byref(plain)) // 4 + 4, device="cuda")
    out = torch.empty_like(attn.out)
    plain.workspace_dev, plain.workspace_bytes, plain.out_dev = ws.data_ptr(), ws.numel() * 4, out.data_ptr()
    assert L.lib().akv_cuda_decode_attention(ct.byref(plain), None) == 0
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), got, atol=1e-6, rtol=1e-5)


def test_tail_descriptor_mismatch_is_rejected(cuda):
    from astc_kv_cuda import _lib as L
    P, T = 96, 384
    _, _, attn = _case(2, 9, 3, 64, T, P, 32, [T, 10], [3, 4], vfmt=(6, "scalar", "token"), seed=9)
    tail = L.AkvAttnDesc.from_buffer_copy(attn.tail)
    tail.kv_heads = 1
    assert L.lib().akv_cuda_attention_tail_workspace(ct.byref(attn.desc), ct.byref(tail)) == 0
    assert L.lib().akv_cuda_decode_attention_tail(ct.byref(attn.desc), ct.byref(tail), None) == 1
