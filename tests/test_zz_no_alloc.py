"""GPU test of `akv_cuda_decode_attention_noalloc`, the entry point for callers
that cannot allocate device memory.

Who needs it: code that reaches the GPU only through this C ABI from another
runtime (cgo, JNI, N-API bindings own no CUDA allocator), hosts whose device
memory is managed by a framework's caching allocator (a direct cudaMalloc
there fragments the pool and can stall every stream), and serving loops that
run under a fixed device-memory budget. They cannot provide the split-partial
workspace that `akv_cuda_decode_attention` asks for, so this variant keeps
those partials in a static device array inside the library.

The test drives both entry points through the C ABI on the same descriptor.
With the same split plan both launch the same kernels, so the workspace-free
call must reproduce the ordinary call bit for bit, on two calls in a row (the
second call reuses the static array the first one left behind); both must
also agree with the float64 attention over the oracle's decode of the same
blocks within the attention tolerance of the other tests. A descriptor that
leaves the split to the library gets a split that fits the array; one whose
explicit split needs more scratch than the array holds is refused with its
own status code before anything runs. The file is named to be collected
last and builds its inputs itself, so it passes alone in a fresh process as
well as after the rest of the suite.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from common import ATOL, REL_L2, RTOL, golden, oracle_restore
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case():
    from astc_kv_cuda.ops import Attention, contiguous_astc_plane, contiguous_fp16_plane
    g = golden("story_l17_v_token6")

    def f16(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()
    k = contiguous_fp16_plane(f16(g["k"][None]), 96)
    v = contiguous_astc_plane(torch.from_numpy(g["v_blocks"][None].copy()).cuda(), f16(g["v_offset"][None, ..., 0]),
                              f16(g["v_scale"][None, ..., 0]), block=6, layout="scalar", normalization="token",
                              head_dim=64, page_tokens=96)
    # Several query rows over the same cache (batch stride 0), ragged lengths.
    for p in (k, v):
        p.stride_batch = p.meta_stride_batch = 0
    rng = np.random.default_rng(77)
    qn = rng.standard_normal((5, 9, 64)).astype(np.float32)
    q = torch.from_numpy(qn).cuda()
    lens = [384, 1, 200, 97, 383]
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    attn = Attention(q, k, v, page_tokens=96, max_tokens=384, seq_lens=lens_t, split_tokens=48)
    # Oracle: CPU decode of the same blocks, unfused fp32 restore, float64 attention.
    vr = oracle_restore(g["v_blocks"], g["v_offset"], g["v_scale"], "token", 6, "scalar", 64, 96)
    kk = g["k"].astype(np.float32)
    expect = O.attention_f64(qn, np.broadcast_to(kk, (5,) + kk.shape), np.broadcast_to(vr, (5,) + vr.shape), lens)
    return attn, expect


def _noalloc(attn, split_tokens=None):
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    # Hand the descriptor over without any workspace.
    d = L.AkvAttnDesc.from_buffer_copy(attn.desc)
    d.workspace_dev, d.workspace_bytes = None, 0
    if split_tokens is not None:
        d.split_tokens = split_tokens
    stream = torch.cuda.current_stream().cuda_stream or None
    rc = lib.akv_cuda_decode_attention_noalloc(ct.byref(d), stream)
    assert rc == 0, lib.akv_cuda_error(rc).decode()
    torch.cuda.synchronize()
    return attn.out.cpu().numpy()


def _close_to(out, expect, what):
    np.testing.assert_allclose(out, expect, atol=ATOL, rtol=RTOL, err_msg=what)
    rel = np.linalg.norm(out - expect) / np.linalg.norm(expect)
    assert rel <= REL_L2, f"{what}: relative L2 {rel:.3e}"


def test_noalloc_matches_workspace_entry_point(cuda):
    attn, expect = _case()
    ref = attn.run().clone().cpu().numpy()
    torch.cuda.synchronize()
    _close_to(ref, expect, "workspace entry point vs oracle")
    for call in range(2):
        attn.out.fill_(float("nan"))
        out = _noalloc(attn)
        # Same kernels, same split plan: identical results.
        assert np.array_equal(out, ref), f"call {call}: differs from the workspace entry point"
        _close_to(out, expect, f"call {call} vs oracle")


def test_noalloc_default_split_fits_the_static_array(cuda):
    """split_tokens = 0 leaves the split to the library, which then picks one
    whose partials fit the static array; the result still matches the oracle.
    The second case is config 2's shape (Hq32/Hkv8, D128) at eight sequences
    of 32768 tokens, whose usual split would need about 15 MB of partials."""
    attn, expect = _case()
    for call in range(2):
        attn.out.fill_(float("nan"))
        out = _noalloc(attn, split_tokens=0)
        _close_to(out, expect, f"default split, call {call}")
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    from astc_kv_cuda import _lib as L
    wl = bench.Workload("c2", cuda, batch=8)
    assert wl.attn.workspace.numel() * 4 > L.AKV_STATIC_WORKSPACE_BYTES
    ref = wl.attn.run().clone().cpu().numpy()
    for call in range(2):
        wl.attn.out.fill_(float("nan"))
        out = _noalloc(wl.attn, split_tokens=0)
        np.testing.assert_allclose(out, ref, atol=ATOL, rtol=RTOL, err_msg=f"config 2 shape, call {call}")
        rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
        assert rel <= REL_L2, rel


def test_noalloc_rejects_scratch_beyond_its_maximum(cuda):
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    attn, _ = _case()
    d = L.AkvAttnDesc.from_buffer_copy(attn.desc)
    # 4096 sequences x 9 heads x 8 splits x (64 + 2) floats > 8 MiB.
    d.batch = 4096
    d.split_tokens = 48
    need = lib.akv_cuda_attention_workspace(ct.byref(d))
    assert need > L.AKV_STATIC_WORKSPACE_BYTES
    assert lib.akv_cuda_decode_attention_noalloc(ct.byref(d), None) == L.AKV_ERR_STATIC_WORKSPACE
    assert b"static workspace" in lib.akv_cuda_error(L.AKV_ERR_STATIC_WORKSPACE)
