"""GPU test of `akv_cuda_decode_attention_noalloc`, the entry point for callers
that cannot allocate device memory.

Who needs it: code that reaches the GPU only through this C ABI from another
runtime (cgo, JNI, N-API bindings own no CUDA allocator), hosts whose device
memory is managed by a framework's caching allocator (a direct cudaMalloc
there fragments the pool and can stall every stream), and serving loops that
run under a fixed device-memory budget. They cannot provide the split-partial
workspace that `akv_cuda_decode_attention` asks for, so this variant keeps
those partials in a static device array inside the library.

The test drives both entry points through the C ABI on the same descriptor
and requires the workspace-free call to agree with the ordinary call within
the attention tolerance of the other tests, on two calls in a row (the second
call reuses the static array the first one left behind). It also checks that
a descriptor needing more scratch than the array holds is refused with its
own status code before anything runs. The file is named to be collected
last and builds its inputs itself, so it passes alone in a fresh process as
well as after the rest of the suite.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from common import ATOL, RTOL, golden

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
    q = torch.from_numpy(rng.standard_normal((5, 9, 64)).astype(np.float32)).cuda()
    lens = torch.tensor([384, 1, 200, 97, 383], dtype=torch.int32, device="cuda")
    return Attention(q, k, v, page_tokens=96, max_tokens=384, seq_lens=lens, split_tokens=48)


def test_noalloc_matches_workspace_entry_point(cuda):
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    attn = _case()
    ref = attn.run().clone()
    torch.cuda.synchronize()
    out = attn.out
    for call in range(2):
        out.fill_(float("nan"))
        # Hand the descriptor over without any workspace.
        d = L.AkvAttnDesc.from_buffer_copy(attn.desc)
        d.workspace_dev, d.workspace_bytes = None, 0
        stream = torch.cuda.current_stream().cuda_stream or None
        rc = lib.akv_cuda_decode_attention_noalloc(ct.byref(d), stream)
        assert rc == 0, lib.akv_cuda_error(rc).decode()
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), atol=ATOL, rtol=RTOL,
                                   err_msg=f"call {call}")


def test_noalloc_rejects_scratch_beyond_its_maximum(cuda):
    from astc_kv_cuda import _lib as L
    lib = L.lib()
    attn = _case()
    d = L.AkvAttnDesc.from_buffer_copy(attn.desc)
    # 4096 sequences x 9 heads x 8 splits x (64 + 2) floats > 8 MiB.
    d.batch = 4096
    d.split_tokens = 48
    need = lib.akv_cuda_attention_workspace(ct.byref(d))
    assert need > L.AKV_STATIC_WORKSPACE_BYTES
    assert lib.akv_cuda_decode_attention_noalloc(ct.byref(d), None) == L.AKV_ERR_STATIC_WORKSPACE
    assert b"static workspace" in lib.akv_cuda_error(L.AKV_ERR_STATIC_WORKSPACE)
