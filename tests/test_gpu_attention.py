"""GPU parity of the fused decode + split-K attention, through the C ABI.

Each case compares the CUDA output with float64 NumPy attention
(codec.py:253-267 restated in oracle/oracle.py) on the oracle's decode of the
very same blocks, within max-abs 2e-3 / relative 1e-3 and relative L2 <= 1e-4.
Shapes follow the five benchmark configurations at oracle-sized token counts,
plus the reference's ragged cases (T = 1, 7, 391; tiles 1/7/13 in the
reference, here split sizes of one block row up to several pages).
"""
import numpy as np
import pytest
import torch

from common import assert_attention_close, device_astc_plane, golden, kv_values, make_astc_plane, oracle_restore
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def f16t(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()


def run(q, k, v, **kw):
    from astc_kv_cuda.ops import Attention
    out = Attention(q, k, v, **kw).run()
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_golden_v_token_fixture_against_reference_output(cuda):
    """Reference fixture story_l17_v_token6: FP16 K, astcenc 6x6 V (token norm)."""
    from astc_kv_cuda.ops import contiguous_fp16_plane
    g = golden("story_l17_v_token6")
    k = contiguous_fp16_plane(f16t(g["k"][None]), 96)
    vp = {"blocks": g["v_blocks"][None], "offsets": g["v_offset"][None, ..., 0], "scales": g["v_scale"][None, ..., 0]}
    v = device_astc_plane(vp, block=6, layout="scalar", normalization="token", page_tokens=96, dim=64)
    q = torch.from_numpy(g["q"][None]).cuda()
    for split in (0, 6, 96, 384):
        got = run(q, k, v, page_tokens=96, max_tokens=384, split_tokens=split)[0]
        assert_attention_close(got, g["attn_out"], f"split={split} vs reference codec.attention")
        ref = O.attention_f64(g["q"][None], g["k"].astype(np.float32)[None], g["v_decoded"][None])[0]
        assert_attention_close(got, ref, f"split={split} vs float64")


def test_golden_kv_page_channel_fixture_positions(cuda):
    """Reference fixture story_l17_kv_page6: astcenc 6x6 K and V, page_channel,
    four query positions (the reference's arbitrary-position attention)."""
    g = golden("story_l17_kv_page6")
    P = int(g["page_tokens"])
    planes = {}
    for side in ("k", "v"):
        p = {"blocks": g[side + "_blocks"][None], "offsets": g[side + "_offset"][None], "scales": g[side + "_scale"][None]}
        planes[side] = device_astc_plane(p, block=6, layout="scalar", normalization="page_channel", page_tokens=P, dim=64)
    # Each query is a batch entry over the same cache (batch stride 0).
    for p in planes.values():
        p.stride_batch = p.meta_stride_batch = 0
    pos = g["positions"]
    q = torch.from_numpy(np.repeat(g["q"][None], len(pos), 0)).cuda()
    lens = torch.from_numpy((pos + 1).astype(np.int32)).cuda()
    got = run(q, planes["k"], planes["v"], page_tokens=P, max_tokens=384, seq_lens=lens)
    assert_attention_close(got, g["attn_out"].transpose(1, 0, 2), "kv_page6 vs reference codec.attention")


def _cfg_case(B, Hq, Hkv, D, T, *, kfmt, vfmt, seed, page_tokens, q_dtype=torch.float32, lens=None, split=0,
              paged=False, side=0, bad=None):
    """Build a synthetic cache, run the kernel, compare with float64 NumPy.
    bad=(b, logical page): that block-table entry points past the pool; the
    reference then reads that page's K and V as zeros (the kernel's rule)."""
    from astc_kv_cuda.ops import contiguous_fp16_plane, paged_astc_plane, paged_fp16_plane
    rng = np.random.default_rng(seed)
    xk, ch = kv_values(rng, B, Hkv, T, D, outliers=2)
    xv, _ = kv_values(rng, B, Hkv, T, D)
    qn = rng.standard_normal((B, Hq, D)).astype(np.float32)
    qt = torch.from_numpy(qn).to(q_dtype).cuda()
    qn = qt.float().cpu().numpy()
    planes, restored = {}, {}
    for side_name, x, fmt in (("k", xk, kfmt), ("v", xv, vfmt)):
        if fmt is None:
            x16 = x.astype(np.float16)
            restored[side_name] = x16.astype(np.float32)
            planes[side_name] = ("fp16", x16)
        else:
            block, layout, norm = fmt
            p = make_astc_plane(x, block=block, layout=layout, normalization=norm, page_tokens=page_tokens,
                                side_channels=ch if (side_name == "k" and side) else None)
            restored[side_name] = p["restored"]
            planes[side_name] = ("astc", p, fmt)
    table = None
    num_pages = 0
    if paged:
        pps = T // page_tokens
        num_pages = B * pps
        perm = rng.permutation(num_pages).astype(np.int32)
        table = perm.reshape(B, pps)
    dev = {}
    for name, entry in planes.items():
        if entry[0] == "fp16":
            x16 = entry[1]
            if paged:
                pages = np.zeros((num_pages, Hkv, page_tokens, D), np.float16)
                for b in range(B):
                    for lp in range(T // page_tokens):
                        pages[table[b, lp]] = x16[b, :, lp * page_tokens:(lp + 1) * page_tokens]
                dev[name] = paged_fp16_plane(f16t(pages))
            else:
                dev[name] = contiguous_fp16_plane(f16t(x16), page_tokens)
        else:
            p, (block, layout, norm) = entry[1], entry[2]
            if paged:
                assert norm == "block_affine" and layout == "scalar"
                rows = page_tokens // block
                cols = p["blocks"].shape[3]
                atlas = np.zeros((num_pages, Hkv, rows, cols, 16), np.uint8)
                off = np.zeros((num_pages, Hkv, rows, cols), np.float16)
                scl = np.zeros_like(off)
                for b in range(B):
                    for lp in range(T // page_tokens):
                        sl = slice(lp * rows, (lp + 1) * rows)
                        atlas[table[b, lp]] = p["blocks"][b, :, sl]
                        off[table[b, lp]] = p["offsets"][b, :, sl]
                        scl[table[b, lp]] = p["scales"][b, :, sl]
                dev[name] = paged_astc_plane(torch.from_numpy(atlas).cuda(), f16t(off), f16t(scl), block=block,
                                             layout=layout, normalization=norm, head_dim=D, page_tokens=page_tokens)
            else:
                dev[name] = device_astc_plane(p, block=block, layout=layout, normalization=norm,
                                              page_tokens=page_tokens, dim=D)
    lens_t = torch.from_numpy(np.asarray(lens, np.int32)).cuda() if lens is not None else None
    extra = {}
    if bad is not None:
        table = table.copy()
        table[bad] = num_pages + 5
        for name in ("k", "v"):
            restored[name] = restored[name].copy()
            restored[name][bad[0], :, bad[1] * page_tokens:(bad[1] + 1) * page_tokens] = 0.0
        extra["status"] = torch.zeros(1, dtype=torch.int32, device="cuda")
    bt = torch.from_numpy(table).cuda() if table is not None else None
    got = run(qt, dev["k"], dev["v"], page_tokens=page_tokens, max_tokens=T, seq_lens=lens_t, block_table=bt,
              num_pages=num_pages, split_tokens=split, **extra)
    if bad is not None:
        assert int(extra["status"].item()) == 5  # AKV_ERR_BAD_BLOCK_TABLE
    ref = O.attention_f64(qn, restored["k"], restored["v"], lens)
    if lens is not None:
        for b, n in enumerate(lens):
            if n == 0:
                ref[b] = 0.0
    return got, ref


def test_config0_smollm2_rgba_4x4(cuda):
    """Config 0 shape: B1, Hq9/Hkv3, D64, T384, FP16 K, RGBA 4x4 V, 16-token page_channel."""
    got, ref = _cfg_case(1, 9, 3, 64, 384, kfmt=None, vfmt=(4, "rgba", "page_channel"), seed=20261028, page_tokens=16)
    assert_attention_close(got, ref, "config0")


def test_config1_layers_as_batch_split_128(cuda):
    """Config 1 structure at oracle size: several layers in one launch (layers
    as the batch dimension), split-K over 128-token chunks."""
    got, ref = _cfg_case(4, 9, 3, 64, 1024, kfmt=None, vfmt=(4, "rgba", "page_channel"), seed=1, page_tokens=16, split=128)
    assert_attention_close(got, ref, "config1")


@pytest.mark.parametrize("q_dtype", [torch.bfloat16, torch.float32])
def test_config2_llama8b_6x6_block_affine(cuda, q_dtype):
    """Config 2 shape: Hq32/Hkv8, D128, bf16 q, FP16 K, scalar 6x6 V, per-block affine."""
    got, ref = _cfg_case(2, 32, 8, 128, 576, kfmt=None, vfmt=(6, "scalar", "block_affine"), seed=2, page_tokens=96,
                         q_dtype=q_dtype)
    assert_attention_close(got, ref, "config2")


def test_config3_llama70b_astc_k_side_plane_v8x8(cuda):
    """Config 3 shape: Hq64/Hkv8, D128, ASTC 4x4 K with a 2-channel FP16 side
    plane, ASTC 8x8 V, per-block affine."""
    got, ref = _cfg_case(1, 64, 8, 128, 512, kfmt=(4, "scalar", "block_affine"), vfmt=(8, "scalar", "block_affine"),
                         seed=3, page_tokens=64, side=2)
    assert_attention_close(got, ref, "config3")


def test_config4_ragged_paged_atlas(cuda):
    """Config 4 shape: ragged lengths, 256-token pages in a shared 4x4 V atlas
    with randomly permuted pages, FP16 K, int32 block table."""
    lens = [1024, 257, 1, 700]
    got, ref = _cfg_case(4, 32, 8, 128, 1024, kfmt=None, vfmt=(4, "scalar", "block_affine"), seed=4, page_tokens=256,
                         lens=lens, paged=True)
    assert_attention_close(got, ref, "config4")


@pytest.mark.parametrize("vfmt", [(4, "scalar", "block_affine"), (6, "scalar", "block_affine")])
def test_fused_kernel_unmapped_page_reads_zeros(cuda, vfmt):
    """Fused kernel, paged ASTC V: an out-of-range block-table entry sets the
    status and that page's tokens read as zero K and V; the sequence's other
    pages, with a partial last chunk, are unaffected."""
    P = 96 if vfmt[0] == 6 else 64
    got, ref = _cfg_case(2, 32, 8, 128, 4 * P, kfmt=None, vfmt=vfmt, seed=17, page_tokens=P,
                         lens=[4 * P, 2 * P + 29], paged=True, bad=(1, 1))
    assert_attention_close(got, ref, f"unmapped page {vfmt}")


@pytest.mark.parametrize("T,split,lens", [(384, 6, None), (96, 12, [1]), (96, 48, [7]), (480, 24, [391]),
                                          (384, 96, [0]), (192, 18, [190])])
def test_ragged_lengths_and_splits(cuda, T, split, lens):
    """The reference's ragged cases: single token, partial block rows, T=391,
    an empty sequence (output 0), splits of one to many block rows."""
    got, ref = _cfg_case(1, 9, 3, 64, T, kfmt=None, vfmt=(6, "scalar", "token"), seed=T + split, page_tokens=96,
                         lens=lens, split=split)
    assert_attention_close(got, ref, f"T={T} split={split} lens={lens}")


def test_fp16_control_and_8x8_v(cuda):
    got, ref = _cfg_case(2, 32, 8, 128, 256, kfmt=None, vfmt=None, seed=5, page_tokens=64)
    assert_attention_close(got, ref, "fp16 control")
    got, ref = _cfg_case(2, 32, 8, 128, 256, kfmt=None, vfmt=(8, "scalar", "block_affine"), seed=6, page_tokens=64)
    assert_attention_close(got, ref, "8x8 V")


def test_bad_block_table_sets_status_without_fault(cuda):
    """An out-of-range block-table entry is reported in the status word and
    the page reads as zeros; the kernel neither faults nor hangs."""
    from astc_kv_cuda.ops import Attention, paged_fp16_plane
    rng = np.random.default_rng(8)
    pages = f16t(rng.standard_normal((4, 8, 256, 128)).astype(np.float16))
    k = paged_fp16_plane(pages)
    v = paged_fp16_plane(pages)
    q = torch.from_numpy(rng.standard_normal((1, 32, 128)).astype(np.float32)).cuda()
    table = torch.tensor([[0, 1, 99, 2]], dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = Attention(q, k, v, page_tokens=256, max_tokens=1024, block_table=table, num_pages=4, status=status).run()
    torch.cuda.synchronize()
    assert int(status.item()) == 5  # AKV_ERR_BAD_BLOCK_TABLE
    assert torch.isfinite(out).all()


def test_invalid_descriptors_return_status(cuda):
    from astc_kv_cuda import AkvError
    from astc_kv_cuda.ops import Attention, contiguous_fp16_plane
    x = f16t(np.zeros((1, 3, 96, 64), np.float16))
    k = contiguous_fp16_plane(x, 96)
    q = torch.zeros(1, 8, 64, device="cuda")  # 8 query heads do not divide by 3 kv heads
    with pytest.raises((AkvError, ValueError)):
        Attention(q, k, k, page_tokens=96, max_tokens=96)
    q = torch.zeros(1, 5 * 3, 64, device="cuda")  # group of 5: not compiled in
    with pytest.raises(AkvError) as e:
        Attention(q, k, k, page_tokens=96, max_tokens=96)
    assert e.value.code == 2


@pytest.mark.parametrize("block,D,G,layout,P", [(6, 128, 4, "scalar", 96), (4, 128, 4, "scalar", 64),
                                                 (8, 128, 8, "scalar", 64), (6, 64, 3, "scalar", 96),
                                                 (4, 64, 3, "rgba", 16), (4, 128, 4, "rgba", 64)])
@pytest.mark.parametrize("norm", ["block_affine", "token", "page_channel"])
def test_fused_kernel_on_every_block_mode(cuda, block, D, G, layout, P, norm):
    """V planes of random legal LDR blocks (every block mode, endpoint mode,
    partition count, dual plane, void extent) mixed with illegal encodings,
    through the fused kernel's table / direct / descriptor / generic paths
    (scalar and RGBA layouts; 16-token RGBA pages put four pages in a chunk),
    against the oracle decode + restore + float64 attention."""
    from astc_kv_cuda.ops import Attention, contiguous_astc_plane, contiguous_fp16_plane, random_blocks
    rng = np.random.default_rng(block * 100 + D + len(norm) + len(layout))
    B, Hkv = 2, 2
    Hq = Hkv * G
    T = 128 if P == 16 else 2 * P
    rows, cols = T // block, (D // (4 * block) if layout == "rgba" else -(-D // block))
    n = B * Hkv * rows * cols
    blk = random_blocks(n, block, seed=7 + block)
    bad = rng.random(n) < 0.05  # sprinkle illegal byte patterns (error colour)
    blk[bad] = rng.integers(0, 256, (int(bad.sum()), 16), dtype=np.uint8)
    blocks = blk.reshape(B, Hkv, rows, cols, 16)
    meta_shape = {"block_affine": (B, Hkv, rows, cols), "token": (B, Hkv, T), "page_channel": (B, Hkv, T // P, D)}[norm]
    off = (rng.standard_normal(meta_shape) * 0.5).astype(np.float16)
    scl = (rng.random(meta_shape) * 3 + 0.25).astype(np.float16)
    vr = np.stack([oracle_restore(blocks[b], off[b], scl[b], norm, block, layout, D, P) for b in range(B)])
    k = (rng.standard_normal((B, Hkv, T, D)) * 0.7).astype(np.float16)
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    lens = [T, T - 7]
    vp = contiguous_astc_plane(torch.from_numpy(blocks).cuda(), f16t(off), f16t(scl), block=block, layout=layout,
                               normalization=norm, head_dim=D, page_tokens=P)
    attn = Attention(torch.from_numpy(q).cuda(), contiguous_fp16_plane(f16t(k), P), vp, page_tokens=P, max_tokens=T,
                     seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"))
    assert attn.plan()["kernel"] == "attn_fast_kernel"
    got = attn.run().cpu().numpy()
    ref = O.attention_f64(q, k.astype(np.float32), vr, lens)
    assert_attention_close(got, ref, f"every-mode {layout} {block}x{block} {norm} D{D} P{P}")


def test_rgba_pages_smaller_than_a_chunk_with_a_partial_last_chunk(cuda):
    """RGBA 4x4 V with 16-token pages puts several pages in one fused-kernel
    chunk, which copies whole chunks of pages. A capacity of 400 tokens (25
    pages) is not whole 64-token chunks, so the library must not take that
    path (its last chunk would copy past the plane); the result must still
    match the oracle. 384 tokens (whole chunks) keeps the fused kernel."""
    from astc_kv_cuda.ops import Attention, contiguous_astc_plane, contiguous_fp16_plane
    got, ref = _cfg_case(1, 9, 3, 64, 400, kfmt=None, vfmt=(4, "rgba", "page_channel"), seed=400, page_tokens=16)
    assert_attention_close(got, ref, "rgba T=400 P=16")
    for T, kernel in ((400, "attn_split_kernel"), (384, "attn_fast_kernel")):
        blocks = torch.zeros(1, 3, T // 4, 4, 16, dtype=torch.uint8, device="cuda")
        meta = torch.zeros(1, 3, T // 16, 64, dtype=torch.float16, device="cuda")
        vp = contiguous_astc_plane(blocks, meta, meta, block=4, layout="rgba", normalization="page_channel",
                                   head_dim=64, page_tokens=16)
        kp = contiguous_fp16_plane(torch.zeros(1, 3, T, 64, dtype=torch.float16, device="cuda"), 16)
        q = torch.zeros(1, 9, 64, device="cuda")
        assert Attention(q, kp, vp, page_tokens=16, max_tokens=T).plan()["kernel"] == kernel, T


@pytest.mark.parametrize("D,G,T,P,split,lens", [(128, 4, 1000, 96, 0, [1000, 999, 64, 1]), (64, 3, 384, 16, 48, [384, 7]),
                                                  (128, 8, 512, 64, 200, [512, 130])])
def test_fp16_control_kernel(cuda, D, G, T, P, split, lens):
    """FP16 K + FP16 V takes the tensor-core FP16 kernel (per-row bulk copies,
    chunks that cross pages, ragged and partial last chunks, splits that are
    not whole chunks) and matches float64 attention."""
    from astc_kv_cuda.ops import Attention, contiguous_fp16_plane
    rng = np.random.default_rng(D + G + T)
    Hkv, B = 2, len(lens)
    k = (rng.standard_normal((B, Hkv, T, D)) * 0.8).astype(np.float16)
    v = (rng.standard_normal((B, Hkv, T, D)) * 2.0).astype(np.float16)
    q = rng.standard_normal((B, Hkv * G, D)).astype(np.float32)
    Tc = -(-T // P) * P
    kp = np.zeros((B, Hkv, Tc, D), np.float16)
    vp = np.zeros_like(kp)
    kp[:, :, :T], vp[:, :, :T] = k, v
    attn = Attention(torch.from_numpy(q).cuda(), contiguous_fp16_plane(f16t(kp), P), contiguous_fp16_plane(f16t(vp), P),
                     page_tokens=P, max_tokens=T, seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"),
                     split_tokens=split)
    assert attn.plan()["kernel"] == "attn_fp16_kernel"
    got = attn.run().cpu().numpy()
    ref = O.attention_f64(q, k.astype(np.float32), v.astype(np.float32), lens)
    assert_attention_close(got, ref, f"fp16 control D{D} G{G} T{T}")
