// Shared device-side plumbing: plane addressing, page lookup, tile decode.
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "../../include/akv_cuda.h"
#include "akv_astc_device.cuh"

namespace akv {

// Kernel-side copy of an AkvPlane.
struct PlaneDev {
    const uint8_t* data;
    int64_t sB, sH, sP;          // bytes
    const __half* off;
    const __half* scl;
    int64_t mB, mH, mP;          // elements
    const uint8_t* side;
    const int32_t* side_ch;
    int64_t xB, xH, xP;          // bytes
    int side_count;
    int norm;
};

inline PlaneDev to_dev(const AkvPlane& p) {
    PlaneDev d;
    d.data = static_cast<const uint8_t*>(p.data);
    d.sB = p.stride_batch; d.sH = p.stride_head; d.sP = p.stride_page;
    d.off = static_cast<const __half*>(p.offsets);
    d.scl = static_cast<const __half*>(p.scales);
    d.mB = p.meta_stride_batch; d.mH = p.meta_stride_head; d.mP = p.meta_stride_page;
    d.side = static_cast<const uint8_t*>(p.side);
    d.side_ch = p.side_channels_dev;
    d.xB = p.side_stride_batch; d.xH = p.side_stride_head; d.xP = p.side_stride_page;
    d.side_count = p.side ? p.side_count : 0;
    d.norm = p.normalization;
    return d;
}

// Logical page -> physical page, or -1 (and a status write) when the table
// entry is out of range.
__device__ __forceinline__ int phys_page(const int32_t* table, int pps, int num_pages, int b, int p, int32_t* status) {
    if (!table) return p;
    const int v = __ldg(table + static_cast<int64_t>(b) * pps + p);
    if (v < 0 || v >= num_pages) {
        if (status) atomicExch(status, AKV_ERR_BAD_BLOCK_TABLE);
        return -1;
    }
    return v;
}

// Per-(b, h) view used by the tile decoders.
struct SeqCtx {
    int b, h;
    const int32_t* table;
    int pps, num_pages, page_tokens;
    int32_t* status;
};

// Affine parameters (offset, scale) of texel (t, c) for TOKEN and
// PAGE_CHANNEL planes; BLOCK_AFFINE comes from the block descriptor.
__device__ __forceinline__ float2 affine_tc(const PlaneDev& pl, int64_t meta_base, int t_in_page, int c) {
    const int64_t i = meta_base + (pl.norm == AKV_NORM_TOKEN ? t_in_page : c);
    return make_float2(__half2float(pl.off[i]), __half2float(pl.scl[i]));
}

// Decode rows [t0, t0 + rows) of an ASTC scalar/rgba plane into an fp32 tile
// `tile[t - t0][c]` (row stride `ld`) holding restored values
// offset + scale * u. `restore_exact` selects unfused mul+add (bit-exact with
// the reference's NumPy restore). Rows must start at a multiple of BS.
// Requires blockDim.x threads to call it together; uses `desc`/`wts`/`aff`
// scratch for up to `kMaxBlocks` blocks per pass.
constexpr int kMaxBlocks = 256;

template <int BS, int LAYOUT>
struct TileScratch {
    static constexpr int NCH = LAYOUT == AKV_LAYOUT_RGBA ? 4 : 1;
    BlockDesc<NCH> desc[kMaxBlocks];
    uint8_t wts[kMaxBlocks][64 + kCodePad];
    float2 aff[kMaxBlocks];
};

template <int BS, int LAYOUT, bool EXACT>
__device__ __forceinline__ void decode_tile(const PlaneDev& pl, const SeqCtx& sq, int D, int t0, int rows, int t_limit,
                                            float* tile, int ld, TileScratch<BS, LAYOUT>& scr) {
    constexpr int NCH = TileScratch<BS, LAYOUT>::NCH;
    constexpr int fp = footprint_index(BS);
    const int comp = NCH;
    const int width = ((D / comp + BS - 1) / BS) * BS;
    const int cols = width / BS;
    const int brows = (rows + BS - 1) / BS;
    const int nblk = brows * cols;
    const int rows_per_page = sq.page_tokens / BS;
    for (int pass = 0; pass < nblk; pass += kMaxBlocks) {
        const int nb = min(kMaxBlocks, nblk - pass);
        // Stage A: one thread per block.
        for (int i = threadIdx.x; i < nb; i += blockDim.x) {
            const int bi = pass + i;
            const int br = bi / cols, bc = bi % cols;
            const int t = t0 + br * BS;
            const int page = t / sq.page_tokens;
            const int phys = (t < t_limit) ? phys_page(sq.table, sq.pps, sq.num_pages, sq.b, page, sq.status) : -2;
            if (phys < 0) {
                // Out-of-range page or rows past the sequence: decode as
                // zeros (never read as attention input; masked by the caller).
                scr.desc[i].info = 1u << kInfoVoid;
#pragma unroll
                for (int c = 0; c < NCH; ++c) scr.desc[i].ep[c] = 0;
                scr.aff[i] = make_float2(0.f, 0.f);
                continue;
            }
            const int row_in_page = (t % sq.page_tokens) / BS;
            const uint8_t* base = pl.data + sq.b * pl.sB + sq.h * pl.sH + static_cast<int64_t>(phys) * pl.sP;
            const uint4 blk = __ldg(reinterpret_cast<const uint4*>(base) + static_cast<int64_t>(row_in_page) * cols + bc);
            decode_header<NCH>(blk, fp, scr.desc[i], scr.wts[i]);
            if (pl.norm == AKV_NORM_BLOCK_AFFINE) {
                const int64_t mi = sq.b * pl.mB + sq.h * pl.mH + static_cast<int64_t>(phys) * pl.mP +
                                   static_cast<int64_t>(row_in_page) * cols + bc;
                scr.aff[i] = make_float2(__half2float(pl.off[mi]), __half2float(pl.scl[mi]));
            }
            (void)rows_per_page;
        }
        __syncthreads();
        // Stage B: one thread per texel (pixel for RGBA).
        const int ntex = nb * BS * BS;
        for (int i = threadIdx.x; i < ntex; i += blockDim.x) {
            // Texel order: block-major so consecutive threads share a block.
            const int li = i / (BS * BS), tx = i % (BS * BS);
            const int bi = pass + li;
            const int br = bi / cols, bc = bi % cols;
            const int x = tx % BS, y = tx / BS;
            const int t_rel = br * BS + y;
            const int px = bc * BS + x;  // pixel column
            if (t_rel >= rows) continue;
            const int t = t0 + t_rel;
            uint32_t cval[NCH];
            texel_values<BS, NCH>(scr.desc[li], scr.wts[li], x, y, cval);
            float2 af = scr.aff[li];
            int64_t meta_base = 0;
            const bool need_meta = pl.norm != AKV_NORM_BLOCK_AFFINE;
            if (need_meta && t < t_limit) {
                const int page = t / sq.page_tokens;
                const int phys = phys_page(sq.table, sq.pps, sq.num_pages, sq.b, page, nullptr);
                meta_base = phys < 0 ? -1 : sq.b * pl.mB + sq.h * pl.mH + static_cast<int64_t>(phys) * pl.mP;
            }
#pragma unroll
            for (int k = 0; k < NCH; ++k) {
                const int c = px * comp + k;
                if (c >= D) break;
                const float u = c16_to_unit(cval[k]);
                if (need_meta) {
                    af = (t < t_limit && meta_base >= 0) ? affine_tc(pl, meta_base, t % sq.page_tokens, c) : make_float2(0.f, 0.f);
                }
                float v;
                if (EXACT) v = __fadd_rn(__fmul_rn(u, af.y), af.x);
                else v = fmaf(u, af.y, af.x);
                tile[t_rel * ld + c] = v;
            }
        }
        __syncthreads();
    }
}

// Overwrite side-plane channels of a decoded K tile with their exact fp16
// values.
__device__ __forceinline__ void apply_side(const PlaneDev& pl, const SeqCtx& sq, int D, int t0, int rows, int t_limit,
                                           float* tile, int ld) {
    if (pl.side_count <= 0) return;
    const int n = rows * pl.side_count;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int r = i / pl.side_count, j = i % pl.side_count;
        const int t = t0 + r;
        if (t >= t_limit) continue;
        const int page = t / sq.page_tokens;
        const int phys = phys_page(sq.table, sq.pps, sq.num_pages, sq.b, page, nullptr);
        if (phys < 0) continue;
        const int c = __ldg(pl.side_ch + sq.h * pl.side_count + j);
        if (c < 0 || c >= D) continue;  // ids outside the head are ignored
        const __half* row = reinterpret_cast<const __half*>(pl.side + sq.b * pl.xB + sq.h * pl.xH +
                                                           static_cast<int64_t>(phys) * pl.xP) +
                            static_cast<int64_t>(t % sq.page_tokens) * pl.side_count;
        tile[r * ld + c] = __half2float(row[j]);
    }
    __syncthreads();
}

}  // namespace akv
