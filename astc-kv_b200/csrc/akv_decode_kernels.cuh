// Standalone decode kernels: blocks -> texels, image decode (akv_decode
// contract), and whole-plane restore to fp32.
#pragma once
#include "akv_common.cuh"

namespace akv {

constexpr int kDecodeThreads = 256;
constexpr int kDecodeBlocksPerIter = 256;  // one header per thread: no warp idles in stage A

// Persistent grid-stride decode of consecutive blocks into
// out[block][y][x][rgba]. Stage A decodes 256 headers into shared memory
// (one per thread); stage B evaluates a texel row per task (texel_row), with
// consecutive threads on consecutive rows so the output stays contiguous
// across a warp: with VEC (out 16-byte aligned) each row leaves in 16-byte
// (8-byte for 6x6 UNORM8) vector stores, else in 32-bit words.
// Four CTAs per SM (registers capped at 64, no spills: the header decoder
// keeps its colour integers in the block's weight row and its endpoints in
// packed registers, so it needs no local memory); weight rows padded to 68
// bytes so the row tasks of different blocks in a warp read different banks.
// Before stage A the iteration's blocks are ordered by header class
// (partition count, endpoint-mode class, void extent: header_class), so a
// warp's lanes mostly decode blocks that take the same branches; each block
// still lands in its own descriptor slot, so the output does not depend on
// the order.
constexpr int kHeaderClasses = 17;
static_assert(kHeaderClasses <= 32, "one warp scans the class counts");

__device__ __forceinline__ int header_class(uint4 blk) {
    const uint32_t x = blk.x;
    if ((x & 0x1FF) == 0x1FC) return 16;  // void extent
    const int parts = static_cast<int>((x >> 11) & 3);  // partition count - 1
    int cls;                                            // endpoint mode >> 2 (of partition 0's class)
    if (parts == 0) {
        cls = static_cast<int>((x >> 15) & 3);
    } else {
        const int field = static_cast<int>((x >> 23) & 63);
        cls = (field & 3) ? (field & 3) - 1 : field >> 4;
    }
    return (parts << 2) | cls;
}

template <int BS, int MODE, bool VEC>
__global__ void __launch_bounds__(kDecodeThreads, 4) decode_blocks_kernel(const uint4* __restrict__ blocks, int64_t n,
                                                                          void* __restrict__ out) {
    __shared__ BlockDesc<4> desc[kDecodeBlocksPerIter];
    __shared__ uint8_t wts[kDecodeBlocksPerIter][64 + kCodePad];
    __shared__ int cls_start[32];
    __shared__ uint8_t order[kDecodeBlocksPerIter];
    constexpr int fp = footprint_index(BS);
    constexpr int TPB = BS * BS;
    const int tid = threadIdx.x;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kDecodeBlocksPerIter; base < n;
         base += static_cast<int64_t>(gridDim.x) * kDecodeBlocksPerIter) {
        const int nb = static_cast<int>(min(static_cast<int64_t>(kDecodeBlocksPerIter), n - base));
        // Counting sort of the iteration's blocks by header class.
        const int key = tid < nb ? header_class(__ldg(blocks + base + tid)) : 0;
        if (tid < 32) cls_start[tid] = 0;
        __syncthreads();
        const int rank = tid < nb ? atomicAdd(&cls_start[key], 1) : 0;
        __syncthreads();
        if (tid < 32) {
            const int c = cls_start[tid];
            int incl = c;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int o = __shfl_up_sync(0xFFFFFFFFu, incl, d);
                if (tid >= d) incl += o;
            }
            cls_start[tid] = incl - c;
        }
        __syncthreads();
        if (tid < nb) order[cls_start[key] + rank] = static_cast<uint8_t>(tid);
        __syncthreads();
        if (tid < nb) {
            const int i = order[tid];
            decode_header<4>(__ldg(blocks + base + i), fp, desc[i], wts[i]);
        }
        __syncthreads();
        constexpr int WPT = MODE == AKV_OUT_UNORM8 ? 1 : 2;  // 32-bit output words per texel
        constexpr int NW = BS * WPT;                             // words per texel row
        for (int r = threadIdx.x; r < nb * BS; r += blockDim.x) {
            const int bi = r / BS, y = r - bi * BS;
            uint32_t c[BS][4];
            texel_row<BS, 4>(desc[bi], wts[bi], y, c);
            uint32_t pk[NW];
#pragma unroll
            for (int x = 0; x < BS; ++x) {
                if (MODE == AKV_OUT_UNORM8) {
                    pk[x] = (c[x][0] >> 8) | ((c[x][1] >> 8) << 8) | ((c[x][2] >> 8) << 16) | ((c[x][3] >> 8) << 24);
                } else if (MODE == AKV_OUT_FP16) {
                    pk[2 * x] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(c16_to_unit(c[x][0])))) |
                                (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(c16_to_unit(c[x][1])))) << 16);
                    pk[2 * x + 1] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(c16_to_unit(c[x][2])))) |
                                    (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(c16_to_unit(c[x][3])))) << 16);
                } else {
                    pk[2 * x] = c[x][0] | (c[x][1] << 16);
                    pk[2 * x + 1] = c[x][2] | (c[x][3] << 16);
                }
            }
            // First output word of the row: texel (base + bi) * TPB + y * BS.
            uint32_t* dst = reinterpret_cast<uint32_t*>(out) + ((base + bi) * TPB + y * BS) * WPT;
            if constexpr (VEC && NW % 4 == 0) {
#pragma unroll
                for (int k = 0; k < NW / 4; ++k)
                    reinterpret_cast<uint4*>(dst)[k] = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
            } else if constexpr (VEC) {
#pragma unroll
                for (int k = 0; k < NW / 2; ++k) reinterpret_cast<uint2*>(dst)[k] = make_uint2(pk[2 * k], pk[2 * k + 1]);
            } else {
#pragma unroll
                for (int k = 0; k < NW; ++k) dst[k] = pk[k];
            }
        }
        __syncthreads();
    }
}

// Image decode: float32 RGBA [h][w][4] (fp16 view of C), blocks row-major.
template <int BS>
__global__ void __launch_bounds__(kDecodeThreads) decode_image_kernel(const uint4* __restrict__ blocks, int cols, int rows,
                                                                      float* __restrict__ rgba, int w, int h) {
    __shared__ BlockDesc<4> desc[kDecodeBlocksPerIter];
    __shared__ uint8_t wts[kDecodeBlocksPerIter][64 + kCodePad];
    constexpr int fp = footprint_index(BS);
    constexpr int TPB = BS * BS;
    const int64_t n = static_cast<int64_t>(cols) * rows;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kDecodeBlocksPerIter; base < n;
         base += static_cast<int64_t>(gridDim.x) * kDecodeBlocksPerIter) {
        const int nb = static_cast<int>(min(static_cast<int64_t>(kDecodeBlocksPerIter), n - base));
        if (threadIdx.x < nb) decode_header<4>(__ldg(blocks + base + threadIdx.x), fp, desc[threadIdx.x], wts[threadIdx.x]);
        __syncthreads();
        for (int i = threadIdx.x; i < nb * TPB; i += blockDim.x) {
            const int bi = i / TPB, t = i % TPB;
            const int64_t blk = base + bi;
            const int px = static_cast<int>(blk % cols) * BS + t % BS;
            const int py = static_cast<int>(blk / cols) * BS + t / BS;
            if (px >= w || py >= h) continue;
            uint32_t c[4];
            texel_values<BS, 4>(desc[bi], wts[bi], t % BS, t / BS, c);
            reinterpret_cast<float4*>(rgba)[static_cast<int64_t>(py) * w + px] =
                make_float4(c16_to_unit(c[0]), c16_to_unit(c[1]), c16_to_unit(c[2]), c16_to_unit(c[3]));
        }
        __syncthreads();
    }
}

// Restore a plane to fp32 [B][H][T][D]. One CTA per (row chunk, h, b).
template <int BS, int LAYOUT>
__global__ void __launch_bounds__(kDecodeThreads) restore_plane_kernel(PlaneDev pl, int D, int T, int page_tokens,
                                                                       const int32_t* table, int pps, int num_pages,
                                                                       float* __restrict__ out, int32_t* status) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr int CH = 8 * BS;
    auto& scr = *reinterpret_cast<TileScratch<BS, LAYOUT>*>(smem);
    float* tile = reinterpret_cast<float*>(smem + sizeof(TileScratch<BS, LAYOUT>));
    const int h = blockIdx.y, b = blockIdx.z, H = gridDim.y;
    const int t0 = blockIdx.x * CH;
    const int rows = min(CH, T - t0);
    SeqCtx sq{b, h, table, pps, num_pages, page_tokens, status};
    decode_tile<BS, LAYOUT, true>(pl, sq, D, t0, rows, T, tile, D, scr);
    float* dst = out + ((static_cast<int64_t>(b) * H + h) * T + t0) * D;
    for (int i = threadIdx.x; i < rows * D; i += blockDim.x) dst[i] = tile[i];
}

// FP16 plane widened to fp32 [B][H][T][D].
__global__ void restore_fp16_kernel(PlaneDev pl, int D, int T, int page_tokens, const int32_t* table, int pps,
                                    int num_pages, float* __restrict__ out, int32_t* status) {
    const int h = blockIdx.y, b = blockIdx.z, H = gridDim.y;
    const int t = blockIdx.x;
    const int phys = phys_page(table, pps, num_pages, b, t / page_tokens, status);
    float* dst = out + ((static_cast<int64_t>(b) * H + h) * T + t) * D;
    if (phys < 0) {
        for (int c = threadIdx.x; c < D; c += blockDim.x) dst[c] = 0.f;
        return;
    }
    const __half* row = reinterpret_cast<const __half*>(pl.data + b * pl.sB + h * pl.sH + static_cast<int64_t>(phys) * pl.sP) +
                        static_cast<int64_t>(t % page_tokens) * D;
    for (int c = threadIdx.x; c < D; c += blockDim.x) dst[c] = __half2float(row[c]);
}

}  // namespace akv
