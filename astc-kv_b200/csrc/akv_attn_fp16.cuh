// Split-K decode attention over an FP16 K / FP16 V cache on sm_100a: the FP16
// control that the ASTC kernels are measured against (the reference's own
// FP16 kernel, metal/probe_gqa_v10.mm:669, gqaFP16Pipeline).
//
// Per CTA: one (split, kv head, batch) unit, processed in chunks of CH = 64
// tokens, one warp per 16-token tile.
//
//   * Staging: every thread issues 16-byte asynchronous copies (cp.async,
//     zero-fill form) of K and V rows into padded shared-memory rows (D + 8
//     halves, so ldmatrix rows fall on distinct banks), one chunk ahead in a
//     two-stage ring (commit / wait groups), three CTAs per SM (measured on
//     config 2's shape: 0.85 ms, against 1.11 ms with three stages and two
//     CTAs per SM and 1.25 ms with 32-token chunks in four stages). Rows past the split's last
//     token and rows of unmapped pages copy zero bytes, i.e. read as zeros.
//     A row's page is looked up per row, so chunks may cross pages. (One 1D
//     bulk copy per 256-byte row was measured first: the copy engine then
//     sustains about 1.8 TB/s, a quarter of HBM, for lack of bytes per
//     request.)
//   * Tensor cores (mma.sync m16n8k16, fp32 accumulation): S^T = K . Q^T
//     with q split into fp16 hi + lo (K is exact in fp16), online softmax in
//     base 2, O^T += V^T . P^T with P split into hi + lo (V is exact), so
//     the only rounding left is fp32 accumulation.
//   * The warps merge their (m, l, O) at the end into one split partial, the
//     workspace format merge_kernel reads, summing in a fixed order (the
//     result does not depend on warp timing).
#pragma once
#include "akv_attn_fast.cuh"

namespace akv {
namespace f16k {

using fast::cp_async16;
using fast::cp_async_commit;
using fast::cp_async_wait;
using fast::ldsm_x4;
using fast::ldsm_x4_t;
using fast::mma16816;
using fast::split_pair;

template <int D, int G>
struct Cfg {
    static constexpr int CH = 64;            // tokens per chunk
    static constexpr int NW = CH / 16;       // warps: one 16-token tile each
    static constexpr int THREADS = 32 * NW;
    static constexpr int STAGES = 2;
    static constexpr int LD = D + 8;         // halves per staged row
    static constexpr int KS = D / 16;        // k-steps of the score MMA, dim tiles of the output
    static constexpr int PPR = D / 8;        // 16-byte pieces per row
    static constexpr int PPT = CH * PPR / THREADS;  // pieces per thread per plane and chunk
    static_assert(D % 16 == 0 && G <= 8 && (CH * PPR) % THREADS == 0 && THREADS % PPR == 0, "shape");
};

template <int D, int G>
struct Smem {
    using C = Cfg<D, G>;
    __align__(16) __half k[C::STAGES][C::CH][C::LD];
    __align__(16) __half v[C::STAGES][C::CH][C::LD];
    __align__(16) uint4 qfrag[C::KS][32];     // per lane: q hi (2 words) | q lo (2 words)
    __align__(16) __half pbuf[C::NW][2][8][16];  // per warp: P hi, P lo as [head][token]
    float wm[C::NW][8];
    float wl[C::NW][8];
};

template <int D, int G>
__global__ void __launch_bounds__(Cfg<D, G>::THREADS, 3) attn_fp16_kernel(AttnParams p) {
    using C = Cfg<D, G>;
    using S = Smem<D, G>;
    constexpr int CH = C::CH, NW = C::NW, THREADS = C::THREADS, STAGES = C::STAGES, KS = C::KS;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    S& sm = *reinterpret_cast<S*>(smem_raw);

    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int len = seq_len_of(p, b);
    const int t_begin = split * p.split_tokens;
    const int t_end = min(t_begin + p.split_tokens, len);
    const int64_t unit0 = (static_cast<int64_t>(b) * p.Hq + h * G) * p.split_stride + p.split_base + split;
    auto write_empty = [&]() {
        for (int i = tid; i < G * D; i += THREADS)
            p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.split_stride) * D + i % D] = 0.f;
        if (tid < G) {
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 0] = -CUDART_INF_F;
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 1] = 0.f;
        }
    };
    if (t_begin >= t_end) {
        write_empty();
        return;
    }
    const int nchunks = (t_end - t_begin + CH - 1) / CH;
    const int P = p.page_tokens;

    // Chunk c -> stage s: thread i copies pieces i, i + THREADS, ... of each
    // plane (row = piece / PPR, so THREADS / PPR threads share a row).
    const uint8_t* kbase = p.k.data + b * p.k.sB + h * p.k.sH;
    const uint8_t* vbase = p.v.data + b * p.v.sB + h * p.v.sH;
    auto issue = [&](int c, int s) {
        const int t0 = t_begin + c * CH;
#pragma unroll
        for (int i = 0; i < C::PPT; ++i) {
            const int piece = tid + i * THREADS;
            const int r = piece / C::PPR, j = piece % C::PPR;
            const int t = t0 + r;
            const int phys = t < t_end ? phys_page(p.table, p.pps, p.num_pages, b, t / P, p.status) : -1;
            const int64_t row = static_cast<int64_t>(t % P) * (D * 2) + j * 16;
            const uint8_t* ks = phys >= 0 ? kbase + static_cast<int64_t>(phys) * p.k.sP + row : kbase;
            const uint8_t* vs = phys >= 0 ? vbase + static_cast<int64_t>(phys) * p.v.sP + row : vbase;
            const uint32_t n = phys >= 0 ? 16u : 0u;
            cp_async16(&sm.k[s][r][8 * j], ks, n);
            cp_async16(&sm.v[s][r][8 * j], vs, n);
        }
    };
#pragma unroll
    for (int c = 0; c < STAGES - 1; ++c) {
        if (c < nchunks) issue(c, c);
        cp_async_commit();
    }

    // Query fragments (B operand of the score MMA, hi + lo) for heads
    // n = lane / 4 of the group, computed once by the last warp.
    const int qn = lane >> 2, qj = lane & 3;
    if (warp == NW - 1) {
        const bool has = qn < G;
        const int64_t qb = (static_cast<int64_t>(b) * p.Hq + h * G + (has ? qn : 0)) * D;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int d0 = 16 * ks + 2 * qj, d1 = d0 + 8;
            const float q0 = has ? load_q(p.q, p.q_dtype, qb + d0) : 0.f;
            const float q1 = has ? load_q(p.q, p.q_dtype, qb + d0 + 1) : 0.f;
            const float q2 = has ? load_q(p.q, p.q_dtype, qb + d1) : 0.f;
            const float q3 = has ? load_q(p.q, p.q_dtype, qb + d1 + 1) : 0.f;
            uint4 f;
            split_pair(q0, q1, f.x, f.z);
            split_pair(q2, q3, f.y, f.w);
            sm.qfrag[ks][lane] = f;
        }
    }
    __syncthreads();

    float o[KS][4];
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F}, l_run[2] = {0.f, 0.f};
    const int mi = lane >> 3, rr = lane & 7;

    for (int c = 0; c < nchunks; ++c) {
        const int s = c % STAGES;
        const int t0 = t_begin + c * CH;
        const int n = min(CH, t_end - t0);
        // This thread's copies of chunk c have landed; the barrier makes
        // everyone's visible and frees the stage chunk c - 1 used, which
        // then takes chunk c + STAGES - 1.
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        if (c + STAGES - 1 < nchunks) issue(c + STAGES - 1, (c + STAGES - 1) % STAGES);
        cp_async_commit();
        // S^T[token][head] for this warp's 16 tokens.
        float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        {
            const int row = 16 * warp + rr + ((mi & 1) ? 8 : 0);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const uint4 qf = sm.qfrag[ks][lane];
                uint32_t a[4];
                ldsm_x4(a, &sm.k[s][row][16 * ks + ((mi & 2) ? 8 : 0)]);
                mma16816(sa[ks & 1], a[0], a[1], a[2], a[3], qf.x, qf.y);
                mma16816(sa[ks & 1], a[0], a[1], a[2], a[3], qf.z, qf.w);
            }
        }
        const bool v0 = 16 * warp + qn < n, v1 = 16 * warp + qn + 8 < n;
        float sv[4];
        sv[0] = v0 ? (sa[0][0] + sa[1][0]) * p.qscale : -CUDART_INF_F;
        sv[1] = v0 ? (sa[0][1] + sa[1][1]) * p.qscale : -CUDART_INF_F;
        sv[2] = v1 ? (sa[0][2] + sa[1][2]) * p.qscale : -CUDART_INF_F;
        sv[3] = v1 ? (sa[0][3] + sa[1][3]) * p.qscale : -CUDART_INF_F;
        float alpha[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float mx = fmaxf(sv[j], sv[j + 2]);
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
            const float mn = fmaxf(m_run[j], mx);
            const bool none = mn == -CUDART_INF_F;
            alpha[j] = none ? 1.f : exp2f(m_run[j] - mn);
            const float p0 = none ? 0.f : exp2f(sv[j] - mn);
            const float p1 = none ? 0.f : exp2f(sv[j + 2] - mn);
            sv[j] = p0;
            sv[j + 2] = p1;
            float sum = p0 + p1;
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 8);
            sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 16);
            l_run[j] = l_run[j] * alpha[j] + sum;
            m_run[j] = mn;
        }
#pragma unroll
        for (int i = 0; i < KS; ++i) {
            o[i][0] *= alpha[0];
            o[i][1] *= alpha[1];
            o[i][2] *= alpha[0];
            o[i][3] *= alpha[1];
        }
        // P^T -> per-warp buffers as P[head][token], split into fp16 hi + lo.
        {
            __half(*ph)[16] = sm.pbuf[warp][0];
            __half(*pl)[16] = sm.pbuf[warp][1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int head = 2 * qj + (j & 1), tok = qn + ((j & 2) ? 8 : 0);
                const __half hi = __float2half_rn(sv[j]);
                ph[head][tok] = hi;
                pl[head][tok] = __float2half_rn(sv[j] - __half2float(hi));
            }
        }
        __syncwarp();
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&sm.pbuf[warp][0][qn][2 * qj]);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&sm.pbuf[warp][0][qn][2 * qj + 8]);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&sm.pbuf[warp][1][qn][2 * qj]);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&sm.pbuf[warp][1][qn][2 * qj + 8]);
        // O^T[dim][head] += V^T . P^T over every dim tile.
        {
            const int vrow = 16 * warp + rr + ((mi & 2) ? 8 : 0);
            const int vcol = (mi & 1) ? 8 : 0;
#pragma unroll
            for (int dt = 0; dt < KS; ++dt) {
                uint32_t a[4];
                ldsm_x4_t(a, &sm.v[s][vrow][16 * dt + vcol]);
                mma16816(o[dt], a[0], a[1], a[2], a[3], bh0, bh1);
                mma16816(o[dt], a[0], a[1], a[2], a[3], bl0, bl1);
            }
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    __syncthreads();  // every stage and P buffer is free

    // Merge the warps' (m, l, O) into one split partial: each warp stores its
    // rescaled O, then the per-warp values are summed in warp order.
    float* red = reinterpret_cast<float*>(&sm.k[0][0][0]);  // [NW][G][D] floats
    static_assert(sizeof(float) * NW * G * D <= sizeof(sm.k), "merge buffer fits the K stages");
    if (lane < 4) {
        sm.wm[warp][2 * lane] = m_run[0];
        sm.wm[warp][2 * lane + 1] = m_run[1];
        sm.wl[warp][2 * lane] = l_run[0];
        sm.wl[warp][2 * lane + 1] = l_run[1];
    }
    __syncthreads();
    {
        float scl[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int hh = 2 * qj + j;
            float M = -CUDART_INF_F;
#pragma unroll
            for (int w = 0; w < NW; ++w) M = fmaxf(M, sm.wm[w][hh]);
            scl[j] = (M == -CUDART_INF_F || m_run[j] == -CUDART_INF_F) ? 0.f : exp2f(m_run[j] - M);
        }
        float* mine = red + warp * G * D;
#pragma unroll
        for (int dt = 0; dt < KS; ++dt) {
            const int d0 = 16 * dt + qn;
            if (2 * qj < G) {
                mine[(2 * qj) * D + d0] = o[dt][0] * scl[0];
                mine[(2 * qj) * D + d0 + 8] = o[dt][2] * scl[0];
            }
            if (2 * qj + 1 < G) {
                mine[(2 * qj + 1) * D + d0] = o[dt][1] * scl[1];
                mine[(2 * qj + 1) * D + d0 + 8] = o[dt][3] * scl[1];
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += THREADS) {
        float acc = red[i];
#pragma unroll
        for (int w = 1; w < NW; ++w) acc += red[w * G * D + i];
        p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.split_stride) * D + i % D] = acc;
    }
    if (tid < G) {
        float M = -CUDART_INF_F;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm.wm[w][tid]);
        float L = 0.f;
        if (M != -CUDART_INF_F)
            for (int w = 0; w < NW; ++w)
                if (sm.wm[w][tid] != -CUDART_INF_F) L += exp2f(sm.wm[w][tid] - M) * sm.wl[w][tid];
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 0] = M;
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 1] = L;
    }
}

}  // namespace f16k
}  // namespace akv
