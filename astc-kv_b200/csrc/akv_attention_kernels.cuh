// Fused ASTC-decode + split-K GQA decode attention (flash-decoding) and the
// log-sum-exp merge.
//
// One CTA owns one (split, kv head, batch) unit: every query head of the GQA
// group reads the same decoded K/V tile, so each texel is decoded once per
// group (the q-group tile the reference's v10 kernel introduced,
// metal/attention_gqa_v10.metal:568-674). Per chunk of CH tokens:
//   1. V (and ASTC K) blocks -> restored fp32 tile in shared memory
//      (stage A/B decoder, akv_common.cuh);
//   2. scores s[t][g] = (q[g] . k[t]) * scale * log2(e): lanes split the head
//      dimension and reduce with warp shuffles;
//   3. online softmax update of (m, l) per query head;
//   4. acc[g][c] = acc*alpha + sum_t p[t][g] * v[t][c].
// Partials (acc, m, l) go to the workspace; `merge_kernel` combines splits:
// out = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s.
#pragma once
#include <math_constants.h>

#include "akv_common.cuh"

namespace akv {

constexpr int kAttnThreads = 256;

struct AttnParams {
    int B, Hq, Hkv, T, page_tokens, split_tokens, nsplits;
    // Partials of split s of (b, query head hq) sit at row
    // (b * Hq + hq) * split_stride + split_base + s of the workspace; the
    // merge reads `split_stride` rows when merge_all is set (several KV
    // segments share one workspace), else the rows the sequence length uses.
    int split_base, split_stride, merge_all;
    int q_dtype;
    const void* q;
    const int32_t* seq_lens;
    const int32_t* table;
    int pps, num_pages;
    PlaneDev k, v;
    float qscale;  // softmax scale * log2(e)
    float* part_acc;
    float* part_ml;
    float* out;
    int32_t* status;
};

__device__ __forceinline__ float load_q(const void* q, int dtype, int64_t i) {
    if (dtype == AKV_Q_F32) return static_cast<const float*>(q)[i];
    if (dtype == AKV_Q_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(q)[i]);
    return __half2float(static_cast<const __half*>(q)[i]);
}

__device__ __forceinline__ int seq_len_of(const AttnParams& p, int b) {
    int len = p.seq_lens ? __ldg(p.seq_lens + b) : p.T;
    return len < 0 ? 0 : (len > p.T ? p.T : len);
}

template <int D, int G, int KBS, int VBS, int VL>
struct AttnCfg {
    static constexpr int CH = VBS ? 8 * VBS : (KBS ? 8 * KBS : 64);
    static_assert(CH % (KBS ? KBS : 1) == 0, "chunk must align to K blocks");
    static constexpr int CP = D / 2;
    static constexpr int TG = kAttnThreads / CP;
    static constexpr int LPT = D / 8;          // lanes per token row in the score loop
    static constexpr int TPI = 32 / LPT;       // tokens per warp iteration
    using VScr = TileScratch<VBS ? VBS : 4, VL>;
    using KScr = TileScratch<KBS ? KBS : 4, AKV_LAYOUT_SCALAR>;
    static constexpr size_t kScr = (VBS ? sizeof(VScr) : 0) > (KBS ? sizeof(KScr) : 0) ? (VBS ? sizeof(VScr) : 0)
                                                                                           : (KBS ? sizeof(KScr) : 0);
    static constexpr size_t kFloats = G * D /*q*/ + CH * D /*v*/ + (KBS ? CH * D : 0) /*k*/ + CH * G /*p*/ + 4 * G;
    static constexpr size_t kSmem = ((kScr + 15) / 16) * 16 + kFloats * sizeof(float);
};

template <int D, int G, int KBS, int VBS, int VL>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(AttnParams p) {
    using Cfg = AttnCfg<D, G, KBS, VBS, VL>;
    constexpr int CH = Cfg::CH, CP = Cfg::CP, TG = Cfg::TG, LPT = Cfg::LPT, TPI = Cfg::TPI;
    extern __shared__ __align__(16) uint8_t smem[];
    float* fl = reinterpret_cast<float*>(smem + ((Cfg::kScr + 15) / 16) * 16);
    float* q_s = fl;
    float* v_s = q_s + G * D;
    float* k_s = v_s + CH * D;
    float* s_s = k_s + (KBS ? CH * D : 0);
    float* m_s = s_s + CH * G;
    float* l_s = m_s + G;
    float* a_s = l_s + G;

    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int len = seq_len_of(p, b);
    const int t_begin = split * p.split_tokens;
    const int t_end = min(t_begin + p.split_tokens, len);
    const int64_t unit0 = (static_cast<int64_t>(b) * p.Hq + h * G) * p.split_stride + p.split_base + split;  // + g * split_stride

    if (t_begin >= t_end) {
        for (int i = tid; i < G * D; i += kAttnThreads)
            p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.split_stride) * D + i % D] = 0.f;
        if (tid < G) {
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 0] = -CUDART_INF_F;
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 1] = 0.f;
        }
        return;
    }

    for (int i = tid; i < G * D; i += kAttnThreads)
        q_s[i] = load_q(p.q, p.q_dtype, (static_cast<int64_t>(b) * p.Hq + h * G) * D + i) * p.qscale;
    if (tid < G) { m_s[tid] = -CUDART_INF_F; l_s[tid] = 0.f; }
    __syncthreads();

    const SeqCtx sq{b, h, p.table, p.pps, p.num_pages, p.page_tokens, p.status};
    auto& vscr = *reinterpret_cast<typename Cfg::VScr*>(smem);
    auto& kscr = *reinterpret_cast<typename Cfg::KScr*>(smem);

    // Per-lane query slice for the score loop.
    const int li = lane % LPT, sub = lane / LPT;
    float qreg[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) qreg[g][j] = q_s[g * D + li * 8 + j];

    const int cp = tid % CP, tg = tid / CP;
    float acc[G][2];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = 0.f;

    for (int t0 = t_begin; t0 < t_end; t0 += CH) {
        const int n = min(CH, t_end - t0);
        // 1. V tile.
        if constexpr (VBS > 0) {
            decode_tile<(VBS ? VBS : 4), VL, false>(p.v, sq, D, t0, n, t_end, v_s, D, vscr);
        } else {
            for (int i = tid; i < n * (D / 8); i += kAttnThreads) {
                const int r = i / (D / 8), c8 = i % (D / 8);
                const int t = t0 + r;
                const int phys = phys_page(p.table, p.pps, p.num_pages, b, t / p.page_tokens, p.status);
                float* dst = v_s + r * D + c8 * 8;
                if (phys < 0) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) dst[j] = 0.f;
                    continue;
                }
                const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p.v.data + b * p.v.sB + h * p.v.sH +
                                                                      static_cast<int64_t>(phys) * p.v.sP +
                                                                      static_cast<int64_t>(t % p.page_tokens) * D * 2) + c8);
                const __half2* hv = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(hv[j]);
                    dst[2 * j] = f.x;
                    dst[2 * j + 1] = f.y;
                }
            }
        }
        // ASTC K tile.
        if constexpr (KBS > 0) {
            decode_tile<(KBS ? KBS : 4), AKV_LAYOUT_SCALAR, false>(p.k, sq, D, t0, n, t_end, k_s, D, kscr);
            apply_side(p.k, sq, D, t0, n, t_end, k_s, D);
        }
        // 2. Scores.
        for (int base = warp * TPI; base < CH; base += (kAttnThreads / 32) * TPI) {
            const int t = base + sub;
            float part[G];
#pragma unroll
            for (int g = 0; g < G; ++g) part[g] = 0.f;
            if (t < n) {
                float kv[8];
                if constexpr (KBS > 0) {
                    const float4 a = *reinterpret_cast<const float4*>(k_s + t * D + li * 8);
                    const float4 c = *reinterpret_cast<const float4*>(k_s + t * D + li * 8 + 4);
                    kv[0] = a.x; kv[1] = a.y; kv[2] = a.z; kv[3] = a.w; kv[4] = c.x; kv[5] = c.y; kv[6] = c.z; kv[7] = c.w;
                } else {
                    const int tt = t0 + t;
                    const int phys = phys_page(p.table, p.pps, p.num_pages, b, tt / p.page_tokens, p.status);
                    if (phys >= 0) {
                        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p.k.data + b * p.k.sB + h * p.k.sH +
                                                                              static_cast<int64_t>(phys) * p.k.sP +
                                                                              static_cast<int64_t>(tt % p.page_tokens) * D * 2) + li);
                        const __half2* hv = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 f = __half22float2(hv[j]);
                            kv[2 * j] = f.x;
                            kv[2 * j + 1] = f.y;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j) kv[j] = 0.f;
                    }
                }
#pragma unroll
                for (int g = 0; g < G; ++g)
#pragma unroll
                    for (int j = 0; j < 8; ++j) part[g] = fmaf(qreg[g][j], kv[j], part[g]);
            }
#pragma unroll
            for (int off = LPT / 2; off > 0; off >>= 1)
#pragma unroll
                for (int g = 0; g < G; ++g) part[g] += __shfl_xor_sync(0xFFFFFFFFu, part[g], off);
            if (li == 0 && t < CH) {
#pragma unroll
                for (int g = 0; g < G; ++g) s_s[t * G + g] = (t < n) ? part[g] : -CUDART_INF_F;
            }
        }
        __syncthreads();
        // 3. Online softmax per query head (one warp per head).
        for (int g = warp; g < G; g += kAttnThreads / 32) {
            float mx = -CUDART_INF_F;
            for (int t = lane; t < n; t += 32) mx = fmaxf(mx, s_s[t * G + g]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
            const float m_old = m_s[g];
            const float m_new = fmaxf(m_old, mx);
            const float alpha = exp2f(m_old - m_new);
            float sum = 0.f;
            for (int t = lane; t < CH; t += 32) {
                const float e = (t < n) ? exp2f(s_s[t * G + g] - m_new) : 0.f;
                s_s[t * G + g] = e;
                sum += e;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, off);
            if (lane == 0) {
                l_s[g] = l_s[g] * alpha + sum;
                m_s[g] = m_new;
                a_s[g] = alpha;
            }
        }
        __syncthreads();
        // 4. P.V accumulate.
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float al = a_s[g];
            acc[g][0] *= al;
            acc[g][1] *= al;
        }
        for (int t = tg; t < n; t += TG) {
            const float2 v2 = *reinterpret_cast<const float2*>(v_s + t * D + 2 * cp);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pr = s_s[t * G + g];
                acc[g][0] = fmaf(pr, v2.x, acc[g][0]);
                acc[g][1] = fmaf(pr, v2.y, acc[g][1]);
            }
        }
        __syncthreads();
    }

    // Reduce the TG token groups (v_s is free now: CH*D >= TG*G*D floats is
    // checked on the host).
    float* red = v_s;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        red[(tg * G + g) * D + 2 * cp] = acc[g][0];
        red[(tg * G + g) * D + 2 * cp + 1] = acc[g][1];
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kAttnThreads) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < TG; ++k) s += red[k * G * D + i];
        p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.split_stride) * D + i % D] = s;
    }
    if (tid < G) {
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 0] = m_s[tid];
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 1] = l_s[tid];
    }
}

constexpr int kMergeThreads = 512;
// Split weights the merge keeps in dynamic shared memory (44 KB, inside the
// 48 KB a launch gets without opting in); beyond that it recomputes them per
// dimension.
constexpr int kMergeSmemSplits = 11 * 1024;

// Block-wide max / sum of one value per thread, in a fixed order (the result
// does not depend on thread timing). `red` holds 32 floats.
__device__ __forceinline__ float block_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < nw; ++w) r = fmaxf(r, red[w]);
    return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < nw; ++w) r += red[w];
    return r;
}

// Combines the split partials of one (query head, sequence):
// out = sum_s w_s acc_s / sum_s w_s l_s with w_s = 2^(m_s - max_s m_s); empty
// splits (m = -inf) weigh 0, also when every split is empty, so nothing to
// attend gives zeros. The weights are computed once per split (into shared
// memory when wcap covers the splits); each dimension's sum is split into
// blockDim / D phases over the splits, each phase loading eight splits at a
// time (the merge is bound by load latency, not bandwidth), added in a
// fixed order.
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(AttnParams p, int D, int wcap) {
    extern __shared__ float wsm[];  // [wcap] split weights
    __shared__ float red[32];
    __shared__ float part[kMergeThreads];
    const int hq = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int len = seq_len_of(p, b);
    const int ns = p.merge_all ? p.split_stride : min(p.nsplits, (len + p.split_tokens - 1) / p.split_tokens);
    const int64_t unit0 = (static_cast<int64_t>(b) * p.Hq + hq) * p.split_stride;
    const float* ml = p.part_ml + unit0 * 2;
    float m = -CUDART_INF_F;
    for (int s = tid; s < ns; s += blockDim.x) m = fmaxf(m, ml[2 * s]);
    const float M = block_max(m, red);
    auto weight = [&](int s) {
        const float ms = ml[2 * s];
        return ms == -CUDART_INF_F ? 0.f : exp2f(ms - M);
    };
    float dpart = 0.f;
    for (int s = tid; s < ns; s += blockDim.x) {
        const float w = weight(s);
        if (s < wcap) wsm[s] = w;
        dpart += w * ml[2 * s + 1];
    }
    const float den = block_sum(dpart, red);  // its barriers also publish wsm
    const float inv = (ns > 0 && den > 0.f) ? 1.f / den : 0.f;
    const float* acc = p.part_acc + unit0 * D;
    float* out = p.out + (static_cast<int64_t>(b) * p.Hq + hq) * D;
    if (D <= static_cast<int>(blockDim.x)) {
        const int nph = blockDim.x / D, c = tid % D, ph = tid / D;
        float num = 0.f;
        if (ph < nph) {
            auto w = [&](int sp) { return sp < wcap ? wsm[sp] : weight(sp); };
            float n[4] = {0.f, 0.f, 0.f, 0.f};
            int sp = ph;
            for (; sp + 7 * nph < ns; sp += 8 * nph) {
                float a[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) a[k] = acc[static_cast<int64_t>(sp + k * nph) * D + c];
#pragma unroll
                for (int k = 0; k < 8; ++k) n[k & 3] += w(sp + k * nph) * a[k];
            }
            for (; sp < ns; sp += nph) n[0] += w(sp) * acc[static_cast<int64_t>(sp) * D + c];
            num = (n[0] + n[1]) + (n[2] + n[3]);
        }
        part[tid] = num;
        __syncthreads();
        if (tid < D) {
            float t = part[tid];
            for (int q = 1; q < nph; ++q) t += part[q * D + tid];
            out[tid] = t * inv;
        }
    } else {
        for (int c = tid; c < D; c += blockDim.x) {
            float num = 0.f;
            for (int s = 0; s < ns; ++s) num += (s < wcap ? wsm[s] : weight(s)) * acc[static_cast<int64_t>(s) * D + c];
            out[c] = num * inv;
        }
    }
}

// Launches merge_kernel for every (query head, sequence) of p.
inline void launch_merge(const AttnParams& p, int D, cudaStream_t s) {
    const int ns = p.merge_all ? p.split_stride : p.nsplits;
    const int wcap = ns <= kMergeSmemSplits ? ns : 0;
    merge_kernel<<<dim3(p.Hq, p.B), kMergeThreads, static_cast<size_t>(wcap) * sizeof(float), s>>>(p, D, wcap);
}

}  // namespace akv
