// Fast split-K decode attention for scalar-layout ASTC V (and FP16 or scalar
// ASTC K) on sm_100a.
//
// Per CTA: one (split, kv head, batch) unit, processed in chunks of CH tokens
// (CH = 48 for 6x6 footprints, 64 otherwise; a chunk never crosses a page).
//
//   * Staging: one elected thread issues cp.async.bulk copies of the chunk's
//     V blocks and fp16 metadata (and ASTC K blocks) into a two-stage shared
//     ring, completed on mbarriers; consumers wait with a bounded try_wait.
//   * Decode, stage A (thread per block): header, endpoints and weight codes.
//     For the common block kinds (single weight plane, full-resolution grid)
//     the block becomes a value table u[partition][weight code] (exact fp16
//     values of the decoded texels) plus one index byte per texel; other
//     blocks (reduced grids with infill, dual plane) store one table entry per
//     texel with identity indices, so stage B is uniform.
//   * Decode, stage B (thread per block row of texels): u = table[index],
//     v = scale*u + offset, split into fp16 hi + lo parts, written to padded
//     [token][channel] tiles.
//   * Tensor cores (mma.sync m16n8k16, fp32 accumulation), one warp per 16
//     tokens of the chunk, query heads of the GQA group as the N=8 dimension:
//       S^T[tok][head] = K . Q^T   (q hi+lo; K fp16 straight from global
//                                   memory in fragment order, or decoded
//                                   K hi+lo from shared memory)
//       online softmax per head in base 2, P^T as fp16 through a 256-byte
//       per-warp buffer,
//       O^T[dim][head] += V^T . P^T  (V hi and lo, ldmatrix.trans).
//   * Each MMA warp keeps its own (m, l, O) over its token slices; the warps
//     merge at the end and the CTA writes one split partial (m, l, acc), the
//     same workspace format the merge kernel reads.
#pragma once
#include <math_constants.h>

#include "akv_attention_kernels.cuh"
#include "akv_common.cuh"

namespace akv {
namespace fast {

// Iterations of mbarrier.try_wait before a wait is declared stuck. Each
// try_wait may itself block for a hardware-defined interval, so this bounds a
// wait at roughly seconds, far beyond any healthy copy.
constexpr uint32_t kWaitIters = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bounded wait on phase `parity`; false when the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < kWaitIters; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred P1;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, P1;\n\t}"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Global -> shared bulk copy (no multicast), completion on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// v -> (fp16 hi, fp16 lo) with hi + lo == v to ~2^-22 relative.
__device__ __forceinline__ void split_pair(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_h2(v0 - hf.x, v1 - hf.y);
}

// ------------------------------------------------------------------ decode

// Stage A of the fast path for one block (R channel of a scalar-layout
// plane). Writes `tab` (fp16 u values) and `idx` (per-texel table index).
template <int BS>
__device__ __forceinline__ void decode_block_table(uint4 blk, __half* tab, uint8_t* idx) {
    constexpr int fp = footprint_index(BS);
    constexpr int N = BS * BS;
    const Tables& T = g_akv_tables;
    const uint64_t lo = (static_cast<uint64_t>(blk.y) << 32) | blk.x;
    const uint64_t hi = (static_cast<uint64_t>(blk.w) << 32) | blk.z;
    const int mode = static_cast<int>(lo & 0x7FF);
    auto constant = [&](float u) {
        tab[0] = __float2half_rn(u);  // exact: u is an fp16 value
#pragma unroll
        for (int t = 0; t < N; t += 4) *reinterpret_cast<uint32_t*>(idx + t) = 0u;
    };
    const uint32_t me = __ldg(&T.mode[fp][mode]);
    const int parts = static_cast<int>((lo >> 11) & 3) + 1;
    const bool fast_kind = (me & kModeValid) && !(me & kModeDual) && !(me & kModeReduced);
    if (!fast_kind || (mode & 0x1FF) == 0x1FC) {
        // Void extent, error, reduced grid or dual plane: per-texel values.
        BlockDesc<1> d;
        uint8_t w[64];
        decode_header<1>(blk, fp, d, w);
        if (d.info & ((1u << kInfoVoid) | (1u << kInfoError))) {
            uint32_t c[1];
            texel_values<BS, 1>(d, w, 0, 0, c);
            constant(c16_to_unit(c[0]));
            return;
        }
#pragma unroll 1
        for (int t = 0; t < N; ++t) {
            uint32_t c[1];
            texel_values<BS, 1>(d, w, t % BS, t / BS, c);
            tab[t] = __float2half_rn(c16_to_unit(c[0]));
            idx[t] = static_cast<uint8_t>(t);
        }
        return;
    }
    const int wq = mode_wq(me), wbits = mode_wbits(me);
    const int top = 128 - wbits;
    int cem[4];
    int cstart, extra = 0, seed = 0;
    if (parts == 1) {
        cem[0] = static_cast<int>((lo >> 13) & 15);
        cstart = 17;
    } else {
        seed = static_cast<int>((lo >> 13) & 0x3FF);
        const int field = static_cast<int>((lo >> 23) & 0x3F);
        cstart = 29;
        if ((field & 3) == 0) {
#pragma unroll
            for (int p = 0; p < 4; ++p) cem[p] = field >> 2;
        } else {
            extra = 3 * parts - 4;
            const int all = (field >> 2) | (static_cast<int>(bits_u128(lo, hi, top - extra, extra)) << 4);
            const int cls = (field & 3) - 1;
#pragma unroll
            for (int p = 0; p < 4; ++p) cem[p] = ((cls + ((all >> p) & 1)) << 2) | ((all >> (parts + 2 * p)) & 3);
        }
    }
    int npairs = 0;
    for (int p = 0; p < parts; ++p) npairs += (cem[p] >> 2) + 1;
    const int avail = top - extra - cstart;
    const int cq = (npairs <= 9 && avail >= 0) ? T.cquant[npairs][avail] : 0xFF;
    const uint32_t wshape = __ldg(&T.shape[wq]);
    const int levels = (1 << (wshape & 15)) * ((wshape >> 4) & 1 ? 3 : ((wshape >> 5) & 1 ? 5 : 1));
    if (cq == 0xFF || parts * levels > N) {
        // Illegal colour budget, or a table larger than the block: per texel.
        BlockDesc<1> d;
        uint8_t w[64];
        decode_header<1>(blk, fp, d, w);
        if (d.info & ((1u << kInfoVoid) | (1u << kInfoError))) {
            uint32_t c[1];
            texel_values<BS, 1>(d, w, 0, 0, c);
            constant(c16_to_unit(c[0]));
            return;
        }
#pragma unroll 1
        for (int t = 0; t < N; ++t) {
            uint32_t c[1];
            texel_values<BS, 1>(d, w, t % BS, t / BS, c);
            tab[t] = __float2half_rn(c16_to_unit(c[0]));
            idx[t] = static_cast<uint8_t>(t);
        }
        return;
    }
    // Colour integers -> R endpoints per partition.
    int vals[18];
    {
        uint64_t clo = window_u128(lo, hi, cstart);
        uint64_t chi = hi >> cstart;
        mask_u128(clo, chi, bise_stream_bits_dev(2 * npairs, cq));
        bise_stream(clo, chi, 2 * npairs, cq, [&](int i, int code) { vals[i] = __ldg(&T.cunq[cq][code]); });
    }
    int e0[4], e1[4];
    {
        int k = 0;
#pragma unroll 1
        for (int p = 0; p < parts; ++p) {
            int a[4], b[4];
            if (!endpoints(cem[p], vals + k, a, b)) {
                constant(1.0f);  // HDR endpoint mode in the LDR profile: error colour (R = 1)
                return;
            }
            e0[p] = a[0];
            e1[p] = b[0];
            k += 2 * ((cem[p] >> 2) + 1);
        }
    }
    // Value table u[p * levels + code].
#pragma unroll 1
    for (int p = 0; p < parts; ++p)
#pragma unroll 1
        for (int code = 0; code < levels; ++code) {
            const int w = __ldg(&T.wunq[wq][code]);
            const int X = e0[p] * (64 - w) + e1[p] * w;
            tab[p * levels + code] = __float2half_rn(c16_to_unit(static_cast<uint32_t>(4 * X + ((X + 32) >> 6))));
        }
    // Per-texel index: partition * levels + weight code (full grid: weight i = texel i).
    uint32_t pat[4] = {0u, 0u, 0u, 0u};
    if (parts > 1) {
        const uint32_t* pt = T.part[fp][parts - 2][seed];
        pat[0] = __ldg(pt + 0);
        pat[1] = __ldg(pt + 1);
        pat[2] = __ldg(pt + 2);
        pat[3] = __ldg(pt + 3);
    }
    uint64_t wlo = __brevll(hi), whi = __brevll(lo);
    mask_u128(wlo, whi, wbits);
    bise_stream(wlo, whi, N, wq, [&](int i, int code) {
        const int part = (pat[i >> 4] >> (2 * (i & 15))) & 3;
        idx[i] = static_cast<uint8_t>(part * levels + code);
    });
}

// ------------------------------------------------------------------ kernel

template <int D, int G, int VBS, int KBS>
struct Cfg {
    static constexpr int CH = (VBS == 6 || KBS == 6) ? 48 : 64;
    static constexpr int NWM = CH / 16;                        // MMA warps
    static constexpr int THREADS = (VBS == 6) ? 192 : 256;
    static constexpr int LD = D + 8;                           // halves per tile row (16-byte pad)
    static constexpr int VCOLS = (D + VBS - 1) / VBS;
    static constexpr int VROWS = CH / VBS;
    static constexpr int VBLK = VROWS * VCOLS;
    static constexpr int KCOLS = KBS ? (D + KBS - 1) / KBS : 1;
    static constexpr int KROWS = KBS ? CH / KBS : 0;
    static constexpr int KBLK = KROWS * KCOLS;
    static constexpr int META = (VBLK > CH ? (VBLK > D ? VBLK : D) : (CH > D ? CH : D));
    static constexpr int KMETA = KBS ? (KBLK > CH ? (KBLK > D ? KBLK : D) : (CH > D ? CH : D)) : 0;
    static constexpr int SIDE = KBS ? CH * 8 : 0;              // up to 8 side channels
    static constexpr int SCR = THREADS;                        // blocks decoded per pass
    static constexpr int MAXBS = (VBS > KBS ? VBS : KBS);
    static_assert(CH % VBS == 0 && CH % (KBS ? KBS : 1) == 0, "chunk must hold whole block rows");
    static_assert(G <= 8, "query group must fit the N=8 MMA dimension");
};

template <int D, int G, int VBS, int KBS>
struct Smem {
    using C = Cfg<D, G, VBS, KBS>;
    uint64_t bar[2];
    int valid[2];
    __align__(16) uint4 vraw[2][C::VBLK];
    __align__(16) __half vmeta[2][2][C::META];
    __align__(16) uint4 kraw[2][KBS ? C::KBLK : 1];
    __align__(16) __half kmeta[2][2][KBS ? C::KMETA : 1];
    __align__(16) __half kside[2][KBS ? C::SIDE : 1];
    __align__(16) __half vhi[C::CH][C::LD];
    __align__(16) __half vlo[C::CH][C::LD];
    __align__(16) __half khi[KBS ? C::CH : 1][C::LD];
    __align__(16) __half klo[KBS ? C::CH : 1][C::LD];
    __align__(16) __half tab[C::SCR][C::MAXBS * C::MAXBS];
    __align__(16) uint8_t idx[C::SCR][C::MAXBS * C::MAXBS];
    __align__(16) __half pbuf[C::NWM][8][16];
    float wm[C::NWM][8];
    float wl[C::NWM][8];
};

// Bytes of metadata per chunk for a plane.
template <int BS>
__device__ __forceinline__ int meta_elems(int norm, int cols, int CH, int D) {
    return norm == AKV_NORM_BLOCK_AFFINE ? (CH / BS) * cols : (norm == AKV_NORM_TOKEN ? CH : D);
}

template <int BS>
__device__ __forceinline__ int64_t meta_chunk_offset(int norm, int cols, int t_in_page) {
    return norm == AKV_NORM_BLOCK_AFFINE ? static_cast<int64_t>(t_in_page / BS) * cols
                                         : (norm == AKV_NORM_TOKEN ? t_in_page : 0);
}

// Decode the chunk's blocks of one plane (from the staged raw blocks) into the
// hi/lo tiles. All threads call it.
template <int BS, int D, int THREADS, int SCRN, int TABN, int LD>
__device__ __forceinline__ void decode_plane_chunk(const uint4* raw, const __half* moff, const __half* mscl, int norm,
                                                   int cols, int rows_blk, int n, bool valid,
                                                   __half (*tab)[TABN], uint8_t (*idx)[TABN],
                                                   __half (*thi)[LD], __half (*tlo)[LD]) {
    const int nblk = rows_blk * cols;
    for (int pass = 0; pass < nblk; pass += SCRN) {
        const int nb = min(SCRN, nblk - pass);
        for (int i = threadIdx.x; i < nb; i += THREADS) decode_block_table<BS>(raw[pass + i], tab[i], idx[i]);
        __syncthreads();
        const int ntask = nb * BS;
        for (int task = threadIdx.x; task < ntask; task += THREADS) {
            const int li = task / BS, y = task - li * BS;
            const int bi = pass + li;
            const int br = bi / cols, bc = bi - br * cols;
            const int row = br * BS + y;
            const bool ok = valid && row < n;
            float sc = 0.f, of = 0.f;
            if (norm == AKV_NORM_BLOCK_AFFINE) { sc = __half2float(mscl[bi]); of = __half2float(moff[bi]); }
            else if (norm == AKV_NORM_TOKEN) { sc = __half2float(mscl[row]); of = __half2float(moff[row]); }
            const uint8_t* ix = idx[li] + y * BS;
            const __half* tb = tab[li];
#pragma unroll
            for (int x = 0; x < BS; x += 2) {
                const int col = bc * BS + x;
                if (col >= D) break;
                float s0 = sc, o0 = of, s1 = sc, o1 = of;
                if (norm == AKV_NORM_PAGE_CHANNEL) {
                    s0 = __half2float(mscl[col]); o0 = __half2float(moff[col]);
                    s1 = __half2float(mscl[col + 1]); o1 = __half2float(moff[col + 1]);
                }
                const float v0 = ok ? fmaf(__half2float(tb[ix[x]]), s0, o0) : 0.f;
                const float v1 = ok ? fmaf(__half2float(tb[ix[x + 1]]), s1, o1) : 0.f;
                uint32_t h, l;
                split_pair(v0, v1, h, l);
                *reinterpret_cast<uint32_t*>(&thi[row][col]) = h;
                *reinterpret_cast<uint32_t*>(&tlo[row][col]) = l;
            }
        }
        __syncthreads();
    }
}

template <int D, int G, int VBS, int KBS>
__global__ void __launch_bounds__(Cfg<D, G, VBS, KBS>::THREADS, 2) attn_fast_kernel(AttnParams p) {
    using C = Cfg<D, G, VBS, KBS>;
    using S = Smem<D, G, VBS, KBS>;
    constexpr int CH = C::CH, NWM = C::NWM, THREADS = C::THREADS, LD = C::LD;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    S& sm = *reinterpret_cast<S*>(smem_raw);

    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int len = seq_len_of(p, b);
    const int t_begin = split * p.split_tokens;
    const int t_end = min(t_begin + p.split_tokens, len);
    const int64_t unit0 = (static_cast<int64_t>(b) * p.Hq + h * G) * p.nsplits + split;
    if (t_begin >= t_end) {
        for (int i = tid; i < G * D; i += THREADS)
            p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.nsplits) * D + i % D] = 0.f;
        if (tid < G) {
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.nsplits) * 2 + 0] = -CUDART_INF_F;
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.nsplits) * 2 + 1] = 0.f;
        }
        return;
    }
    const int nchunks = (t_end - t_begin + CH - 1) / CH;
    const int P = p.page_tokens;

    if (tid == 0) {
        mbar_init(&sm.bar[0], 1);
        mbar_init(&sm.bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // Producer: stage `s` <- chunk `c` (one elected thread).
    auto issue = [&](int c, int s) {
        const int t0 = t_begin + c * CH;
        const int page = t0 / P;
        const int phys = phys_page(p.table, p.pps, p.num_pages, b, page, p.status);
        const int tin = t0 - page * P;
        sm.valid[s] = phys >= 0;
        uint32_t bytes = 0;
        const uint8_t* vsrc = nullptr;
        const __half* voff = nullptr;
        const __half* vscl = nullptr;
        const int vrows = CH / VBS, vcols = C::VCOLS;
        const int vme = meta_elems<VBS>(p.v.norm, vcols, CH, D);
        const uint8_t* ksrc = nullptr;
        const __half* koff = nullptr;
        const __half* kscl = nullptr;
        const uint8_t* kside = nullptr;
        const int krows = KBS ? CH / KBS : 0, kcols = C::KCOLS;
        const int kme = KBS ? meta_elems<(KBS ? KBS : 4)>(p.k.norm, kcols, CH, D) : 0;
        if (phys >= 0) {
            vsrc = p.v.data + b * p.v.sB + h * p.v.sH + static_cast<int64_t>(phys) * p.v.sP +
                   static_cast<int64_t>(tin / VBS) * vcols * 16;
            const int64_t mbase = b * p.v.mB + h * p.v.mH + static_cast<int64_t>(phys) * p.v.mP +
                                  meta_chunk_offset<VBS>(p.v.norm, vcols, tin);
            voff = p.v.off + mbase;
            vscl = p.v.scl + mbase;
            bytes += vrows * vcols * 16 + 2 * vme * 2;
            if constexpr (KBS > 0) {
                ksrc = p.k.data + b * p.k.sB + h * p.k.sH + static_cast<int64_t>(phys) * p.k.sP +
                       static_cast<int64_t>(tin / KBS) * kcols * 16;
                const int64_t kb = b * p.k.mB + h * p.k.mH + static_cast<int64_t>(phys) * p.k.mP +
                                   meta_chunk_offset<(KBS ? KBS : 4)>(p.k.norm, kcols, tin);
                koff = p.k.off + kb;
                kscl = p.k.scl + kb;
                bytes += krows * kcols * 16 + 2 * kme * 2;
                if (p.k.side_count > 0) {
                    kside = p.k.side + b * p.k.xB + h * p.k.xH + static_cast<int64_t>(phys) * p.k.xP +
                            static_cast<int64_t>(tin) * p.k.side_count * 2;
                    bytes += CH * p.k.side_count * 2;
                }
            }
        }
        mbar_arrive_expect_tx(&sm.bar[s], bytes);
        if (phys >= 0) {
            bulk_g2s(sm.vraw[s], vsrc, vrows * vcols * 16, &sm.bar[s]);
            bulk_g2s(sm.vmeta[s][0], voff, vme * 2, &sm.bar[s]);
            bulk_g2s(sm.vmeta[s][1], vscl, vme * 2, &sm.bar[s]);
            if constexpr (KBS > 0) {
                bulk_g2s(sm.kraw[s], ksrc, krows * kcols * 16, &sm.bar[s]);
                bulk_g2s(sm.kmeta[s][0], koff, kme * 2, &sm.bar[s]);
                bulk_g2s(sm.kmeta[s][1], kscl, kme * 2, &sm.bar[s]);
                if (kside) bulk_g2s(sm.kside[s], kside, CH * p.k.side_count * 2, &sm.bar[s]);
            }
        }
    };
    if (tid == 0) {
        issue(0, 0);
        if (nchunks > 1) issue(1, 1);
    }

    // Query fragments (B operand, hi + lo), heads n = lane/4 of the group.
    const int qn = lane >> 2, qj = lane & 3;
    constexpr int KS = D / 16;
    uint32_t qhi[KS][2], qlo[KS][2];
    {
        const bool has = qn < G;
        const int64_t qb = (static_cast<int64_t>(b) * p.Hq + h * G + (has ? qn : 0)) * D;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            // Natural dim order for decoded K; a permuted order for direct
            // FP16 K loads (see the K loader below).
            int d0, d1;
            if (KBS > 0) { d0 = 16 * ks + 2 * qj; d1 = d0 + 8; }
            else { const int g32 = ks >> 1, half = ks & 1; d0 = 32 * g32 + 8 * qj + 4 * half; d1 = d0 + 2; }
            float q0 = has ? load_q(p.q, p.q_dtype, qb + d0) : 0.f;
            float q1 = has ? load_q(p.q, p.q_dtype, qb + d0 + 1) : 0.f;
            float q2 = has ? load_q(p.q, p.q_dtype, qb + d1) : 0.f;
            float q3 = has ? load_q(p.q, p.q_dtype, qb + d1 + 1) : 0.f;
            split_pair(q0, q1, qhi[ks][0], qlo[ks][0]);
            split_pair(q2, q3, qhi[ks][1], qlo[ks][1]);
        }
    }

    float o[KS][4];
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F}, l_run[2] = {0.f, 0.f};
    bool stuck = false;

    for (int c = 0; c < nchunks; ++c) {
        const int s = c & 1;
        const uint32_t parity = (c >> 1) & 1;
        const int t0 = t_begin + c * CH;
        const int n = min(CH, t_end - t0);
        // Direct FP16 K fragments for this warp's 16 tokens, issued before the
        // wait so the loads overlap it. Permuted dims: lane quad j of row r
        // loads dims [32g + 8j, 32g + 8j + 8) for each 32-dim group g.
        uint4 kreg[KBS ? 1 : D / 32][2];
        if constexpr (KBS == 0) {
            if (warp < NWM) {
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int tr = 16 * warp + qn + 8 * rr;
                    const int tt = t0 + tr;
                    const uint4* row = nullptr;
                    if (tr < n) {
                        const int phys = phys_page(p.table, p.pps, p.num_pages, b, tt / P, nullptr);
                        if (phys >= 0)
                            row = reinterpret_cast<const uint4*>(p.k.data + b * p.k.sB + h * p.k.sH +
                                                                 static_cast<int64_t>(phys) * p.k.sP +
                                                                 static_cast<int64_t>(tt % P) * D * 2);
                    }
#pragma unroll
                    for (int g32 = 0; g32 < D / 32; ++g32)
                        kreg[g32][rr] = row ? __ldg(row + 4 * g32 + qj) : make_uint4(0, 0, 0, 0);
                }
            }
        }
        const bool waited = mbar_wait(&sm.bar[s], parity);
        if (__syncthreads_or(!waited)) {
            stuck = true;
            break;
        }
        const bool valid = sm.valid[s] != 0;
        // Decode V (and K) tiles.
        decode_plane_chunk<VBS, D, THREADS, C::SCR, C::MAXBS * C::MAXBS, LD>(
            sm.vraw[s], sm.vmeta[s][0], sm.vmeta[s][1], p.v.norm, C::VCOLS, CH / VBS, n, valid, sm.tab, sm.idx,
            sm.vhi, sm.vlo);
        if constexpr (KBS > 0) {
            decode_plane_chunk<(KBS ? KBS : 4), D, THREADS, C::SCR, C::MAXBS * C::MAXBS, LD>(
                sm.kraw[s], sm.kmeta[s][0], sm.kmeta[s][1], p.k.norm, C::KCOLS, CH / KBS, n, valid, sm.tab, sm.idx,
                sm.khi, sm.klo);
            // Exact side-plane channels.
            const int sc = p.k.side_count;
            if (sc > 0) {
                for (int i = tid; i < n * sc; i += THREADS) {
                    const int r = i / sc, jj = i - r * sc;
                    const int ch = __ldg(p.k.side_ch + h * sc + jj);
                    if (ch < 0 || ch >= D) continue;
                    const float v = valid ? __half2float(sm.kside[s][r * sc + jj]) : 0.f;
                    const __half hv = __float2half_rn(v);
                    sm.khi[r][ch] = hv;
                    sm.klo[r][ch] = __float2half_rn(v - __half2float(hv));
                }
                __syncthreads();
            }
        }
        // The raw stage is consumed: refill it with chunk c + 2.
        if (tid == 0 && c + 2 < nchunks) {
            fence_proxy_async();
            issue(c + 2, s);
        }
        // Tensor-core phase: warp w owns chunk tokens [16w, 16w + 16).
        if (warp < NWM) {
            float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                if constexpr (KBS > 0) {
                    const int mi = lane >> 3, rr = lane & 7;
                    const int row = 16 * warp + rr + ((mi & 1) ? 8 : 0);
                    const int col = 16 * ks + ((mi & 2) ? 8 : 0);
                    ldsm_x4(a, &sm.khi[row][col]);
                    mma16816(sacc, a[0], a[1], a[2], a[3], qhi[ks][0], qhi[ks][1]);
                    mma16816(sacc, a[0], a[1], a[2], a[3], qlo[ks][0], qlo[ks][1]);
                    ldsm_x4(a, &sm.klo[row][col]);
                    mma16816(sacc, a[0], a[1], a[2], a[3], qhi[ks][0], qhi[ks][1]);
                } else {
                    const uint4& r0 = kreg[ks >> 1][0];
                    const uint4& r1 = kreg[ks >> 1][1];
                    if ((ks & 1) == 0) { a[0] = r0.x; a[2] = r0.y; a[1] = r1.x; a[3] = r1.y; }
                    else { a[0] = r0.z; a[2] = r0.w; a[1] = r1.z; a[3] = r1.w; }
                    mma16816(sacc, a[0], a[1], a[2], a[3], qhi[ks][0], qhi[ks][1]);
                    mma16816(sacc, a[0], a[1], a[2], a[3], qlo[ks][0], qlo[ks][1]);
                }
            }
            // sacc: S^T[tok = qn (+8)][head = 2qj (+1)], in log2 units after scaling.
            const bool v0 = 16 * warp + qn < n, v1 = 16 * warp + qn + 8 < n;
            float sv[4];
            sv[0] = v0 ? sacc[0] * p.qscale : -CUDART_INF_F;
            sv[1] = v0 ? sacc[1] * p.qscale : -CUDART_INF_F;
            sv[2] = v1 ? sacc[2] * p.qscale : -CUDART_INF_F;
            sv[3] = v1 ? sacc[3] * p.qscale : -CUDART_INF_F;
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
            // P^T -> per-warp buffer as P[head][tok] (fp16), then B fragments.
            __half(*pb)[16] = sm.pbuf[warp];
            pb[2 * qj][qn] = __float2half_rn(sv[0]);
            pb[2 * qj + 1][qn] = __float2half_rn(sv[1]);
            pb[2 * qj][qn + 8] = __float2half_rn(sv[2]);
            pb[2 * qj + 1][qn + 8] = __float2half_rn(sv[3]);
            __syncwarp();
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&pb[qn][2 * qj]);
            const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&pb[qn][2 * qj + 8]);
            // O^T[dim][head] += V^T . P^T with V = hi + lo.
            const int mi = lane >> 3, rr = lane & 7;
            const int vrow = 16 * warp + rr + ((mi & 2) ? 8 : 0);
            const int vcol = (mi & 1) ? 8 : 0;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                uint32_t a[4];
                ldsm_x4_t(a, &sm.vhi[vrow][16 * mt + vcol]);
                mma16816(o[mt], a[0], a[1], a[2], a[3], b0, b1);
                ldsm_x4_t(a, &sm.vlo[vrow][16 * mt + vcol]);
                mma16816(o[mt], a[0], a[1], a[2], a[3], b0, b1);
            }
            __syncwarp();
        }
        __syncthreads();  // tiles and P buffers free for the next chunk
    }

    if (stuck) {
        // A copy never completed: report, give in-flight copies a bounded
        // grace period, and leave this split empty.
        if (tid == 0) {
            if (p.status) atomicExch(p.status, AKV_ERR_TIMEOUT);
            mbar_wait(&sm.bar[0], 0);
        }
        for (int i = tid; i < G * D; i += THREADS)
            p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.nsplits) * D + i % D] = 0.f;
        if (tid < G) {
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.nsplits) * 2 + 0] = -CUDART_INF_F;
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.nsplits) * 2 + 1] = 0.f;
        }
        return;
    }

    // Merge the MMA warps' (m, l, O) into one split partial.
    float* red = reinterpret_cast<float*>(&sm.vhi[0][0]);  // G * D floats, fits in the V tiles
    for (int i = tid; i < G * D; i += THREADS) red[i] = 0.f;
    if (warp < NWM && lane < 4) {
        sm.wm[warp][2 * lane] = m_run[0];
        sm.wm[warp][2 * lane + 1] = m_run[1];
        sm.wl[warp][2 * lane] = l_run[0];
        sm.wl[warp][2 * lane + 1] = l_run[1];
    }
    __syncthreads();
    if (warp < NWM) {
        float scl[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int hh = 2 * qj + j;
            float M = -CUDART_INF_F;
#pragma unroll
            for (int w = 0; w < NWM; ++w) M = fmaxf(M, sm.wm[w][hh]);
            scl[j] = (M == -CUDART_INF_F || m_run[j] == -CUDART_INF_F) ? 0.f : exp2f(m_run[j] - M);
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            const int d0 = 16 * mt + qn;
            if (2 * qj < G) {
                atomicAdd(&red[(2 * qj) * D + d0], o[mt][0] * scl[0]);
                atomicAdd(&red[(2 * qj) * D + d0 + 8], o[mt][2] * scl[0]);
            }
            if (2 * qj + 1 < G) {
                atomicAdd(&red[(2 * qj + 1) * D + d0], o[mt][1] * scl[1]);
                atomicAdd(&red[(2 * qj + 1) * D + d0 + 8], o[mt][3] * scl[1]);
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += THREADS)
        p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.nsplits) * D + i % D] = red[i];
    if (tid < G) {
        float M = -CUDART_INF_F;
        for (int w = 0; w < NWM; ++w) M = fmaxf(M, sm.wm[w][tid]);
        float L = 0.f;
        if (M != -CUDART_INF_F)
            for (int w = 0; w < NWM; ++w)
                if (sm.wm[w][tid] != -CUDART_INF_F) L += exp2f(sm.wm[w][tid] - M) * sm.wl[w][tid];
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.nsplits) * 2 + 0] = M;
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.nsplits) * 2 + 1] = L;
    }
}

}  // namespace fast
}  // namespace akv
