// Per-block "value table" decode of scalar-layout ASTC blocks (R channel),
// used by the sorted decode of akv_attn_fast.cuh.
//
// Fast-class blocks (single weight plane, full-resolution grid, table small
// enough) become a table of values indexed by partition * levels + weight
// code plus one index byte per texel; every BISE position is a compile-time
// constant because the weight range is a template parameter.
#pragma once
#include <cuda_fp16.h>

#include "akv_astc_device.cuh"

namespace akv {
namespace fast {

// ---------------------------------------------------------- sorted decode
//
// Blocks of a chunk are first classified (constant, per-texel "slow", or a
// fast class per weight range), counting-sorted by class, and then decoded
// in class order so the lanes of a warp run the same code path.

constexpr int kClsConst = 0;   // void extent or illegal encoding: one value
constexpr int kClsSlow = 1;    // reduced weight grid, dual plane or large table
constexpr int kClsFast = 2;    // + weight range index (0..11)
constexpr int kNumCls = 14;

__device__ __forceinline__ int range_levels(int q) {
    const uint32_t shp = __ldg(&g_akv_tables.shape[q]);
    return (1 << (shp & 15)) * (((shp >> 4) & 1) ? 3 : (((shp >> 5) & 1) ? 5 : 1));
}

template <int BS>
__device__ __forceinline__ int classify(uint4 blk) {
    constexpr int fp = footprint_index(BS);
    const int mode = static_cast<int>(blk.x & 0x7FF);
    if ((mode & 0x1FF) == 0x1FC) return kClsConst;
    const uint32_t me = __ldg(&g_akv_tables.mode[fp][mode]);
    if (!(me & kModeValid)) return kClsConst;
    if (me & (kModeDual | kModeReduced)) return kClsSlow;
    return kClsFast + mode_wq(me);
}

// Table entry for a decoded value u: either v = scale*u + offset split into
// fp16 hi | lo << 16 (block-affine planes, the affine is per block), or u's
// float bits (token / page-channel planes, affine applied per texel later).
__device__ __forceinline__ uint32_t table_entry(float u, bool affine, float sc, float of) {
    if (!affine) return __float_as_uint(u);
    const float v = fmaf(u, sc, of);
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    return static_cast<uint32_t>(__half_as_ushort(hi)) | (static_cast<uint32_t>(__half_as_ushort(lo)) << 16);
}

// Weight unquantisation (spec formula) evaluated at compile time for a
// compile-time weight range, so value tables need no table loads.
constexpr int cx_replicate(int v, int n, int width) {
    int out = 0, filled = 0;
    while (filled < width) {
        const int k = n < width - filled ? n : width - filled;
        out = (out << k) | (v >> (n - k));
        filled += k;
    }
    return out;
}

constexpr int cx_weight(int q, int code) {
    const int lv[12] = {2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32};
    const int L = lv[q];
    const bool tr = L % 3 == 0, qu = L % 5 == 0;
    const int base = tr ? L / 3 : (qu ? L / 5 : L);
    int b = 0;
    while ((1 << b) < base) ++b;
    int r = 0;
    if (!tr && !qu) {
        r = cx_replicate(code, b, 6);
    } else if (b == 0) {
        r = tr ? (code == 0 ? 0 : code == 1 ? 32 : 63) : (code * 16 - (code >= 3 ? 1 : 0));
    } else {
        const int digit = code >> b, m = code & ((1 << b) - 1);
        const int a = m & 1, bb = (m >> 1) & 1, c = (m >> 2) & 1;
        int B = 0, C = 0;
        if (L == 6) C = 50;
        else if (L == 10) C = 28;
        else if (L == 12) { C = 23; B = bb * 0x45; }
        else if (L == 20) { C = 13; B = bb * 0x42; }
        else if (L == 24) { C = 11; B = c * 0x42 + bb * 0x21; }
        const int A = a ? 0x7F : 0;
        const int T = (digit * C + B) ^ A;
        r = (A & 0x20) | (T >> 2);
    }
    return r > 32 ? r + 1 : r;
}

// Up to eight colour integers of range `cq` from a colour stream that starts
// at bit 0 of (clo, chi) and is masked to its length, unquantised to 0..255
// into registers (no local-memory arrays).
__device__ __forceinline__ void colors8(uint64_t clo, uint64_t chi, int cq, int (&v)[8]) {
    const Tables& T = g_akv_tables;
    const uint32_t shp = __ldg(&T.shape[cq]);
    const int b = shp & 15;
    const uint64_t mm = (1ull << b) - 1ull;
    const uint8_t* un = T.cunq[cq];
    if (shp & 0x10) {
        const int gb = 5 * b + 8;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            const uint64_t w = window_u128(clo, chi, g * gb);
            const uint32_t t = static_cast<uint32_t>((w >> b) & 3u) | static_cast<uint32_t>(((w >> (2 * b + 2)) & 3u) << 2) |
                               static_cast<uint32_t>(((w >> (3 * b + 4)) & 1u) << 4) |
                               static_cast<uint32_t>(((w >> (4 * b + 5)) & 3u) << 5) |
                               static_cast<uint32_t>(((w >> (5 * b + 7)) & 1u) << 7);
            const uint32_t dg = __ldg(&T.trit[t]);
            const int off[5] = {0, 2, 4, 5, 7};
#pragma unroll
            for (int j = 0; j < 5; ++j) {
                const int i = 5 * g + j;
                if (i < 8) {
                    const uint32_t m = static_cast<uint32_t>((w >> (j * b + off[j])) & mm);
                    v[i] = __ldg(un + ((((dg >> (2 * j)) & 3u) << b) | m));
                }
            }
        }
    } else if (shp & 0x20) {
        const int gb = 3 * b + 7;
#pragma unroll
        for (int g = 0; g < 3; ++g) {
            const uint64_t w = window_u128(clo, chi, g * gb);
            const uint32_t qv = static_cast<uint32_t>((w >> b) & 7u) | static_cast<uint32_t>(((w >> (2 * b + 3)) & 3u) << 3) |
                                static_cast<uint32_t>(((w >> (3 * b + 5)) & 3u) << 5);
            const uint32_t dg = __ldg(&T.quint[qv]);
            const int off[3] = {0, 3, 5};
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int i = 3 * g + j;
                if (i < 8) {
                    const uint32_t m = static_cast<uint32_t>((w >> (j * b + off[j])) & mm);
                    v[i] = __ldg(un + ((((dg >> (3 * j)) & 7u) << b) | m));
                }
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __ldg(un + static_cast<uint32_t>(window_u128(clo, chi, i * b) & mm));
    }
}

// Fast-class block: header, endpoints, value table and per-texel indices.
// WQ is the block's weight range (compile time: every BISE position below is
// a constant).
template <int BS, int WQ>
__device__ __forceinline__ void decode_fast(uint4 blk, bool affine, float sc, float of, uint32_t* tab, uint8_t* idx) {
    constexpr int fp = footprint_index(BS);
    constexpr int N = BS * BS;
    constexpr int kLv[12] = {2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32};
    constexpr int L = kLv[WQ];
    constexpr bool TR = (L % 3) == 0;
    constexpr bool QU = (L % 5) == 0;
    constexpr int B = TR ? (L == 3 ? 0 : L == 6 ? 1 : L == 12 ? 2 : 3)
                         : QU ? (L == 5 ? 0 : L == 10 ? 1 : 2)
                              : (L == 2 ? 1 : L == 4 ? 2 : L == 8 ? 3 : L == 16 ? 4 : 5);
    constexpr int WBITS = N * B + (TR ? (8 * N + 4) / 5 : 0) + (QU ? (7 * N + 2) / 3 : 0);
    const Tables& T = g_akv_tables;
    const uint64_t lo = (static_cast<uint64_t>(blk.y) << 32) | blk.x;
    const uint64_t hi = (static_cast<uint64_t>(blk.w) << 32) | blk.z;
    const int parts = static_cast<int>((lo >> 11) & 3) + 1;
    constexpr int top = 128 - WBITS;
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
            for (int q = 0; q < 4; ++q) cem[q] = field >> 2;
        } else {
            extra = 3 * parts - 4;
            const int all = (field >> 2) | (static_cast<int>(bits_u128(lo, hi, top - extra, extra)) << 4);
            const int cls = (field & 3) - 1;
#pragma unroll
            for (int q = 0; q < 4; ++q) cem[q] = ((cls + ((all >> q) & 1)) << 2) | ((all >> (parts + 2 * q)) & 3);
        }
    }
    int npairs = 0;
    for (int q = 0; q < parts; ++q) npairs += (cem[q] >> 2) + 1;
    const int avail = top - extra - cstart;
    const int cq = (npairs <= 9 && avail >= 0) ? T.cquant[npairs][avail] : 0xFF;
    auto error_block = [&]() {
        tab[0] = table_entry(1.0f, affine, sc, of);  // error colour: R = 1
#pragma unroll
        for (int t = 0; t < N; t += 4) *reinterpret_cast<uint32_t*>(idx + t) = 0u;
    };
    if (cq == 0xFF) { error_block(); return; }
    int e0[4] = {0, 0, 0, 0}, e1[4] = {0, 0, 0, 0};
    uint64_t clo = window_u128(lo, hi, cstart);
    uint64_t chi = hi >> cstart;
    mask_u128(clo, chi, bise_stream_bits_dev(2 * npairs, cq));
    const bool lum_direct = parts == 1 ? cem[0] == 0 : (cem[0] | cem[1] | (parts > 2 ? cem[2] : 0) | (parts > 3 ? cem[3] : 0)) == 0;
    if (lum_direct) {
        // Luminance direct (mode 0) on every partition: e0 = v[2q], e1 = v[2q+1].
        int v[8];
        colors8(clo, chi, cq, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) { e0[q] = v[2 * q]; e1[q] = v[2 * q + 1]; }
    } else {
        int vals[18];
        bise_stream(clo, chi, 2 * npairs, cq, [&](int i, int code) { vals[i] = __ldg(&T.cunq[cq][code]); });
        int k = 0;
#pragma unroll 1
        for (int q = 0; q < parts; ++q) {
            int a[4], bb[4];
            if (!endpoints(cem[q], vals + k, a, bb)) { error_block(); return; }
            k += 2 * ((cem[q] >> 2) + 1);
            if (q == 0) { e0[0] = a[0]; e1[0] = bb[0]; }
            else if (q == 1) { e0[1] = a[0]; e1[1] = bb[0]; }
            else if (q == 2) { e0[2] = a[0]; e1[2] = bb[0]; }
            else { e0[3] = a[0]; e1[3] = bb[0]; }
        }
    }
    // Direct mode: a table would be larger than the block, so each texel's
    // value is computed in place (identity indices).
    const bool direct = parts * L > N;
    // Value table: entry q*L + code (weights are compile-time constants).
    if (!direct) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (q < parts) {
#pragma unroll
                for (int code = 0; code < L; ++code) {
                    constexpr int dummy = 0;
                    (void)dummy;
                    const int w = cx_weight(WQ, code);
                    const int X = e0[q] * (64 - w) + e1[q] * w;
                    tab[q * L + code] =
                        table_entry(c16_to_unit(static_cast<uint32_t>(4 * X + ((X + 32) >> 6))), affine, sc, of);
                }
            }
        }
    }
    // Weight stream (bit-reversed, masked) and partition pattern.
    uint64_t w0 = __brevll(hi), w1 = __brevll(lo);
    mask_u128(w0, w1, WBITS);
    uint32_t pat[4] = {0u, 0u, 0u, 0u};
    if (parts > 1) {
        const uint32_t* pt = T.part[fp][parts - 2][seed];
        pat[0] = __ldg(pt + 0); pat[1] = __ldg(pt + 1); pat[2] = __ldg(pt + 2); pat[3] = __ldg(pt + 3);
    }
    auto wbits = [&](int pos, int n) -> uint32_t {  // pos, n compile-time after unrolling
        const uint64_t v = pos >= 64 ? (w1 >> (pos - 64)) : (pos == 0 ? w0 : ((w0 >> pos) | (w1 << (64 - pos))));
        return static_cast<uint32_t>(v) & ((n >= 32) ? 0xFFFFFFFFu : ((1u << n) - 1u));
    };
    uint32_t word = 0;
    auto emit = [&](int i, int code) {
        const int part = (pat[i >> 4] >> (2 * (i & 15))) & 3;
        if (direct) {
            const int a = part == 0 ? e0[0] : part == 1 ? e0[1] : part == 2 ? e0[2] : e0[3];
            const int bq = part == 0 ? e1[0] : part == 1 ? e1[1] : part == 2 ? e1[2] : e1[3];
            const int w = __ldg(&T.wunq[WQ][code]);  // code is a runtime value here
            const int X = a * (64 - w) + bq * w;
            tab[i] = table_entry(c16_to_unit(static_cast<uint32_t>(4 * X + ((X + 32) >> 6))), affine, sc, of);
            code = i;
            word |= static_cast<uint32_t>(i) << (8 * (i & 3));
        } else {
            word |= static_cast<uint32_t>(part * L + code) << (8 * (i & 3));
        }
        if ((i & 3) == 3 || i == N - 1) {
            *reinterpret_cast<uint32_t*>(idx + (i & ~3)) = word;
            word = 0;
        }
    };
    if constexpr (TR) {
        constexpr int GB = 5 * B + 8;
#pragma unroll
        for (int g = 0; g < (N + 4) / 5; ++g) {
            const int base = g * GB;
            const uint32_t tbits = wbits(base + B, 2) | (wbits(base + 2 * B + 2, 2) << 2) |
                                   (wbits(base + 3 * B + 4, 1) << 4) | (wbits(base + 4 * B + 5, 2) << 5) |
                                   (wbits(base + 5 * B + 7, 1) << 7);
            const uint32_t dg = __ldg(&T.trit[tbits]);
            constexpr int off[5] = {0, 2, 4, 5, 7};
#pragma unroll
            for (int j = 0; j < 5; ++j) {
                const int i = 5 * g + j;
                if (i < N) emit(i, static_cast<int>((((dg >> (2 * j)) & 3u) << B) | (B ? wbits(base + j * B + off[j], B) : 0u)));
            }
        }
    } else if constexpr (QU) {
        constexpr int GB = 3 * B + 7;
#pragma unroll
        for (int g = 0; g < (N + 2) / 3; ++g) {
            const int base = g * GB;
            const uint32_t qbits = wbits(base + B, 3) | (wbits(base + 2 * B + 3, 2) << 3) | (wbits(base + 3 * B + 5, 2) << 5);
            const uint32_t dg = __ldg(&T.quint[qbits]);
            constexpr int off[3] = {0, 3, 5};
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int i = 3 * g + j;
                if (i < N) emit(i, static_cast<int>((((dg >> (3 * j)) & 7u) << B) | (B ? wbits(base + j * B + off[j], B) : 0u)));
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) emit(i, static_cast<int>(wbits(i * B, B)));
    }
}

// Per-class dispatch of the fast decode (only the weight ranges a footprint
// can use with a full-resolution grid are instantiated).
template <int BS>
__device__ __forceinline__ void decode_fast_any(int wq, uint4 blk, bool affine, float sc, float of, uint32_t* tab,
                                                uint8_t* idx) {
    constexpr int N = BS * BS;
    // WQ valid for a full grid iff its stream fits in 24..96 bits.
#define AKV_FAST_CASE(Q)                                                                                 \
    case Q: {                                                                                            \
        constexpr int kL[12] = {2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32};                               \
        constexpr int L = kL[Q];                                                                         \
        constexpr int bb = (L % 3 == 0) ? (L == 3 ? 0 : L == 6 ? 1 : L == 12 ? 2 : 3)                     \
                           : (L % 5 == 0) ? (L == 5 ? 0 : L == 10 ? 1 : 2)                                \
                                          : (L == 2 ? 1 : L == 4 ? 2 : L == 8 ? 3 : L == 16 ? 4 : 5);     \
        constexpr int wb = N * bb + ((L % 3 == 0) ? (8 * N + 4) / 5 : 0) + ((L % 5 == 0) ? (7 * N + 2) / 3 : 0); \
        if constexpr (wb >= 24 && wb <= 96) decode_fast<BS, Q>(blk, affine, sc, of, tab, idx);           \
        return;                                                                                          \
    }
    switch (wq) {
        AKV_FAST_CASE(0) AKV_FAST_CASE(1) AKV_FAST_CASE(2) AKV_FAST_CASE(3) AKV_FAST_CASE(4) AKV_FAST_CASE(5)
        AKV_FAST_CASE(6) AKV_FAST_CASE(7) AKV_FAST_CASE(8) AKV_FAST_CASE(9) AKV_FAST_CASE(10) AKV_FAST_CASE(11)
        default: return;
    }
#undef AKV_FAST_CASE
}

}  // namespace fast
}  // namespace akv
