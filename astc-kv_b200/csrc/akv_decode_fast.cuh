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

__device__ __forceinline__ int range_levels(int q) {
    const uint32_t shp = __ldg(&g_akv_tables.shape[q]);
    return (1 << (shp & 15)) * (((shp >> 4) & 1) ? 3 : (((shp >> 5) & 1) ? 5 : 1));
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

// Value-table capacity per block (entries = partitions * weight levels).
constexpr int kTabCap = 32;

// Sort keys of the per-chunk counting sort: constant blocks, per-texel
// ("slow") blocks, and one key per weight range for fast blocks.
constexpr int kKeyConst = 0;
constexpr int kKeySlow = 1;
constexpr int kKeyFast = 2;  // + weight range index 0..11
constexpr int kNumKeys = 14;

// Sort key of a block. Fast blocks: one weight plane, full-resolution grid,
// luminance-direct endpoints (mode 0) on every partition and a value table
// of at most kTabCap entries. Constant: void extent or an illegal encoding
// (error colour).
template <int BS>
__device__ __forceinline__ int block_key(uint4 blk) {
    constexpr int fp = footprint_index(BS);
    const uint32_t x = blk.x;
    const int mode = static_cast<int>(x & 0x7FF);
    if ((mode & 0x1FF) == 0x1FC) return kKeyConst;
    const uint32_t me = __ldg(&g_akv_tables.mode[fp][mode]);
    if (!(me & kModeValid)) return kKeyConst;
    if (me & (kModeDual | kModeReduced)) return kKeySlow;
    const int parts = static_cast<int>((x >> 11) & 3) + 1;
    const bool lum = parts == 1 ? ((x >> 13) & 15) == 0 : ((x >> 23) & 0x3F) == 0;
    if (!lum) return kKeySlow;
    const int wq = mode_wq(me);
    const int avail = 128 - mode_wbits(me) - (parts == 1 ? 17 : 29);
    if (avail < 0 || __ldg(&g_akv_tables.cquant[parts][avail]) == 0xFF) return kKeyConst;
    if (parts * range_levels(wq) > kTabCap) return kKeySlow;
    return kKeyFast + wq;
}

// UNORM16 value of a constant block: the void-extent R colour, or the error
// colour's R = 1.0 for illegal encodings.
__device__ __forceinline__ uint32_t const_c16(uint4 blk) {
    const uint32_t x = blk.x;
    if ((x & 0x1FF) == 0x1FC) {
        const uint64_t lo = (static_cast<uint64_t>(blk.y) << 32) | blk.x;
        const uint32_t s0 = static_cast<uint32_t>(lo >> 12) & 0x1FFF, s1 = static_cast<uint32_t>(lo >> 25) & 0x1FFF;
        const uint32_t t0 = static_cast<uint32_t>(lo >> 38) & 0x1FFF, t1 = static_cast<uint32_t>(lo >> 51) & 0x1FFF;
        const bool all_ones = (s0 & s1 & t0 & t1) == 0x1FFF;
        const bool bad = (x & 0x200) || ((x >> 10) & 3) != 3 || (!all_ones && (s0 >= s1 || t0 >= t1));
        return bad ? 0xFFFFu : (blk.z & 0xFFFFu);
    }
    return 0xFFFFu;
}

// Per-texel table-index bytes of one block (texel t in byte t & 3 of word t >> 2).
template <int BS>
struct Idx {
    static constexpr int NW = (BS * BS + 3) / 4;
    uint32_t w[NW];
};

// Fast block of weight range WQ (every BISE position is a compile-time
// constant): endpoints, value table (entry q * L + code at tab[entry * nt])
// and the per-texel index bytes q * L + code. Returns L.
template <int BS, int WQ>
__device__ __forceinline__ int decode_fast(uint4 blk, bool affine, float sc, float of, uint32_t* tab, int nt,
                                           Idx<BS>& ix) {
    constexpr int fp = footprint_index(BS);
    constexpr int N = BS * BS;
    constexpr int NW = Idx<BS>::NW;
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
    const int seed = static_cast<int>((lo >> 13) & 0x3FF);
    const int cstart = parts == 1 ? 17 : 29;
    const int cq = T.cquant[parts][128 - WBITS - cstart];
    // Luminance-direct endpoints: e0 = v[2q], e1 = v[2q + 1].
    int v[8];
    {
        uint64_t clo = window_u128(lo, hi, cstart);
        uint64_t chi = hi >> cstart;
        mask_u128(clo, chi, bise_stream_bits_dev(2 * parts, cq));
        colors8(clo, chi, cq, v);
    }
    // Value table, two entries per step (fp16 hi/lo packing on pairs).
    const float s16 = sc * 0x1p-16f;  // u = t * 2^-16 with t = C truncated to 11 significant bits
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (q < parts) {
            const int e0 = v[2 * q], e1 = v[2 * q + 1];
#pragma unroll
            for (int code = 0; code < L; code += 2) {
                const int wa = cx_weight(WQ, code);
                const int wb = cx_weight(WQ, code + 1 < L ? code + 1 : code);
                const uint32_t ca = static_cast<uint32_t>(257 * (e0 * (64 - wa) + e1 * wa) + 32) >> 6;
                const uint32_t cb = static_cast<uint32_t>(257 * (e0 * (64 - wb) + e1 * wb) + 32) >> 6;
                // 65535 decodes to exactly 1.0 (t = 65536).
                const float ta = __int_as_float(__float_as_int(static_cast<float>(ca + (ca == 0xFFFFu))) & 0xFFFFE000);
                const float tb = __int_as_float(__float_as_int(static_cast<float>(cb + (cb == 0xFFFFu))) & 0xFFFFE000);
                uint32_t e_a, e_b;
                if (affine) {
                    const float va = fmaf(ta, s16, of), vb = fmaf(tb, s16, of);
                    const __half2 h = __floats2half2_rn(va, vb);
                    const float2 hf = __half22float2(h);
                    const __half2 l = __floats2half2_rn(va - hf.x, vb - hf.y);
                    const uint32_t hw = *reinterpret_cast<const uint32_t*>(&h);
                    const uint32_t lw = *reinterpret_cast<const uint32_t*>(&l);
                    e_a = (hw & 0xFFFFu) | (lw << 16);
                    e_b = (hw >> 16) | (lw & 0xFFFF0000u);
                } else {
                    e_a = __float_as_uint(ta * 0x1p-16f);
                    e_b = __float_as_uint(tb * 0x1p-16f);
                }
                tab[(q * L + code) * nt] = e_a;
                if (code + 1 < L) tab[(q * L + code + 1) * nt] = e_b;
            }
        }
    }
    // Weight stream (bit-reversed, masked) and partition pattern.
    uint64_t w0 = __brevll(hi), w1 = __brevll(lo);
    mask_u128(w0, w1, WBITS);
    uint32_t pat[4] = {0u, 0u, 0u, 0u};
    if (parts > 1) {
        const uint32_t* pt = T.part[fp][parts - 2][seed];
#pragma unroll
        for (int k = 0; k < (N + 15) / 16; ++k) pat[k] = __ldg(pt + k);
    }
    auto wbits = [&](int pos, int n) -> uint32_t {  // pos, n compile-time after unrolling
        const uint64_t u = pos >= 64 ? (w1 >> (pos - 64)) : (pos == 0 ? w0 : ((w0 >> pos) | (w1 << (64 - pos))));
        return static_cast<uint32_t>(u) & ((n >= 32) ? 0xFFFFFFFFu : ((1u << n) - 1u));
    };
    uint32_t* cw = ix.w;
#pragma unroll
    for (int k = 0; k < NW; ++k) cw[k] = 0u;
    constexpr bool kSwar = (L == 2 || L == 3 || L == 4 || L == 5 || L == 6);
    if constexpr (kSwar) {
        // Weight codes become index bytes four or more at a time through
        // host-built spread tables; partition * L is added per word.
        uint32_t ext[3] = {0u, 0u, 0u};  // spill-over words past NW
        auto word = [&](int k) -> uint32_t& { return k < NW ? cw[k < NW ? k : 0] : ext[k - NW < 3 ? k - NW : 0]; };
        // OR `nb` code bytes (value u) in at texel offset `off` (compile time).
        auto place = [&](int off, uint64_t u, int nb) {
            const int k = off >> 2, o = off & 3;
            if (o == 0) {
                word(k) |= static_cast<uint32_t>(u);
                if (nb > 4) word(k + 1) |= static_cast<uint32_t>(u >> 32);
            } else {
                const uint64_t t = u << (8 * o);
                word(k) |= static_cast<uint32_t>(t);
                if (nb + o > 4) word(k + 1) |= static_cast<uint32_t>(t >> 32);
                if (nb + o > 8) word(k + 2) |= static_cast<uint32_t>(u >> (64 - 8 * o));
            }
        };
        if constexpr (L == 4) {
#pragma unroll
            for (int k = 0; k < NW; ++k) cw[k] = __ldg(&T.spread2[wbits(8 * k, 8)]);
        } else if constexpr (L == 2) {
#pragma unroll
            for (int g = 0; g < (N + 7) / 8; ++g) place(8 * g, __ldg(&T.spread1[wbits(8 * g, 8)]), 8);
        } else if constexpr (L == 3) {
#pragma unroll
            for (int g = 0; g < (N + 4) / 5; ++g) place(5 * g, __ldg(&T.tlut[wbits(8 * g, 8)]), 5);
        } else if constexpr (L == 5) {
#pragma unroll
            for (int g = 0; g < (N + 2) / 3; ++g) place(3 * g, __ldg(&T.qlut[wbits(7 * g, 7)]), 3);
        } else if constexpr (L == 6) {
#pragma unroll
            for (int g = 0; g < (N + 4) / 5; ++g) {
                const uint32_t bits13 = wbits(13 * g, 13);
                const uint64_t c = __ldg(&T.t13lo[bits13 & 0x7F]) | __ldg(&T.t13hi[bits13 >> 7]);
                const uint64_t d5 = __ldg(&T.tlut[static_cast<uint32_t>(c >> 56)]);
                place(5 * g, (d5 << 1) | (c & 0xFFFFFFFFFFull), 5);
            }
        }
        if (N % 4) cw[NW - 1] &= (1u << (8 * (N % 4))) - 1u;
        if (parts > 1) {
#pragma unroll
            for (int k = 0; k < NW; ++k) cw[k] += __ldg(&T.spread2[(pat[k >> 2] >> (8 * (k & 3))) & 0xFF]) * L;
        }
        return L;
    }
    auto emit = [&](int i, int code) {
        const int part = (pat[i >> 4] >> (2 * (i & 15))) & 3;
        cw[i >> 2] |= static_cast<uint32_t>(part * L + code) << (8 * (i & 3));
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
    return L;
}

// Per-key dispatch of the fast decode (only the weight ranges a footprint can
// use with a full-resolution grid are instantiated). Returns L, or 0 for a
// range that cannot occur (the caller then treats the block as slow).
template <int BS>
__device__ __forceinline__ int decode_fast_any(int wq, uint4 blk, bool affine, float sc, float of, uint32_t* tab,
                                               int nt, Idx<BS>& ix) {
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
        if constexpr (wb >= 24 && wb <= 96) return decode_fast<BS, Q>(blk, affine, sc, of, tab, nt, ix);  \
        return 0;                                                                                        \
    }
    switch (wq) {
        AKV_FAST_CASE(0) AKV_FAST_CASE(1) AKV_FAST_CASE(2) AKV_FAST_CASE(3) AKV_FAST_CASE(4) AKV_FAST_CASE(5)
        AKV_FAST_CASE(6) AKV_FAST_CASE(7) AKV_FAST_CASE(8) AKV_FAST_CASE(9) AKV_FAST_CASE(10) AKV_FAST_CASE(11)
        default: return 0;
    }
#undef AKV_FAST_CASE
}

// Texel value of a table entry as fp32: block-affine entries hold v as fp16
// hi | lo << 16, the others the unit value u (the caller applies the
// per-token / per-channel affine).
__device__ __forceinline__ float entry_value(uint32_t e, bool affine) {
    if (affine) {
        const __half2 h = *reinterpret_cast<const __half2*>(&e);
        const float2 f = __half22float2(h);
        return f.x + f.y;
    }
    return __uint_as_float(e);
}

}  // namespace fast
}  // namespace akv
