// Runtime-parameterised decode of scalar-layout ASTC blocks (R channel) for
// the fused attention kernel (akv_attn_fast.cuh).
//
// One compact code path serves every weight range, partition count and
// footprint: per-range quantities (bits per value, trit/quint groups, group
// widths) are runtime values, so the lanes of a warp run the same
// instructions whatever their blocks look like and the kernel's machine code
// stays small. A luminance-direct (endpoint mode 0), single-plane block with
// a full-resolution grid becomes a value table (entry = partition * levels +
// weight code, affine and fp16 hi/lo split folded in) plus one weight-code
// byte per texel; with a reduced grid, or a table larger than kTabCap<BS>, it
// becomes a descriptor evaluated a texel row (or pair) at a time
// (desc_seg_c16). Everything else takes the generic decoder of
// akv_astc_device.cuh.
#pragma once
#include <cuda_fp16.h>

#include "akv_astc_device.cuh"

namespace akv {
namespace fast {


// Block kinds of the runtime path.
enum : int { kKindTable = 0, kKindDesc = 1, kKindGeneric = 2, kKindConst = 3 };

// Footprints whose table-kind blocks skip the value table: each texel's value
// is computed from its endpoints and weight directly (a 4x4 block has 16
// texels, fewer than most of its tables would have entries).
template <int BS>
constexpr bool kDirect = BS == 4;

// Value-table capacity per block (entries = partitions * weight levels) by
// footprint: none for directly evaluated 4x4 blocks; a full-resolution 8x8
// grid only fits two weight levels (at most 8 entries); 12 for 6x6, the
// largest table of any full-grid block in the reference's astcenc corpus
// (three partitions x four levels, four x three), larger ones become
// descriptors.
template <int BS>
constexpr int kTabCap = BS == 4 ? 0 : (BS == 8 ? 8 : 12);
constexpr int kTabCapMax = 12;

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

// Kind of a block, with its mode-table entry and colour range for the
// luminance kinds (table / descriptor).
template <int BS>
__device__ __forceinline__ int block_kind(uint4 blk, uint32_t& me, int& cq) {
    constexpr int fp = footprint_index(BS);
    const uint32_t x = blk.x;
    const int mode = static_cast<int>(x & 0x7FF);
    me = 0u;
    cq = 0;
    if ((mode & 0x1FF) == 0x1FC) return kKindConst;
    me = __ldg(&g_akv_tables.mode[fp][mode]);
    if (!(me & kModeValid)) return kKindConst;
    if (me & kModeDual) return kKindGeneric;
    const int parts = static_cast<int>((x >> 11) & 3) + 1;
    const bool lum = parts == 1 ? ((x >> 13) & 15) == 0 : ((x >> 23) & 0x3F) == 0;
    if (!lum) return kKindGeneric;
    const int avail = 128 - mode_wbits(me) - (parts == 1 ? 17 : 29);
    cq = avail < 0 ? 0xFF : __ldg(&g_akv_tables.cquant[parts][avail]);
    if (cq == 0xFF) return kKindConst;
    if (me & kModeReduced) return kKindDesc;
    // 4x4 blocks are evaluated per texel in the thread (kDirect), so their
    // table size does not matter.
    if (!kDirect<BS> && parts * range_levels(mode_wq(me)) > kTabCap<BS>) return kKindDesc;
    return kKindTable;
}

// Value table of a luminance-direct block: entry q * L + code at
// tab[entry * nt], two entries per step (fp16 hi/lo packing on pairs).
__device__ __forceinline__ void build_table(const int (&v)[8], int parts, int wq, int L, bool affine, float sc,
                                            float of, uint32_t* tab, int nt) {
    const uint8_t* wun = g_akv_tables.wunq[wq];
    const float s16 = sc * 0x1p-16f;  // u = t * 2^-16 with t = C truncated to 11 significant bits
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (q < parts) {
            const int e0 = v[2 * q], e1 = v[2 * q + 1];
            uint32_t* tq = tab + q * L * nt;
            for (int c = 0; c < L; c += 2) {
                const uint32_t wpair = __ldg(reinterpret_cast<const uint16_t*>(wun + c));
                const int wa = static_cast<int>(wpair & 0xFF), wb = static_cast<int>(wpair >> 8);
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
                tq[c * nt] = e_a;
                if (c + 1 < L) tq[(c + 1) * nt] = e_b;
            }
        }
    }
}

// What the tile writer needs of a table / constant block.
struct LumOut {
    uint32_t pat[4];  // partition per texel, 2 bits each
    int L;            // table entries per partition
    uint32_t cmask;   // 0xFF, or 0 for a constant block (every texel -> entry 0)
    // Direct evaluation (kDirect footprints): endpoints of partitions 0..3
    // as bytes, the weight unquantisation row, the constant's unit value.
    uint32_t e0p, e1p;
    const uint8_t* wun;
    float cu;
};

// Texel t of a directly evaluated, non-constant block as 2^16 times its unit
// value: the fp16 view of C (C truncated to 11 significant bits, 65535 ->
// 65536) as an integer-valued float. The partition's endpoint bytes come out
// of e0p / e1p by one byte permute each (selector nibbles 4 pick zero bytes).
__device__ __forceinline__ float direct_t(const LumOut& o, const uint8_t* codes, int nt, int t) {
    const uint32_t sel = ((o.pat[t >> 4] >> (2 * (t & 15))) & 3u) | 0x4440u;
    const uint32_t e0 = __byte_perm(o.e0p, 0u, sel), e1 = __byte_perm(o.e1p, 0u, sel);
    const uint32_t w = __ldg(o.wun + codes[t * nt]);
    const uint32_t c = (257u * (e0 * (64u - w) + e1 * w) + 32u) >> 6;
    return __int_as_float(__float_as_int(static_cast<float>(c + (c == 0xFFFFu))) & 0xFFFFE000);
}

// Unit value of texel t of a directly evaluated block.
__device__ __forceinline__ float direct_unit(const LumOut& o, const uint8_t* codes, int nt, int t) {
    return o.cmask ? direct_t(o, codes, nt, t) * 0x1p-16f : o.cu;
}

// Runtime path for table, descriptor and constant blocks (kind from
// block_kind). Table / constant: tab and codes filled, `o` describes them.
// Descriptor: d's partitions and info filled as decode_header fills them,
// d->ep[0] / ep[1] = the endpoints e0 / e1 of partitions 0..3 packed as bytes
// (desc_seg_c16's e0p / e1p), and the weight codes left in codes[j * nt]
// for desc_weight.
template <int BS>
__device__ __forceinline__ void decode_lum(uint4 blk, int kind, uint32_t me, int cq, bool affine, float sc, float of,
                                           uint32_t* tab, uint8_t* codes, int nt, BlockDesc<1>* d, LumOut& o) {
    constexpr int fp = footprint_index(BS);
    constexpr int N = BS * BS;
    const Tables& T = g_akv_tables;
    const uint64_t lo = (static_cast<uint64_t>(blk.y) << 32) | blk.x;
    const uint64_t hi = (static_cast<uint64_t>(blk.w) << 32) | blk.z;
    const bool lum = kind != kKindConst;
    const int parts = lum ? static_cast<int>((lo >> 11) & 3) + 1 : 1;
    const int wq = mode_wq(me);
    const int L = lum ? range_levels(wq) : 1;
    o.L = L;
    o.cmask = lum ? 0xFFu : 0u;
    o.wun = T.wunq[wq];
    o.e0p = o.e1p = 0u;
    o.cu = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) o.pat[k] = 0u;
    if (!lum) {
        if constexpr (kDirect<BS>) o.cu = c16_to_unit(const_c16(blk));
        else {
            // Every texel reads entry 0: a one-entry table and zero codes.
            tab[0] = table_entry(c16_to_unit(const_c16(blk)), affine, sc, of);
            for (int t = 0; t < N; ++t) codes[t * nt] = 0;
        }
        return;
    }
    int v[8];
    {
        // Colour integers through the thread's code rows (overwritten by the
        // weight codes below), read back into registers.
        const int cstart = parts == 1 ? 17 : 29;
        uint64_t clo = window_u128(lo, hi, cstart);
        uint64_t chi = hi >> cstart;
        mask_u128(clo, chi, bise_stream_bits_dev(2 * parts, cq));
        color_values(clo, chi, cq, 2 * parts, codes, nt);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = codes[k * nt];
    }
    if constexpr (kDirect<BS>) {
        o.e0p = static_cast<uint32_t>(v[0] | (v[2] << 8) | (v[4] << 16) | (v[6] << 24));
        o.e1p = static_cast<uint32_t>(v[1] | (v[3] << 8) | (v[5] << 16) | (v[7] << 24));
    } else {
        if (kind == kKindTable) build_table(v, parts, wq, L, affine, sc, of, tab, nt);
    }
    if (parts > 1) {
        const uint32_t* pt = T.part[fp][parts - 2][(lo >> 13) & 0x3FF];
#pragma unroll
        for (int k = 0; k < (N + 15) / 16; ++k) o.pat[k] = __ldg(pt + k);
    }
    const int wx = mode_wx(me), wy = mode_wy(me);
    const int count = wx * wy;
    {
        uint64_t s0 = __brevll(hi), s1 = __brevll(lo);
        mask_u128(s0, s1, mode_wbits(me));
        weight_codes(s0, s1, wq, count, codes, nt);
    }
    if (kind == kKindDesc) {
        d->pat[0] = o.pat[0];
        d->pat[1] = o.pat[1];
        d->pat_hi[0] = o.pat[2];
        d->pat_hi[1] = o.pat[3];
        // Endpoints of partitions 0..3 packed as bytes (desc_seg_c16).
        d->ep[0] = static_cast<uint32_t>(v[0] | (v[2] << 8) | (v[4] << 16) | (v[6] << 24));
        d->ep[1] = static_cast<uint32_t>(v[1] | (v[3] << 8) | (v[5] << 16) | (v[7] << 24));
        d->info = static_cast<uint32_t>(parts - 1) | ((me & kModeReduced) ? (1u << kInfoReduced) : 0u) |
                  (static_cast<uint32_t>(wx) << kInfoWx) | (static_cast<uint32_t>(wy) << kInfoWy);
    }
}

// UNORM16 value C of texel t of a single-plane descriptor from decode_header
// (grid weights with a row stride of wx; what texel_values gives for it)
// through the host-built infill taps; w must have 8 readable bytes of slack
// past the grid (taps past the grid carry weight 0).
template <int BS>
__device__ __forceinline__ uint32_t desc_texel_c16(const BlockDesc<1>& d, const uint8_t* w, int t) {
    constexpr int fp = footprint_index(BS);
    const uint32_t info = d.info;
    uint32_t wt;
    if (info & (1u << kInfoReduced)) {
        const int wx = (info >> kInfoWx) & 15, wy = (info >> kInfoWy) & 15;
        const uint32_t tap = __ldg(&g_akv_tables.infill[fp][wx - 2][wy - 2][t]);
        const uint32_t i00 = tap & 63u, fs = (tap >> 6) & 15u, ft = tap >> 10;
        const uint32_t w11 = (fs * ft + 8u) >> 4;
        wt = (w[i00] * (16u - fs - ft + w11) + w[i00 + 1] * (fs - w11) + w[i00 + wx] * (ft - w11) +
              w[i00 + wx + 1] * w11 + 8u) >> 4;
    } else {
        wt = w[t];
    }
    const uint32_t word = t < 16 ? d.pat[0] : t < 32 ? d.pat[1] : t < 48 ? d.pat_hi[0] : d.pat_hi[1];
    const uint32_t ep = d.ep[(word >> (2 * (t & 15))) & 3u];
    const uint32_t X = (ep & 0xFFu) * (64u - wt) + ((ep >> 8) & 0xFFu) * wt;
    return 4u * X + ((X + 32u) >> 6);
}

// Unquantised grid weight k = 8 r + c (the row-stride-8 layout desc_seg_c16
// reads) of a descriptor block, from its weight codes codes[j * nt] with
// j = r * wx + c; meaningful for c < wx, r < wy.
__device__ __forceinline__ uint8_t desc_weight(const uint8_t* codes, int nt, const uint8_t* un, int wx, int k) {
    return __ldg(un + codes[((k >> 3) * wx + (k & 7)) * nt]);
}

// Texels per phase-1b task of a luminance descriptor: whole rows, except
// pairs for 6x6 (6x6 planes have few descriptor blocks per chunk, and short
// tasks keep that phase's critical path short).
template <int BS>
constexpr int kDescSeg = BS == 6 ? 2 : BS;

// UNORM16 values C of texels x0 .. x0 + SEG - 1 of row y (SEG = BS with
// x0 = 0, or SEG = 2 with x0 even) of a single-plane luminance descriptor
// block (what texel_values gives for them): info as decode_header fills it,
// grid weights w in rows of 8 bytes plus one readable slack row, the row's
// partition bits `prow`, and the endpoints of partitions 0..3 as bytes of
// e0p / e1p. Infill is separable: the row fixes the two grid rows and the t
// fraction, each column its two grid columns (one byte permute per grid row)
// and the s fraction.
template <int BS, int SEG>
__device__ __forceinline__ void desc_seg_c16(uint32_t info, const uint8_t* w, uint32_t prow, uint32_t e0p,
                                             uint32_t e1p, int y, int x0, uint32_t (&c)[SEG]) {
    static_assert(SEG == BS || SEG == 2, "whole rows or pairs");
    constexpr int fp = footprint_index(BS);
    const Tables& T = g_akv_tables;
    const int wx = (info >> kInfoWx) & 15, wy = (info >> kInfoWy) & 15;
    const uint32_t ty = __ldg(&T.sep[fp][wy - 2][y]);
    const uint32_t jt = ty & 15u, ft = ty >> 8;
    const uint2 r0 = *reinterpret_cast<const uint2*>(w + 8 * jt);
    const uint2 r1 = *reinterpret_cast<const uint2*>(w + 8 * jt + 8);
    uint32_t txw[SEG == BS ? 4 : 1];
    if constexpr (SEG == BS) {
        const uint4 tx = __ldg(reinterpret_cast<const uint4*>(T.sep[fp][wx - 2]));
        txw[0] = tx.x; txw[1] = tx.y; txw[2] = tx.z; txw[3] = tx.w;
    } else {
        txw[0] = __ldg(reinterpret_cast<const uint32_t*>(T.sep[fp][wx - 2]) + (x0 >> 1));
    }
    prow >>= 2 * x0;
#pragma unroll
    for (int x = 0; x < SEG; ++x) {
        const uint32_t e = (txw[x >> 1] >> (16 * (x & 1))) & 0xFFFFu;
        const uint32_t sel = e & 0xFFu, fs = e >> 8;
        const uint32_t w11 = (fs * ft + 8u) >> 4;
        const uint32_t a = __byte_perm(r0.x, r0.y, sel), b = __byte_perm(r1.x, r1.y, sel);
        const uint32_t wt = ((a & 0xFFu) * (16u - fs - ft + w11) + ((a >> 8) & 0xFFu) * (fs - w11) +
                             (b & 0xFFu) * (ft - w11) + ((b >> 8) & 0xFFu) * w11 + 8u) >> 4;
        const uint32_t part = (prow >> (2 * x)) & 3u;
        const uint32_t e0 = (e0p >> (8 * part)) & 0xFFu, e1 = (e1p >> (8 * part)) & 0xFFu;
        const uint32_t X = e0 * (64u - wt) + e1 * wt;
        c[x] = 4u * X + ((X + 32u) >> 6);
    }
}

// fp32 value of texel t of a table / constant block (for host-side checks;
// the kernel's tile writer reads the table the same way).
__device__ __forceinline__ float lum_unit(const LumOut& o, const uint32_t* tab, const uint8_t* codes, int nt, int t) {
    const uint32_t c = codes[t * nt] & o.cmask;
    const uint32_t part = (o.pat[t >> 4] >> (2 * (t & 15))) & 3u;
    return __uint_as_float(tab[(part * o.L + c) * nt]);
}

// ------------------------------------------------- RGBA layout, 4x4 blocks
//
// A texel holds four consecutive channels (codec.py:185-187). Fast blocks:
// one weight plane, full 4x4 grid, at most two partitions, RGBA-direct
// endpoints (mode 12) on every partition; each texel's four values are
// computed from its endpoints and weight in the decoding thread.

// Kind of an RGBA 4x4 block (kKindTable = the fast path), with its mode
// entry and colour range.
__device__ __forceinline__ int rgba_block_kind(uint4 blk, uint32_t& me, int& cq) {
    constexpr int fp = footprint_index(4);
    const uint32_t x = blk.x;
    const int mode = static_cast<int>(x & 0x7FF);
    me = 0u;
    cq = 0;
    if ((mode & 0x1FF) == 0x1FC) return kKindConst;
    me = __ldg(&g_akv_tables.mode[fp][mode]);
    if (!(me & kModeValid)) return kKindConst;
    if (me & (kModeDual | kModeReduced)) return kKindGeneric;
    const int parts = static_cast<int>((x >> 11) & 3) + 1;
    if (parts > 2) return kKindGeneric;
    const bool rgba = parts == 1 ? ((x >> 13) & 15) == 12 : ((x >> 23) & 0x3F) == (12 << 2);
    if (!rgba) return kKindGeneric;
    const int avail = 128 - mode_wbits(me) - (parts == 1 ? 17 : 29);
    cq = avail < 0 ? 0xFF : __ldg(&g_akv_tables.cquant[4 * parts][avail]);
    return cq == 0xFF ? kKindConst : kKindTable;
}

// What the tile writer needs of a fast or constant RGBA block.
struct RgbaOut {
    uint32_t e0[4], e1[4];  // per channel: endpoints of partitions 0, 1 as bytes 0, 1
    uint32_t pat;           // partition per texel, 2 bits each
    const uint8_t* wun;     // weight unquantisation row
    bool cst;               // constant block: c16 holds the four channel values
    uint32_t c16[4];
};

// Fast or constant RGBA 4x4 block -> RgbaOut and the 16 weight codes in
// codes[t * nt] (which also stage the colour integers).
__device__ __forceinline__ void decode_rgba4(uint4 blk, int kind, uint32_t me, int cq, uint8_t* codes, int nt,
                                             RgbaOut& o) {
    const Tables& T = g_akv_tables;
    const uint64_t lo = (static_cast<uint64_t>(blk.y) << 32) | blk.x;
    const uint64_t hi = (static_cast<uint64_t>(blk.w) << 32) | blk.z;
    o.cst = kind == kKindConst;
    o.pat = 0u;
    o.wun = T.wunq[mode_wq(me)];
#pragma unroll
    for (int c = 0; c < 4; ++c) o.e0[c] = o.e1[c] = o.c16[c] = 0u;
    if (o.cst) {
        const uint32_t err[4] = {0xFFFFu, 0u, 0xFFFFu, 0xFFFFu};  // error colour (1, 0, 1, 1)
        // A valid void extent carries RGBA UNORM16 in bits 64..127.
        bool valid_void = false;
        if ((blk.x & 0x1FF) == 0x1FC) {
            const uint32_t s0 = static_cast<uint32_t>(lo >> 12) & 0x1FFF, s1 = static_cast<uint32_t>(lo >> 25) & 0x1FFF;
            const uint32_t t0 = static_cast<uint32_t>(lo >> 38) & 0x1FFF, t1 = static_cast<uint32_t>(lo >> 51) & 0x1FFF;
            const bool all_ones = (s0 & s1 & t0 & t1) == 0x1FFF;
            valid_void = !(blk.x & 0x200) && ((blk.x >> 10) & 3) == 3 && (all_ones || (s0 < s1 && t0 < t1));
        }
        o.c16[0] = valid_void ? (blk.z & 0xFFFFu) : err[0];
        o.c16[1] = valid_void ? (blk.z >> 16) : err[1];
        o.c16[2] = valid_void ? (blk.w & 0xFFFFu) : err[2];
        o.c16[3] = valid_void ? (blk.w >> 16) : err[3];
        return;
    }
    const int parts = static_cast<int>((lo >> 11) & 3) + 1;
    {
        const int cstart = parts == 1 ? 17 : 29;
        uint64_t clo = window_u128(lo, hi, cstart);
        uint64_t chi = hi >> cstart;
        mask_u128(clo, chi, bise_stream_bits_dev(8 * parts, cq));
        color_values(clo, chi, cq, 8 * parts, codes, nt);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        if (q < parts) {
            int v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = codes[(8 * q + k) * nt];
            int a[4], b[4];
            if (v[1] + v[3] + v[5] >= v[0] + v[2] + v[4]) {
                a[0] = v[0]; a[1] = v[2]; a[2] = v[4]; a[3] = v[6];
                b[0] = v[1]; b[1] = v[3]; b[2] = v[5]; b[3] = v[7];
            } else {  // blue contraction, endpoints swapped
                a[0] = (v[1] + v[5]) >> 1; a[1] = (v[3] + v[5]) >> 1; a[2] = v[5]; a[3] = v[7];
                b[0] = (v[0] + v[4]) >> 1; b[1] = (v[2] + v[4]) >> 1; b[2] = v[4]; b[3] = v[6];
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                o.e0[c] |= static_cast<uint32_t>(a[c]) << (8 * q);
                o.e1[c] |= static_cast<uint32_t>(b[c]) << (8 * q);
            }
        }
    }
    if (parts > 1) o.pat = __ldg(&T.part[footprint_index(4)][parts - 2][(lo >> 13) & 0x3FF][0]);
    uint64_t s0 = __brevll(hi), s1 = __brevll(lo);
    mask_u128(s0, s1, mode_wbits(me));
    weight_codes(s0, s1, mode_wq(me), 16, codes, nt);
}

// The four channels of texel t of a fast / constant RGBA block as 2^16 times
// their unit values (the fp16 view of C as an integer-valued float, 65535 ->
// 65536): the weight once per texel, each channel's endpoint bytes of the
// texel's partition by one byte permute (selector nibbles 4 pick zero bytes).
__device__ __forceinline__ void rgba_t4(const RgbaOut& o, const uint8_t* codes, int nt, int t, float (&tv)[4]) {
    const uint32_t sel = ((o.pat >> (2 * t)) & 3u) | 0x4440u;
    const uint32_t w = __ldg(o.wun + codes[t * nt]);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t e0 = __byte_perm(o.e0[c], 0u, sel), e1 = __byte_perm(o.e1[c], 0u, sel);
        const uint32_t X = e0 * (64u - w) + e1 * w;
        const uint32_t c16 = o.cst ? o.c16[c] : 4u * X + ((X + 32u) >> 6);
        tv[c] = __int_as_float(__float_as_int(static_cast<float>(c16 + (c16 == 0xFFFFu))) & 0xFFFFE000);
    }
}

}  // namespace fast
}  // namespace akv
