// sm_100a software ASTC LDR decoder (device side).
//
// B200 has no ASTC texture hardware, so blocks are decoded with integer ALU
// work in two stages that every kernel in this library shares:
//
//   Stage A, one thread per 16-byte block (`decode_header`): block mode,
//   partition count/seed, colour endpoint modes, BISE colour integers ->
//   8-bit endpoint pairs per partition, BISE weight integers -> unquantised
//   0..64 grid weights. Results land in a `BlockDesc` plus a 64-byte weight
//   array in shared memory.
//
//   Stage B, one thread per texel (`texel_c16`): partition from the
//   precomputed pattern table, weight (direct or bilinear infill), endpoint
//   interpolation to the 16-bit value C.
//
// Views of C (the values the reference's astcenc F32 output carries, see
// astc_kv/bridge.cpp:27-35): UNORM8 = C >> 8; fp16 = 1.0 for C == 65535,
// otherwise C/65536 truncated to fp16.
//
// Illegal encodings (reserved modes, over-long weight/colour streams, HDR
// endpoint modes or HDR void-extent in this LDR profile, malformed
// void-extent) decode to the error colour: magenta (1, 0, 1, 1).
#pragma once
#include <cstdint>

#include "akv_tables.h"

namespace akv {

// The decode tables, in static device memory of the (single) translation
// unit that includes this header; akv_cuda_init fills them per device.
__device__ Tables g_akv_tables;

// BlockDesc.info layout.
enum : uint32_t {
    kInfoParts = 0,     // 2 bits: partition count - 1
    kInfoVoid = 2,      // 1 bit: void-extent block (ep holds UNORM16 colours)
    kInfoDual = 3,      // 1 bit
    kInfoCcs = 4,       // 2 bits: channel on plane 1
    kInfoReduced = 6,   // 1 bit: weight grid smaller than the footprint
    kInfoWx = 8,        // 4 bits
    kInfoWy = 12,       // 4 bits
    kInfoError = 16,    // 1 bit: decoded as the error colour
};

// NCH = channels the caller needs (1: R only, as in the scalar layout; 4: RGBA).
template <int NCH>
struct BlockDesc {
    uint32_t pat[2];        // 2-bit partition per texel (texels 0..31; enough for <= 6x6)
    uint32_t pat_hi[2];     // texels 32..63 (8x8)
    uint32_t ep[4 * NCH];   // per partition/channel: e0 | e1 << 8, or UNORM16 colour when void
    uint32_t info;
};

__device__ __forceinline__ uint32_t bits_u128(uint64_t lo, uint64_t hi, int pos, int n) {
    // n <= 32, 0 <= pos < 128
    uint64_t w = pos >= 64 ? (hi >> (pos - 64)) : (pos == 0 ? lo : ((lo >> pos) | (hi << (64 - pos))));
    return static_cast<uint32_t>(w) & (n >= 32 ? 0xFFFFFFFFu : ((1u << n) - 1u));
}

__device__ __forceinline__ uint64_t window_u128(uint64_t lo, uint64_t hi, int pos) {
    // 64 bits starting at pos (bits past 127 read as zero)
    if (pos == 0) return lo;
    if (pos >= 64) return pos >= 128 ? 0ull : (hi >> (pos - 64));
    return (lo >> pos) | (hi << (64 - pos));
}

// Keep only bits [0, n) of a 128-bit value.
__device__ __forceinline__ void mask_u128(uint64_t& lo, uint64_t& hi, int n) {
    if (n <= 0) { lo = hi = 0; return; }
    if (n < 64) { lo &= (1ull << n) - 1ull; hi = 0; return; }
    if (n == 64) { hi = 0; return; }
    if (n < 128) hi &= (1ull << (n - 64)) - 1ull;
}

// BISE weight codes: `count` values of range wq from the bit-reversed weight
// stream (s0, s1), already masked to its length, into codes[i * nt] (UNQ:
// the unquantised weights un[code] instead). Groups of five (trits, plain
// bits) or three (quints) values per step, with the trit/quint block bits
// gathered by runtime shifts and decoded through the combined digit table.
// Every step stores five codes without predicates: a quint step's two extra
// codes are overwritten by the next step, and the last step may write up to
// four rows past `count` (the caller provides kCodePad rows of slack). Every
// code a step forms, the extra ones included, lies inside its range's row of
// the unquantisation table.
constexpr int kCodePad = 4;

template <bool UNQ = false>
__device__ __forceinline__ void weight_codes(uint64_t s0, uint64_t s1, int wq, int count, uint8_t* codes, int nt,
                                             const uint8_t* un = nullptr) {
    const Tables& T = g_akv_tables;
    const uint32_t shp = __ldg(&T.shape[wq]);
    const int b = shp & 15;
    const bool tr = (shp >> 4) & 1, qu = (shp >> 5) & 1;
    const int gs = qu ? 3 : 5;
    const int gb = tr ? 5 * b + 8 : (qu ? 3 * b + 7 : 5 * b);
    const int ng = qu ? (count + 2) / 3 : (count + 4) / 5;
    // Masks of the trit / quint block bits after shifting by k * b.
    const uint32_t m1 = tr ? 0x03u : (qu ? 0x07u : 0u);
    const uint32_t m2 = tr ? 0x0Cu : (qu ? 0x18u : 0u);
    const uint32_t m3 = tr ? 0x10u : (qu ? 0x60u : 0u);
    const uint32_t m4 = tr ? 0x60u : 0u;
    const uint32_t m5 = tr ? 0x80u : 0u;
    // Offsets of the low bits of values 1..4 within a group.
    const int o1 = b + (tr ? 2 : (qu ? 3 : 0));
    const int o2 = 2 * b + (tr ? 4 : (qu ? 5 : 0));
    const int o3 = 3 * b + (tr ? 5 : 0);
    const int o4 = 4 * b + (tr ? 7 : 0);
    const int b2 = 2 * b, b3 = 3 * b, b4 = 4 * b, b5 = 5 * b;
    const uint16_t* dig = T.dig3 + (qu ? 256 : 0);
    const uint32_t bm = (1u << b) - 1u, km = 7u << b;
    // The stream as four 32-bit words, shifted down by `gb` per step.
    uint32_t w0 = static_cast<uint32_t>(s0), w1 = static_cast<uint32_t>(s0 >> 32);
    uint32_t w2 = static_cast<uint32_t>(s1), w3 = static_cast<uint32_t>(s1 >> 32);
    uint8_t* cp = codes;
    const int step = gs * nt;
    for (int g = 0; g < ng; ++g) {
        const uint32_t win = w0;
        const uint32_t X = ((win >> b) & m1) | ((win >> b2) & m2) | ((win >> b3) & m3) | ((win >> b4) & m4) |
                           ((win >> b5) & m5);
        const uint32_t dgb = static_cast<uint32_t>(__ldg(dig + X)) << b;
        const uint32_t c0 = (dgb & km) | (win & bm);
        const uint32_t c1 = ((dgb >> 3) & km) | ((win >> o1) & bm);
        const uint32_t c2 = ((dgb >> 6) & km) | ((win >> o2) & bm);
        const uint32_t c3 = ((dgb >> 9) & km) | ((win >> o3) & bm);
        const uint32_t c4 = ((dgb >> 12) & km) | ((win >> o4) & bm);
        if constexpr (UNQ) {
            cp[0] = __ldg(un + c0);
            cp[nt] = __ldg(un + c1);
            cp[2 * nt] = __ldg(un + c2);
            cp[3 * nt] = __ldg(un + c3);
            cp[4 * nt] = __ldg(un + c4);
        } else {
            cp[0] = static_cast<uint8_t>(c0);
            cp[nt] = static_cast<uint8_t>(c1);
            cp[2 * nt] = static_cast<uint8_t>(c2);
            cp[3 * nt] = static_cast<uint8_t>(c3);
            cp[4 * nt] = static_cast<uint8_t>(c4);
        }
        cp += step;
        w0 = __funnelshift_r(w0, w1, gb);
        w1 = __funnelshift_r(w1, w2, gb);
        w2 = __funnelshift_r(w2, w3, gb);
        w3 >>= gb;
    }
}

// Number of bits in a BISE stream (device copy of bise_stream_bits).
__device__ __forceinline__ int bise_stream_bits_dev(int count, int q) {
    const uint32_t shp = __ldg(&g_akv_tables.shape[q]);
    const int b = shp & 15;
    return count * b + (((shp >> 4) & 1) ? (8 * count + 4) / 5 : 0) + (((shp >> 5) & 1) ? (7 * count + 2) / 3 : 0);
}

// The first nv colour integers of range cq from the colour stream (s0, s1),
// masked to its length, unquantised to 0..255 into out[j * nt]: one runtime
// step loop for trit, quint and plain-bit ranges alike (64-bit windows:
// colour groups reach 40 bits). Writes up to four values past nv (callers
// have the slack).
__device__ __forceinline__ void color_values(uint64_t s0, uint64_t s1, int cq, int nv, uint8_t* out, int nt) {
    const Tables& T = g_akv_tables;
    const uint32_t shp = __ldg(&T.shape[cq]);
    const int b = shp & 15;
    const bool tr = (shp >> 4) & 1, qu = (shp >> 5) & 1;
    const int gs = qu ? 3 : 5;
    const int gb = tr ? 5 * b + 8 : (qu ? 3 * b + 7 : 5 * b);
    const int ng = qu ? (nv + 2) / 3 : (nv + 4) / 5;
    const uint64_t m1 = tr ? 0x03u : (qu ? 0x07u : 0u);
    const uint64_t m2 = tr ? 0x0Cu : (qu ? 0x18u : 0u);
    const uint64_t m3 = tr ? 0x10u : (qu ? 0x60u : 0u);
    const uint64_t m4 = tr ? 0x60u : 0u;
    const uint64_t m5 = tr ? 0x80u : 0u;
    const int o1 = b + (tr ? 2 : (qu ? 3 : 0));
    const int o2 = 2 * b + (tr ? 4 : (qu ? 5 : 0));
    const int o3 = 3 * b + (tr ? 5 : 0);
    const int o4 = 4 * b + (tr ? 7 : 0);
    const uint16_t* dig = T.dig3 + (qu ? 256 : 0);
    const uint8_t* un = T.cunq[cq];
    const uint64_t bm = (1ull << b) - 1ull;
    uint8_t* cp = out;
    for (int g = 0; g < ng; ++g) {
        const uint64_t win = s0;
        const uint32_t X = static_cast<uint32_t>(((win >> b) & m1) | ((win >> (2 * b)) & m2) |
                                                 ((win >> (3 * b)) & m3) | ((win >> (4 * b)) & m4) |
                                                 ((win >> (5 * b)) & m5));
        const uint32_t dg = __ldg(dig + X);
        cp[0] = __ldg(un + (((dg & 7u) << b) | static_cast<uint32_t>(win & bm)));
        cp[nt] = __ldg(un + ((((dg >> 3) & 7u) << b) | static_cast<uint32_t>((win >> o1) & bm)));
        cp[2 * nt] = __ldg(un + ((((dg >> 6) & 7u) << b) | static_cast<uint32_t>((win >> o2) & bm)));
        cp[3 * nt] = __ldg(un + ((((dg >> 9) & 7u) << b) | static_cast<uint32_t>((win >> o3) & bm)));
        cp[4 * nt] = __ldg(un + ((((dg >> 12) & 7u) << b) | static_cast<uint32_t>((win >> o4) & bm)));
        cp += gs * nt;
        s0 = (s0 >> gb) | (s1 << (64 - gb));
        s1 >>= gb;
    }
}

__device__ __forceinline__ int clamp8(int v) { return v < 0 ? 0 : (v > 255 ? 255 : v); }

// Signed bit transfer between a (offset) and b (base), spec form.
__device__ __forceinline__ void bit_xfer(int& a, int& b) {
    b = (b >> 1) | (a & 0x80);
    a = (a >> 1) & 0x3F;
    if (a & 0x20) a -= 0x40;
}

// LDR endpoint modes -> 8-bit endpoint pair per channel, from the mode's
// colour integers v[0..]. Returns false for HDR modes (2, 3, 7, 11, 14, 15).
__device__ __forceinline__ bool endpoints(int cem, const uint8_t* v, int (&e0)[4], int (&e1)[4]) {
    switch (cem) {
        case 0:
            e0[0] = e0[1] = e0[2] = v[0]; e1[0] = e1[1] = e1[2] = v[1]; e0[3] = e1[3] = 255;
            return true;
        case 1: {
            const int l0 = (v[0] >> 2) | (v[1] & 0xC0);
            const int l1 = min(l0 + (v[1] & 0x3F), 255);
            e0[0] = e0[1] = e0[2] = l0; e1[0] = e1[1] = e1[2] = l1; e0[3] = e1[3] = 255;
            return true;
        }
        case 4:
            e0[0] = e0[1] = e0[2] = v[0]; e1[0] = e1[1] = e1[2] = v[1]; e0[3] = v[2]; e1[3] = v[3];
            return true;
        case 5: {
            int a0 = v[1], b0 = v[0], a1 = v[3], b1 = v[2];
            bit_xfer(a0, b0);
            bit_xfer(a1, b1);
            e0[0] = e0[1] = e0[2] = b0; e0[3] = b1;
            e1[0] = e1[1] = e1[2] = clamp8(b0 + a0); e1[3] = clamp8(b1 + a1);
            return true;
        }
        case 6:
        case 10:
#pragma unroll
            for (int c = 0; c < 3; ++c) { e0[c] = (v[c] * v[3]) >> 8; e1[c] = v[c]; }
            e0[3] = cem == 10 ? v[4] : 255;
            e1[3] = cem == 10 ? v[5] : 255;
            return true;
        case 8:
        case 12: {
            const int a0 = cem == 12 ? v[6] : 255, a1 = cem == 12 ? v[7] : 255;
            if (v[1] + v[3] + v[5] >= v[0] + v[2] + v[4]) {
                e0[0] = v[0]; e0[1] = v[2]; e0[2] = v[4]; e0[3] = a0;
                e1[0] = v[1]; e1[1] = v[3]; e1[2] = v[5]; e1[3] = a1;
            } else {  // blue contraction, endpoints swapped
                e0[0] = (v[1] + v[5]) >> 1; e0[1] = (v[3] + v[5]) >> 1; e0[2] = v[5]; e0[3] = a1;
                e1[0] = (v[0] + v[4]) >> 1; e1[1] = (v[2] + v[4]) >> 1; e1[2] = v[4]; e1[3] = a0;
            }
            return true;
        }
        case 9:
        case 13: {
            int o[4], bse[4];
#pragma unroll
            for (int c = 0; c < 3; ++c) { o[c] = v[2 * c + 1]; bse[c] = v[2 * c]; bit_xfer(o[c], bse[c]); }
            if (cem == 13) { o[3] = v[7]; bse[3] = v[6]; bit_xfer(o[3], bse[3]); }
            else { o[3] = 0; bse[3] = 255; }
            int lo[4], hi[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) { lo[c] = bse[c]; hi[c] = bse[c] + o[c]; }
            if (o[0] + o[1] + o[2] < 0) {  // blue contraction, endpoints swapped
                int t[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) { t[c] = hi[c]; hi[c] = lo[c]; lo[c] = t[c]; }
                lo[0] = (lo[0] + lo[2]) >> 1; lo[1] = (lo[1] + lo[2]) >> 1;
                hi[0] = (hi[0] + hi[2]) >> 1; hi[1] = (hi[1] + hi[2]) >> 1;
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) { e0[c] = clamp8(lo[c]); e1[c] = clamp8(hi[c]); }
            return true;
        }
        default:
            return false;
    }
}

// Stage A. `blk` is the raw 16-byte block; `fp` the footprint index (0/1/2 for
// 4x4/6x6/8x8). Writes `d` and the unquantised grid weights `w` (plane
// interleaved, up to 64 entries); `w` needs 64 + kCodePad bytes.
template <int NCH>
__device__ __forceinline__ void decode_header(uint4 blk, int fp, BlockDesc<NCH>& d, uint8_t* w) {
    const Tables& T = g_akv_tables;
    const uint64_t lo = (static_cast<uint64_t>(blk.y) << 32) | blk.x;
    const uint64_t hi = (static_cast<uint64_t>(blk.w) << 32) | blk.z;
    const int mode = static_cast<int>(lo & 0x7FF);

    auto set_error = [&]() {
        d.info = (1u << kInfoError);
        d.pat[0] = d.pat[1] = d.pat_hi[0] = d.pat_hi[1] = 0;
#pragma unroll
        for (int c = 0; c < NCH; ++c) d.ep[c] = (c == 1) ? 0u : 0xFFFFu;  // e0 = e1 = 255 or 0
        w[0] = 0;
    };

    if ((mode & 0x1FF) == 0x1FC) {
        // Void extent: bit 9 = HDR (error here), bits 10..11 reserved = 1,
        // four 13-bit extent coordinates, then RGBA UNORM16 at bits 64..127.
        const uint32_t s0 = bits_u128(lo, hi, 12, 13), s1 = bits_u128(lo, hi, 25, 13);
        const uint32_t t0 = bits_u128(lo, hi, 38, 13), t1 = bits_u128(lo, hi, 51, 13);
        const bool all_ones = (s0 & s1 & t0 & t1) == 0x1FFF;
        if ((mode & 0x200) || ((lo >> 10) & 3) != 3 || (!all_ones && (s0 >= s1 || t0 >= t1))) { set_error(); return; }
        d.info = (1u << kInfoVoid);
        d.pat[0] = d.pat[1] = d.pat_hi[0] = d.pat_hi[1] = 0;
#pragma unroll
        for (int c = 0; c < NCH; ++c) d.ep[c] = static_cast<uint32_t>((hi >> (16 * c)) & 0xFFFF);
        w[0] = 0;
        return;
    }

    const uint32_t me = __ldg(&T.mode[fp][mode]);
    if (!(me & kModeValid)) { set_error(); return; }
    const int dual = (me & kModeDual) ? 1 : 0;
    const int wq = mode_wq(me), wx = mode_wx(me), wy = mode_wy(me), wbits = mode_wbits(me);
    const int parts = static_cast<int>((lo >> 11) & 3) + 1;
    if (dual && parts == 4) { set_error(); return; }

    const int top = 128 - wbits - 2 * dual;  // first bit above the colour data
    // Endpoint modes of partitions 0..3, four bits each (no array: the
    // partition loop below indexes them at run time).
    uint32_t cems;
    int cstart, extra = 0, seed = 0;
    if (parts == 1) {
        cems = static_cast<uint32_t>((lo >> 13) & 15);
        cstart = 17;
    } else {
        seed = static_cast<int>((lo >> 13) & 0x3FF);
        const int field = static_cast<int>((lo >> 23) & 0x3F);
        cstart = 29;
        if ((field & 3) == 0) {
            cems = static_cast<uint32_t>(field >> 2) * 0x1111u;
        } else {
            extra = 3 * parts - 4;
            const int all = (field >> 2) | (static_cast<int>(bits_u128(lo, hi, top - extra, extra)) << 4);
            const int cls = (field & 3) - 1;
            cems = 0u;
#pragma unroll
            for (int p = 0; p < 4; ++p)
                cems |= static_cast<uint32_t>(((cls + ((all >> p) & 1)) << 2) | ((all >> (parts + 2 * p)) & 3))
                        << (4 * p);
        }
    }
    int npairs = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p)
        if (p < parts) npairs += static_cast<int>((cems >> (4 * p + 2)) & 3u) + 1;
    const int avail = top - extra - cstart;
    if (npairs > 9 || avail < 0) { set_error(); return; }
    const int cq = T.cquant[npairs][avail];
    if (cq == 0xFF) { set_error(); return; }

    // Colour integers, unquantised, into w[0 .. 2 npairs) (at most 18 values
    // plus 4 of slack; the weights overwrite them below).
    {
        uint64_t clo = window_u128(lo, hi, cstart);
        uint64_t chi = hi >> cstart;
        mask_u128(clo, chi, bise_stream_bits_dev(2 * npairs, cq));
        color_values(clo, chi, cq, 2 * npairs, w, 1);
    }
    // Endpoints: each partition's pair per channel, packed as the bytes of
    // e0p[c] / e1p[c] (byte p = partition p).
    uint32_t e0p[NCH], e1p[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) e0p[c] = e1p[c] = 0u;
    {
        int k = 0;
        for (int p = 0; p < parts; ++p) {
            const int cem = static_cast<int>((cems >> (4 * p)) & 15u);
            int e0[4], e1[4];
            if (!endpoints(cem, w + k, e0, e1)) { set_error(); return; }
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                e0p[c] |= static_cast<uint32_t>(e0[c]) << (8 * p);
                e1p[c] |= static_cast<uint32_t>(e1[c]) << (8 * p);
            }
            k += 2 * ((cem >> 2) + 1);
        }
    }

    // Weights: the stream runs downward from bit 127; bit-reverse the block.
    // Unquantised five per step (writes up to kCodePad bytes past n).
    {
        uint64_t wlo = __brevll(hi), whi = __brevll(lo);
        mask_u128(wlo, whi, wbits);
        const int n = wx * wy * (dual + 1);
        weight_codes<true>(wlo, whi, wq, n, w, 1, T.wunq[wq]);
    }

    const int ccs = dual ? static_cast<int>(bits_u128(lo, hi, 128 - wbits - 2, 2)) : 0;
    d.info = static_cast<uint32_t>(parts - 1) | (dual << kInfoDual) | (ccs << kInfoCcs) |
             ((me & kModeReduced) ? (1u << kInfoReduced) : 0u) | (wx << kInfoWx) | (wy << kInfoWy);
    if (parts > 1) {
        const uint32_t* pt = T.part[fp][parts - 2][seed];
        d.pat[0] = __ldg(pt + 0); d.pat[1] = __ldg(pt + 1);
        d.pat_hi[0] = __ldg(pt + 2); d.pat_hi[1] = __ldg(pt + 3);
    } else {
        d.pat[0] = d.pat[1] = d.pat_hi[0] = d.pat_hi[1] = 0;
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int c = 0; c < NCH; ++c)
            d.ep[p * NCH + c] = (p < parts) ? (((e0p[c] >> (8 * p)) & 0xFFu) | (((e1p[c] >> (8 * p)) & 0xFFu) << 8))
                                            : 0u;
}


// Stage B: 16-bit values C of texel (x, y) for the NCH channels the
// descriptor holds (channel c of the descriptor is RGBA channel c).
template <int BS, int NCH>
__device__ __forceinline__ void texel_values(const BlockDesc<NCH>& d, const uint8_t* w, int x, int y, uint32_t* out) {
    const uint32_t info = d.info;
    if (info & (1u << kInfoVoid)) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) out[c] = d.ep[c];
        return;
    }
    const int t = y * BS + x;
    int part = 0;
    if (info & 3u) {
        const uint32_t word = t < 16 ? d.pat[0] : t < 32 ? d.pat[1] : t < 48 ? d.pat_hi[0] : d.pat_hi[1];
        part = (word >> (2 * (t & 15))) & 3;
    }
    const int dual = (info >> kInfoDual) & 1;
    const int ccs = (info >> kInfoCcs) & 3;
    int wt0 = 0, wt1 = 0;
    if (info & (1u << kInfoError)) {
        wt0 = wt1 = 0;
    } else if (!(info & (1u << kInfoReduced))) {
        wt0 = w[t << dual];
        wt1 = dual ? w[(t << 1) + 1] : wt0;
    } else {
        const int wx = (info >> kInfoWx) & 15, wy = (info >> kInfoWy) & 15;
        constexpr int kDs = (1024 + BS / 2) / (BS - 1);
        const int gs = (kDs * x * (wx - 1) + 32) >> 6;
        const int gt = (kDs * y * (wy - 1) + 32) >> 6;
        const int js = gs >> 4, fs = gs & 15, jt = gt >> 4, ft = gt & 15;
        const int w11 = (fs * ft + 8) >> 4;
        const int f00 = 16 - fs - ft + w11, f01 = fs - w11, f10 = ft - w11;
        const int i00 = js + jt * wx;
        const bool has_x = js + 1 < wx, has_y = jt + 1 < wy;
#pragma unroll
        for (int pl = 0; pl < 2; ++pl) {
            if (pl == 1 && !dual) { wt1 = wt0; break; }
            const int p00 = w[(i00 << dual) + pl];
            const int p01 = has_x ? w[((i00 + 1) << dual) + pl] : 0;
            const int p10 = has_y ? w[((i00 + wx) << dual) + pl] : 0;
            const int p11 = (has_x && has_y) ? w[((i00 + wx + 1) << dual) + pl] : 0;
            const int v = (p00 * f00 + p01 * f01 + p10 * f10 + p11 * w11 + 8) >> 4;
            if (pl == 0) wt0 = v; else wt1 = v;
        }
    }
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int wt = (dual && ccs == c) ? wt1 : wt0;
        const uint32_t ep = d.ep[part * NCH + c];
        const int e0 = ep & 0xFF, e1 = (ep >> 8) & 0xFF;
        // C = ((e0*257)*(64-w) + (e1*257)*w + 32) >> 6 = 4X + ((X + 32) >> 6),
        // with X = e0*(64-w) + e1*w.
        const int X = e0 * (64 - wt) + e1 * wt;
        out[c] = static_cast<uint32_t>(4 * X + ((X + 32) >> 6));
    }
}

// Partition bits of texel row y (2 bits per texel, texel x at bit 2x) from
// the four pattern words of a block (texels 0..15, 16..31, 32..47, 48..63).
template <int BS>
__device__ __forceinline__ uint32_t row_pattern(uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3, int y) {
    const int b = 2 * BS * y;
    const int k = b >> 5;
    const uint32_t lo = k == 0 ? p0 : (k == 1 ? p1 : (k == 2 ? p2 : p3));
    const uint32_t hi = k == 0 ? p1 : (k == 1 ? p2 : p3);
    return __funnelshift_r(lo, hi, static_cast<uint32_t>(b & 31));
}

// Stage B by rows: the 16-bit values C of the BS texels of row y for the NCH
// channels (out[x][c]), each equal to what texel_values gives for that
// texel. The row's partition bits and, for a reduced grid, its grid row and
// t fraction are found once; the per-axis tap table Tables::sep gives the
// column taps (the spec computes the s and t grid coordinates separately).
template <int BS, int NCH>
__device__ __forceinline__ void texel_row(const BlockDesc<NCH>& d, const uint8_t* w, int y,
                                          uint32_t (&out)[BS][NCH]) {
    constexpr int fp = footprint_index(BS);
    const uint32_t info = d.info;
    if (info & (1u << kInfoVoid)) {
#pragma unroll
        for (int x = 0; x < BS; ++x)
#pragma unroll
            for (int c = 0; c < NCH; ++c) out[x][c] = d.ep[c];
        return;
    }
    const uint32_t prow = (info & 3u) ? row_pattern<BS>(d.pat[0], d.pat[1], d.pat_hi[0], d.pat_hi[1], y) : 0u;
    const int dual = (info >> kInfoDual) & 1;
    const int ccs = (info >> kInfoCcs) & 3;
    const bool err = (info >> kInfoError) & 1;
    const bool red = (info >> kInfoReduced) & 1;
    const int wx = (info >> kInfoWx) & 15, wy = (info >> kInfoWy) & 15;
    int jt = y, ft = 0;
    uint32_t tx[4] = {0u, 0u, 0u, 0u};
    if (red && !err) {
        const uint32_t e = __ldg(&g_akv_tables.sep[fp][wy - 2][y]);
        jt = static_cast<int>(e & 15u);
        ft = static_cast<int>(e >> 8);
        const uint4 r = __ldg(reinterpret_cast<const uint4*>(g_akv_tables.sep[fp][wx - 2]));
        tx[0] = r.x; tx[1] = r.y; tx[2] = r.z; tx[3] = r.w;
    }
    const bool has_y = jt + 1 < wy;
#pragma unroll
    for (int x = 0; x < BS; ++x) {
        int wt0 = 0, wt1 = 0;
        if (err) {
        } else if (!red) {
            const int t = y * BS + x;
            wt0 = w[t << dual];
            wt1 = dual ? w[(t << 1) + 1] : wt0;
        } else {
            const uint32_t e = (tx[x >> 1] >> (16 * (x & 1))) & 0xFFFFu;
            const int js = static_cast<int>(e & 15u), fs = static_cast<int>(e >> 8);
            const int w11 = (fs * ft + 8) >> 4;
            const int f00 = 16 - fs - ft + w11, f01 = fs - w11, f10 = ft - w11;
            const int i00 = js + jt * wx;
            const bool has_x = js + 1 < wx;
#pragma unroll
            for (int pl = 0; pl < 2; ++pl) {
                if (pl == 1 && !dual) { wt1 = wt0; break; }
                const int p00 = w[(i00 << dual) + pl];
                const int p01 = has_x ? w[((i00 + 1) << dual) + pl] : 0;
                const int p10 = has_y ? w[((i00 + wx) << dual) + pl] : 0;
                const int p11 = (has_x && has_y) ? w[((i00 + wx + 1) << dual) + pl] : 0;
                const int v = (p00 * f00 + p01 * f01 + p10 * f10 + p11 * w11 + 8) >> 4;
                if (pl == 0) wt0 = v; else wt1 = v;
            }
        }
        const int part = static_cast<int>((prow >> (2 * x)) & 3u);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const int wt = (dual && ccs == c) ? wt1 : wt0;
            const uint32_t ep = d.ep[part * NCH + c];
            const int X = static_cast<int>(ep & 0xFF) * (64 - wt) + static_cast<int>((ep >> 8) & 0xFF) * wt;
            out[x][c] = static_cast<uint32_t>(4 * X + ((X + 32) >> 6));
        }
    }
}

// fp16 view of C as float (exact): 1.0 for 65535, else C/65536 truncated to 11
// significant bits.
__device__ __forceinline__ float c16_to_unit(uint32_t c) {
    const float f = __int_as_float(__float_as_int(static_cast<float>(c)) & 0xFFFFE000) * 0x1p-16f;
    return c == 0xFFFFu ? 1.0f : f;
}


}  // namespace akv
