// TEST INFRASTRUCTURE ONLY. Compiles the product's device-side ASTC decoder
// (astc-kv_b200/csrc/akv_astc_device.cuh) as plain host C++ so CPU tests can
// compare its stage A/B logic with the oracle bit for bit before any GPU run.
// Nothing in the product loads this library.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <cmath>
#include <vector_types.h>

#define __device__
#define __host__
#define __forceinline__ inline
#define __global__
template <class T>
inline T __ldg(const T* p) { return *p; }
inline unsigned long long __brevll(unsigned long long x) {
    unsigned long long r = 0;
    for (int i = 0; i < 64; ++i) r |= ((x >> i) & 1ull) << (63 - i);
    return r;
}
inline unsigned __funnelshift_r(unsigned lo, unsigned hi, unsigned s) {
    s &= 31;
    return s ? (lo >> s) | (hi << (32 - s)) : lo;
}
// Byte permute with plain-copy selector nibbles (0..7), the only form the
// decoder uses: result byte n = byte (s >> 4n) & 7 of the 8 bytes {hi, lo}.
inline unsigned __byte_perm(unsigned lo, unsigned hi, unsigned s) {
    const unsigned long long v = (static_cast<unsigned long long>(hi) << 32) | lo;
    unsigned r = 0;
    for (int n = 0; n < 4; ++n) r |= static_cast<unsigned>((v >> (8 * ((s >> (4 * n)) & 7))) & 0xFF) << (8 * n);
    return r;
}
inline float __int_as_float(int i) { float f; std::memcpy(&f, &i, 4); return f; }
inline int __float_as_int(float f) { int i; std::memcpy(&i, &f, 4); return i; }
using std::max;
using std::min;

#include <cuda_fp16.h>
#include <cmath>
using std::fmaf;
inline float __uint_as_float(unsigned int i) { float f; std::memcpy(&f, &i, 4); return f; }
inline unsigned int __float_as_uint(float f) { unsigned int i; std::memcpy(&i, &f, 4); return i; }
#include "../../astc-kv_b200/csrc/akv_astc_device.cuh"
#include "../../astc-kv_b200/csrc/akv_decode_fast.cuh"

extern "C" int emu_decode_blocks_u16(const uint8_t* blocks, int64_t n, int bs, uint16_t* out) {
    static bool ready = false;
    if (!ready) { akv::build_tables(&akv::g_akv_tables); ready = true; }
    const int fp = akv::footprint_index(bs);
    if (fp < 0) return 1;
    for (int64_t i = 0; i < n; ++i) {
        uint4 b;
        std::memcpy(&b, blocks + 16 * i, 16);
        akv::BlockDesc<4> d;
        uint8_t w[64 + akv::kCodePad];
        std::memset(w, 0, sizeof(w));
        akv::decode_header<4>(b, fp, d, w);
        for (int y = 0; y < bs; ++y)
            for (int x = 0; x < bs; ++x) {
                uint32_t c[4];
                switch (bs) {
                    case 4: akv::texel_values<4, 4>(d, w, x, y, c); break;
                    case 6: akv::texel_values<6, 4>(d, w, x, y, c); break;
                    default: akv::texel_values<8, 4>(d, w, x, y, c); break;
                }
                for (int k = 0; k < 4; ++k) out[((i * bs + y) * bs + x) * 4 + k] = static_cast<uint16_t>(c[k]);
            }
    }
    return 0;
}

// The standalone decoder's row stage (texel_row): UNORM16 RGBA per texel,
// out[n][bs][bs][4], as emu_decode_blocks_u16 but a texel row at a time.
template <int BS>
static void rows_one(const akv::BlockDesc<4>& d, const uint8_t* w, uint16_t* o) {
    for (int y = 0; y < BS; ++y) {
        uint32_t c[BS][4];
        akv::texel_row<BS, 4>(d, w, y, c);
        for (int x = 0; x < BS; ++x)
            for (int k = 0; k < 4; ++k) o[(y * BS + x) * 4 + k] = static_cast<uint16_t>(c[x][k]);
    }
}

extern "C" int emu_decode_rows_u16(const uint8_t* blocks, int64_t n, int bs, uint16_t* out) {
    static bool ready = false;
    if (!ready) { akv::build_tables(&akv::g_akv_tables); ready = true; }
    const int fp = akv::footprint_index(bs);
    if (fp < 0) return 1;
    for (int64_t i = 0; i < n; ++i) {
        uint4 b;
        std::memcpy(&b, blocks + 16 * i, 16);
        akv::BlockDesc<4> d;
        uint8_t w[64 + akv::kCodePad];
        std::memset(w, 0xEE, sizeof(w));  // unwritten weights must not matter
        akv::decode_header<4>(b, fp, d, w);
        uint16_t* o = out + i * bs * bs * 4;
        if (bs == 4) rows_one<4>(d, w, o);
        else if (bs == 6) rows_one<6>(d, w, o);
        else rows_one<8>(d, w, o);
    }
    return 0;
}

extern "C" float emu_unit(uint32_t c) { return akv::c16_to_unit(c); }

// The per-block runtime path of the attention kernel's plane decode
// (akv_decode_fast.cuh): block kind, then table / constant blocks (value table
// + weight codes, or per-texel endpoint/weight evaluation for 4x4, read back as
// the kernel's tile writer reads them) or
// descriptor blocks (grid weights expanded, then evaluated a row or pair of
// texels at a time, as the kernel's phases 1a / 1b do).
// Generic blocks are evaluated as the kernel's phase 1b does. Returns the
// fp16-view values of the R channel per texel; `cls` gets the kind.
template <int BS>
static int fast_r_one(uint4 b, int* kind_out, float* out) {
    namespace F = akv::fast;
    constexpr int N = BS * BS;
    uint32_t me;
    int cq;
    const int kind = F::block_kind<BS>(b, me, cq);
    *kind_out = kind;
    if (kind == F::kKindGeneric) {
        // The kernel's generic slots: decode_header, then phase 1b's choice of
        // evaluator (lean infill taps unless void / error / dual plane).
        akv::BlockDesc<1> d;
        uint8_t w[72];
        std::memset(w, 0xEE, sizeof(w));
        akv::decode_header<1>(b, akv::footprint_index(BS), d, w);
        const bool lean = !(d.info & ((1u << akv::kInfoVoid) | (1u << akv::kInfoError) | (1u << akv::kInfoDual)));
        for (int t = 0; t < N; ++t) {
            uint32_t c;
            if (lean) {
                c = F::desc_texel_c16<BS>(d, w, t);
            } else {
                uint32_t cv[1];
                akv::texel_values<BS, 1>(d, w, t % BS, t / BS, cv);
                c = cv[0];
            }
            out[t] = akv::c16_to_unit(c);
        }
        return 0;
    }
    uint32_t tab[F::kTabCapMax];
    uint8_t codes[64 + akv::kCodePad];
    std::memset(codes, 0xEE, sizeof(codes));  // stale bytes must not matter for constant blocks
    akv::BlockDesc<1> d;
    alignas(16) uint8_t w[72];
    std::memset(w, 0xEE, sizeof(w));  // stale slack bytes must not matter
    F::LumOut o;
    F::decode_lum<BS>(b, kind, me, cq, false, 0.f, 0.f, tab, codes, 1, kind == F::kKindDesc ? &d : nullptr, o);
    if (kind == F::kKindDesc) {
        const int wx = (d.info >> akv::kInfoWx) & 15, wy = (d.info >> akv::kInfoWy) & 15;
        for (int k = 0; k < 8 * wy; ++k)
            if ((k & 7) < wx) w[k] = F::desc_weight(codes, 1, akv::g_akv_tables.wunq[akv::mode_wq(me)], wx, k);
        constexpr int SEG = F::kDescSeg<BS>;
        for (int y = 0; y < BS; ++y)
            for (int x0 = 0; x0 < BS; x0 += SEG) {
                uint32_t c[SEG];
                F::desc_seg_c16<BS, SEG>(d.info, w, akv::row_pattern<BS>(d.pat[0], d.pat[1], d.pat_hi[0], d.pat_hi[1], y),
                                         d.ep[0], d.ep[1], y, x0, c);
                for (int x = 0; x < SEG; ++x) out[y * BS + x0 + x] = akv::c16_to_unit(c[x]);
            }
        return 0;
    }
    for (int t = 0; t < N; ++t) {
        if constexpr (F::kDirect<BS>) {
            out[t] = F::direct_unit(o, codes, 1, t);
        } else {
            const uint32_t c = codes[t] & o.cmask;
            const uint32_t part = (o.pat[t >> 4] >> (2 * (t & 15))) & 3u;
            if (part * o.L + c >= static_cast<uint32_t>(F::kTabCap<BS>)) return 3;
            out[t] = F::lum_unit(o, tab, codes, 1, t);
        }
    }
    return 0;
}

extern "C" int emu_decode_fast_r(const uint8_t* blocks, int64_t n, int bs, float* out, int* cls) {
    static bool ready = false;
    if (!ready) { akv::build_tables(&akv::g_akv_tables); ready = true; }
    for (int64_t i = 0; i < n; ++i) {
        uint4 b;
        std::memcpy(&b, blocks + 16 * i, 16);
        const int rc = bs == 4 ? fast_r_one<4>(b, cls + i, out + i * 16)
                     : bs == 6 ? fast_r_one<6>(b, cls + i, out + i * 36)
                               : fast_r_one<8>(b, cls + i, out + i * 64);
        if (rc) return rc;
    }
    return 0;
}

// The attention kernel's RGBA 4x4 path: block kind, then the fast / constant
// decode (fp16-view values of all four channels per texel, out[n][16][4]), or
// the generic decoder for other blocks, as the kernel's in-thread fallback.
extern "C" int emu_decode_rgba4(const uint8_t* blocks, int64_t n, float* out, int* cls) {
    static bool ready = false;
    if (!ready) { akv::build_tables(&akv::g_akv_tables); ready = true; }
    namespace F = akv::fast;
    for (int64_t i = 0; i < n; ++i) {
        uint4 b;
        std::memcpy(&b, blocks + 16 * i, 16);
        uint32_t me;
        int cq;
        const int kind = F::rgba_block_kind(b, me, cq);
        cls[i] = kind;
        float* o = out + i * 64;
        if (kind == F::kKindGeneric) {
            akv::BlockDesc<4> d;
            uint8_t w[64 + akv::kCodePad];
            akv::decode_header<4>(b, akv::footprint_index(4), d, w);
            for (int t = 0; t < 16; ++t) {
                uint32_t c[4];
                akv::texel_values<4, 4>(d, w, t & 3, t >> 2, c);
                for (int k = 0; k < 4; ++k) o[4 * t + k] = akv::c16_to_unit(c[k]);
            }
            continue;
        }
        uint8_t codes[16 + akv::kCodePad];
        std::memset(codes, 0xEE, sizeof(codes));
        F::RgbaOut r;
        F::decode_rgba4(b, kind, me, cq, codes, 1, r);
        for (int t = 0; t < 16; ++t) {
            float tv[4];
            F::rgba_t4(r, codes, 1, t, tv);
            for (int k = 0; k < 4; ++k) o[4 * t + k] = tv[k] * 0x1p-16f;
        }
    }
    return 0;
}
