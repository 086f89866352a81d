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
        uint8_t w[64];
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

extern "C" float emu_unit(uint32_t c) { return akv::c16_to_unit(c); }

// The fast per-block path of the attention kernel's plane decode: sort key,
// then (fast keys) value table + per-texel index bytes, or (constant keys)
// the block's single value. Returns the fp16-view values of the R channel
// per texel, or -1 for blocks that take the per-texel path; `cls` gets the key.
extern "C" int emu_decode_fast_r(const uint8_t* blocks, int64_t n, int bs, float* out, int* cls) {
    static bool ready = false;
    if (!ready) { akv::build_tables(&akv::g_akv_tables); ready = true; }
    namespace F = akv::fast;
    for (int64_t i = 0; i < n; ++i) {
        uint4 b;
        std::memcpy(&b, blocks + 16 * i, 16);
        const int c = bs == 4 ? F::block_key<4>(b) : bs == 6 ? F::block_key<6>(b) : F::block_key<8>(b);
        cls[i] = c;
        const int N = bs * bs;
        if (c == F::kKeySlow) { for (int t = 0; t < N; ++t) out[i * N + t] = -1.f; continue; }
        if (c == F::kKeyConst) {
            const float u = akv::c16_to_unit(F::const_c16(b));
            for (int t = 0; t < N; ++t) out[i * N + t] = u;
            continue;
        }
        uint32_t tab[F::kTabCap];
        uint32_t words[16];
        int L = 0;
        if (bs == 4) { F::Idx<4> ix; L = F::decode_fast_any<4>(c - F::kKeyFast, b, false, 0.f, 0.f, tab, 1, ix); std::memcpy(words, ix.w, sizeof(ix.w)); }
        else if (bs == 6) { F::Idx<6> ix; L = F::decode_fast_any<6>(c - F::kKeyFast, b, false, 0.f, 0.f, tab, 1, ix); std::memcpy(words, ix.w, sizeof(ix.w)); }
        else { F::Idx<8> ix; L = F::decode_fast_any<8>(c - F::kKeyFast, b, false, 0.f, 0.f, tab, 1, ix); std::memcpy(words, ix.w, sizeof(ix.w)); }
        if (L == 0) return 2;
        for (int t = 0; t < N; ++t) {
            const uint32_t k = (words[t >> 2] >> (8 * (t & 3))) & 0xFF;
            if (k >= static_cast<uint32_t>(F::kTabCap)) return 3;
            out[i * N + t] = __uint_as_float(tab[k]);
        }
    }
    return 0;
}
