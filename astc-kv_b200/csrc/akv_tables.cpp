// Host-side construction of the ASTC decode tables (see akv_tables.h).
//
// Written from the Khronos Data Format Specification, ASTC chapter: the 2D
// block-mode layout, the BISE trit/quint digit procedures, the colour and
// weight unquantisation formulas and the partition hash. The decode path that
// consumes these tables runs on the GPU (akv_astc_device.cuh).
#include "akv_tables.h"

#include <cstring>

namespace akv {
namespace {

// Range index -> number of levels (spec enumeration order).
constexpr int kLevels[21] = {2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32, 40, 48, 64, 80, 96, 128, 160, 192, 256};

struct Shape { int bits, trits, quints; };

Shape shape_of(int q) {
    int n = kLevels[q];
    Shape s{0, 0, 0};
    if (n % 3 == 0) { s.trits = 1; n /= 3; }
    else if (n % 5 == 0) { s.quints = 1; n /= 5; }
    while ((1 << s.bits) < n) s.bits++;
    return s;
}

inline int bit(int v, int i) { return (v >> i) & 1; }

// 8-bit trit block -> five digits (spec "trit decoding" procedure).
void trit_digits(int T, int d[5]) {
    int c;
    if ((T & 0x1C) == 0x1C) {
        c = ((T >> 3) & 0x1C) | (T & 3);
        d[3] = d[4] = 2;
    } else {
        c = T & 0x1F;
        if ((T & 0x60) == 0x60) { d[4] = 2; d[3] = bit(T, 7); }
        else { d[4] = bit(T, 7); d[3] = (T >> 5) & 3; }
    }
    if ((c & 3) == 3) {
        d[2] = 2; d[1] = bit(c, 4); d[0] = (bit(c, 3) << 1) | (bit(c, 2) & (1 - bit(c, 3)));
    } else if ((c & 0xC) == 0xC) {
        d[2] = 2; d[1] = 2; d[0] = c & 3;
    } else {
        d[2] = bit(c, 4); d[1] = (c >> 2) & 3; d[0] = (bit(c, 1) << 1) | (bit(c, 0) & (1 - bit(c, 1)));
    }
}

// 7-bit quint block -> three digits (spec "quint decoding" procedure).
void quint_digits(int Q, int d[3]) {
    const bool low_all = (Q & 6) == 6;
    if (low_all && (Q & 0x60) == 0) {
        const int q0 = bit(Q, 0);
        d[2] = (q0 << 2) | ((bit(Q, 4) & (1 - q0)) << 1) | (bit(Q, 3) & (1 - q0));
        d[1] = d[0] = 4;
        return;
    }
    int c;
    if (low_all) {
        d[2] = 4;
        c = (Q & 0x18) | (((~Q >> 5) & 3) << 1) | (Q & 1);
    } else {
        d[2] = (Q >> 5) & 3;
        c = Q & 0x1F;
    }
    if ((c & 7) == 5) { d[1] = 4; d[0] = (c >> 3) & 3; }
    else { d[1] = (c >> 3) & 3; d[0] = c & 7; }
}

// Bit replication of an n-bit value to `width` bits.
int widen(int v, int n, int width) {
    int out = 0;
    for (int filled = 0; filled < width;) {
        const int k = n < width - filled ? n : width - filled;
        out = (out << k) | (v >> (n - k));
        filled += k;
    }
    return out;
}

// Colour unquantisation (spec table of B/C constants per trit/quint range).
int color_value(int q, int code) {
    const Shape s = shape_of(q);
    if (!s.trits && !s.quints) return widen(code, s.bits, 8);
    const int digit = code >> s.bits;
    const int m = code & ((1 << s.bits) - 1);
    auto mb = [&](int i) { return (m >> i) & 1; };
    const int a = mb(0), b = mb(1), c = mb(2), d = mb(3), e = mb(4), f = mb(5);
    int B = 0, C = 0;
    switch (kLevels[q]) {
        case 6: C = 204; break;
        case 10: C = 113; break;
        case 12: C = 93; B = b * 0x116; break;                                  // b000b0bb0
        case 20: C = 54; B = b * 0x10C; break;                                  // b0000bb00
        case 24: C = 44; B = c * 0x10A + b * 0x85; break;                       // cb000cbcb
        case 40: C = 26; B = c * 0x105 + b * 0x82; break;                       // cb0000cbc
        case 48: C = 22; B = d * 0x104 + c * 0x82 + b * 0x41; break;            // dcb000dcb
        case 80: C = 13; B = d * 0x102 + c * 0x81 + b * 0x40; break;            // dcb0000dc
        case 96: C = 11; B = e * 0x102 + d * 0x81 + c * 0x40 + b * 0x20; break; // edcb000ed
        case 160: C = 6; B = e * 0x101 + d * 0x80 + c * 0x40 + b * 0x20; break; // edcb0000e
        case 192: C = 5; B = f * 0x101 + e * 0x80 + d * 0x40 + c * 0x20 + b * 0x10; break;  // fedcb000f
        default: return 0;  // ranges 3 and 5 never hold colour values
    }
    const int A = a ? 0x1FF : 0;
    const int T = (digit * C + B) ^ A;
    return (A & 0x80) | (T >> 2);
}

// Weight unquantisation to 0..64.
int weight_value(int q, int code) {
    const Shape s = shape_of(q);
    int r;
    if (!s.trits && !s.quints) {
        r = widen(code, s.bits, 6);
    } else if (s.bits == 0) {
        r = s.trits ? (code == 0 ? 0 : code == 1 ? 32 : 63) : (code * 16 - (code >= 3 ? 1 : 0));
    } else {
        const int digit = code >> s.bits;
        const int m = code & ((1 << s.bits) - 1);
        const int a = m & 1, b = (m >> 1) & 1, c = (m >> 2) & 1;
        int B = 0, C = 0;
        switch (kLevels[q]) {
            case 6: C = 50; break;
            case 10: C = 28; break;
            case 12: C = 23; B = b * 0x45; break;              // b000b0b
            case 20: C = 13; B = b * 0x42; break;              // b0000b0
            case 24: C = 11; B = c * 0x42 + b * 0x21; break;   // cb000cb
            default: return 0;
        }
        const int A = a ? 0x7F : 0;
        const int T = (digit * C + B) ^ A;
        r = (A & 0x20) | (T >> 2);
    }
    return r > 32 ? r + 1 : r;
}

// 2D block-mode decode; returns false for reserved encodings.
bool block_mode(int m, int* wx, int* wy, int* dual, int* wq) {
    const int a = (m >> 5) & 3, b = (m >> 7) & 3;
    int r, hi = (m >> 9) & 1, dp = (m >> 10) & 1;
    if (m & 3) {
        r = ((m & 3) << 1) | ((m >> 4) & 1);
        const int sel = (m >> 2) & 3;
        if (sel == 0) { *wx = b + 4; *wy = a + 2; }
        else if (sel == 1) { *wx = b + 8; *wy = a + 2; }
        else if (sel == 2) { *wx = a + 2; *wy = b + 8; }
        else if (m & 0x100) { *wx = (b & 1) + 2; *wy = a + 2; }
        else { *wx = a + 2; *wy = (b & 1) + 6; }
    } else {
        if ((m & 0xC) == 0) return false;
        r = (((m >> 2) & 3) << 1) | ((m >> 4) & 1);
        switch (b) {
            case 0: *wx = 12; *wy = a + 2; break;
            case 1: *wx = a + 2; *wy = 12; break;
            case 2: *wx = a + 6; *wy = ((m >> 9) & 3) + 6; hi = 0; dp = 0; break;
            default:
                if (a > 1) return false;
                *wx = a ? 10 : 6; *wy = a ? 6 : 10;
                break;
        }
    }
    *wq = r - 2 + 6 * hi;
    *dual = dp;
    return true;
}

uint32_t mix52(uint32_t x) {
    x ^= x >> 15;
    x *= 0xEEDE0891u;
    x ^= x >> 5;
    x += x << 16;
    x ^= x >> 7;
    x ^= x >> 3;
    x ^= x << 6;
    x ^= x >> 17;
    return x;
}

// Partition of texel (x, y) for a 2D block (spec partition-selection function).
int partition_of(int seed, int x, int y, int count, bool small) {
    if (small) { x *= 2; y *= 2; }
    seed += (count - 1) * 1024;
    const uint32_t r = mix52(static_cast<uint32_t>(seed));
    // Twelve 4-bit fields of the hash, squared.
    static const int kShift[12] = {0, 4, 8, 12, 16, 20, 24, 28, 18, 22, 26, 30};
    uint32_t f[12];
    for (int i = 0; i < 12; ++i) {
        const uint32_t v = (i == 11 ? ((r >> 30) | (r << 2)) : (r >> kShift[i])) & 0xF;
        f[i] = v * v;
    }
    const int odd_shift = (seed & 2) ? 4 : 5;
    const int tri_shift = count == 3 ? 6 : 5;
    const int s1 = (seed & 1) ? odd_shift : tri_shift;
    const int s2 = (seed & 1) ? tri_shift : odd_shift;
    const int s3 = (seed & 0x10) ? s1 : s2;
    for (int i = 0; i < 8; ++i) f[i] >>= (i & 1) ? s2 : s1;
    for (int i = 8; i < 12; ++i) f[i] >>= s3;
    // z = 0 for 2D blocks, so fields 8..11 contribute nothing but keep the
    // spec's structure readable.
    int lane[4];
    lane[0] = static_cast<int>((f[0] * x + f[1] * y + (r >> 14)) & 0x3F);
    lane[1] = static_cast<int>((f[2] * x + f[3] * y + (r >> 10)) & 0x3F);
    lane[2] = count >= 3 ? static_cast<int>((f[4] * x + f[5] * y + (r >> 6)) & 0x3F) : 0;
    lane[3] = count >= 4 ? static_cast<int>((f[6] * x + f[7] * y + (r >> 2)) & 0x3F) : 0;
    int best = 0;
    for (int i = 1; i < 4; ++i)
        if (lane[i] > lane[best]) best = i;  // ties keep the lower index
    return best;
}

}  // namespace

int bise_stream_bits(int count, int q) {
    const Shape s = shape_of(q);
    return count * s.bits + (s.trits ? (8 * count + 4) / 5 : 0) + (s.quints ? (7 * count + 2) / 3 : 0);
}

void build_tables(Tables* t) {
    std::memset(t, 0, sizeof(*t));
    for (int q = 0; q < 21; ++q) {
        const Shape s = shape_of(q);
        t->shape[q] = static_cast<uint8_t>(s.bits | (s.trits << 4) | (s.quints << 5));
    }
    for (int T = 0; T < 256; ++T) {
        int d[5];
        trit_digits(T, d);
        uint16_t v = 0;
        for (int j = 0; j < 5; ++j) v |= static_cast<uint16_t>(d[j] << (2 * j));
        t->trit[T] = v;
    }
    for (int Q = 0; Q < 128; ++Q) {
        int d[3];
        quint_digits(Q, d);
        t->quint[Q] = static_cast<uint16_t>(d[0] | (d[1] << 3) | (d[2] << 6));
    }
    for (int q = 0; q < 21; ++q)
        for (int code = 0; code < kLevels[q]; ++code) t->cunq[q][code] = static_cast<uint8_t>(color_value(q, code));
    for (int q = 0; q < 12; ++q)
        for (int code = 0; code < kLevels[q]; ++code) t->wunq[q][code] = static_cast<uint8_t>(weight_value(q, code));
    for (int pairs = 1; pairs <= 9; ++pairs)
        for (int avail = 0; avail < 128; ++avail) {
            uint8_t pick = 0xFF;
            for (int q = 20; q >= 4; --q)
                if (bise_stream_bits(2 * pairs, q) <= avail) { pick = static_cast<uint8_t>(q); break; }
            t->cquant[pairs][avail] = pick;
        }
    // Combined digit table, 3 bits per digit: trit blocks, then quint blocks.
    for (int v = 0; v < 256; ++v) {
        uint16_t d = 0;
        for (int j = 0; j < 5; ++j) d |= static_cast<uint16_t>(((t->trit[v] >> (2 * j)) & 3) << (3 * j));
        t->dig3[v] = d;
    }
    for (int v = 0; v < 128; ++v) t->dig3[256 + v] = t->quint[v];
    for (int f = 0; f < kNumFootprints; ++f) {
        const int bs = f == 0 ? 4 : (f == 1 ? 6 : 8);
        const int ds = (1024 + bs / 2) / (bs - 1);
        for (int wx = 2; wx <= bs; ++wx)
            for (int wy = 2; wy <= bs; ++wy)
                for (int y = 0; y < bs; ++y)
                    for (int x = 0; x < bs; ++x) {
                        const int gs = (ds * x * (wx - 1) + 32) >> 6, gt = (ds * y * (wy - 1) + 32) >> 6;
                        const int i00 = (gs >> 4) + (gt >> 4) * wx;
                        t->infill[f][wx - 2][wy - 2][y * bs + x] =
                            static_cast<uint16_t>(i00 | ((gs & 15) << 6) | ((gt & 15) << 10));
                    }        for (int n = 2; n <= bs; ++n)
            for (int c = 0; c < 8; ++c) {
                const int g = c < bs ? (ds * c * (n - 1) + 32) >> 6 : 0;
                const int j = g >> 4;
                t->sep[f][n - 2][c] = static_cast<uint16_t>(j | ((j + 1 < 7 ? j + 1 : 7) << 4) | ((g & 15) << 8));
            }
    }
    static const int kBlocks[kNumFootprints] = {4, 6, 8};
    for (int f = 0; f < kNumFootprints; ++f) {
        const int bs = kBlocks[f];
        for (int m = 0; m < 2048; ++m) {
            int wx, wy, dual, wq;
            uint32_t e = 0;
            if ((m & 0x1FF) != 0x1FC && block_mode(m, &wx, &wy, &dual, &wq)) {
                const int n = wx * wy * (dual + 1);
                const int bits = bise_stream_bits(n, wq);
                if (n <= 64 && bits >= 24 && bits <= 96 && wx <= bs && wy <= bs) {
                    e = kModeValid | (dual ? kModeDual : 0u) | (static_cast<uint32_t>(wq) << 2) |
                        (static_cast<uint32_t>(wx) << 6) | (static_cast<uint32_t>(wy) << 10) |
                        (static_cast<uint32_t>(bits) << 14) | ((wx < bs || wy < bs) ? kModeReduced : 0u);
                }
            }
            t->mode[f][m] = e;
        }
        const bool small = bs * bs < 31;
        for (int c = 2; c <= 4; ++c)
            for (int seed = 0; seed < 1024; ++seed) {
                uint32_t* w = t->part[f][c - 2][seed];
                for (int y = 0; y < bs; ++y)
                    for (int x = 0; x < bs; ++x) {
                        const int i = y * bs + x;
                        w[i >> 4] |= static_cast<uint32_t>(partition_of(seed, x, y, c, small)) << (2 * (i & 15));
                    }
            }
    }
}

}  // namespace akv
