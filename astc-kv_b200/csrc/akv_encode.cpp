// Host-side ASTC LDR encoder and random-block generator (see include/akv_host.h).
//
// The encoder is deliberately small: per block it tries a handful of
// candidates (1 or 2 partitions with the seed whose pattern best matches a
// 2-means split, the full or a few reduced weight grids, every weight range
// whose bit count is legal), fits endpoints by min/max, projects texels onto
// the endpoint line for weights, quantises with the same unquantisation
// tables the GPU decoder uses, and keeps the candidate with the smallest
// squared error on the decoded fp16 view. Output blocks are legal ASTC that
// any decoder reads; they are not astcenc's choices.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/akv_host.h"
#include "akv_tables.h"

namespace akv {
namespace {

constexpr int kLevels[21] = {2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32, 40, 48, 64, 80, 96, 128, 160, 192, 256};

struct Enc {
    Tables t;
    // Trit/quint block encoders for a group holding `c` values: digits (base
    // 3 / base 5 number, first digit least significant) -> block bits with
    // every bit past the group's stored length zero. -1 when unreachable.
    int16_t trit_enc[6][243];
    int16_t quint_enc[4][125];
    uint8_t cnear[21][256];
    uint8_t wnear[12][65];
    int16_t mode_of[3][13][13][12];  // footprint, wx, wy, wq -> mode (single plane) or -1
};

const Enc& enc_tables() {
    static Enc* e = [] {
        Enc* x = new Enc;
        build_tables(&x->t);
        std::memset(x->trit_enc, 0xFF, sizeof(x->trit_enc));
        std::memset(x->quint_enc, 0xFF, sizeof(x->quint_enc));
        static const int kTritBits[6] = {0, 2, 4, 5, 7, 8};
        for (int c = 1; c <= 5; ++c)
            for (int T = 0; T < (1 << kTritBits[c]); ++T) {
                int code = 0, mul = 1;
                for (int j = 0; j < c; ++j, mul *= 3) code += ((x->t.trit[T] >> (2 * j)) & 3) * mul;
                if (x->trit_enc[c][code] < 0) x->trit_enc[c][code] = static_cast<int16_t>(T);
            }
        static const int kQuintBits[4] = {0, 3, 5, 7};
        for (int c = 1; c <= 3; ++c)
            for (int Q = 0; Q < (1 << kQuintBits[c]); ++Q) {
                int code = 0, mul = 1;
                for (int j = 0; j < c; ++j, mul *= 5) code += ((x->t.quint[Q] >> (3 * j)) & 7) * mul;
                if (x->quint_enc[c][code] < 0) x->quint_enc[c][code] = static_cast<int16_t>(Q);
            }
        for (int q = 0; q < 21; ++q)
            for (int v = 0; v < 256; ++v) {
                int best = 0, bd = 1 << 30;
                for (int code = 0; code < kLevels[q]; ++code) {
                    const int d = std::abs(static_cast<int>(x->t.cunq[q][code]) - v);
                    if (d < bd) { bd = d; best = code; }
                }
                x->cnear[q][v] = static_cast<uint8_t>(best);
            }
        for (int q = 0; q < 12; ++q)
            for (int v = 0; v <= 64; ++v) {
                int best = 0, bd = 1 << 30;
                for (int code = 0; code < kLevels[q]; ++code) {
                    const int d = std::abs(static_cast<int>(x->t.wunq[q][code]) - v);
                    if (d < bd) { bd = d; best = code; }
                }
                x->wnear[q][v] = static_cast<uint8_t>(best);
            }
        std::memset(x->mode_of, 0xFF, sizeof(x->mode_of));
        for (int f = 0; f < kNumFootprints; ++f)
            for (int m = 0; m < 2048; ++m) {
                const uint32_t me = x->t.mode[f][m];
                if (!(me & kModeValid) || (me & kModeDual)) continue;
                int16_t& slot = x->mode_of[f][mode_wx(me)][mode_wy(me)][mode_wq(me)];
                if (slot < 0) slot = static_cast<int16_t>(m);
            }
        return x;
    }();
    return *e;
}

void put(uint8_t* blk, int pos, int n, uint32_t v) {
    for (int i = 0; i < n; ++i)
        if ((v >> i) & 1u) blk[(pos + i) >> 3] |= static_cast<uint8_t>(1u << ((pos + i) & 7));
}

// BISE-encode `codes` into `buf` starting at bit 0. Returns the bit count.
int bise_put(const Enc& E, const int* codes, int count, int q, uint8_t* buf) {
    const int shp = E.t.shape[q];
    const int b = shp & 15, trits = (shp >> 4) & 1, quints = (shp >> 5) & 1;
    int pos = 0;
    if (trits) {
        static const int kTb[5] = {2, 2, 1, 2, 1};
        for (int g = 0; g < count; g += 5) {
            const int c = std::min(5, count - g);
            int key = 0, mul = 1;
            for (int j = 0; j < c; ++j, mul *= 3) key += (codes[g + j] >> b) * mul;
            const int T = E.trit_enc[c][key];
            int tpos = 0;
            for (int j = 0; j < c; ++j) {
                put(buf, pos, b, static_cast<uint32_t>(codes[g + j]) & ((1u << b) - 1u));
                pos += b;
                // A partial group stores only the trit bits up to its last
                // value; trit_enc[c] picked a T whose later bits are zero.
                put(buf, pos, kTb[j], static_cast<uint32_t>(T >> tpos) & ((1u << kTb[j]) - 1u));
                pos += kTb[j];
                tpos += kTb[j];
            }
        }
        // Trim to the exact stream length (bits past it are zero anyway).
        return count * b + (8 * count + 4) / 5;
    }
    if (quints) {
        static const int kQb[3] = {3, 2, 2};
        for (int g = 0; g < count; g += 3) {
            const int c = std::min(3, count - g);
            int key = 0, mul = 1;
            for (int j = 0; j < c; ++j, mul *= 5) key += (codes[g + j] >> b) * mul;
            const int Q = E.quint_enc[c][key];
            int qpos = 0;
            for (int j = 0; j < c; ++j) {
                put(buf, pos, b, static_cast<uint32_t>(codes[g + j]) & ((1u << b) - 1u));
                pos += b;
                put(buf, pos, kQb[j], static_cast<uint32_t>(Q >> qpos) & ((1u << kQb[j]) - 1u));
                pos += kQb[j];
                qpos += kQb[j];
            }
        }
        return count * b + (7 * count + 2) / 3;
    }
    for (int i = 0; i < count; ++i, pos += b) put(buf, pos, b, static_cast<uint32_t>(codes[i]));
    return pos;
}

// Bilinear infill of texel weights from a grid (spec weight infill).
void infill(int bs, int wx, int wy, const int* grid, int* out) {
    const int ds = (1024 + bs / 2) / (bs - 1);
    for (int y = 0; y < bs; ++y)
        for (int x = 0; x < bs; ++x) {
            const int gs = (ds * x * (wx - 1) + 32) >> 6, gt = (ds * y * (wy - 1) + 32) >> 6;
            const int js = gs >> 4, fs = gs & 15, jt = gt >> 4, ft = gt & 15;
            const int w11 = (fs * ft + 8) >> 4;
            const int i0 = js + jt * wx;
            const int p00 = grid[i0];
            const int p01 = js + 1 < wx ? grid[i0 + 1] : 0;
            const int p10 = jt + 1 < wy ? grid[i0 + wx] : 0;
            const int p11 = (js + 1 < wx && jt + 1 < wy) ? grid[i0 + wx + 1] : 0;
            out[y * bs + x] = (p00 * (16 - fs - ft + w11) + p01 * (fs - w11) + p10 * (ft - w11) + p11 * w11 + 8) >> 4;
        }
}

// Infill coefficients: texel i gets sum_j coef[i][j] * grid[j] / 16.
void infill_coefs(int bs, int wx, int wy, std::vector<float>& coef) {
    const int n = bs * bs, g = wx * wy;
    coef.assign(static_cast<size_t>(n) * g, 0.f);
    const int ds = (1024 + bs / 2) / (bs - 1);
    for (int y = 0; y < bs; ++y)
        for (int x = 0; x < bs; ++x) {
            const int gs = (ds * x * (wx - 1) + 32) >> 6, gt = (ds * y * (wy - 1) + 32) >> 6;
            const int js = gs >> 4, fs = gs & 15, jt = gt >> 4, ft = gt & 15;
            const int w11 = (fs * ft + 8) >> 4;
            const int i0 = js + jt * wx;
            float* c = &coef[static_cast<size_t>(y * bs + x) * g];
            c[i0] += 16 - fs - ft + w11;
            if (js + 1 < wx) c[i0 + 1] += fs - w11;
            if (jt + 1 < wy) c[i0 + wx] += ft - w11;
            if (js + 1 < wx && jt + 1 < wy) c[i0 + wx + 1] += w11;
        }
}

inline float unit_of(uint32_t c) {
    if (c == 0xFFFFu) return 1.0f;
    float f = static_cast<float>(c);
    uint32_t bits;
    std::memcpy(&bits, &f, 4);
    bits &= 0xFFFFE000u;
    std::memcpy(&f, &bits, 4);
    return f * (1.0f / 65536.0f);
}

inline uint32_t interp(int e0, int e1, int w) {
    const int X = e0 * (64 - w) + e1 * w;
    return static_cast<uint32_t>(4 * X + ((X + 32) >> 6));
}

struct Candidate {
    float err = 1e30f;
    uint8_t blk[16];
};

// Encode one block with a fixed partitioning / grid / weight range / CEM.
// x: texels [n][4] in [0,1]. part: partition per texel. Returns the error.
float try_block(const Enc& E, int bs, int fp, const float* x, int nch, int parts, int seed, const int* part, int wx, int wy,
                int wq, const std::vector<float>* coef, uint8_t* out) {
    const int n = bs * bs;
    const int cem = nch == 1 ? 0 : 12;
    const int vals_per = nch == 1 ? 2 : 8;
    const int mode = E.mode_of[fp][wx][wy][wq];
    if (mode < 0) return 1e30f;
    const int ngrid = wx * wy;
    const int wbits = bise_stream_bits(ngrid, wq);
    const int cstart = parts == 1 ? 17 : 29;
    const int avail = 128 - wbits - cstart;
    if (avail < 0) return 1e30f;
    const int nints = vals_per * parts;
    const int cq = E.t.cquant[nints / 2][avail];
    if (cq == 0xFF) return 1e30f;

    // Endpoints per partition: per-channel min/max, quantised.
    int codes[18];
    int e0[4][4], e1[4][4];
    for (int p = 0; p < parts; ++p) {
        float lo[4] = {1, 1, 1, 1}, hi[4] = {0, 0, 0, 0};
        bool any = false;
        for (int i = 0; i < n; ++i) {
            if (part[i] != p) continue;
            any = true;
            for (int c = 0; c < nch; ++c) { lo[c] = std::min(lo[c], x[i * 4 + c]); hi[c] = std::max(hi[c], x[i * 4 + c]); }
        }
        if (!any) for (int c = 0; c < nch; ++c) { lo[c] = 0; hi[c] = 0; }
        int q0[4], q1[4];
        for (int c = 0; c < nch; ++c) {
            // Round the range outward so quantised endpoints cover it.
            int a = static_cast<int>(std::floor(lo[c] * 255.f + 1e-4f)), b = static_cast<int>(std::ceil(hi[c] * 255.f - 1e-4f));
            a = std::clamp(a, 0, 255); b = std::clamp(b, 0, 255);
            q0[c] = E.cnear[cq][a]; q1[c] = E.cnear[cq][b];
        }
        if (nch == 1) {
            codes[p * 2] = q0[0]; codes[p * 2 + 1] = q1[0];
            e0[p][0] = E.t.cunq[cq][q0[0]]; e1[p][0] = E.t.cunq[cq][q1[0]];
        } else {
            int s0 = 0, s1 = 0;
            for (int c = 0; c < 3; ++c) { s0 += E.t.cunq[cq][q0[c]]; s1 += E.t.cunq[cq][q1[c]]; }
            if (s1 < s0) for (int c = 0; c < 4; ++c) std::swap(q0[c], q1[c]);  // avoid blue contraction
            for (int c = 0; c < 4; ++c) {
                codes[p * 8 + 2 * c] = q0[c]; codes[p * 8 + 2 * c + 1] = q1[c];
                e0[p][c] = E.t.cunq[cq][q0[c]]; e1[p][c] = E.t.cunq[cq][q1[c]];
            }
        }
    }
    // Ideal texel weights (0..64) by projection on the endpoint line.
    float wi[64];
    for (int i = 0; i < n; ++i) {
        const int p = part[i];
        float num = 0, den = 0;
        for (int c = 0; c < nch; ++c) {
            const float d = (e1[p][c] - e0[p][c]) / 255.f;
            num += (x[i * 4 + c] - e0[p][c] / 255.f) * d;
            den += d * d;
        }
        wi[i] = den > 0 ? std::clamp(64.f * num / den, 0.f, 64.f) : 0.f;
    }
    int wcodes[64], grid[64], tw[64];
    if (!coef) {
        for (int i = 0; i < n; ++i) {
            wcodes[i] = E.wnear[wq][static_cast<int>(std::lround(wi[i]))];
            tw[i] = E.t.wunq[wq][wcodes[i]];
        }
    } else {
        for (int j = 0; j < ngrid; ++j) {
            float num = 0, den = 0;
            for (int i = 0; i < n; ++i) {
                const float c = (*coef)[static_cast<size_t>(i) * ngrid + j];
                num += c * wi[i];
                den += c;
            }
            const float g = den > 0 ? num / den : 0.f;
            wcodes[j] = E.wnear[wq][static_cast<int>(std::lround(std::clamp(g, 0.f, 64.f)))];
            grid[j] = E.t.wunq[wq][wcodes[j]];
        }
        infill(bs, wx, wy, grid, tw);
    }
    float err = 0;
    for (int i = 0; i < n; ++i)
        for (int c = 0; c < nch; ++c) {
            const float d = unit_of(interp(e0[part[i]][c], e1[part[i]][c], tw[i])) - x[i * 4 + c];
            err += d * d;
        }
    // Assemble.
    std::memset(out, 0, 16);
    put(out, 0, 11, static_cast<uint32_t>(mode));
    put(out, 11, 2, static_cast<uint32_t>(parts - 1));
    if (parts == 1) put(out, 13, 4, static_cast<uint32_t>(cem));
    else { put(out, 13, 10, static_cast<uint32_t>(seed)); put(out, 23, 6, static_cast<uint32_t>(cem << 2)); }
    uint8_t tmp[32];
    std::memset(tmp, 0, sizeof(tmp));
    const int cbits = bise_put(E, codes, nints, cq, tmp);
    for (int i = 0; i < cbits; ++i)
        if ((tmp[i >> 3] >> (i & 7)) & 1) put(out, cstart + i, 1, 1);
    std::memset(tmp, 0, sizeof(tmp));
    const int wb = bise_put(E, wcodes, ngrid, wq, tmp);
    for (int i = 0; i < wb; ++i)
        if ((tmp[i >> 3] >> (i & 7)) & 1) put(out, 127 - i, 1, 1);
    return err;
}

void encode_block(const Enc& E, int bs, const float* x, int nch, int effort, uint8_t* out) {
    const int fp = footprint_index(bs);
    const int n = bs * bs;
    Candidate best;
    int part0[64] = {0};
    // Grids to try.
    std::vector<std::pair<int, int>> grids;
    grids.push_back({bs, bs});
    if (bs == 6) { if (effort >= 1) { grids.push_back({5, 5}); grids.push_back({6, 5}); grids.push_back({5, 6}); } }
    if (bs == 8) {
        grids.push_back({6, 6});
        grids.push_back({5, 5});
        if (effort >= 1) { grids.push_back({8, 5}); grids.push_back({5, 8}); grids.push_back({4, 4}); }
    }
    // 2-partition seeds from a 2-means split on the first channel.
    std::vector<int> seeds;
    if (nch == 1 && effort >= 1) {
        float lo = 1, hi = 0;
        for (int i = 0; i < n; ++i) { lo = std::min(lo, x[i * 4]); hi = std::max(hi, x[i * 4]); }
        float c0 = lo, c1 = hi;
        uint64_t mask = 0;
        for (int it = 0; it < 4; ++it) {
            mask = 0;
            float s0 = 0, s1 = 0;
            int n0 = 0, n1 = 0;
            for (int i = 0; i < n; ++i) {
                const bool one = std::fabs(x[i * 4] - c1) < std::fabs(x[i * 4] - c0);
                if (one) { mask |= 1ull << i; s1 += x[i * 4]; ++n1; } else { s0 += x[i * 4]; ++n0; }
            }
            if (n0) c0 = s0 / n0;
            if (n1) c1 = s1 / n1;
        }
        std::vector<std::pair<int, int>> scored;
        for (int s = 0; s < 1024; ++s) {
            uint64_t pm = 0;
            for (int i = 0; i < n; ++i)
                if ((E.t.part[fp][0][s][i >> 4] >> (2 * (i & 15))) & 1u) pm |= 1ull << i;
            const uint64_t all = n == 64 ? ~0ull : ((1ull << n) - 1);
            const int d = std::min(__builtin_popcountll((pm ^ mask) & all), __builtin_popcountll((pm ^ ~mask) & all));
            scored.push_back({d, s});
        }
        std::partial_sort(scored.begin(), scored.begin() + 2, scored.end());
        seeds.push_back(scored[0].second);
        if (effort >= 2) seeds.push_back(scored[1].second);
    }
    std::vector<float> coef;
    for (auto [wx, wy] : grids) {
        const bool reduced = wx != bs || wy != bs;
        if (reduced) infill_coefs(bs, wx, wy, coef);
        for (int wq = 0; wq < 12; ++wq) {
            const int wbits = bise_stream_bits(wx * wy, wq);
            if (wbits < 24 || wbits > 96) continue;
            Candidate c;
            c.err = try_block(E, bs, fp, x, nch, 1, 0, part0, wx, wy, wq, reduced ? &coef : nullptr, c.blk);
            if (c.err < best.err) best = c;
            for (int seed : seeds) {
                int part[64];
                for (int i = 0; i < n; ++i) part[i] = (E.t.part[fp][0][seed][i >> 4] >> (2 * (i & 15))) & 3;
                c.err = try_block(E, bs, fp, x, nch, 2, seed, part, wx, wy, wq, reduced ? &coef : nullptr, c.blk);
                if (c.err < best.err) best = c;
            }
        }
    }
    if (best.err >= 1e29f) {
        // Fallback: constant void-extent block with the mean value.
        std::memset(out, 0, 16);
        put(out, 0, 12, 0xDFC);  // mode bits 0..8 = 0x1FC, bit 9 = 0 (LDR), bits 10..11 = 1
        for (int k = 0; k < 4; ++k) { put(out, 12 + 13 * k, 13, 0x1FFF); }
        for (int c = 0; c < 4; ++c) {
            float m = 0;
            for (int i = 0; i < n; ++i) m += c < nch ? x[i * 4 + c] : (nch == 1 ? x[i * 4] : 1.f);
            put(out, 64 + 16 * c, 16, static_cast<uint32_t>(std::lround(std::clamp(m / n, 0.f, 1.f) * 65535.f)));
        }
        return;
    }
    std::memcpy(out, best.blk, 16);
}

template <typename F>
void parallel_for(int64_t n, int threads, F&& f) {
    if (threads <= 1 || n < 64) { for (int64_t i = 0; i < n; ++i) f(i); return; }
    std::atomic<int64_t> next{0};
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t)
        pool.emplace_back([&] {
            for (;;) {
                const int64_t start = next.fetch_add(256);
                if (start >= n) break;
                const int64_t end = std::min(n, start + 256);
                for (int64_t i = start; i < end; ++i) f(i);
            }
        });
    for (auto& th : pool) th.join();
}

uint64_t splitmix(uint64_t& s) {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

}  // namespace
}  // namespace akv

using namespace akv;

extern "C" int akv_host_encode(const float* rgba, unsigned width, unsigned height, int block, int layout, int effort,
                               uint8_t* out, size_t bytes, int threads) {
    if (!rgba || !out || (block != 4 && block != 6 && block != 8) || (layout != 0 && layout != 1)) return 1;
    if (width % block || height % block || width == 0 || height == 0) return 1;
    const int64_t cols = width / block, rows = height / block;
    if (static_cast<size_t>(cols * rows * 16) != bytes) return 1;
    const Enc& E = enc_tables();
    const int nch = layout == 0 ? 1 : 4;
    parallel_for(cols * rows, threads, [&](int64_t bi) {
        const int64_t r = bi / cols, c = bi % cols;
        float x[64 * 4];
        for (int y = 0; y < block; ++y)
            for (int xx = 0; xx < block; ++xx) {
                const float* src = rgba + ((r * block + y) * static_cast<int64_t>(width) + c * block + xx) * 4;
                for (int k = 0; k < 4; ++k) x[(y * block + xx) * 4 + k] = std::clamp(src[k], 0.f, 1.f);
            }
        encode_block(E, block, x, nch, effort, out + bi * 16);
    });
    return 0;
}

extern "C" int akv_host_random_blocks(int64_t n, int block, uint64_t seed, uint8_t* out, int threads) {
    if (n < 0 || !out || (block != 4 && block != 6 && block != 8)) return 1;
    const Enc& E = enc_tables();
    const int fp = footprint_index(block);
    std::vector<int> modes;
    for (int m = 0; m < 2048; ++m)
        if (E.t.mode[fp][m] & kModeValid) modes.push_back(m);
    static const int kLdrCems[10] = {0, 1, 4, 5, 6, 8, 9, 10, 12, 13};
    parallel_for(n, threads, [&](int64_t i) {
        uint64_t s = seed ^ (0xA24BAED4963EE407ull * static_cast<uint64_t>(i + 1));
        uint8_t* b = out + i * 16;
        for (int attempt = 0;; ++attempt) {
            for (int k = 0; k < 2; ++k) {
                const uint64_t r = splitmix(s);
                std::memcpy(b + 8 * k, &r, 8);
            }
            if (splitmix(s) % 64 == 0 || attempt > 64) {
                // Constant void-extent block.
                std::memset(b, 0, 8);
                put(b, 0, 12, 0xDFC);
                for (int k = 0; k < 4; ++k) put(b, 12 + 13 * k, 13, 0x1FFF);
                return;
            }
            const int mode = modes[splitmix(s) % modes.size()];
            const uint32_t me = E.t.mode[fp][mode];
            const int dual = (me & kModeDual) ? 1 : 0;
            const int parts = static_cast<int>(splitmix(s) % (dual ? 3 : 4)) + 1;
            const int wbits = mode_wbits(me);
            int cems[4], npairs = 0;
            for (int p = 0; p < parts; ++p) {
                cems[p] = parts == 1 || p == 0 ? kLdrCems[splitmix(s) % 10] : cems[0];
                npairs += (cems[p] >> 2) + 1;
            }
            const int cstart = parts == 1 ? 17 : 29;
            const int avail = 128 - wbits - 2 * dual - cstart;
            if (npairs > 9 || avail < 0 || E.t.cquant[npairs][avail] == 0xFF) continue;
            // Header fields over the random payload.
            for (int k = 0; k < 13; ++k) b[k >> 3] &= static_cast<uint8_t>(~(1u << (k & 7)));
            put(b, 0, 11, static_cast<uint32_t>(mode));
            put(b, 11, 2, static_cast<uint32_t>(parts - 1));
            if (parts == 1) {
                for (int k = 13; k < 17; ++k) b[k >> 3] &= static_cast<uint8_t>(~(1u << (k & 7)));
                put(b, 13, 4, static_cast<uint32_t>(cems[0]));
            } else {
                // Seed stays random (bits 13..22); shared CEM, selector 00.
                for (int k = 23; k < 29; ++k) b[k >> 3] &= static_cast<uint8_t>(~(1u << (k & 7)));
                put(b, 23, 6, static_cast<uint32_t>(cems[0] << 2));
            }
            return;
        }
    });
    return 0;
}
