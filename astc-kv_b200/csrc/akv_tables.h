// Decode tables for the sm_100a ASTC LDR decoder.
//
// Every table is derived on the host from the ASTC rules (Khronos Data Format
// Specification, ASTC chapter) and copied once per device into the
// `g_akv_tables` __device__ object. Per-block work on the GPU then becomes
// table lookups instead of the spec's bit-serial procedures:
//   * mode[f][m]     11-bit block mode -> weight grid, range, dual plane, bits
//   * part[f][n][s]  partition index of every texel (2 bits per texel) for
//                    footprint f, partition count n+2, 10-bit seed s
//   * trit/quint     packed digits of a BISE trit (8-bit) / quint (7-bit) block
//   * cunq / wunq    colour (0..255) / weight (0..64) unquantisation by code
//   * cquant[n][b]   colour range chosen for n/2 integers in b free bits
#pragma once
#include <cstdint>

#ifdef __CUDACC__
#define AKV_HD __host__ __device__
#else
#define AKV_HD
#endif

namespace akv {

// Footprints supported by the reference encoder (astc_kv/codec.py:123, block
// in {4, 6, 8}, square).
constexpr int kNumFootprints = 3;
AKV_HD constexpr int footprint_index(int block) { return block == 4 ? 0 : block == 6 ? 1 : block == 8 ? 2 : -1; }

// mode[] entry layout.
constexpr uint32_t kModeValid = 1u << 0;
constexpr uint32_t kModeDual = 1u << 1;
AKV_HD constexpr int mode_wq(uint32_t e) { return (e >> 2) & 15; }
AKV_HD constexpr int mode_wx(uint32_t e) { return (e >> 6) & 15; }
AKV_HD constexpr int mode_wy(uint32_t e) { return (e >> 10) & 15; }
AKV_HD constexpr int mode_wbits(uint32_t e) { return (e >> 14) & 127; }
constexpr uint32_t kModeReduced = 1u << 21;  // weight grid smaller than the footprint

struct Tables {
    uint32_t mode[kNumFootprints][2048];
    uint32_t part[kNumFootprints][3][1024][4];  // 2 bits per texel, texel = y*block + x
    uint16_t trit[256];                         // 5 digits x 2 bits
    uint16_t quint[128];                        // 3 digits x 3 bits
    uint8_t cunq[21][256];
    uint8_t wunq[12][32];
    uint8_t cquant[10][128];                    // 0xFF: no range fits (illegal block)
    // Range shape per range index: bits | trits << 4 | quints << 5.
    uint8_t shape[21];
    // Digits of a trit block (index 0..255) or quint block (256 + 0..127),
    // 3 bits per digit: the runtime BISE decoder's single lookup.
    uint16_t dig3[384];
    // Bilinear infill taps of a reduced weight grid (spec weight infill) for
    // footprint f, grid (wx, wy) in 2..8 x 2..8, texel t: base grid index
    // i00 | fs << 6 | ft << 10. At the last texel row / column the fraction
    // is 0, so the taps past the grid get zero weight.
    uint16_t infill[kNumFootprints][7][7][64];
    // The same infill, separated by axis (the spec computes the s and t grid
    // coordinates independently): for footprint f, grid size n in 2..8 and
    // texel coordinate c, entry = j | min(j + 1, 7) << 4 | frac << 8 with j the
    // lower grid index and frac the fraction towards j + 1 (0 at the last
    // coordinate, so the clamped upper tap never carries weight). Rows of 8
    // entries (16 bytes) so one vector load fetches a whole row.
    alignas(16) uint16_t sep[kNumFootprints][7][8];
};

// Fills `t` on the host. Deterministic; no device calls.
void build_tables(Tables* t);

// ---------------------------------------------------------------------------
// Header decode of 6x6 luminance blocks by table, for the fused attention
// kernel's common case (every astcenc 6x6 block of scalar KV data seen so far
// is luminance-direct, single-plane, with a 6x6 or 5x6 / 6x5 weight grid and a
// weight range of 0..2 to 0..7). The 11-bit block mode and the 2-bit
// partition count fix everything else about such a block: the weight range,
// the stream lengths and (with every endpoint mode 0) the colour range. One
// lookup in `info` gives all of it, and each BISE group of the weight stream
// is decoded by one lookup of its whole bit window into packed code bytes.

// info[] entry layout.
constexpr uint32_t kF6Lum = 1u << 0;    // luminance candidate: on the fast path when every endpoint mode is 0
constexpr uint32_t kF6Const = 1u << 1;  // void extent or reserved mode: a constant block
constexpr uint32_t kF6Err = 1u << 2;    // with endpoint mode 0 the colour data cannot fit: error colour
constexpr uint32_t kF6Full = 1u << 3;   // full 6x6 weight grid (else a reduced grid)
AKV_HD constexpr int f6_parts(uint32_t e) { return static_cast<int>((e >> 4) & 3) + 1; }
AKV_HD constexpr int f6_wq(uint32_t e) { return static_cast<int>((e >> 6) & 15); }
AKV_HD constexpr int f6_cq(uint32_t e) { return static_cast<int>((e >> 10) & 31); }
AKV_HD constexpr int f6_levels(uint32_t e) { return static_cast<int>((e >> 15) & 15); }
AKV_HD constexpr int f6_kind(uint32_t e) { return static_cast<int>((e >> 19) & 7); }
AKV_HD constexpr int f6_wbits(uint32_t e) { return static_cast<int>((e >> 22) & 127); }
// Weight stream kinds of the fast path: plain 2-bit and 3-bit codes, quints
// (0..4), trits (0..2) and trits with one extra bit (0..5).
enum : int { kF6W2 = 0, kF6W3 = 1, kF6Q0 = 2, kF6T0 = 3, kF6T1 = 4 };

// Header classes of 6x6 blocks (Fast6Tables::klass): constant blocks, blocks
// left to the runtime classifier, luminance blocks with a reduced grid, and
// the luminance full-grid classes decoded by fully specialised code, each a
// (weight range, partitions, colour range) triple. The colour range follows
// from the other two (and the block mode) when every endpoint mode is 0.
enum : int { kC6Const = 0, kC6Other = 1, kC6Reduced = 2, kC6First = 3 };
struct F6Class {
    int wq, parts, cq;
};
// Ordered by how often astcenc picks them for scalar KV data (the reference
// corpus: 40 %, 26 %, 20 %, 5 % for the first four).
constexpr F6Class kF6Classes[] = {{3, 2, 7},  {4, 1, 20}, {2, 3, 9},  {2, 2, 16}, {1, 4, 11},
                                  {1, 3, 16}, {3, 1, 20}, {2, 1, 20}, {1, 1, 20}, {1, 2, 20}};
constexpr int kF6NumClasses = static_cast<int>(sizeof(kF6Classes) / sizeof(kF6Classes[0]));
constexpr int kC6Count = kC6First + kF6NumClasses;

struct Fast6Tables {
    uint32_t info[8192];         // (mode | (partitions - 1) << 11) -> info entry, 0 = not on the fast path
    uint8_t klass[8192];         // the same index -> header class (kC6*) | 0x80 for luminance candidates
    uint32_t spread2[256];       // four 2-bit fields -> four bytes
    uint32_t spread3[4096];      // four 3-bit fields -> four bytes
    uint32_t quint0[128];        // 7-bit quint block -> its three digits as bytes
    uint32_t trit0[256][2];      // 8-bit trit block -> its five digits as bytes (4 + 1)
    uint32_t trit1[8192][2];     // 13-bit group of a 0..5 stream -> its five codes as bytes (4 + 1)
};

// Fills `f` from the base tables `t` (which build_tables filled).
void build_fast6_tables(const Tables& t, Fast6Tables* f);

// Number of bits a BISE stream of `count` values of range `q` occupies.
int bise_stream_bits(int count, int q);

}  // namespace akv
