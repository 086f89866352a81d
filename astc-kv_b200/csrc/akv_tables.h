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

// Number of bits a BISE stream of `count` values of range `q` occupies.
int bise_stream_bits(int count, int q);

}  // namespace akv
