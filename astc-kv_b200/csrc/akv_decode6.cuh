// Sorted, class-specialised decode of 6x6 scalar planes for the fused
// attention kernel (akv_attn_fast.cuh).
//
// Every 6x6 block astcenc writes for scalar KV data is luminance-direct and
// single-plane, and its 13 low bits (block mode, partition count) fix the rest
// of its layout: weight range, colour range, both stream lengths. A handful of
// such (weight range, partitions, colour range) classes cover nearly all
// blocks. Decoding each lane's own block lets a warp pay for every class its
// 32 blocks contain, so one chunk of blocks is decoded in three phases:
//
//   S  every thread classifies one block (one lookup, Fast6Tables::klass) and
//      the chunk's blocks are counting-sorted by class;
//   H  thread j decodes the j-th block in class order, so a warp runs one or
//      two class paths: colour integers and weight groups at compile-time bit
//      positions (weight groups by one window lookup each), the partition
//      pattern, then the block's value table (entry = L * partition + code)
//      and the entry byte of every texel go to the block's record;
//      reduced-grid and unusual blocks take descriptor / generic slots;
//   T  thread i writes the texels of block i from its record, blocks in the
//      natural 4 x 8 tiling whose pair stores fall on distinct banks.
#pragma once
#include "akv_decode_fast.cuh"

namespace akv {
namespace fast {

constexpr int kLevelsCt[21] = {2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32, 40, 48, 64, 80, 96, 128, 160, 192, 256};

struct RangeShape {
    int bits, trits, quints;
};

constexpr RangeShape range_shape(int q) {
    int n = kLevelsCt[q];
    RangeShape s{0, 0, 0};
    if (n % 3 == 0) { s.trits = 1; n /= 3; }
    else if (n % 5 == 0) { s.quints = 1; n /= 5; }
    while ((1 << s.bits) < n) s.bits++;
    return s;
}

constexpr int bise_bits_ct(int count, int q) {
    return count * range_shape(q).bits + (range_shape(q).trits ? (8 * count + 4) / 5 : 0) +
           (range_shape(q).quints ? (7 * count + 2) / 3 : 0);
}

constexpr int weight_kind_ct(int wq) {
    return wq == 1 ? kF6T0 : wq == 2 ? kF6W2 : wq == 3 ? kF6Q0 : wq == 4 ? kF6T1 : kF6W3;
}

// The NV colour integers of range CQ (unquantised to 0..255) from the colour
// stream `cs` (its first bit at bit 0, masked to its length): plain-bit,
// trit or quint groups at compile-time offsets.
template <int CQ, int NV>
__device__ __forceinline__ void colours_ct(uint64_t cs, int (&v)[8]) {
    constexpr RangeShape sh = range_shape(CQ);
    constexpr int b = sh.bits;
    constexpr uint32_t bm = (1u << b) - 1u;
    const uint8_t* un = g_akv_tables.cunq[CQ];
    if constexpr (!sh.trits && !sh.quints) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int code = static_cast<int>(static_cast<uint32_t>(cs >> (j * b)) & bm);
            v[j] = CQ == 20 ? code : __ldg(un + code);  // 256 levels: the identity
        }
    } else if constexpr (sh.trits) {
        constexpr int GB = 5 * b + 8;
        constexpr int off[5] = {0, b + 2, 2 * b + 4, 3 * b + 5, 4 * b + 7};
#pragma unroll
        for (int g = 0; g * 5 < NV; ++g) {
            const uint64_t x = cs >> (g * GB);
            const uint32_t T = static_cast<uint32_t>(((x >> b) & 3u) | (((x >> (2 * b + 2)) & 3u) << 2) |
                                                     (((x >> (3 * b + 4)) & 1u) << 4) | (((x >> (4 * b + 5)) & 3u) << 5) |
                                                     (((x >> (5 * b + 7)) & 1u) << 7));
            const uint32_t d = __ldg(&g_akv_tables.trit[T]);
#pragma unroll
            for (int j = 0; j < 5; ++j)
                if (g * 5 + j < NV) {
                    const uint32_t m = static_cast<uint32_t>(x >> off[j]) & bm;
                    v[g * 5 + j] = __ldg(un + ((((d >> (2 * j)) & 3u) << b) | m));
                }
        }
    } else {
        constexpr int GB = 3 * b + 7;
        constexpr int off[3] = {0, b + 3, 2 * b + 5};
#pragma unroll
        for (int g = 0; g * 3 < NV; ++g) {
            const uint64_t x = cs >> (g * GB);
            const uint32_t Q = static_cast<uint32_t>(((x >> b) & 7u) | (((x >> (2 * b + 3)) & 3u) << 3) |
                                                     (((x >> (3 * b + 5)) & 3u) << 5));
            const uint32_t d = __ldg(&g_akv_tables.quint[Q]);
#pragma unroll
            for (int j = 0; j < 3; ++j)
                if (g * 3 + j < NV) {
                    const uint32_t m = static_cast<uint32_t>(x >> off[j]) & bm;
                    v[g * 3 + j] = __ldg(un + ((((d >> (3 * j)) & 7u) << b) | m));
                }
        }
    }
}

// Class K (kF6Classes[K]) block: its value table at tab[e * nt] (entry e =
// L * partition + code) and the entry byte of each texel in idx.
template <int K>
__device__ __forceinline__ void decode_class6(uint4 blk, bool affine, float sc, float of, uint32_t* tab, int nt,
                                              uint32_t (&idx)[9]) {
    constexpr F6Class C = kF6Classes[K];
    constexpr int WQ = C.wq, PARTS = C.parts, CQ = C.cq, L = kLevelsCt[WQ];
    constexpr int CSTART = PARTS == 1 ? 17 : 29;
    constexpr int CBITS = bise_bits_ct(2 * PARTS, CQ);
    constexpr int WBITS = bise_bits_ct(36, WQ);
    static_assert(CBITS < 64 && PARTS * L <= 12, "class fits the fast path");
    const uint64_t lo = (static_cast<uint64_t>(blk.y) << 32) | blk.x;
    const uint64_t hi = (static_cast<uint64_t>(blk.w) << 32) | blk.z;
    const uint64_t cs = ((lo >> CSTART) | (hi << (64 - CSTART))) & ((1ull << CBITS) - 1ull);
    int v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    colours_ct<CQ, 2 * PARTS>(cs, v);
    const uint64_t s0 = __brevll(hi), s1 = __brevll(lo);
    uint32_t w[4] = {static_cast<uint32_t>(s0), static_cast<uint32_t>(s0 >> 32), static_cast<uint32_t>(s1),
                     static_cast<uint32_t>(s1 >> 32)};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if (32 * k >= WBITS) w[k] = 0u;
        else if (32 * (k + 1) > WBITS) w[k] &= (1u << (WBITS - 32 * k)) - 1u;
    }
    uint32_t cw[9];
    weight_codes6<weight_kind_ct(WQ)>(w, cw);
    if constexpr (PARTS > 1) {
        const uint32_t* pt = g_akv_tables.part[1][PARTS - 2][(blk.x >> 13) & 0x3FF];
        const uint32_t pw[3] = {__ldg(pt), __ldg(pt + 1), __ldg(pt + 2)};
#pragma unroll
        for (int k = 0; k < 9; ++k)
            idx[k] = cw[k] + static_cast<uint32_t>(L) * __ldg(&g_f6.spread2[(pw[k >> 2] >> (8 * (k & 3))) & 0xFFu]);
    } else {
#pragma unroll
        for (int k = 0; k < 9; ++k) idx[k] = cw[k];
    }
    build_table(v, PARTS, WQ, L, affine, sc, of, tab, nt);
}

template <int... K>
__device__ __forceinline__ void decode_class6_any(int k, uint4 blk, bool affine, float sc, float of, uint32_t* tab,
                                                  int nt, uint32_t (&idx)[9], std::integer_sequence<int, K...>) {
    ((k == K ? (decode_class6<K>(blk, affine, sc, of, tab, nt, idx), 0) : 0), ...);
}

#ifdef __CUDACC__
// (The per-block functions above also build for the host test emulator; the
// CTA-wide plane decode below is device code only.)

// Scratch of the decode of one plane-chunk of up to NB 6x6 blocks. Records
// and code columns are indexed by the block's position in the chunk (its
// natural index), with a stride NS of whole bank rows.
template <int NB>
struct Scratch6 {
    static constexpr int NS = ((NB + 31) / 32) * 32;
    static constexpr int kTab = 12;                      // value-table entries per record
    static constexpr int kSlowCap = NB < 64 ? NB : 64;   // descriptor / generic slots
    uint32_t tab[kTab][NS];         // block i's value table at tab[e][i]
    uint32_t idx[9][NS];            // block i's texel entry bytes
    uint8_t codes[36 + kCodePad][NS];  // block i's colour / weight codes (runtime and descriptor paths)
    uint16_t order[NS];             // sorted position -> block index | class << 8
    uint8_t slotted[NS];            // block i is evaluated by the slot phases
    int cnt[kC6Count];
    int base[kC6Count];
    int nslot;
    uint32_t slot_pos[kSlowCap];
    float2 slot_aff[kSlowCap];
    uint32_t slot_src[kSlowCap];
    BlockDesc<1> desc[kSlowCap];
    alignas(16) uint8_t w[kSlowCap][72];
};

// Decode one 6x6 plane's chunk into the hi/lo tiles. All threads call it.
template <int D, int THREADS, int NB, int LD>
__device__ __forceinline__ void decode_plane6(const uint4* raw, const __half* moff, const __half* mscl, int norm,
                                              int cols, int rows_blk, int n, bool valid, Scratch6<NB>& ds,
                                              __half (*thi)[LD], __half (*tlo)[LD]) {
    constexpr int BS = 6;
    constexpr int NS = Scratch6<NB>::NS;
    constexpr int kCap = Scratch6<NB>::kSlowCap;
    static_assert(NB <= THREADS, "one block per thread in each phase");
    static_assert(D % 8 == 0, "whole 8-texel rows");
    const int nblk = rows_blk * cols;
    const bool affine = norm == AKV_NORM_BLOCK_AFFINE;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    if (tid < kC6Count) ds.cnt[tid] = 0;
    if (tid == 0) ds.nslot = 0;
    __syncthreads();
    // Phase S: classify and rank within the class (warp-aggregated counts).
    int my_k = 0, my_r = 0;
    {
        const bool act = tid < nblk;
        if (act) {
            const uint4 blk = raw[tid];
            int k = __ldg(&g_f6.klass[blk.x & 0x1FFFu]);
            if (k & 0x80) {
                const bool cem0 = (blk.x & 0x1800u) == 0 ? ((blk.x >> 13) & 15) == 0 : ((blk.x >> 23) & 0x3F) == 0;
                k = cem0 ? (k & 0x7F) : kC6Other;
            }
            my_k = k;
        }
        const unsigned amask = __ballot_sync(0xFFFFFFFFu, act);
        if (act) {
            const unsigned peers = __match_any_sync(amask, my_k);
            const int leader = __ffs(peers) - 1;
            int b0 = 0;
            if (lane == leader) b0 = atomicAdd(&ds.cnt[my_k], __popc(peers));
            b0 = __shfl_sync(peers, b0, leader);
            my_r = b0 + __popc(peers & ((1u << lane) - 1u));
        }
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
#pragma unroll
        for (int c = 0; c < kC6Count; ++c) {
            ds.base[c] = acc;
            acc += ds.cnt[c];
        }
    }
    __syncthreads();
    if (tid < nblk) ds.order[ds.base[my_k] + my_r] = static_cast<uint16_t>(tid | (my_k << 8));
    __syncthreads();
    // Phase H: blocks in class order.
    if (tid < nblk) {
        const int e = ds.order[tid];
        const int i = e & 0xFF, k = e >> 8;
        const uint4 blk = raw[i];
        const int br = i / cols, bc = i - br * cols;
        const int row0 = br * BS, col0 = bc * BS;
        const int rows = valid ? min(BS, n - row0) : 0;
        const int ncol = min(BS, D - col0);
        const float sc = affine ? __half2float(mscl[i]) : 0.f;
        const float of = affine ? __half2float(moff[i]) : 0.f;
        uint32_t* tab = &ds.tab[0][i];
        uint8_t* cc = &ds.codes[0][i];
        bool slotted = false;
        uint32_t idx[9] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        bool have_idx = true;
        if (k >= kC6First) {
            decode_class6_any(k - kC6First, blk, affine, sc, of, tab, NS, idx,
                              std::make_integer_sequence<int, kF6NumClasses>{});
        } else if (k == kC6Const) {
            tab[0] = table_entry(c16_to_unit(const_c16(blk)), affine, sc, of);
        } else {
            // Reduced grids (table header path) and everything else (runtime
            // classifier): a value table when it fits, else a slot.
            have_idx = false;
            int slot = -1, kind = kKindDesc, cq = 0;
            uint32_t me = 0u;
            F6Lum o;
            bool fast_hdr = k == kC6Reduced;
            if (!fast_hdr) kind = block_kind<BS>(blk, me, cq);
            if (!fast_hdr && kind == kKindConst) {
                tab[0] = table_entry(c16_to_unit(const_c16(blk)), affine, sc, of);
                have_idx = true;
            } else if (!fast_hdr && kind == kKindTable &&
                       (((blk.x >> 11) & 3) + 1) * range_levels(mode_wq(me)) <= Scratch6<NB>::kTab) {
                LumOut lo;
                decode_lum<BS>(blk, kind, me, cq, affine, sc, of, tab, cc, NS, nullptr, lo);
#pragma unroll
                for (int t = 0; t < 36; ++t) {
                    const uint32_t part = (lo.pat[t >> 4] >> (2 * (t & 15))) & 3u;
                    idx[t >> 2] |= ((cc[t * NS] & lo.cmask) + part * static_cast<uint32_t>(lo.L)) << (8 * (t & 3));
                }
                have_idx = true;
            } else {
                slot = atomicAdd(&ds.nslot, 1);
                slotted = true;
                if (slot >= kCap) {
                    eval_block_generic<BS, LD>(blk, norm, sc, of, moff, mscl, row0, col0, rows, ncol, thi, tlo);
                } else if (!fast_hdr && kind == kKindGeneric) {
                    ds.slot_pos[slot] = static_cast<uint32_t>(row0) | (static_cast<uint32_t>(col0) << 16);
                    ds.slot_aff[slot] = make_float2(sc, of);
                    decode_header_slow<BS>(blk, ds.desc[slot], ds.w[slot]);
                } else {
                    BlockDesc<1>& d = ds.desc[slot];
                    int wq;
                    if (fast_hdr) {
                        const uint32_t f6 = __ldg(&g_f6.info[blk.x & 0x1FFFu]);
                        decode_f6_lum(blk, f6, cc, NS, o);
                        const uint32_t me6 = __ldg(&g_akv_tables.mode[1][blk.x & 0x7FFu]);
                        const int wx = mode_wx(me6), wy = mode_wy(me6);
                        if (o.parts > 1) {
                            const uint32_t* pt = g_akv_tables.part[1][o.parts - 2][(blk.x >> 13) & 0x3FF];
                            d.pat[0] = __ldg(pt); d.pat[1] = __ldg(pt + 1);
                            d.pat_hi[0] = __ldg(pt + 2); d.pat_hi[1] = __ldg(pt + 3);
                        } else {
                            d.pat[0] = d.pat[1] = d.pat_hi[0] = d.pat_hi[1] = 0u;
                        }
                        d.ep[0] = static_cast<uint32_t>(o.v[0] | (o.v[2] << 8) | (o.v[4] << 16) | (o.v[6] << 24));
                        d.ep[1] = static_cast<uint32_t>(o.v[1] | (o.v[3] << 8) | (o.v[5] << 16) | (o.v[7] << 24));
                        d.info = static_cast<uint32_t>(o.parts - 1) | (1u << kInfoReduced) |
                                 (static_cast<uint32_t>(wx) << kInfoWx) | (static_cast<uint32_t>(wy) << kInfoWy);
                        const int count = wx * wy;
#pragma unroll
                        for (int j = 0; j < 36; ++j)
                            if (j < count) cc[j * NS] = static_cast<uint8_t>(byte_of(o.cw, j));
                        wq = o.wq;
                    } else {
                        // Luminance descriptor (reduced grid or a table too
                        // large for the record) through the runtime decoder.
                        LumOut lo;
                        decode_lum<BS>(blk, kKindDesc, me, cq, affine, sc, of, tab, cc, NS, &d, lo);
                        wq = mode_wq(me);
                    }
                    ds.slot_pos[slot] = static_cast<uint32_t>(row0) | (static_cast<uint32_t>(col0) << 16) | kSlotRows;
                    ds.slot_aff[slot] = make_float2(sc, of);
                    ds.slot_src[slot] = static_cast<uint32_t>(i) | (static_cast<uint32_t>(wq) << 16);
                }
            }
        }
        ds.slotted[i] = slotted ? 1 : 0;
        if (have_idx) {
#pragma unroll
            for (int q = 0; q < 9; ++q) ds.idx[q][i] = idx[q];
        }
    }
    __syncthreads();
    const int nslow = min(ds.nslot, kCap);
    if (nslow > 0) {
        // Phase 1a: grid weights of the descriptor slots, one grid row per
        // task, from the code column of the slot's block.
        const bool wide = nslow * 8 > THREADS;
        const int nwtask = wide ? ((nslow + 31) & ~31) * 8 : nslow * 8;
        for (int task = tid; task < nwtask; task += THREADS) {
            const int g = task >> 5;
            const int slot = wide ? (((g >> 3) << 5) | (task & 31)) : task >> 3;
            const int r = wide ? g & 7 : task & 7;
            if (slot >= nslow || !(ds.slot_pos[slot] & kSlotRows)) continue;
            const uint32_t info = ds.desc[slot].info, src = ds.slot_src[slot];
            const int wx = (info >> kInfoWx) & 15, wy = (info >> kInfoWy) & 15;
            if (r >= wy) continue;
            const uint8_t* un = g_akv_tables.wunq[src >> 16];
            const uint8_t* cc = &ds.codes[0][src & 0xFFFFu];
#pragma unroll
            for (int c = 0; c < BS; ++c)
                if (c < wx) ds.w[slot][8 * r + c] = desc_weight(cc, NS, un, wx, 8 * r + c);
        }
        __syncthreads();
    }
    // Phase T: texels of the table / constant blocks, natural tiling.
    {
        const int tiles_c = (cols + 7) >> 3, ntiles = ((rows_blk + 3) >> 2) * tiles_c;
        const bool tiled = ntiles * 32 <= THREADS;
        const int nitems = tiled ? ntiles * 32 : nblk;
        for (int it = tid; it < nitems; it += THREADS) {
            int br, bc;
            if (tiled) {
                const int tile = it >> 5, tr = tile / tiles_c, tc = tile - tr * tiles_c;
                br = 4 * tr + ((it >> 3) & 3);
                bc = 8 * tc + (it & 7);
                if (br >= rows_blk || bc >= cols) continue;
            } else {
                br = it / cols;
                bc = it - br * cols;
            }
            const int i = br * cols + bc;
            if (ds.slotted[i]) continue;
            uint32_t idx[9];
#pragma unroll
            for (int q = 0; q < 9; ++q) idx[q] = ds.idx[q][i];
            write6<LD>(idx, &ds.tab[0][i], NS, norm, moff, mscl, br * BS, bc * BS, thi, tlo);
        }
    }
    if (nslow > 0) {
        // Phase 1b: one segment (two texels) of a slotted block per task;
        // generic slots take a whole row per segment-0 task.
        constexpr int SEG = kDescSeg<BS>;
        constexpr int NSEG = BS / SEG;
        const int ntask = nslow * BS * NSEG;
        for (int task = tid; task < ntask; task += THREADS) {
            const int slot = task / (BS * NSEG), r = task - slot * (BS * NSEG);
            const int y = r / NSEG, x0 = (r - y * NSEG) * SEG;
            const uint32_t pos = ds.slot_pos[slot];
            const int row = static_cast<int>(pos & 0x7FFFu) + y, col0 = static_cast<int>(pos >> 16);
            const BlockDesc<1>& d = ds.desc[slot];
            const bool ok = valid && row < n;
            const float2 aff = ds.slot_aff[slot];
            if (!(pos & kSlotRows)) {
                if (x0 == 0)
                    eval_row_generic<BS, D, LD>(d, ds.w[slot], y, row, col0, ok, norm, aff, moff, mscl, thi, tlo);
                continue;
            }
            const int col = col0 + x0;
            if (col >= D) continue;
            uint32_t c[SEG];
            desc_seg_c16<BS, SEG>(d.info, ds.w[slot],
                                  row_pattern<BS>(d.pat[0], d.pat[1], d.pat_hi[0], d.pat_hi[1], y), d.ep[0], d.ep[1], y,
                                  x0, c);
            float rs = aff.x, ro = aff.y;
            if (norm == AKV_NORM_TOKEN) { rs = __half2float(mscl[row]); ro = __half2float(moff[row]); }
#pragma unroll
            for (int x = 0; x < SEG; x += 2) {
                float s0 = rs, o0 = ro, s1 = rs, o1 = ro;
                if (norm == AKV_NORM_PAGE_CHANNEL && col + x < D) {
                    s0 = __half2float(mscl[col + x]); o0 = __half2float(moff[col + x]);
                    s1 = __half2float(mscl[col + x + 1]); o1 = __half2float(moff[col + x + 1]);
                }
                uint32_t hw, lw;
                split_pair(fmaf(c16_to_unit(c[x]), s0, o0), fmaf(c16_to_unit(c[x + 1]), s1, o1), hw, lw);
                if (!ok) hw = lw = 0u;
                if (col + x < D) {
                    *reinterpret_cast<uint32_t*>(&thi[row][col + x]) = hw;
                    *reinterpret_cast<uint32_t*>(&tlo[row][col + x]) = lw;
                }
            }
        }
    }
    __syncthreads();
}
#endif  // __CUDACC__

}  // namespace fast
}  // namespace akv
