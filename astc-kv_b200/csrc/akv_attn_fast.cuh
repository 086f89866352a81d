// Fast split-K decode attention for scalar-layout ASTC V (and FP16 or scalar
// ASTC K) on sm_100a.
//
// Per CTA: one (split, kv head, batch) unit, processed in chunks of CH tokens
// (CH = 48 with a 6x6 plane, 32 when K is ASTC too, 64 otherwise; a chunk
// never crosses a page), 64 threads per 16-token tile.
//
//   * Staging: one elected thread issues cp.async.bulk copies of the chunk's
//     V blocks and fp16 metadata (and ASTC K blocks) into a two-stage shared
//     ring, completed on mbarriers; consumers wait with a bounded try_wait.
//   * Decode (decode_plane): one thread per block with the runtime decoder of
//     akv_decode_fast.cuh, the same instructions for every weight range and
//     partition count (small machine code, no per-class divergence).
//     Luminance blocks with a full-resolution grid become a value table
//     (v = scale*u + offset split into fp16 hi and lo for block-affine
//     planes) plus a weight-code byte per texel, and the thread writes its
//     texels into the padded [token][channel] hi/lo tiles; reduced-grid,
//     large-table and generic blocks become descriptors whose texels are
//     evaluated one thread per texel afterwards.
//   * Tensor cores (mma.sync m16n8k16, fp32 accumulation). Every warp owns
//     one (16-token tile, half of the head dims) pair; the query heads of
//     the GQA group are the N=8 dimension:
//       S^T[tok][head] = K . Q^T   (q hi+lo; FP16 K staged in shared memory
//                                   by 16-byte cp.async copies issued a
//                                   chunk ahead (they land during the
//                                   chunk's decode), or decoded K hi+lo;
//                                   both warps of a tile compute it)
//       online softmax per head in base 2, P^T as fp16 hi + lo through a
//       512-byte per-warp buffer,
//       O^T[dim][head] += V^T . P^T  for the warp's dim half (V hi and lo,
//                                     ldmatrix.trans).
//   * Each warp keeps its own (m, l, O half) over its token slices; the
//     warps merge at the end and the CTA writes one split partial (m, l,
//     acc), the same workspace format the merge kernel reads.
#pragma once
#include <math_constants.h>

#include "akv_attention_kernels.cuh"
#include "akv_common.cuh"
#include "akv_decode_fast.cuh"

namespace akv {
namespace fast {

// Iterations of mbarrier.try_wait before a wait is declared stuck. Each
// try_wait may itself block for a hardware-defined interval, so this bounds a
// wait at roughly seconds, far beyond any healthy copy.
constexpr uint32_t kWaitIters = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bounded wait on phase `parity`; false when the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < kWaitIters; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred P1;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, P1;\n\t}"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Global -> shared bulk copy (no multicast), completion on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 16-byte global -> shared asynchronous copy; `bytes` 0 writes zeros (the
// source is then not read).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// L2 prefetch of one global-memory line.
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// A register-only operation (no memory, no side effects): not volatile, so
// the compiler may interleave independent accumulator chains.
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// v -> (fp16 hi, fp16 lo) with hi + lo == v to ~2^-22 relative.
__device__ __forceinline__ void split_pair(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_h2(v0 - hf.x, v1 - hf.y);
}

// Metadata elements per chunk for a plane (a chunk of CH tokens spans
// max(1, CH / P) pages of P tokens; page-channel metadata is per page).
template <int BS>
__device__ __forceinline__ int meta_elems(int norm, int cols, int CH, int D, int P) {
    return norm == AKV_NORM_BLOCK_AFFINE ? (CH / BS) * cols : (norm == AKV_NORM_TOKEN ? CH : D * (P < CH ? CH / P : 1));
}

template <int BS>
__device__ __forceinline__ int64_t meta_chunk_offset(int norm, int cols, int t_in_page) {
    return norm == AKV_NORM_BLOCK_AFFINE ? static_cast<int64_t>(t_in_page / BS) * cols
                                         : (norm == AKV_NORM_TOKEN ? t_in_page : 0);
}

// Generic header decode for the rare blocks the runtime path does not cover
// (kept out of line: it is large and rarely executed).
template <int BS>
__device__ __noinline__ void decode_header_slow(uint4 blk, BlockDesc<1>& d, uint8_t* w) {
    decode_header<1>(blk, footprint_index(BS), d, w);
}

// One thread decodes and evaluates a whole block (beyond the slot capacity;
// out of line, rarely executed).
template <int BS, int LD>
__device__ __noinline__ void eval_block_generic(uint4 blk, int norm, float sc, float of, const __half* moff,
                                                const __half* mscl, int row0, int col0, int rows, int ncol,
                                                __half (*thi)[LD], __half (*tlo)[LD]) {
    BlockDesc<1> d;
    uint8_t wl[64 + kCodePad];
    decode_header<1>(blk, footprint_index(BS), d, wl);
    for (int t = 0; t < BS * BS; ++t) {
        const int x = t % BS, y = t / BS;
        if (x >= ncol) continue;
        uint32_t cv[1];
        texel_values<BS, 1>(d, wl, x, y, cv);
        const float u = c16_to_unit(cv[0]);
        float s = sc, o = of;
        if (norm == AKV_NORM_TOKEN) { s = __half2float(mscl[row0 + y]); o = __half2float(moff[row0 + y]); }
        if (norm == AKV_NORM_PAGE_CHANNEL) { s = __half2float(mscl[col0 + x]); o = __half2float(moff[col0 + x]); }
        const float v = fmaf(u, s, o);
        const __half hv = __float2half_rn(v);
        const bool ok = y < rows;
        thi[row0 + y][col0 + x] = ok ? hv : __float2half_rn(0.f);
        tlo[row0 + y][col0 + x] = ok ? __float2half_rn(v - __half2float(hv)) : __float2half_rn(0.f);
    }
}

// Scratch of the decode of one plane-chunk of up to NB blocks by NT threads
// (N = texels per block).
template <int NB, int NT, int BS>
struct DecodeScratch {
    static constexpr int N = BS * BS;
    // Descriptor slots: every block of a small chunk (8x8 planes are mostly
    // reduced grids), at most 64; 40 for 6x6 planes (astcenc's 6x6 chunks
    // hold about ten descriptor blocks in 176).
    static constexpr int kSlowMax = BS == 6 ? 40 : 64;
    static constexpr int kSlowCap = NB < kSlowMax ? NB : kSlowMax;
    // Columns: one per decoding thread (a chunk with fewer blocks than
    // threads leaves the others idle).
    static constexpr int NC = NT < ((NB + 31) / 32) * 32 ? NT : ((NB + 31) / 32) * 32;
    uint32_t tab[kTabCap<BS> > 0 ? kTabCap<BS> : 1][NC];  // value tables, thread-interleaved (conflict-free lookups)
    uint8_t codes[N + kCodePad][NC];  // weight codes, thread-interleaved (+ slack rows)
    int nslot;                  // descriptor slots taken in this plane-chunk
    // Per slot: tile row | kSlotRows | tile column << 16; block-affine
    // (scale, offset); owner thread | weight range << 16 (late expansion).
    uint32_t slot_pos[kSlowCap];
    float2 slot_aff[kSlowCap];
    uint32_t slot_src[kSlowCap];
    BlockDesc<1> desc[kSlowCap];
    // Grid weights: rows of 8 bytes for luminance descriptors (desc_seg_c16),
    // the decode_header layout for generic blocks; 8 bytes of slack either way.
    alignas(16) uint8_t w[kSlowCap][72];
};

// Slot flag: a luminance descriptor (decode_lum) evaluated by desc_seg_c16.
constexpr uint32_t kSlotRows = 1u << 15;

// One texel value v (fp32) -> the hi/lo tiles.
template <int LD>
__device__ __forceinline__ void put_texel(float v, bool ok, int row, int col, __half (*thi)[LD], __half (*tlo)[LD]) {
    const __half hv = __float2half_rn(v);
    thi[row][col] = ok ? hv : __float2half_rn(0.f);
    tlo[row][col] = ok ? __float2half_rn(v - __half2float(hv)) : __float2half_rn(0.f);
}

// Texel row y of a generic slot (decode_header layout) -> the hi/lo tiles
// (out of line: generic blocks are rare).
template <int BS, int D, int LD>
__device__ __noinline__ void eval_row_generic(const BlockDesc<1>& d, const uint8_t* w, int y, int row, int col0,
                                              bool ok, int norm, float2 aff, const __half* moff, const __half* mscl,
                                              __half (*thi)[LD], __half (*tlo)[LD]) {
    const bool lean = !(d.info & ((1u << kInfoVoid) | (1u << kInfoError) | (1u << kInfoDual)));
    for (int x = 0; x < BS && col0 + x < D; ++x) {
        uint32_t c16;
        if (lean) {
            c16 = desc_texel_c16<BS>(d, w, y * BS + x);
        } else {
            uint32_t cv[1];
            texel_values<BS, 1>(d, w, x, y, cv);
            c16 = cv[0];
        }
        float s = aff.x, o = aff.y;
        if (norm == AKV_NORM_TOKEN) { s = __half2float(mscl[row]); o = __half2float(moff[row]); }
        if (norm == AKV_NORM_PAGE_CHANNEL) { s = __half2float(mscl[col0 + x]); o = __half2float(moff[col0 + x]); }
        put_texel<LD>(fmaf(c16_to_unit(c16), s, o), ok, row, col0 + x, thi, tlo);
    }
}

// The 2^16 u values tv of a directly evaluated block, normalised (NORM fixed
// per instantiation) -> the hi/lo tiles (rows past the chunk's tokens are
// zeroed afterwards by the kernel).
template <int BS, int LD, int NORM>
__device__ __forceinline__ void write_direct_n(const float (&tv)[BS * BS], float sc, float of, const __half* moff,
                                               const __half* mscl, int row0, int col0, int rows, __half (*thi)[LD],
                                               __half (*tlo)[LD]) {
    // Scales times 2^-16 (tv is 2^16 u; exact, the FMA still rounds once).
    float cs[BS], co[BS];
#pragma unroll
    for (int x = 0; x < BS; ++x) {
        cs[x] = NORM == AKV_NORM_PAGE_CHANNEL ? __half2float(mscl[col0 + x]) * 0x1p-16f : sc * 0x1p-16f;
        co[x] = NORM == AKV_NORM_PAGE_CHANNEL ? __half2float(moff[col0 + x]) : of;
    }
#pragma unroll
    for (int y = 0; y < BS; ++y) {
        float rs = 0.f, ro = 0.f;
        if (NORM == AKV_NORM_TOKEN) {
            rs = __half2float(mscl[row0 + y]) * 0x1p-16f;
            ro = __half2float(moff[row0 + y]);
        }
#pragma unroll
        for (int x = 0; x < BS; x += 2) {
            uint32_t h, l;
            const float s0 = NORM == AKV_NORM_TOKEN ? rs : cs[x], s1 = NORM == AKV_NORM_TOKEN ? rs : cs[x + 1];
            const float o0 = NORM == AKV_NORM_TOKEN ? ro : co[x], o1 = NORM == AKV_NORM_TOKEN ? ro : co[x + 1];
            split_pair(fmaf(tv[y * BS + x], s0, o0), fmaf(tv[y * BS + x + 1], s1, o1), h, l);
            *reinterpret_cast<uint32_t*>(&thi[row0 + y][col0 + x]) = h;
            *reinterpret_cast<uint32_t*>(&tlo[row0 + y][col0 + x]) = l;
        }
    }
}

// Texels of a directly evaluated (kDirect) table / constant block -> the
// hi/lo tiles: every texel's value first (the constant case decided once
// per block), then the block's normalisation applied with its scales and
// offsets loaded once (the footprint divides the head dimension, so every
// column is in range).
template <int BS, int LD>
__device__ __forceinline__ void write_direct(const LumOut& o, const uint8_t* codes, int nt, int norm, float sc,
                                             float of, const __half* moff, const __half* mscl, int row0, int col0,
                                             int rows, __half (*thi)[LD], __half (*tlo)[LD]) {
    float tv[BS * BS];
    if (o.cmask) {
#pragma unroll
        for (int t = 0; t < BS * BS; ++t) tv[t] = direct_t(o, codes, nt, t);
    } else {
        const float ct = o.cu * 65536.f;
#pragma unroll
        for (int t = 0; t < BS * BS; ++t) tv[t] = ct;
    }
    if (norm == AKV_NORM_TOKEN)
        write_direct_n<BS, LD, AKV_NORM_TOKEN>(tv, sc, of, moff, mscl, row0, col0, rows, thi, tlo);
    else if (norm == AKV_NORM_PAGE_CHANNEL)
        write_direct_n<BS, LD, AKV_NORM_PAGE_CHANNEL>(tv, sc, of, moff, mscl, row0, col0, rows, thi, tlo);
    else
        write_direct_n<BS, LD, AKV_NORM_BLOCK_AFFINE>(tv, sc, of, moff, mscl, row0, col0, rows, thi, tlo);
}

// Texels of one table / constant block -> the hi/lo tiles (pairs of columns
// per 32-bit store), from the value table or, for kDirect footprints, from
// endpoints and weights. Rows past the chunk's tokens are written like the
// others and zeroed afterwards by the kernel.
template <int BS, int LD>
__device__ __forceinline__ void write_block(const LumOut& o, const uint32_t* tab, const uint8_t* codes, int nt,
                                            int norm, float sc, float of, const __half* moff, const __half* mscl,
                                            int row0, int col0, int rows, int cols, __half (*thi)[LD],
                                            __half (*tlo)[LD]) {
    if constexpr (kDirect<BS>) {
        static_assert(BS == 4, "direct evaluation is for 4x4 blocks (whole columns: D % 4 == 0)");
        write_direct<BS, LD>(o, codes, nt, norm, sc, of, moff, mscl, row0, col0, rows, thi, tlo);
        return;
    }
    const bool affine = norm == AKV_NORM_BLOCK_AFFINE;
    const uint32_t L = static_cast<uint32_t>(o.L);
#pragma unroll
    for (int y = 0; y < BS; ++y) {
        float rs = 0.f, ro = 0.f;
        if (norm == AKV_NORM_TOKEN) {
            rs = __half2float(mscl[row0 + y]);
            ro = __half2float(moff[row0 + y]);
        }
#pragma unroll
        for (int x = 0; x < BS; x += 2) {
            // No column check: a block overhanging the head dimension (6x6)
            // writes its extra columns into the tile rows' padding (LD =
            // D + 8) and reads metadata inside the chunk's metadata array;
            // neither is read for results.
            {
                const int i = y * BS + x;
                uint32_t h, l;
                const uint32_t c0 = codes[i * nt], c1 = codes[(i + 1) * nt];
                const uint32_t p0 = (o.pat[i >> 4] >> (2 * (i & 15))) & 3u;
                const uint32_t p1 = (o.pat[(i + 1) >> 4] >> (2 * ((i + 1) & 15))) & 3u;
                const uint32_t a = tab[(p0 * L + c0) * nt], b2 = tab[(p1 * L + c1) * nt];
                if (affine) {
                    h = __byte_perm(a, b2, 0x5410);
                    l = __byte_perm(a, b2, 0x7632);
                } else {
                    float s0 = rs, o0 = ro, s1 = rs, o1 = ro;
                    if (norm == AKV_NORM_PAGE_CHANNEL) {
                        s0 = __half2float(mscl[col0 + x]); o0 = __half2float(moff[col0 + x]);
                        s1 = __half2float(mscl[col0 + x + 1]); o1 = __half2float(moff[col0 + x + 1]);
                    }
                    split_pair(fmaf(__uint_as_float(a), s0, o0), fmaf(__uint_as_float(b2), s1, o1), h, l);
                }
                *reinterpret_cast<uint32_t*>(&thi[row0 + y][col0 + x]) = h;
                *reinterpret_cast<uint32_t*>(&tlo[row0 + y][col0 + x]) = l;
            }
        }
    }
}

// Decode one plane's chunk into the hi/lo tiles. All threads call it.
//   phase 1  thread per block: table and constant blocks go straight to the
//            tiles; descriptor and generic blocks take a scratch slot;
//   phase 1a thread per grid-weight row of the descriptor slots (when each
//            thread decoded at most one block);
//   phase 1b thread per texel row (6x6: texel pair) of the slotted blocks.
// RESET: clear the slot count here (one barrier); otherwise the caller
// cleared it before its last barrier. wait_async: wait for the thread's
// cp.async copies before the slot phase's first barrier, which then also
// publishes them (the caller's next reads of those copies need no barrier
// of their own).
template <int BS, int D, int THREADS, int NB, int LD, bool RESET = true>
__device__ __forceinline__ void decode_plane(const uint4* raw, const __half* moff, const __half* mscl, int norm,
                                             int cols, int rows_blk, int n, bool valid,
                                             DecodeScratch<NB, THREADS, BS>& ds, __half (*thi)[LD],
                                             __half (*tlo)[LD], bool wait_async = false) {
    static_assert(BS % 2 == 0 && D % 8 == 0, "texel pairs; whole 8-texel rows");
    constexpr int kCap = DecodeScratch<NB, THREADS, BS>::kSlowCap;
    const int nblk = rows_blk * cols;
    const bool affine = norm == AKV_NORM_BLOCK_AFFINE;
    const int tid = threadIdx.x;
    if constexpr (RESET) {
        if (tid == 0) ds.nslot = 0;
        __syncthreads();
    }
    // Work items: when the chunk's 4 x 8 tiles of blocks (block rows x block
    // columns) fit the scratch columns, lane l of item group g takes block
    // (4 tr + l / 8, 8 tc + l % 8) of tile g, so the lanes' pair stores into
    // the tiles fall on distinct banks (6x6: row offsets 24 banks, column
    // offsets 3); otherwise items are blocks in row-major order. Either way
    // a thread's scratch column is its thread index.
    constexpr int NC = DecodeScratch<NB, THREADS, BS>::NC;
    const int tiles_c = (cols + 7) >> 3, ntiles = ((rows_blk + 3) >> 2) * tiles_c;
    const bool tiled = ntiles * 32 <= NC;
    const int nitems = tiled ? ntiles * 32 : nblk;
    // With at most one block per thread the code columns survive phase 1, so
    // descriptor grid weights are expanded by all threads afterwards (a lane
    // expanding its block alone would hold up its warp); otherwise by the
    // owner right away.
    const bool late_w = nitems <= THREADS;
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
        const uint4 blk = raw[i];
        const int row0 = br * BS, col0 = bc * BS;
        const int rows = valid ? min(BS, n - row0) : 0;
        const int ncol = min(BS, D - col0);
        const float sc = affine ? __half2float(mscl[i]) : 0.f;
        const float of = affine ? __half2float(moff[i]) : 0.f;
        uint32_t me;
        int cq;
        const int kind = block_kind<BS>(blk, me, cq);
        int slot = -1;
        if (kind == kKindDesc || kind == kKindGeneric) {
            slot = atomicAdd(&ds.nslot, 1);
            if (slot >= kCap) {
                eval_block_generic<BS, LD>(blk, norm, sc, of, moff, mscl, row0, col0, rows, ncol, thi, tlo);
                continue;
            }
            ds.slot_pos[slot] = static_cast<uint32_t>(row0) | (static_cast<uint32_t>(col0) << 16) |
                                (kind == kKindDesc ? kSlotRows : 0u);
            ds.slot_aff[slot] = make_float2(sc, of);
            if (kind == kKindGeneric) {
                decode_header_slow<BS>(blk, ds.desc[slot], ds.w[slot]);
                continue;
            }
        }
        LumOut o;
        decode_lum<BS>(blk, kind, me, cq, affine, sc, of, &ds.tab[0][tid], &ds.codes[0][tid], NC,
                       slot >= 0 ? &ds.desc[slot] : nullptr, o);
        if (slot < 0) {
            write_block<BS, LD>(o, &ds.tab[0][tid], &ds.codes[0][tid], NC, norm, sc, of, moff, mscl, row0, col0,
                                rows, ncol, thi, tlo);
        } else if (late_w) {
            ds.slot_src[slot] = static_cast<uint32_t>(tid) | (static_cast<uint32_t>(mode_wq(me)) << 16);
        } else {
            const uint8_t* un = g_akv_tables.wunq[mode_wq(me)];
            const int wx = mode_wx(me), wy = mode_wy(me);
            for (int r = 0; r < wy; ++r) {
#pragma unroll
                for (int c = 0; c < BS; ++c)
                    if (c < wx) ds.w[slot][8 * r + c] = desc_weight(&ds.codes[0][tid], NC, un, wx, 8 * r + c);
            }
        }
    }
    if (wait_async) cp_async_wait<0>();
    __syncthreads();
    const int nslow = min(ds.nslot, kCap);
    if (nslow > 0) {
        if (late_w) {
            // Phase 1a: grid weights of the descriptor slots, one grid row per
            // task. When that takes more than one round anyway, a warp takes
            // one row of 32 slots, so its lanes read the owners' code columns
            // side by side (one row of the code scratch) instead of one
            // column down (a single bank); else a slot's rows are adjacent.
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
                    if (c < wx) ds.w[slot][8 * r + c] = desc_weight(cc, NC, un, wx, 8 * r + c);
            }
            __syncthreads();
        }
        // Phase 1b: one segment (kDescSeg texels of a row) of a slotted block
        // per task; generic slots take a whole row per segment-0 task.
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
            uint32_t hw[SEG / 2], lw[SEG / 2];
#pragma unroll
            for (int x = 0; x < SEG; x += 2) {
                float s0 = rs, o0 = ro, s1 = rs, o1 = ro;
                if (norm == AKV_NORM_PAGE_CHANNEL && col + x < D) {
                    s0 = __half2float(mscl[col + x]); o0 = __half2float(moff[col + x]);
                    s1 = __half2float(mscl[col + x + 1]); o1 = __half2float(moff[col + x + 1]);
                }
                split_pair(fmaf(c16_to_unit(c[x]), s0, o0), fmaf(c16_to_unit(c[x + 1]), s1, o1), hw[x / 2], lw[x / 2]);
                if (!ok) hw[x / 2] = lw[x / 2] = 0u;
            }
            if constexpr (SEG == 8) {
                // A whole 8x8 row: one 16-byte store per tile (column 8 bc).
                *reinterpret_cast<uint4*>(&thi[row][col]) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(&tlo[row][col]) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            } else {
#pragma unroll
                for (int x = 0; x < SEG; x += 2) {
                    if (col + x < D) {
                        *reinterpret_cast<uint32_t*>(&thi[row][col + x]) = hw[x / 2];
                        *reinterpret_cast<uint32_t*>(&tlo[row][col + x]) = lw[x / 2];
                    }
                }
            }
        }
        __syncthreads();
    }
}

// One RGBA texel (four channel values v[0..3] of channels col..col+3) -> the
// hi/lo tiles, two 8-byte stores.
template <int LD>
__device__ __forceinline__ void put_rgba(const float (&v)[4], bool ok, int row, int col, __half (*thi)[LD],
                                         __half (*tlo)[LD]) {
    uint32_t h0, l0, h1, l1;
    split_pair(v[0], v[1], h0, l0);
    split_pair(v[2], v[3], h1, l1);
    if (!ok) h0 = l0 = h1 = l1 = 0u;
    *reinterpret_cast<uint2*>(&thi[row][col]) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(&tlo[row][col]) = make_uint2(l0, l1);
}

// Affine of channel `ch` in token row `row` of block i (meta indexing as in
// decode_plane).
__device__ __forceinline__ void meta_affine(int norm, const __half* moff, const __half* mscl, int i, int row, int ch,
                                            float& s, float& o) {
    const int m = norm == AKV_NORM_BLOCK_AFFINE ? i : (norm == AKV_NORM_TOKEN ? row : ch);
    s = __half2float(mscl[m]);
    o = __half2float(moff[m]);
}

// Whole RGBA 4x4 block decoded and evaluated by one thread with the generic
// decoder (out of line: blocks the fast path does not cover).
template <int LD>
__device__ __noinline__ void eval_rgba_generic(uint4 blk, int i, int norm, const __half* moff, const __half* mscl,
                                               int row0, int col0, int rows, __half (*thi)[LD], __half (*tlo)[LD]) {
    BlockDesc<4> d;
    uint8_t w[64 + kCodePad];
    decode_header<4>(blk, footprint_index(4), d, w);
    for (int t = 0; t < 16; ++t) {
        const int x = t & 3, y = t >> 2;
        uint32_t c[4];
        texel_values<4, 4>(d, w, x, y, c);
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float s, o;
            meta_affine(norm, moff, mscl, i, row0 + y, col0 + 4 * x + k, s, o);
            v[k] = fmaf(c16_to_unit(c[k]), s, o);
        }
        put_rgba<LD>(v, y < rows, row0 + y, col0 + 4 * x, thi, tlo);
    }
}

// The 16 texels x 4 channels of a fast / constant RGBA 4x4 block -> the
// hi/lo tiles, with the normalisation NORM fixed per instantiation and its
// scales (times 2^-16: exact, the FMA still rounds once) and offsets loaded
// once per texel column (page-channel), row (token) or block (affine).
template <int LD, int NORM>
__device__ __forceinline__ void write_rgba_n(const RgbaOut& o, const uint8_t* codes, int nt, int i, const __half* moff,
                                             const __half* mscl, int row0, int col0, int rows, __half (*thi)[LD],
                                             __half (*tlo)[LD]) {
    const float bs = NORM == AKV_NORM_BLOCK_AFFINE ? __half2float(mscl[i]) * 0x1p-16f : 0.f;
    const float bo = NORM == AKV_NORM_BLOCK_AFFINE ? __half2float(moff[i]) : 0.f;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
        float cs[4], co[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            cs[k] = NORM == AKV_NORM_PAGE_CHANNEL ? __half2float(mscl[col0 + 4 * x + k]) * 0x1p-16f : bs;
            co[k] = NORM == AKV_NORM_PAGE_CHANNEL ? __half2float(moff[col0 + 4 * x + k]) : bo;
        }
#pragma unroll
        for (int y = 0; y < 4; ++y) {
            float tv[4], v[4];
            rgba_t4(o, codes, nt, 4 * y + x, tv);
            float rs = 0.f, ro = 0.f;
            if (NORM == AKV_NORM_TOKEN) {
                rs = __half2float(mscl[row0 + y]) * 0x1p-16f;
                ro = __half2float(moff[row0 + y]);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k)
                v[k] = fmaf(tv[k], NORM == AKV_NORM_TOKEN ? rs : cs[k], NORM == AKV_NORM_TOKEN ? ro : co[k]);
            put_rgba<LD>(v, y < rows, row0 + y, col0 + 4 * x, thi, tlo);
        }
    }
}

// Decode one RGBA 4x4 plane's chunk into the hi/lo tiles (block i covers
// token rows 4 br.. and channels 16 bc..). All threads call it.
template <int D, int THREADS, int NB, int LD>
__device__ __forceinline__ void decode_plane_rgba(const uint4* raw, const __half* moff, const __half* mscl, int norm,
                                                  int cols, int rows_blk, int n, bool valid, int P,
                                                  DecodeScratch<NB, THREADS, 4>& ds, __half (*thi)[LD],
                                                  __half (*tlo)[LD], bool wait_async = false) {
    constexpr int NC = DecodeScratch<NB, THREADS, 4>::NC;
    const int nblk = rows_blk * cols;
    const int tid = threadIdx.x;
    for (int i = tid; i < nblk; i += THREADS) {
        const uint4 blk = raw[i];
        const int br = i / cols, bc = i - br * cols;
        const int row0 = br * 4, col0 = bc * 16;
        const int rows = valid ? min(4, n - row0) : 0;
        // Page-channel metadata of the page this block row lies in.
        const int pm = norm == AKV_NORM_PAGE_CHANNEL ? (row0 / P) * D : 0;
        const __half* bmoff = moff + pm;
        const __half* bmscl = mscl + pm;
        uint32_t me;
        int cq;
        const int kind = rgba_block_kind(blk, me, cq);
        if (kind == kKindGeneric) {
            eval_rgba_generic<LD>(blk, i, norm, bmoff, bmscl, row0, col0, rows, thi, tlo);
            continue;
        }
        RgbaOut o;
        uint8_t* codes = &ds.codes[0][tid];
        decode_rgba4(blk, kind, me, cq, codes, NC, o);
        if (norm == AKV_NORM_PAGE_CHANNEL)
            write_rgba_n<LD, AKV_NORM_PAGE_CHANNEL>(o, codes, NC, i, bmoff, bmscl, row0, col0, rows, thi, tlo);
        else if (norm == AKV_NORM_TOKEN)
            write_rgba_n<LD, AKV_NORM_TOKEN>(o, codes, NC, i, bmoff, bmscl, row0, col0, rows, thi, tlo);
        else
            write_rgba_n<LD, AKV_NORM_BLOCK_AFFINE>(o, codes, NC, i, bmoff, bmscl, row0, col0, rows, thi, tlo);
    }
    if (wait_async) cp_async_wait<0>();
    __syncthreads();
}

// ------------------------------------------------------------------ kernel

template <int D, int G, int VBS, int KBS, int VL = AKV_LAYOUT_SCALAR>
struct Cfg {
    // Tokens per chunk: 48 with a 6x6 plane; 32 with ASTC K (two decoded
    // planes in shared memory); else 64.
    static constexpr int CH = (VBS == 6 || KBS == 6) ? 48 : (KBS ? 32 : 64);
    static constexpr int NWM = CH / 16;                        // token tiles of 16 per chunk
    static constexpr int THREADS = 64 * NWM;                   // two warps per token tile
    static constexpr int LD = D + 8;                           // halves per tile row (16-byte pad)
    // V block columns: a scalar block covers VBS channels, an RGBA block 4 x VBS.
    static constexpr int VCOLS = VL == AKV_LAYOUT_RGBA ? D / (4 * VBS) : (D + VBS - 1) / VBS;
    static constexpr int VROWS = CH / VBS;
    static constexpr int VBLK = VROWS * VCOLS;
    static constexpr int KCOLS = KBS ? (D + KBS - 1) / KBS : 1;
    static constexpr int KROWS = KBS ? CH / KBS : 0;
    static constexpr int KBLK = KROWS * KCOLS;
    // V metadata per chunk; RGBA planes may have pages of 16 tokens inside a
    // chunk (page-channel metadata of up to CH / 16 pages).
    static constexpr int META0 = (VBLK > CH ? (VBLK > D ? VBLK : D) : (CH > D ? CH : D));
    static constexpr int META = VL == AKV_LAYOUT_RGBA && D * (CH / 16) > META0 ? D * (CH / 16) : META0;
    static constexpr int KMETA = KBS ? (KBLK > CH ? (KBLK > D ? KBLK : D) : (CH > D ? CH : D)) : 0;
    static constexpr int SIDE = KBS ? CH * 8 : 0;              // up to 8 side channels
    static constexpr int MAXBS = (VBS > KBS ? VBS : KBS);
    // CTAs per SM (shared memory allows three; scalar 4x4 V with FP16 K runs
    // two with more registers), and the register cap that fits them.
    static constexpr int CTAS = (VBS == 4 && KBS == 0 && VL == AKV_LAYOUT_SCALAR) ? 2 : 3;
    static constexpr int MAXREG = (65536 / (CTAS * THREADS)) / 8 * 8;
    static constexpr size_t VDS = sizeof(DecodeScratch<VBLK, THREADS, VBS>);
    static constexpr size_t KDS = KBS ? sizeof(DecodeScratch<(KBS ? KBLK : 1), THREADS, (KBS ? KBS : 4)>) : 0;
    static constexpr size_t DSBYTES = VDS > KDS ? VDS : KDS;     // decode scratch, shared by the planes
    static_assert(CH % VBS == 0 && CH % (KBS ? KBS : 1) == 0, "chunk must hold whole block rows");
    static_assert(G <= 8, "query group must fit the N=8 MMA dimension");
    // Overhanging block columns stay inside the tile rows and metadata.
    static_assert((D + VBS - 1) / VBS * VBS <= LD && (!KBS || (D + MAXBS - 1) / MAXBS * MAXBS <= LD), "tile row padding");
    static_assert(VL == AKV_LAYOUT_RGBA || (D + VBS - 1) / VBS * VBS <= META, "metadata padding");
    static_assert(VL == AKV_LAYOUT_SCALAR || (VBS == 4 && KBS == 0 && D % 16 == 0), "RGBA: 4x4 V, FP16 K");
};

template <int D, int G, int VBS, int KBS, int VL = AKV_LAYOUT_SCALAR>
struct Smem {
    using C = Cfg<D, G, VBS, KBS, VL>;
    uint64_t bar[2];
    int valid[2];
    int stuck_c;  // chunk whose copies did not arrive in time
    __align__(16) uint4 vraw[2][C::VBLK];
    __align__(16) __half vmeta[2][2][C::META];
    __align__(16) uint4 kraw[2][KBS ? C::KBLK : 1];
    __align__(16) __half kmeta[2][2][KBS ? C::KMETA : 1];
    __align__(16) __half kside[2][KBS ? C::SIDE : 1];
    __align__(16) __half vhi[C::CH][C::LD];
    __align__(16) __half vlo[C::CH][C::LD];
    __align__(16) __half khi[C::CH][C::LD];   // decoded K hi, or the staged FP16 K rows
    __align__(16) __half klo[KBS ? C::CH : 1][C::LD];
    __align__(16) uint8_t ds[C::DSBYTES];
    __align__(16) __half pbuf[2 * C::NWM][2][16][8];  // per warp: P hi, P lo as [token][head]
    __align__(16) uint4 qfrag[D / 16][32];                         // per lane: q hi (2 words) | q lo (2 words)

    float wm[C::NWM][8];
    float wl[C::NWM][8];
};

// Three CTAs per SM, except scalar 4x4 V with FP16 K (256 threads): two CTAs
// with up to 128 registers instead of spilling at 80 (C4 9.7 ms against 10.5;
// the RGBA 4x4 instances are faster with three). The register cap is the
// most the CTAs per SM leave (Cfg::MAXREG).
template <int D, int G, int VBS, int KBS, int VL = AKV_LAYOUT_SCALAR>
__global__ void __launch_bounds__(Cfg<D, G, VBS, KBS, VL>::THREADS, Cfg<D, G, VBS, KBS, VL>::CTAS)
    attn_fast_kernel(AttnParams p) {
    using C = Cfg<D, G, VBS, KBS, VL>;
    using S = Smem<D, G, VBS, KBS, VL>;
    constexpr int CH = C::CH, NWM = C::NWM, THREADS = C::THREADS, LD = C::LD;
    static_assert(THREADS == 64 * NWM, "every warp owns one (token tile, dim half)");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    S& sm = *reinterpret_cast<S*>(smem_raw);

    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int len = seq_len_of(p, b);
    const int t_begin = split * p.split_tokens;
    const int t_end = min(t_begin + p.split_tokens, len);
    const int64_t unit0 = (static_cast<int64_t>(b) * p.Hq + h * G) * p.split_stride + p.split_base + split;
    if (t_begin >= t_end) {
        for (int i = tid; i < G * D; i += THREADS)
            p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.split_stride) * D + i % D] = 0.f;
        if (tid < G) {
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 0] = -CUDART_INF_F;
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 1] = 0.f;
        }
        return;
    }
    const int nchunks = (t_end - t_begin + CH - 1) / CH;
    const int P = p.page_tokens;

    if (tid == 0) {
        mbar_init(&sm.bar[0], 1);
        mbar_init(&sm.bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // Producer: stage `s` <- chunk `c` (one elected thread).
    auto issue = [&](int c, int s) {
        const int t0 = t_begin + c * CH;
        const int page = t0 / P;
        const int phys = phys_page(p.table, p.pps, p.num_pages, b, page, p.status);
        const int tin = t0 - page * P;
        sm.valid[s] = phys >= 0;
        uint32_t bytes = 0;
        const uint8_t* vsrc = nullptr;
        const __half* voff = nullptr;
        const __half* vscl = nullptr;
        const int vrows = CH / VBS, vcols = C::VCOLS;
        const int vme = meta_elems<VBS>(p.v.norm, vcols, CH, D, P);
        const uint8_t* ksrc = nullptr;
        const __half* koff = nullptr;
        const __half* kscl = nullptr;
        const uint8_t* kside = nullptr;
        const int krows = KBS ? CH / KBS : 0, kcols = C::KCOLS;
        const int kme = KBS ? meta_elems<(KBS ? KBS : 4)>(p.k.norm, kcols, CH, D, P) : 0;
        if (phys >= 0) {
            vsrc = p.v.data + b * p.v.sB + h * p.v.sH + static_cast<int64_t>(phys) * p.v.sP +
                   static_cast<int64_t>(tin / VBS) * vcols * 16;
            const int64_t mbase = b * p.v.mB + h * p.v.mH + static_cast<int64_t>(phys) * p.v.mP +
                                  meta_chunk_offset<VBS>(p.v.norm, vcols, tin);
            voff = p.v.off + mbase;
            vscl = p.v.scl + mbase;
            bytes += vrows * vcols * 16 + 2 * vme * 2;
            if constexpr (KBS > 0) {
                ksrc = p.k.data + b * p.k.sB + h * p.k.sH + static_cast<int64_t>(phys) * p.k.sP +
                       static_cast<int64_t>(tin / KBS) * kcols * 16;
                const int64_t kb = b * p.k.mB + h * p.k.mH + static_cast<int64_t>(phys) * p.k.mP +
                                   meta_chunk_offset<(KBS ? KBS : 4)>(p.k.norm, kcols, tin);
                koff = p.k.off + kb;
                kscl = p.k.scl + kb;
                bytes += krows * kcols * 16 + 2 * kme * 2;
                if (p.k.side_count > 0) {
                    kside = p.k.side + b * p.k.xB + h * p.k.xH + static_cast<int64_t>(phys) * p.k.xP +
                            static_cast<int64_t>(tin) * p.k.side_count * 2;
                    bytes += CH * p.k.side_count * 2;
                }
            }
        }
        mbar_arrive_expect_tx(&sm.bar[s], bytes);
        if (phys >= 0) {
            bulk_g2s(sm.vraw[s], vsrc, vrows * vcols * 16, &sm.bar[s]);
            bulk_g2s(sm.vmeta[s][0], voff, vme * 2, &sm.bar[s]);
            bulk_g2s(sm.vmeta[s][1], vscl, vme * 2, &sm.bar[s]);
            if constexpr (KBS > 0) {
                bulk_g2s(sm.kraw[s], ksrc, krows * kcols * 16, &sm.bar[s]);
                bulk_g2s(sm.kmeta[s][0], koff, kme * 2, &sm.bar[s]);
                bulk_g2s(sm.kmeta[s][1], kscl, kme * 2, &sm.bar[s]);
                if (kside) bulk_g2s(sm.kside[s], kside, CH * p.k.side_count * 2, &sm.bar[s]);
            }
        }
    };
    if (tid == 0) {
        issue(0, 0);
        if (nchunks > 1) issue(1, 1);
    }

    // Query fragments (B operand, hi + lo) for heads n = lane/4 of the
    // group, computed once by warp 0 into shared memory.
    const int qn = lane >> 2, qj = lane & 3;
    constexpr int KS = D / 16;
    constexpr int KH = KS / 2;  // dim tiles per half
    const int tw = warp % NWM, dh = warp / NWM;
    if (warp == 0) {
        const bool has = qn < G;
        const int64_t qb = (static_cast<int64_t>(b) * p.Hq + h * G + (has ? qn : 0)) * D;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int d0 = 16 * ks + 2 * qj, d1 = d0 + 8;
            const float q0 = has ? load_q(p.q, p.q_dtype, qb + d0) : 0.f;
            const float q1 = has ? load_q(p.q, p.q_dtype, qb + d0 + 1) : 0.f;
            const float q2 = has ? load_q(p.q, p.q_dtype, qb + d1) : 0.f;
            const float q3 = has ? load_q(p.q, p.q_dtype, qb + d1 + 1) : 0.f;
            uint4 f;
            split_pair(q0, q1, f.x, f.z);
            split_pair(q2, q3, f.y, f.w);
            sm.qfrag[ks][lane] = f;
        }
    }

    // FP16 K rows of chunk c -> sm.khi by 16-byte asynchronous copies (rows
    // past the split or on unmapped pages copy zero bytes: zeros).
    auto stage_k = [&](int c) {
        if constexpr (KBS == 0) {
            constexpr int PPR = D / 8, PIECES = CH * PPR;
            const int t0 = t_begin + c * CH;
            const uint8_t* kbase = p.k.data + b * p.k.sB + h * p.k.sH;
            if (P % CH == 0) {
                // The chunk lies in one page: one table lookup, contiguous rows.
                const int page = t0 / P;
                const int phys = phys_page(p.table, p.pps, p.num_pages, b, page, nullptr);
                const int nrow = phys >= 0 ? min(CH, t_end - t0) : 0;
                const uint8_t* src0 = phys >= 0 ? kbase + static_cast<int64_t>(phys) * p.k.sP +
                                                      static_cast<int64_t>(t0 - page * P) * (D * 2)
                                                : kbase;
                for (int piece = tid; piece < PIECES; piece += THREADS) {
                    const int r = piece / PPR;
                    const bool ok = r < nrow;
                    cp_async16(&sm.khi[r][8 * (piece - r * PPR)], ok ? src0 + static_cast<int64_t>(piece) * 16 : kbase,
                               ok ? 16u : 0u);
                }
            } else {
                for (int piece = tid; piece < PIECES; piece += THREADS) {
                    const int r = piece / PPR, j = piece - r * PPR;
                    const int t = t0 + r;
                    const int phys = t < t_end ? phys_page(p.table, p.pps, p.num_pages, b, t / P, nullptr) : -1;
                    const uint8_t* src = phys >= 0 ? kbase + static_cast<int64_t>(phys) * p.k.sP +
                                                         static_cast<int64_t>(t % P) * (D * 2) + j * 16
                                                   : kbase;
                    cp_async16(&sm.khi[r][8 * j], src, phys >= 0 ? 16u : 0u);
                }
            }
            cp_async_commit();
        }
    };
    stage_k(0);

    float o[KH][4];
#pragma unroll
    for (int i = 0; i < KH; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F}, l_run[2] = {0.f, 0.f};
    bool stuck = false;  // a chunk's copies did not arrive in time (its index: sm.stuck_c)

    for (int c = 0; c < nchunks; ++c) {
        const int s = c & 1;
        const uint32_t parity = (c >> 1) & 1;
        const int t0 = t_begin + c * CH;
        const int n = min(CH, t_end - t0);
        const bool waited = mbar_wait(&sm.bar[s], parity);
        // The V plane's slot count restarts at zero; nothing reads it between
        // the previous chunk's last barrier and the next one.
        if constexpr (VL != AKV_LAYOUT_RGBA)
            if (tid == 0) reinterpret_cast<DecodeScratch<C::VBLK, THREADS, VBS>*>(sm.ds)->nslot = 0;
        if (__syncthreads_or(!waited)) {
            stuck = true;
            if (tid == 0) sm.stuck_c = c;
            break;
        }
        const bool valid = sm.valid[s] != 0;
        // Decode V (and K) tiles.
        if constexpr (VL == AKV_LAYOUT_RGBA)
            decode_plane_rgba<D, THREADS, C::VBLK, LD>(sm.vraw[s], sm.vmeta[s][0], sm.vmeta[s][1], p.v.norm, C::VCOLS,
                                                      CH / 4, n, valid, P,
                                                      *reinterpret_cast<DecodeScratch<C::VBLK, THREADS, 4>*>(sm.ds),
                                                      sm.vhi, sm.vlo, KBS == 0);
        else
            decode_plane<VBS, D, THREADS, C::VBLK, LD, false>(
                sm.vraw[s], sm.vmeta[s][0], sm.vmeta[s][1], p.v.norm, C::VCOLS, CH / VBS, n, valid,
                *reinterpret_cast<DecodeScratch<C::VBLK, THREADS, VBS>*>(sm.ds), sm.vhi, sm.vlo, KBS == 0);
        if constexpr (KBS > 0) {
            constexpr int KB = KBS ? KBS : 4;
            constexpr int KN = KBS ? C::KBLK : 1;
            decode_plane<KB, D, THREADS, KN, LD>(sm.kraw[s], sm.kmeta[s][0], sm.kmeta[s][1], p.k.norm, C::KCOLS,
                                                CH / KB, n, valid, *reinterpret_cast<DecodeScratch<KN, THREADS, KB>*>(sm.ds),
                                                sm.khi, sm.klo);
            // Exact side-plane channels.
            const int sc = p.k.side_count;
            if (sc > 0) {
                for (int i = tid; i < n * sc; i += THREADS) {
                    const int r = i / sc, jj = i - r * sc;
                    const int ch = __ldg(p.k.side_ch + h * sc + jj);
                    if (ch < 0 || ch >= D) continue;
                    const float v = valid ? __half2float(sm.kside[s][r * sc + jj]) : 0.f;
                    const __half hv = __float2half_rn(v);
                    sm.khi[r][ch] = hv;
                    sm.klo[r][ch] = __float2half_rn(v - __half2float(hv));
                }
                __syncthreads();
            }
        }
        // Rows past the chunk's last token (every row of an unmapped page)
        // must be zero in the tiles: the table and direct writers store
        // whatever the staged blocks decode to there. Only a split's last,
        // partial chunk has such rows.
        if (n < CH || !valid) {
            const int r0 = valid ? n : 0;
            constexpr int Q = LD / 8;  // 16-byte words per tile row
            for (int i = tid; i < (CH - r0) * Q; i += THREADS) {
                const int r = r0 + i / Q, k = 8 * (i % Q);
                *reinterpret_cast<uint4*>(&sm.vhi[r][k]) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(&sm.vlo[r][k]) = make_uint4(0u, 0u, 0u, 0u);
                if constexpr (KBS > 0) {
                    *reinterpret_cast<uint4*>(&sm.khi[r][k]) = make_uint4(0u, 0u, 0u, 0u);
                    *reinterpret_cast<uint4*>(&sm.klo[r][k]) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            __syncthreads();
        }
        // FP16 K: this chunk's rows (issued a chunk ahead) were waited for
        // inside the V decode, before a barrier.
        // The raw stage is consumed: refill it with chunk c + 2.
        if (tid == 0 && c + 2 < nchunks) {
            fence_proxy_async();
            issue(c + 2, s);
        }
        // Tensor-core phase: warp w owns chunk tokens [16 tw, 16 tw + 16) and
        // dim half dh (both warps of a token tile compute its scores).
        {
            __syncwarp();
            // Two independent accumulator chains (even / odd k-steps).
            float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const uint4 qf = sm.qfrag[ks][lane];
                float* acc = sa[ks & 1];
                uint32_t a[4];
                const int mi = lane >> 3, rr = lane & 7;
                const int row = 16 * tw + rr + ((mi & 1) ? 8 : 0);
                const int col = 16 * ks + ((mi & 2) ? 8 : 0);
                ldsm_x4(a, &sm.khi[row][col]);
                mma16816(acc, a[0], a[1], a[2], a[3], qf.x, qf.y);
                mma16816(acc, a[0], a[1], a[2], a[3], qf.z, qf.w);
                if constexpr (KBS > 0) {
                    ldsm_x4(a, &sm.klo[row][col]);
                    mma16816(acc, a[0], a[1], a[2], a[3], qf.x, qf.y);
                }
            }
            float sacc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) sacc[i] = sa[0][i] + sa[1][i];
            // sacc: S^T[tok = qn (+8)][head = 2qj (+1)], in log2 units after scaling.
            const bool v0 = 16 * tw + qn < n, v1 = 16 * tw + qn + 8 < n;
            float sv[4];
            sv[0] = v0 ? sacc[0] * p.qscale : -CUDART_INF_F;
            sv[1] = v0 ? sacc[1] * p.qscale : -CUDART_INF_F;
            sv[2] = v1 ? sacc[2] * p.qscale : -CUDART_INF_F;
            sv[3] = v1 ? sacc[3] * p.qscale : -CUDART_INF_F;
            float alpha[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float mx = fmaxf(sv[j], sv[j + 2]);
                mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
                const float mn = fmaxf(m_run[j], mx);
                const bool none = mn == -CUDART_INF_F;
                alpha[j] = none ? 1.f : exp2f(m_run[j] - mn);
                const float p0 = none ? 0.f : exp2f(sv[j] - mn);
                const float p1 = none ? 0.f : exp2f(sv[j + 2] - mn);
                sv[j] = p0;
                sv[j + 2] = p1;
                float sum = p0 + p1;
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 8);
                sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 16);
                l_run[j] = l_run[j] * alpha[j] + sum;
                m_run[j] = mn;
            }
#pragma unroll
            for (int i = 0; i < KH; ++i) {
                o[i][0] *= alpha[0];
                o[i][1] *= alpha[1];
                o[i][2] *= alpha[0];
                o[i][3] *= alpha[1];
            }
            // P^T -> per-warp buffers as [token][head] in fp16 hi + lo (the
            // unrounded p is what l accumulates); ldmatrix.trans gives the B
            // fragments (k = token, n = head).
            __half(*pbh)[8] = sm.pbuf[warp][0];
            __half(*pbl)[8] = sm.pbuf[warp][1];
            {
                const __half2 h01 = __floats2half2_rn(sv[0], sv[1]), h23 = __floats2half2_rn(sv[2], sv[3]);
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                *reinterpret_cast<__half2*>(&pbh[qn][2 * qj]) = h01;
                *reinterpret_cast<__half2*>(&pbh[qn + 8][2 * qj]) = h23;
                *reinterpret_cast<__half2*>(&pbl[qn][2 * qj]) = __floats2half2_rn(sv[0] - f01.x, sv[1] - f01.y);
                *reinterpret_cast<__half2*>(&pbl[qn + 8][2 * qj]) = __floats2half2_rn(sv[2] - f23.x, sv[3] - f23.y);
            }
            __syncwarp();
            uint32_t b0, b1, b0l, b1l;
            ldsm_x2_t(b0, b1, &pbh[lane & 15][0]);
            ldsm_x2_t(b0l, b1l, &pbl[lane & 15][0]);
            // O^T[dim][head] += V^T . P^T with V = hi + lo and P = hi + lo
            // (the lo x lo product, below 2^-22 relative, is left out).
            const int mi = lane >> 3, rr = lane & 7;
            const int vrow = 16 * tw + rr + ((mi & 2) ? 8 : 0);
            const int vcol = (mi & 1) ? 8 : 0;
#pragma unroll
            for (int mt = 0; mt < KH; ++mt) {
                const int dt = dh * KH + mt;
                uint32_t a[4];
                ldsm_x4_t(a, &sm.vhi[vrow][16 * dt + vcol]);
                mma16816(o[mt], a[0], a[1], a[2], a[3], b0, b1);
                mma16816(o[mt], a[0], a[1], a[2], a[3], b0l, b1l);
                ldsm_x4_t(a, &sm.vlo[vrow][16 * dt + vcol]);
                mma16816(o[mt], a[0], a[1], a[2], a[3], b0, b1);
            }
            __syncwarp();
        }
        __syncthreads();  // tiles and P buffers free for the next chunk
        if (c + 1 < nchunks) stage_k(c + 1);
    }
    if constexpr (KBS == 0) cp_async_wait<0>();  // nothing in flight past the loop

    if (stuck) {
        // A copy never completed: report, give the copies still in flight
        // (chunk `stuck` and, if it was issued, chunk stuck + 1, one per
        // stage) a bounded grace period each so none lands in shared memory
        // after the CTA exits, and leave this split empty.
        if (tid == 0) {
            if (p.status) atomicExch(p.status, AKV_ERR_TIMEOUT);
            const int sc = sm.stuck_c;
            mbar_wait(&sm.bar[sc & 1], (sc >> 1) & 1);
            if (sc + 1 < nchunks) mbar_wait(&sm.bar[(sc + 1) & 1], ((sc + 1) >> 1) & 1);
        }
        __syncthreads();
        for (int i = tid; i < G * D; i += THREADS)
            p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.split_stride) * D + i % D] = 0.f;
        if (tid < G) {
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 0] = -CUDART_INF_F;
            p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 1] = 0.f;
        }
        return;
    }

    // Merge the MMA warps' (m, l, O) into one split partial: each warp
    // stores its rescaled O (its token tile, its dim half), then the token
    // tiles are summed in a fixed order (the result does not depend on warp
    // timing).
    float* red = reinterpret_cast<float*>(&sm.vhi[0][0]);  // [NWM][G][D] floats
    static_assert(sizeof(float) * NWM * G * D <= sizeof(sm.vhi), "merge buffer fits the V tile");
    if (dh == 0 && lane < 4) {
        sm.wm[tw][2 * lane] = m_run[0];
        sm.wm[tw][2 * lane + 1] = m_run[1];
        sm.wl[tw][2 * lane] = l_run[0];
        sm.wl[tw][2 * lane + 1] = l_run[1];
    }
    __syncthreads();
    {
        float scl[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int hh = 2 * qj + j;
            float M = -CUDART_INF_F;
#pragma unroll
            for (int w = 0; w < NWM; ++w) M = fmaxf(M, sm.wm[w][hh]);
            scl[j] = (M == -CUDART_INF_F || m_run[j] == -CUDART_INF_F) ? 0.f : exp2f(m_run[j] - M);
        }
        float* mine = red + tw * G * D;
#pragma unroll
        for (int mt = 0; mt < KH; ++mt) {
            const int d0 = 16 * (dh * KH + mt) + qn;
            if (2 * qj < G) {
                mine[(2 * qj) * D + d0] = o[mt][0] * scl[0];
                mine[(2 * qj) * D + d0 + 8] = o[mt][2] * scl[0];
            }
            if (2 * qj + 1 < G) {
                mine[(2 * qj + 1) * D + d0] = o[mt][1] * scl[1];
                mine[(2 * qj + 1) * D + d0 + 8] = o[mt][3] * scl[1];
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += THREADS) {
        float acc = red[i];
#pragma unroll
        for (int w = 1; w < NWM; ++w) acc += red[w * G * D + i];
        p.part_acc[(unit0 + static_cast<int64_t>(i / D) * p.split_stride) * D + i % D] = acc;
    }
    if (tid < G) {
        float M = -CUDART_INF_F;
        for (int w = 0; w < NWM; ++w) M = fmaxf(M, sm.wm[w][tid]);
        float L = 0.f;
        if (M != -CUDART_INF_F)
            for (int w = 0; w < NWM; ++w)
                if (sm.wm[w][tid] != -CUDART_INF_F) L += exp2f(sm.wm[w][tid] - M) * sm.wl[w][tid];
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 0] = M;
        p.part_ml[(unit0 + static_cast<int64_t>(tid) * p.split_stride) * 2 + 1] = L;
    }
}

}  // namespace fast
}  // namespace akv
