// C-ABI entry points of libakv_cuda.so (declared in include/akv_cuda.h).
//
// Host side: argument validation, per-device table set-up, launch-shape
// choice and template dispatch. Device side: the kernels in
// akv_decode_kernels.cuh and akv_attention_kernels.cuh.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/akv_cuda.h"
#include "akv_attention_kernels.cuh"
#include "akv_attn_fast.cuh"
#include "akv_attn_fp16.cuh"
#include "akv_decode_kernels.cuh"
#include "akv_tables.h"

namespace akv {
namespace {

// Split scratch of akv_cuda_decode_attention_noalloc: static device memory,
// one copy per device that loads the library. Host code sees only a stand-in
// for this symbol; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) float g_static_workspace[AKV_STATIC_WORKSPACE_BYTES / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_init_mu;
// Per-device "tables uploaded" flags. They live as long as the process: after
// a cudaDeviceReset the device's static memory is gone but the flag is not,
// so a caller that resets a device must not use this library on it again.
std::atomic<bool> g_init_done[kMaxDevices];
Tables* g_host_tables = nullptr;

const Tables& host_tables() {
    static std::once_flag once;
    std::call_once(once, [] {
        g_host_tables = new Tables;
        build_tables(g_host_tables);
    });
    return *g_host_tables;
}

int init_device(int device) {
    if (device < 0 || device >= kMaxDevices) return AKV_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(g_init_mu);
    if (g_init_done[device].load(std::memory_order_acquire)) return AKV_OK;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return AKV_ERR_CUDA;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return AKV_ERR_CUDA;
    const Tables& t = host_tables();
    cudaError_t e = cudaMemcpyToSymbol(g_akv_tables, &t, sizeof(Tables), 0, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return AKV_ERR_CUDA;
    g_init_done[device].store(true, std::memory_order_release);
    return AKV_OK;
}

// True when `s` (or, in global capture mode elsewhere, the legacy stream) is
// being captured; a failing query counts as capturing.
bool capturing(cudaStream_t s) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) {
        cudaGetLastError();
        return true;
    }
    if (cap != cudaStreamCaptureStatusNone) return true;
    if (s != nullptr && s != cudaStreamLegacy) {
        if (cudaStreamIsCapturing(cudaStreamLegacy, &cap) != cudaSuccess) {
            cudaGetLastError();
            return true;
        }
        return cap != cudaStreamCaptureStatusNone;
    }
    return false;
}

// Tables of the current device, uploaded on first use. The upload is
// synchronous, so it is refused while the call's stream is being captured.
int ensure_init(cudaStream_t stream) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return AKV_ERR_CUDA;
    if (dev >= 0 && dev < kMaxDevices && g_init_done[dev].load(std::memory_order_acquire)) return AKV_OK;
    if (capturing(stream)) return AKV_ERR_NOT_INITIALIZED;
    return init_device(dev);
}

std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices];

// Device address of g_static_workspace on the current device (looked up once
// per device, with that device current).
int static_workspace(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AKV_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_static_workspace) != cudaSuccess || !ptr) {
            cudaGetLastError();
            return AKV_ERR_CUDA;
        }
        g_static_ptr[dev] = ptr;
    }
    *out = g_static_ptr[dev];
    return AKV_OK;
}

int sm_count() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

inline int launch_status() {
    return cudaPeekAtLastError() == cudaSuccess ? AKV_OK : (cudaGetLastError(), AKV_ERR_CUDA);
}

bool valid_block(int b) { return b == 4 || b == 6 || b == 8; }

// ---------------------------------------------------------------- attention

template <int D, int G, int KBS, int VBS, int VL>
int launch_attention(const AttnParams& p, cudaStream_t s, int phases) {
    using Cfg = AttnCfg<D, G, KBS, VBS, VL>;
    static_assert(Cfg::TG * G <= 2 * Cfg::CH || KBS == 0, "reduction fits");
    static_assert(Cfg::TG * G <= Cfg::CH, "reduction fits in the V tile");
    auto kern = attn_split_kernel<D, G, KBS, VBS, VL>;
    const size_t smem = Cfg::kSmem;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        return AKV_ERR_CUDA;
    }
    if (phases & AKV_PHASE_SPLIT) {
        dim3 grid(p.nsplits, p.Hkv, p.B);
        kern<<<grid, kAttnThreads, smem, s>>>(p);
        if (int st = launch_status()) return st;
    }
    if (phases & AKV_PHASE_MERGE) {
        launch_merge(p, D, s);
        if (int st = launch_status()) return st;
    }
    return AKV_OK;
}

using Launcher = int (*)(const AttnParams&, cudaStream_t, int);

template <int D, int G, int VBS, int KBS, int VL>
int launch_fast(const AttnParams& p, cudaStream_t s, int phases) {
    using C = fast::Cfg<D, G, VBS, KBS, VL>;
    auto kern = fast::attn_fast_kernel<D, G, VBS, KBS, VL>;
    const size_t smem = sizeof(fast::Smem<D, G, VBS, KBS, VL>);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        return AKV_ERR_CUDA;
    }
    if (phases & AKV_PHASE_SPLIT) {
        dim3 grid(p.nsplits, p.Hkv, p.B);
        kern<<<grid, C::THREADS, smem, s>>>(p);
        if (int st = launch_status()) return st;
    }
    if (phases & AKV_PHASE_MERGE) {
        launch_merge(p, D, s);
        if (int st = launch_status()) return st;
    }
    return AKV_OK;
}

struct FastVariant {
    int D, G, vbs, kbs, vl;
    Launcher fn;
    size_t smem;
};

// Tensor-core variants for scalar-layout ASTC V with FP16 (kbs 0) or scalar
// ASTC K, and RGBA-layout 4x4 V with FP16 K.
#define AKV_FAST(D, G, VB, KB, VL) \
    {D, G, VB, KB, VL, &launch_fast<D, G, VB, KB, VL>, sizeof(fast::Smem<D, G, VB, KB, VL>)}
constexpr int kS = AKV_LAYOUT_SCALAR, kR = AKV_LAYOUT_RGBA;
const FastVariant kFastVariants[] = {
    AKV_FAST(64, 3, 6, 0, kS), AKV_FAST(64, 3, 6, 6, kS), AKV_FAST(64, 3, 4, 0, kS), AKV_FAST(64, 3, 8, 0, kS),
    AKV_FAST(128, 4, 6, 0, kS), AKV_FAST(128, 4, 4, 0, kS), AKV_FAST(128, 4, 8, 0, kS),
    AKV_FAST(128, 8, 8, 4, kS), AKV_FAST(128, 8, 8, 0, kS), AKV_FAST(128, 8, 4, 0, kS),
    AKV_FAST(64, 3, 4, 0, kR), AKV_FAST(128, 4, 4, 0, kR),
};
#undef AKV_FAST

template <int D, int G>
int launch_fp16(const AttnParams& p, cudaStream_t s, int phases) {
    using C = f16k::Cfg<D, G>;
    auto kern = f16k::attn_fp16_kernel<D, G>;
    const size_t smem = sizeof(f16k::Smem<D, G>);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        return AKV_ERR_CUDA;
    }
    if (phases & AKV_PHASE_SPLIT) {
        dim3 grid(p.nsplits, p.Hkv, p.B);
        kern<<<grid, C::THREADS, smem, s>>>(p);
        if (int st = launch_status()) return st;
    }
    if (phases & AKV_PHASE_MERGE) {
        launch_merge(p, D, s);
        if (int st = launch_status()) return st;
    }
    return AKV_OK;
}

struct Fp16Variant {
    int D, G;
    Launcher fn;
    size_t smem;
};

// FP16 K + FP16 V (the FP16 control) on the tensor-core kernel.
#define AKV_FP16(D, G) {D, G, &launch_fp16<D, G>, sizeof(f16k::Smem<D, G>)}
const Fp16Variant kFp16Variants[] = {AKV_FP16(64, 3), AKV_FP16(128, 4), AKV_FP16(128, 8)};
#undef AKV_FP16

const Fp16Variant* find_fp16(int D, int G) {
    for (const Fp16Variant& v : kFp16Variants)
        if (v.D == D && v.G == G) return &v;
    return nullptr;
}

bool fp16_path_ok(const AkvAttnDesc* d) {
    const char* env = std::getenv("AKV_ATTN_PATH");
    if (env && std::strcmp(env, "generic") == 0) return false;
    if (d->k.storage != AKV_STORAGE_FP16 || d->v.storage != AKV_STORAGE_FP16) return false;
    const Fp16Variant* fv = find_fp16(d->head_dim, d->q_heads / d->kv_heads);
    if (!fv) return false;
    int dev = 0, smem_max = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        fv->smem > static_cast<size_t>(smem_max)) {
        cudaGetLastError();
        return false;
    }
    // One bulk copy per row: every row start 16-byte aligned.
    const AkvPlane* planes[2] = {&d->k, &d->v};
    for (const AkvPlane* pl : planes)
        if (pl->stride_batch % 16 || pl->stride_head % 16 || pl->stride_page % 16) return false;
    return true;
}

constexpr int kMinSplitChunks = 6;

int fast_chunk(int kbs, int vbs) { return (vbs == 6 || kbs == 6) ? 48 : (kbs ? 32 : 64); }

const FastVariant* find_fast(int D, int G, int vbs, int kbs, int vl) {
    for (const FastVariant& v : kFastVariants)
        if (v.D == D && v.G == G && v.vbs == vbs && v.kbs == kbs && v.vl == vl) return &v;
    return nullptr;
}

bool aligned16(int64_t bytes) { return bytes % 16 == 0; }

// Metadata elements per chunk for a plane, and their offset granularity
// inside a page (both must keep the bulk copies 16-byte aligned).
bool meta_copy_ok(const AkvPlane& pl, int D, int CH, int P) {
    const int cols = pl.layout == AKV_LAYOUT_RGBA ? D / (4 * pl.block) : (D + pl.block - 1) / pl.block;
    int64_t elems, step;
    if (pl.normalization == AKV_NORM_BLOCK_AFFINE) { elems = (CH / pl.block) * cols; step = elems; }
    else if (pl.normalization == AKV_NORM_TOKEN) { elems = CH; step = CH; }
    else { elems = static_cast<int64_t>(D) * (P < CH ? CH / P : 1); step = 0; }
    return aligned16(elems * 2) && aligned16(step * 2) && aligned16(pl.meta_stride_batch * 2) &&
           aligned16(pl.meta_stride_head * 2) && aligned16(pl.meta_stride_page * 2) &&
           reinterpret_cast<uintptr_t>(pl.offsets) % 16 == 0 && reinterpret_cast<uintptr_t>(pl.scales) % 16 == 0;
}

bool fast_path_ok(const AkvAttnDesc* d, int kbs, int vbs, int vl, int split) {
    const char* env = std::getenv("AKV_ATTN_PATH");
    if (env && std::strcmp(env, "generic") == 0) return false;
    if (!vbs) return false;
    if (d->k.storage == AKV_STORAGE_ASTC && d->k.layout != AKV_LAYOUT_SCALAR) return false;
    const FastVariant* fv = find_fast(d->head_dim, d->q_heads / d->kv_heads, vbs, kbs, vl);
    if (!fv) return false;
    int dev = 0, smem_max = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        fv->smem > static_cast<size_t>(smem_max)) {
        cudaGetLastError();
        return false;
    }
    const int CH = fast_chunk(kbs, vbs);
    const int P = d->page_tokens;
    if (split % CH) return false;
    if (P % CH) {
        // Several pages per chunk: RGBA V of a contiguous cache only, pages of
        // at least 16 tokens, consecutive pages adjacent in memory (one copy
        // per chunk) with their metadata. Every chunk copies CH / P whole
        // pages, so the capacity (max_tokens) must be whole chunks: the last
        // chunk's copy then ends inside the plane.
        if (vl != AKV_LAYOUT_RGBA || d->block_table_dev || CH % P || P < 16 || d->max_tokens % CH) return false;
        const AkvPlane& v = d->v;
        const int cols = d->head_dim / (4 * v.block);
        const int64_t per_page = v.normalization == AKV_NORM_BLOCK_AFFINE ? (P / v.block) * cols
                                 : v.normalization == AKV_NORM_TOKEN ? P : d->head_dim;
        if (v.stride_page != static_cast<int64_t>(P / v.block) * cols * 16 || v.meta_stride_page != per_page) return false;
    }
    const AkvPlane* planes[2] = {&d->k, &d->v};
    for (const AkvPlane* pl : planes) {
        if (!aligned16(pl->stride_batch) || !aligned16(pl->stride_head) || !aligned16(pl->stride_page)) return false;
        if (pl->storage == AKV_STORAGE_ASTC && !meta_copy_ok(*pl, d->head_dim, CH, P)) return false;
    }
    if (d->k.side) {
        if (d->k.side_count > 8) return false;
        const int64_t sc2 = static_cast<int64_t>(d->k.side_count) * 2;
        if (!aligned16(CH * sc2) || !aligned16(d->k.side_stride_batch) || !aligned16(d->k.side_stride_head) ||
            !aligned16(d->k.side_stride_page) || reinterpret_cast<uintptr_t>(d->k.side) % 16)
            return false;
    }
    return true;
}

int chunk_tokens(int kbs, int vbs) { return vbs ? 8 * vbs : (kbs ? 8 * kbs : 64); }


struct Variant {
    int D, G, kbs, vbs, vl;
    Launcher fn;
};

// Compiled (head_dim, group, K footprint (0 = fp16), V footprint (0 = fp16),
// V layout) combinations: the reference fixtures' shapes and the five
// benchmark configurations.
#define AKV_VARIANT(D, G, KB, VB, VL) {D, G, KB, VB, VL, &launch_attention<D, G, KB, VB, VL>}
const Variant kVariants[] = {
    AKV_VARIANT(64, 3, 0, 4, AKV_LAYOUT_RGBA),     // SmolLM2 shape, rgba 4x4 V (configs 0/1)
    AKV_VARIANT(64, 3, 0, 4, AKV_LAYOUT_SCALAR),
    AKV_VARIANT(64, 3, 0, 6, AKV_LAYOUT_SCALAR),   // reference fixtures, scalar 6x6 V
    AKV_VARIANT(64, 3, 6, 6, AKV_LAYOUT_SCALAR),   // reference fixtures, 6x6 K and V
    AKV_VARIANT(64, 3, 0, 8, AKV_LAYOUT_SCALAR),
    AKV_VARIANT(64, 3, 0, 0, AKV_LAYOUT_SCALAR),   // FP16 control
    AKV_VARIANT(128, 4, 0, 6, AKV_LAYOUT_SCALAR),  // Llama-3-8B shape, 6x6 V (config 2)
    AKV_VARIANT(128, 4, 0, 4, AKV_LAYOUT_SCALAR),  // ragged paged atlas, 4x4 V (config 4)
    AKV_VARIANT(128, 4, 0, 8, AKV_LAYOUT_SCALAR),
    AKV_VARIANT(128, 4, 0, 4, AKV_LAYOUT_RGBA),
    AKV_VARIANT(128, 4, 0, 0, AKV_LAYOUT_SCALAR),  // FP16 control
    AKV_VARIANT(128, 8, 4, 8, AKV_LAYOUT_SCALAR),  // Llama-3-70B shape, 4x4 K + 8x8 V (config 3)
    AKV_VARIANT(128, 8, 0, 8, AKV_LAYOUT_SCALAR),
    AKV_VARIANT(128, 8, 0, 0, AKV_LAYOUT_SCALAR),  // FP16 control
};
#undef AKV_VARIANT

const Variant* find_variant(int D, int G, int kbs, int vbs, int vl) {
    for (const Variant& v : kVariants)
        if (v.D == D && v.G == G && v.kbs == kbs && v.vbs == vbs && (vbs == 0 || v.vl == vl)) return &v;
    return nullptr;
}

struct AttnPlan {
    int kbs, vbs, vl, split, nsplits;
    int kernel;  // AKV_KERNEL_*
    size_t ws;
};

// `ws_limit` > 0: when the caller leaves the split to the library and the
// default split's partials need more than ws_limit bytes, the plan takes the
// most splits whose partials fit instead (fewer, longer splits).
int plan_attention(const AkvAttnDesc* d, AttnPlan* out, size_t ws_limit = 0) {
    if (!d) return AKV_ERR_INVALID_ARGUMENT;
    if (d->batch <= 0 || d->q_heads <= 0 || d->kv_heads <= 0 || d->head_dim <= 0 || d->max_tokens <= 0 ||
        d->page_tokens <= 0 || d->q_heads % d->kv_heads)
        return AKV_ERR_INVALID_ARGUMENT;
    if (d->q_dtype < AKV_Q_F32 || d->q_dtype > AKV_Q_F16) return AKV_ERR_INVALID_ARGUMENT;
    const AkvPlane* planes[2] = {&d->k, &d->v};
    int fps[2] = {0, 0};
    for (int i = 0; i < 2; ++i) {
        const AkvPlane* pl = planes[i];
        if (!pl->data) return AKV_ERR_INVALID_ARGUMENT;
        if (pl->storage == AKV_STORAGE_ASTC) {
            if (!valid_block(pl->block) || d->page_tokens % pl->block) return AKV_ERR_INVALID_ARGUMENT;
            if (pl->layout != AKV_LAYOUT_SCALAR && pl->layout != AKV_LAYOUT_RGBA) return AKV_ERR_INVALID_ARGUMENT;
            if (pl->layout == AKV_LAYOUT_RGBA && d->head_dim % 4) return AKV_ERR_INVALID_ARGUMENT;
            if (pl->normalization < AKV_NORM_PAGE_CHANNEL || pl->normalization > AKV_NORM_BLOCK_AFFINE)
                return AKV_ERR_INVALID_ARGUMENT;
            if (!pl->offsets || !pl->scales) return AKV_ERR_INVALID_ARGUMENT;
            if (i == 0 && pl->layout != AKV_LAYOUT_SCALAR) return AKV_ERR_UNSUPPORTED;
            if (reinterpret_cast<uintptr_t>(pl->data) % 16) return AKV_ERR_INVALID_ARGUMENT;
            fps[i] = pl->block;
        } else if (pl->storage == AKV_STORAGE_FP16) {
            if (reinterpret_cast<uintptr_t>(pl->data) % 16 || (d->head_dim * 2) % 16) return AKV_ERR_INVALID_ARGUMENT;
        } else {
            return AKV_ERR_INVALID_ARGUMENT;
        }
        if (pl->side && (i != 0 || pl->storage != AKV_STORAGE_ASTC || pl->side_count <= 0 || !pl->side_channels_dev))
            return AKV_ERR_INVALID_ARGUMENT;
    }
    if (d->block_table_dev && (d->pages_per_seq <= 0 || d->num_pages <= 0 ||
                               static_cast<int64_t>(d->pages_per_seq) * d->page_tokens < d->max_tokens))
        return AKV_ERR_INVALID_ARGUMENT;
    out->kbs = fps[0];
    out->vbs = fps[1];
    out->vl = d->v.storage == AKV_STORAGE_ASTC ? d->v.layout : AKV_LAYOUT_SCALAR;
    if (!find_variant(d->head_dim, d->q_heads / d->kv_heads, out->kbs, out->vbs, out->vl)) return AKV_ERR_UNSUPPORTED;
    const bool fast_shape = out->vbs && find_fast(d->head_dim, d->q_heads / d->kv_heads, out->vbs, out->kbs, out->vl);
    const bool fp16_shape = !out->vbs && !out->kbs && find_fp16(d->head_dim, d->q_heads / d->kv_heads);
    const int ch = fast_shape ? fast_chunk(out->kbs, out->vbs)
                              : (fp16_shape ? f16k::Cfg<64, 3>::CH : chunk_tokens(out->kbs, out->vbs));
    int split = d->split_tokens;
    if (split <= 0) {
        // Enough (split, head, batch) units for ~64 CTAs per SM: many short
        // splits keep the SMs evenly busy to the end of the launch (measured
        // against 8 per SM: C2 5.06 -> 4.76 ms, C3 11.2 -> 10.1, C4 9.6 ->
        // 8.2), for a split-partial workspace that grows with the count.
        // Splits of at least kMinSplitChunks chunks: when few (head, batch)
        // units share the GPU (one KV head per GPU of eight), shorter splits
        // cost more in per-split set-up and merge work than they gain in
        // balance (config 2 at one head per GPU: 0.695 ms with 3-chunk splits,
        // 0.670 with 6).
        const int64_t units = static_cast<int64_t>(d->batch) * d->kv_heads;
        const int64_t want = (static_cast<int64_t>(sm_count()) * 64 + units - 1) / units;
        int64_t per = (d->max_tokens + want - 1) / want;
        per = ((per + ch - 1) / ch) * ch;
        const int64_t min_per = static_cast<int64_t>(kMinSplitChunks) * ch;
        const int64_t whole = ((d->max_tokens + ch - 1) / ch) * ch;
        if (per < min_per) per = min_per < whole ? min_per : whole;
        split = static_cast<int>(per < ch ? ch : per);
    }
    int lcm_fp = out->kbs ? out->kbs : 1;
    if (out->vbs) {
        int a = lcm_fp, b = out->vbs;
        while (b) { const int r = a % b; a = b; b = r; }
        lcm_fp = lcm_fp / a * out->vbs;
    }
    const size_t per_split = static_cast<size_t>(d->batch) * d->q_heads * (d->head_dim + 2) * sizeof(float);
    if (d->split_tokens <= 0 && ws_limit > 0 &&
        per_split * static_cast<size_t>((d->max_tokens + split - 1) / split) > ws_limit) {
        const int64_t nmax = static_cast<int64_t>(ws_limit / per_split);
        if (nmax < 1) return AKV_ERR_STATIC_WORKSPACE;
        // Splits stay whole chunks and whole block rows of every plane.
        int align = ch, b = lcm_fp;
        {
            int a = align;
            while (b) { const int r = a % b; a = b; b = r; }
            align = align / a * lcm_fp;
        }
        int64_t per = (d->max_tokens + nmax - 1) / nmax;
        per = ((per + align - 1) / align) * align;
        split = static_cast<int>(per);
    }
    if (split % lcm_fp) return AKV_ERR_INVALID_ARGUMENT;
    out->split = split;
    out->nsplits = (d->max_tokens + split - 1) / split;
    out->kernel = fast_path_ok(d, out->kbs, out->vbs, out->vl, split) ? AKV_KERNEL_FAST
                  : (fp16_shape && fp16_path_ok(d)) ? AKV_KERNEL_FP16 : AKV_KERNEL_GENERIC;
    out->ws = static_cast<size_t>(d->batch) * d->q_heads * out->nsplits * (d->head_dim + 2) * sizeof(float);
    return AKV_OK;
}

// ------------------------------------------------------------------ decode

template <int BS>
int launch_decode(const void* blocks, int64_t n, int mode, void* out, cudaStream_t s) {
    const int64_t iters = (n + kDecodeBlocksPerIter - 1) / kDecodeBlocksPerIter;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    const int grid = static_cast<int>(iters < cap ? iters : cap);
    const uint4* b = static_cast<const uint4*>(blocks);
    // Vector row stores need a 16-byte aligned output (cudaMalloc'd buffers
    // are); any other 4-byte aligned output gets the word-store instance.
    if (reinterpret_cast<uintptr_t>(out) % 16 == 0) {
        if (mode == AKV_OUT_UNORM8) decode_blocks_kernel<BS, AKV_OUT_UNORM8, true><<<grid, kDecodeThreads, 0, s>>>(b, n, out);
        else if (mode == AKV_OUT_FP16) decode_blocks_kernel<BS, AKV_OUT_FP16, true><<<grid, kDecodeThreads, 0, s>>>(b, n, out);
        else decode_blocks_kernel<BS, AKV_OUT_UNORM16, true><<<grid, kDecodeThreads, 0, s>>>(b, n, out);
    } else {
        if (mode == AKV_OUT_UNORM8) decode_blocks_kernel<BS, AKV_OUT_UNORM8, false><<<grid, kDecodeThreads, 0, s>>>(b, n, out);
        else if (mode == AKV_OUT_FP16) decode_blocks_kernel<BS, AKV_OUT_FP16, false><<<grid, kDecodeThreads, 0, s>>>(b, n, out);
        else decode_blocks_kernel<BS, AKV_OUT_UNORM16, false><<<grid, kDecodeThreads, 0, s>>>(b, n, out);
    }
    return launch_status();
}

template <int BS, int LAYOUT>
int launch_restore(const PlaneDev& pl, int B, int H, int T, int D, int P, const int32_t* table, int pps, int num_pages,
                   float* out, int32_t* status, cudaStream_t s) {
    constexpr int CH = 8 * BS;
    const size_t smem = sizeof(TileScratch<BS, LAYOUT>) + static_cast<size_t>(CH) * D * sizeof(float);
    auto kern = restore_plane_kernel<BS, LAYOUT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        return AKV_ERR_CUDA;
    }
    dim3 grid((T + CH - 1) / CH, H, B);
    kern<<<grid, kDecodeThreads, smem, s>>>(pl, D, T, P, table, pps, num_pages, out, status);
    return launch_status();
}


// Kernel parameters of one KV segment `d` (its planes, lengths and split
// plan) writing split rows [split_base, split_base + plan.nsplits) of a
// workspace with `stride` rows per (sequence, query head); query, output,
// status and scale come from `io`.
AttnParams segment_params(const AkvAttnDesc* d, const AttnPlan& plan, const AkvAttnDesc* io, int split_base,
                          int stride) {
    AttnParams p;
    p.B = d->batch; p.Hq = d->q_heads; p.Hkv = d->kv_heads; p.T = d->max_tokens;
    p.page_tokens = d->page_tokens; p.split_tokens = plan.split; p.nsplits = plan.nsplits;
    p.split_base = split_base; p.split_stride = stride; p.merge_all = 0;
    p.q_dtype = io->q_dtype; p.q = io->q_dev;
    p.seq_lens = d->seq_lens_dev; p.table = d->block_table_dev;
    p.pps = d->pages_per_seq; p.num_pages = d->num_pages;
    p.k = to_dev(d->k); p.v = to_dev(d->v);
    const float scale = io->scale > 0.f ? io->scale : 1.0f / std::sqrt(static_cast<float>(io->head_dim));
    p.qscale = scale * 1.4426950408889634f;
    float* ws = static_cast<float*>(io->workspace_dev);
    p.part_acc = ws;
    p.part_ml = ws + static_cast<size_t>(io->batch) * io->q_heads * stride * io->head_dim;
    p.out = io->out_dev;
    p.status = io->status_dev;
    return p;
}

int launch_segment(const AkvAttnDesc* d, const AttnPlan& plan, const AttnParams& p, cudaStream_t s, int phase) {
    if (plan.kernel == AKV_KERNEL_FAST)
        return find_fast(d->head_dim, d->q_heads / d->kv_heads, plan.vbs, plan.kbs, plan.vl)->fn(p, s, phase);
    if (plan.kernel == AKV_KERNEL_FP16) return find_fp16(d->head_dim, d->q_heads / d->kv_heads)->fn(p, s, phase);
    return find_variant(d->head_dim, d->q_heads / d->kv_heads, plan.kbs, plan.vbs, plan.vl)->fn(p, s, phase);
}

// A tail descriptor must describe the same sequences and heads as the main one.
bool tail_matches(const AkvAttnDesc* d, const AkvAttnDesc* t) {
    return t && t->batch == d->batch && t->q_heads == d->q_heads && t->kv_heads == d->kv_heads &&
           t->head_dim == d->head_dim;
}

}  // namespace
}  // namespace akv

using namespace akv;

extern "C" {

const char* akv_cuda_error(int code) {
    switch (code) {
        case AKV_OK: return "success";
        case AKV_ERR_INVALID_ARGUMENT: return "invalid argument (pointer, size, alignment or shape)";
        case AKV_ERR_UNSUPPORTED: return "unsupported combination of head_dim, GQA group, footprints and layout";
        case AKV_ERR_CUDA: return "CUDA runtime error";
        case AKV_ERR_NOT_INITIALIZED: return "decode tables not initialised on this device (call akv_cuda_init outside stream capture)";
        case AKV_ERR_BAD_BLOCK_TABLE: return "block table entry outside [0, num_pages)";
        case AKV_ERR_WORKSPACE: return "workspace missing or smaller than akv_cuda_attention_workspace()";
        case AKV_ERR_TIMEOUT: return "a kernel's bounded wait for its own asynchronous copies ran out";
        case AKV_ERR_STATIC_WORKSPACE:
            return "the call needs more split scratch than the library's static workspace (AKV_STATIC_WORKSPACE_BYTES)";
        default: return "unknown status code";
    }
}

int akv_cuda_abi_version(void) { return AKV_CUDA_ABI_VERSION; }

int akv_cuda_init(int device) { return init_device(device); }

size_t akv_cuda_struct_size(int which) {
    return which == 0 ? sizeof(AkvPlane) : which == 1 ? sizeof(AkvAttnDesc) : 0;
}

size_t akv_cuda_host_tables(void* out, size_t bytes) {
    const Tables& t = host_tables();
    if (out && bytes >= sizeof(Tables)) std::memcpy(out, &t, sizeof(Tables));
    return sizeof(Tables);
}

int akv_cuda_decode_blocks(const void* blocks_dev, int64_t nblocks, int block, int out_mode, void* out_dev, void* stream) {
    if (nblocks < 0 || !valid_block(block) || out_mode < AKV_OUT_UNORM8 || out_mode > AKV_OUT_UNORM16)
        return AKV_ERR_INVALID_ARGUMENT;
    if (nblocks == 0) return AKV_OK;
    if (!blocks_dev || !out_dev || reinterpret_cast<uintptr_t>(blocks_dev) % 16 ||
        reinterpret_cast<uintptr_t>(out_dev) % (out_mode == AKV_OUT_UNORM8 ? 4 : 8))
        return AKV_ERR_INVALID_ARGUMENT;
    if (int st = ensure_init(static_cast<cudaStream_t>(stream))) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (block) {
        case 4: return launch_decode<4>(blocks_dev, nblocks, out_mode, out_dev, s);
        case 6: return launch_decode<6>(blocks_dev, nblocks, out_mode, out_dev, s);
        default: return launch_decode<8>(blocks_dev, nblocks, out_mode, out_dev, s);
    }
}

int akv_cuda_decode_image(const void* blocks_dev, size_t bytes, int block, float* rgba_dev, unsigned width,
                          unsigned height, void* stream) {
    if (!valid_block(block) || width == 0 || height == 0 || width > (1u << 24) || height > (1u << 24))
        return AKV_ERR_INVALID_ARGUMENT;
    const int cols = static_cast<int>((width + block - 1) / block), rows = static_cast<int>((height + block - 1) / block);
    if (static_cast<size_t>(cols) * rows * 16 != bytes) return AKV_ERR_INVALID_ARGUMENT;
    if (!blocks_dev || !rgba_dev || reinterpret_cast<uintptr_t>(blocks_dev) % 16 || reinterpret_cast<uintptr_t>(rgba_dev) % 16)
        return AKV_ERR_INVALID_ARGUMENT;
    if (int st = ensure_init(static_cast<cudaStream_t>(stream))) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t n = static_cast<int64_t>(cols) * rows;
    const int64_t iters = (n + kDecodeBlocksPerIter - 1) / kDecodeBlocksPerIter;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    const int grid = static_cast<int>(iters < cap ? iters : cap);
    const uint4* b = static_cast<const uint4*>(blocks_dev);
    const int w = static_cast<int>(width), h = static_cast<int>(height);
    if (block == 4) decode_image_kernel<4><<<grid, kDecodeThreads, 0, s>>>(b, cols, rows, rgba_dev, w, h);
    else if (block == 6) decode_image_kernel<6><<<grid, kDecodeThreads, 0, s>>>(b, cols, rows, rgba_dev, w, h);
    else decode_image_kernel<8><<<grid, kDecodeThreads, 0, s>>>(b, cols, rows, rgba_dev, w, h);
    return launch_status();
}

size_t akv_cuda_attention_workspace(const AkvAttnDesc* desc) {
    AttnPlan plan;
    return plan_attention(desc, &plan) == AKV_OK ? plan.ws : 0;
}

int akv_cuda_attention_plan(const AkvAttnDesc* desc, int* kernel, int* split_tokens, int* nsplits) {
    AttnPlan plan;
    if (int st = plan_attention(desc, &plan)) return st;
    if (kernel) *kernel = plan.kernel;
    if (split_tokens) *split_tokens = plan.split;
    if (nsplits) *nsplits = plan.nsplits;
    return AKV_OK;
}

int akv_cuda_decode_attention(const AkvAttnDesc* d, void* stream) {
    return akv_cuda_decode_attention_phase(d, AKV_PHASE_SPLIT | AKV_PHASE_MERGE, stream);
}


int akv_cuda_decode_attention_phase(const AkvAttnDesc* d, int phase, void* stream) {
    if (phase < AKV_PHASE_SPLIT || phase > (AKV_PHASE_SPLIT | AKV_PHASE_MERGE)) return AKV_ERR_INVALID_ARGUMENT;
    AttnPlan plan;
    if (int st = plan_attention(d, &plan)) return st;
    if (!d->q_dev || !d->out_dev) return AKV_ERR_INVALID_ARGUMENT;
    if (!d->workspace_dev || d->workspace_bytes < plan.ws) return AKV_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(d->workspace_dev) % 16) return AKV_ERR_INVALID_ARGUMENT;
    if (int st = ensure_init(static_cast<cudaStream_t>(stream))) return st;
    const AttnParams p = segment_params(d, plan, d, 0, plan.nsplits);
    return launch_segment(d, plan, p, static_cast<cudaStream_t>(stream), phase);
}

size_t akv_cuda_attention_tail_workspace(const AkvAttnDesc* desc, const AkvAttnDesc* tail) {
    AttnPlan a, b;
    if (!desc || !tail_matches(desc, tail) || plan_attention(desc, &a) || plan_attention(tail, &b)) return 0;
    return a.ws + b.ws;
}

int akv_cuda_decode_attention_tail(const AkvAttnDesc* d, const AkvAttnDesc* tail, void* stream) {
    if (!d || !tail_matches(d, tail)) return AKV_ERR_INVALID_ARGUMENT;
    AttnPlan a, b;
    if (int st = plan_attention(d, &a)) return st;
    if (int st = plan_attention(tail, &b)) return st;
    if (!d->q_dev || !d->out_dev) return AKV_ERR_INVALID_ARGUMENT;
    if (!d->workspace_dev || d->workspace_bytes < a.ws + b.ws) return AKV_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(d->workspace_dev) % 16) return AKV_ERR_INVALID_ARGUMENT;
    if (int st = ensure_init(static_cast<cudaStream_t>(stream))) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int stride = a.nsplits + b.nsplits;
    AttnParams pa = segment_params(d, a, d, 0, stride);
    if (int st = launch_segment(d, a, pa, s, AKV_PHASE_SPLIT)) return st;
    const AttnParams pb = segment_params(tail, b, d, a.nsplits, stride);
    if (int st = launch_segment(tail, b, pb, s, AKV_PHASE_SPLIT)) return st;
    // One merge over both segments' split rows (empty splits hold m = -inf).
    pa.merge_all = 1;
    launch_merge(pa, d->head_dim, s);
    return launch_status();
}

int akv_cuda_decode_attention_noalloc(const AkvAttnDesc* d, void* stream) {
    AttnPlan plan;
    if (int st = plan_attention(d, &plan, static_cast<size_t>(AKV_STATIC_WORKSPACE_BYTES))) return st;
    if (plan.ws > static_cast<size_t>(AKV_STATIC_WORKSPACE_BYTES)) return AKV_ERR_STATIC_WORKSPACE;
    if (int st = ensure_init(static_cast<cudaStream_t>(stream))) return st;
    void* ws = nullptr;
    if (int st = static_workspace(&ws)) return st;
    AkvAttnDesc local = *d;
    local.split_tokens = plan.split;  // the split chosen to fit the static array
    local.workspace_dev = ws;
    local.workspace_bytes = AKV_STATIC_WORKSPACE_BYTES;
    return akv_cuda_decode_attention(&local, stream);
}

int akv_cuda_restore_plane(const AkvPlane* plane, int32_t batch, int32_t kv_heads, int32_t max_tokens, int32_t head_dim,
                           int32_t page_tokens, const int32_t* block_table_dev, int32_t pages_per_seq, int32_t num_pages,
                           float* out_dev, int32_t* status_dev, void* stream) {
    if (!plane || !plane->data || !out_dev || batch <= 0 || kv_heads <= 0 || max_tokens <= 0 || head_dim <= 0 ||
        page_tokens <= 0)
        return AKV_ERR_INVALID_ARGUMENT;
    if (block_table_dev && (pages_per_seq <= 0 || num_pages <= 0 ||
                            static_cast<int64_t>(pages_per_seq) * page_tokens < max_tokens))
        return AKV_ERR_INVALID_ARGUMENT;
    if (int st = ensure_init(static_cast<cudaStream_t>(stream))) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const PlaneDev pl = to_dev(*plane);
    if (plane->storage == AKV_STORAGE_FP16) {
        restore_fp16_kernel<<<dim3(max_tokens, kv_heads, batch), 128, 0, s>>>(pl, head_dim, max_tokens, page_tokens,
                                                                              block_table_dev, pages_per_seq, num_pages,
                                                                              out_dev, status_dev);
        return launch_status();
    }
    if (plane->storage != AKV_STORAGE_ASTC || !valid_block(plane->block) || page_tokens % plane->block ||
        !plane->offsets || !plane->scales || reinterpret_cast<uintptr_t>(plane->data) % 16)
        return AKV_ERR_INVALID_ARGUMENT;
    if (plane->layout == AKV_LAYOUT_RGBA && head_dim % 4) return AKV_ERR_INVALID_ARGUMENT;
    const bool rgba = plane->layout == AKV_LAYOUT_RGBA;
#define AKV_RESTORE(BS, L) launch_restore<BS, L>(pl, batch, kv_heads, max_tokens, head_dim, page_tokens, block_table_dev, \
                                                  pages_per_seq, num_pages, out_dev, status_dev, s)
    switch (plane->block) {
        case 4: return rgba ? AKV_RESTORE(4, AKV_LAYOUT_RGBA) : AKV_RESTORE(4, AKV_LAYOUT_SCALAR);
        case 6: return rgba ? AKV_RESTORE(6, AKV_LAYOUT_RGBA) : AKV_RESTORE(6, AKV_LAYOUT_SCALAR);
        default: return rgba ? AKV_RESTORE(8, AKV_LAYOUT_RGBA) : AKV_RESTORE(8, AKV_LAYOUT_SCALAR);
    }
#undef AKV_RESTORE
}

}  // extern "C"
