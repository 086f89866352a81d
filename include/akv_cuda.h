/*
 * akv_cuda.h — C ABI of the B200 (sm_100a) ASTC-KV decode-attention library.
 *
 * Plain C, plain pointers and sizes. Conventions, kept from the reference
 * bridge (astc_kv/bridge.cpp:1-36):
 *   - the caller owns every buffer; pointers named *_dev are device memory;
 *   - every entry point returns an int status, 0 = success, and never throws;
 *     `akv_cuda_error(code)` gives the message (bridge.cpp:17 `akv_error`);
 *   - work is ordered on the cudaStream_t passed as `stream` (NULL = legacy
 *     default stream); calls do not synchronise the device;
 *   - no entry point allocates device memory; tables live in static
 *     __device__ storage that akv_cuda_init fills once per device.
 */
#ifndef AKV_CUDA_H
#define AKV_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AKV_CUDA_ABI_VERSION 1

/* Status codes. */
#define AKV_OK 0
#define AKV_ERR_INVALID_ARGUMENT 1   /* bad pointer, size or shape */
#define AKV_ERR_UNSUPPORTED 2        /* valid but not compiled in (shape/format combination) */
#define AKV_ERR_CUDA 3               /* a CUDA runtime call failed */
#define AKV_ERR_NOT_INITIALIZED 4    /* akv_cuda_init has not run on this device and could not run now */
#define AKV_ERR_BAD_BLOCK_TABLE 5    /* a kernel saw a block-table entry outside [0, num_pages) */
#define AKV_ERR_WORKSPACE 6          /* workspace missing or smaller than akv_cuda_attention_workspace() */
#define AKV_ERR_TIMEOUT 7            /* a kernel's bounded wait for its own async copies ran out */
#define AKV_ERR_STATIC_WORKSPACE 8   /* the call needs more split scratch than AKV_STATIC_WORKSPACE_BYTES */

/* Decoder output views of the 16-bit interpolation result C of each texel. */
#define AKV_OUT_UNORM8 0   /* C >> 8 (decode_unorm8), 4 bytes per texel */
#define AKV_OUT_FP16 1     /* fp16 bits: 1.0 if C == 65535, else C/65536 truncated (what astcenc's F32 LDR output holds), 8 bytes per texel */
#define AKV_OUT_UNORM16 2  /* C itself, 8 bytes per texel */

/* Plane storage, layout and normalisation (astc_kv/codec.py:116-215). */
#define AKV_STORAGE_FP16 0
#define AKV_STORAGE_ASTC 1
#define AKV_LAYOUT_SCALAR 0        /* value in R of an rrr1 texel (codec.py:181-184) */
#define AKV_LAYOUT_RGBA 1          /* four channels per texel (codec.py:185-187) */
#define AKV_NORM_PAGE_CHANNEL 0    /* (offset, scale) per (head, page, channel), codec.py:155-161 */
#define AKV_NORM_TOKEN 1           /* (offset, scale) per (head, token), codec.py:162-166 */
#define AKV_NORM_BLOCK_AFFINE 2    /* (offset, scale) per (head, ASTC block); extends block_min, codec.py:167-172 */
#define AKV_Q_F32 0
#define AKV_Q_BF16 1
#define AKV_Q_F16 2

/* Error message for a status code. Replaces bridge.cpp:17 `akv_error`. */
const char* akv_cuda_error(int code);

/* ABI version of the loaded library (AKV_CUDA_ABI_VERSION). */
int akv_cuda_abi_version(void);

/* Fills the decode tables of `device` (synchronous, once per device; later
 * calls return at once). Every other entry point calls it for the current
 * device on first use (and returns AKV_ERR_NOT_INITIALIZED instead while the
 * call's stream is being captured), so call it yourself before any stream
 * capture. The per-device state lives until the process exits: a device
 * reset (cudaDeviceReset) drops the tables but not the library's record of
 * them, so do not use the library on a device after resetting it. */
int akv_cuda_init(int device);

/*
 * Standalone block decode: `nblocks` consecutive 16-byte ASTC LDR blocks of a
 * square footprint `block` (4, 6 or 8) -> per-block texels
 * out[nblocks][block][block][4] in `out_mode`.
 * Replaces the decode half of bridge.cpp:27-35 `akv_decode` for device data
 * (the reference decodes through astcenc on the CPU, codec.py:56).
 */
int akv_cuda_decode_blocks(const void* blocks_dev, int64_t nblocks, int block, int out_mode,
                           void* out_dev, void* stream);

/*
 * Image decode with the contract of bridge.cpp:27-35 `akv_decode`: blocks of a
 * width x height image in row-major block order (`bytes` must equal
 * ceil(w/block)*ceil(h/block)*16) -> float32 RGBA [height][width][4], each
 * value the fp16 view of C widened to float (the LDR F32 output of astcenc).
 */
int akv_cuda_decode_image(const void* blocks_dev, size_t bytes, int block, float* rgba_dev,
                          unsigned width, unsigned height, void* stream);

/*
 * One K or V plane of a KV cache. Tokens of a (batch b, kv head h) sequence
 * are grouped in pages of `page_tokens` rows. Logical page p of sequence b is
 * physical page `block_table ? block_table[b*pages_per_seq + p] : p`, and its
 * bytes start at
 *     data + b*stride_batch + h*stride_head + phys*stride_page
 * holding page_tokens rows of head_dim fp16 values (FP16 storage) or
 * page_tokens/block rows of ceil(width/block) 16-byte blocks, width =
 * align(head_dim/components, block) (ASTC storage, codec.py:137).
 * Metadata (fp16 offsets/scales) is addressed the same way with element
 * strides meta_stride_*; inside a page it holds
 *     PAGE_CHANNEL: [head_dim]           (page-level pair per channel)
 *     TOKEN:        [page_tokens]
 *     BLOCK_AFFINE: [page_tokens/block][ceil(width/block)]
 * Side plane (ASTC K only, optional): `side_count` channels per head kept
 * exactly in fp16, [page_tokens][side_count] per page at side + strides
 * side_stride_* (bytes); channel ids in side_channels_dev[kv_head][side_count].
 */
typedef struct AkvPlane {
    int32_t storage;
    int32_t block;
    int32_t layout;
    int32_t normalization;
    const void* data;
    int64_t stride_batch, stride_head, stride_page;
    const void* offsets;
    const void* scales;
    int64_t meta_stride_batch, meta_stride_head, meta_stride_page;
    const void* side;
    const int32_t* side_channels_dev;
    int32_t side_count;
    int32_t reserved0;
    int64_t side_stride_batch, side_stride_head, side_stride_page;
} AkvPlane;

/*
 * Decode-step split-K GQA attention over a compressed KV cache: for every
 * (b, query head hq), kv head h = hq / (q_heads/kv_heads) (codec.py:259),
 *   out[b][hq] = softmax(scale * q[b][hq] . K[b][h][t]) . V[b][h][t],
 *   t < seq_len[b],
 * with K/V values restored as offset + scale * decoded (codec.py:198-208),
 * fp32 accumulation, online-softmax partials per split of `split_tokens`
 * tokens and a log-sum-exp merge. Replaces the reference's CPU attention
 * (codec.py:253-267) and its Metal split/merge kernels.
 */
typedef struct AkvAttnDesc {
    int32_t batch, q_heads, kv_heads, head_dim;
    int32_t max_tokens;           /* tokens per sequence capacity (upper bound of seq_lens) */
    int32_t page_tokens;          /* multiple of every ASTC footprint in use */
    int32_t split_tokens;         /* split-K chunk; 0 = library choice */
    int32_t q_dtype;              /* AKV_Q_* */
    const void* q_dev;            /* [batch][q_heads][head_dim] */
    const int32_t* seq_lens_dev;  /* [batch] or NULL (= max_tokens) */
    const int32_t* block_table_dev; /* [batch][pages_per_seq] or NULL */
    int32_t pages_per_seq;
    int32_t num_pages;            /* physical pages, bounds for block_table entries */
    AkvPlane k, v;
    float scale;                  /* 0 = head_dim^-0.5 (codec.py:260) */
    int32_t reserved0;
    void* workspace_dev;          /* split partials, see akv_cuda_attention_workspace */
    size_t workspace_bytes;
    float* out_dev;               /* [batch][q_heads][head_dim] fp32 */
    int32_t* status_dev;          /* optional: kernels write AKV_ERR_BAD_BLOCK_TABLE here */
} AkvAttnDesc;

/* Workspace bytes the descriptor needs (0 on invalid descriptors). */
size_t akv_cuda_attention_workspace(const AkvAttnDesc* desc);

/*
 * Decode attention over two KV segments in one softmax: `desc` (for example
 * the ASTC-compressed complete pages) and `tail` (for example the exact
 * FP16 tokens of the incomplete last page that is not compressed yet).
 * Both descriptors describe the same batch, query/KV heads and head_dim;
 * each has its own planes, lengths (seq_lens_dev), pages and split size.
 * Query, output, scale, status and workspace are taken from `desc` (the
 * tail's are ignored); the workspace must hold
 * akv_cuda_attention_tail_workspace(desc, tail) bytes. Output is
 * softmax(scale q.[K;K_tail]^T) [V;V_tail] per sequence. No counterpart in
 * the reference: its encoder rejects incomplete pages (codec.py:132-133) and
 * its pilot keeps the suffix in FP16 outside the kernels.
 */
size_t akv_cuda_attention_tail_workspace(const AkvAttnDesc* desc, const AkvAttnDesc* tail);
int akv_cuda_decode_attention_tail(const AkvAttnDesc* desc, const AkvAttnDesc* tail, void* stream);

/* The launch plan of a descriptor, without launching: which split kernel
 * runs (AKV_KERNEL_FAST: fused decode + tensor-core kernel for scalar ASTC V
 * with whole chunks per page and 16-byte aligned metadata; AKV_KERNEL_FP16:
 * tensor-core kernel for FP16 K with FP16 V, the FP16 control;
 * AKV_KERNEL_GENERIC otherwise), the split size in tokens and the number of
 * splits. Any output pointer may be NULL. Returns the status
 * akv_cuda_decode_attention would return for a descriptor error. No
 * counterpart in the reference (its Metal host picks kernels in the probe
 * programs). */
#define AKV_KERNEL_GENERIC 0
#define AKV_KERNEL_FAST 1
#define AKV_KERNEL_FP16 2
int akv_cuda_attention_plan(const AkvAttnDesc* desc, int* kernel, int* split_tokens, int* nsplits);

int akv_cuda_decode_attention(const AkvAttnDesc* desc, void* stream);

/* The two launches of akv_cuda_decode_attention issued one at a time, so a
 * caller can place work or events between them: phase 1 writes the split
 * partials (m, l, acc) to the workspace, phase 2 merges them into out.
 * Calling phase 1 then phase 2 on one stream equals one
 * akv_cuda_decode_attention call. */
#define AKV_PHASE_SPLIT 1
#define AKV_PHASE_MERGE 2
int akv_cuda_decode_attention_phase(const AkvAttnDesc* desc, int phase, void* stream);

/*
 * Decode attention for callers that cannot allocate device memory.
 * No counterpart in the reference: it is an addition of this library.
 *
 * Some callers of this code cannot call cudaMalloc or hand out a workspace:
 * bindings from other language runtimes (cgo, JNI, N-API) that reach the GPU
 * only through this C ABI and own no device allocator; hosts whose memory
 * belongs to a framework's caching allocator, where a stray cudaMalloc
 * fragments the pool or stalls every stream; serving loops with a fixed
 * device-memory budget. This entry point takes the same descriptor as
 * akv_cuda_decode_attention, ignores workspace_dev / workspace_bytes, and
 * keeps the split partials in a static device array of
 * AKV_STATIC_WORKSPACE_BYTES compiled into the library (every GPU that loads
 * the library holds that array until the process exits). It allocates
 * nothing.
 *   - With split_tokens = 0 the library picks the split: its usual choice
 *     when those partials fit the array, else the most splits whose
 *     partials fit (longer splits). A descriptor whose explicit
 *     split_tokens needs more scratch than the array holds (see
 *     akv_cuda_attention_workspace), or that does not fit even with one
 *     split per sequence, returns AKV_ERR_STATIC_WORKSPACE.
 *   - The first call on a device looks up the array's device address (and
 *     fills the decode tables if akv_cuda_init has not run there); make that
 *     first call, or akv_cuda_init plus one call, before any stream capture.
 *   - All calls share the one array and it keeps the last call's contents;
 *     nothing in it needs to start at zero (every partial a call reads, that
 *     call wrote first). Calls whose kernels overlap on the GPU (different
 *     streams, or several host threads) race on the array: serialise them.
 */
#define AKV_STATIC_WORKSPACE_BYTES (8u << 20)
int akv_cuda_decode_attention_noalloc(const AkvAttnDesc* desc, void* stream);

/*
 * Restore a whole plane to fp32 [batch][kv_heads][max_tokens][head_dim]:
 * decode + affine, the device twin of EncodedTensor.decoded
 * (codec.py:198-208; unfused fp32 `rec*scale + offset`, bit-exact with the
 * reference's restore). FP16 planes are widened.
 */
int akv_cuda_restore_plane(const AkvPlane* plane, int32_t batch, int32_t kv_heads, int32_t max_tokens,
                           int32_t head_dim, int32_t page_tokens, const int32_t* block_table_dev,
                           int32_t pages_per_seq, int32_t num_pages, float* out_dev,
                           int32_t* status_dev, void* stream);

/* Host-only: sizeof(AkvPlane) for which = 0, sizeof(AkvAttnDesc) for
 * which = 1 (lets FFI bindings check their struct layout); 0 otherwise. */
size_t akv_cuda_struct_size(int which);

/* Host-only: copy the decode tables the library builds (for CPU tests of the
 * table construction). Returns the table size when out is NULL. */
size_t akv_cuda_host_tables(void* out, size_t bytes);

#ifdef __cplusplus
}
#endif

#endif /* AKV_CUDA_H */
