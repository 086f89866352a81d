/*
 * akv_host.h — host-side (CPU) utilities exported by libakv_cuda.so.
 *
 * The reference encodes completed pages on the CPU with Arm astcenc through
 * astc_kv/bridge.cpp:18-26 (`akv_encode`). astcenc is not part of the
 * reference tree, so this library carries its own small ASTC LDR encoder:
 * spec-conformant output that any ASTC decoder reads, but NOT astcenc's
 * search, so its block choices and error differ from astcenc's. The Python
 * layer uses the reference bridge instead whenever libakv_astc.so (built
 * against astcenc) is present.
 */
#ifndef AKV_HOST_H
#define AKV_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Encode a float RGBA image (values in [0, 1], [height][width][4], width and
 * height multiples of `block`) into ceil(w/block)*ceil(h/block) blocks
 * (row-major), `bytes` = 16 * block count. layout 0 (scalar): the value is in
 * R and luminance endpoint modes are used; layout 1 (rgba): RGBA endpoints.
 * effort 0..2 widens the candidate search (partitions, weight grids).
 * Same argument order and status convention as bridge.cpp:18 `akv_encode`
 * (0 = success).
 */
int akv_host_encode(const float* rgba, unsigned width, unsigned height, int block, int layout, int effort,
                    uint8_t* out, size_t bytes, int threads);

/*
 * `n` random, legal LDR blocks of footprint `block`: uniformly drawn valid
 * block modes, partition counts 1-4, LDR endpoint modes, random payload bits
 * and a few void-extent blocks. For the standalone decode benchmark.
 */
int akv_host_random_blocks(int64_t n, int block, uint64_t seed, uint8_t* out, int threads);

#ifdef __cplusplus
}
#endif

#endif /* AKV_HOST_H */
