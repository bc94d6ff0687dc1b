/*
 * cascade_b200 — C ABI of the B200-native block-ingest path of CASCADE
 * (Cascade-HPC/Cascade): SHA-256 content addressing, the FP16->INT8
 * KVCompressor, and the HBM block pool behind CascadeStore.put/get.
 *
 * Every function returns an int status (CASCADE_OK = 0).  On failure the
 * calling thread's cascade_last_error() holds a one-line description.
 * Pointers named d_* are device pointers; arrays of device addresses are
 * passed as uint64_t.  Functions taking `void *stream` enqueue their work on
 * that CUDA stream (NULL = the legacy default stream) and return without
 * synchronising unless stated otherwise.
 *
 * Each entry point names the reference interface it replaces; citations are
 * path:line within the reference project.
 */
#ifndef CASCADE_B200_H
#define CASCADE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CASCADE_ABI_VERSION 1

#define CASCADE_OK 0
#define CASCADE_ERR_INVALID 1   /* bad argument */
#define CASCADE_ERR_CUDA 2      /* a CUDA runtime call failed */
#define CASCADE_ERR_NOMEM 3     /* host or device allocation failed */
#define CASCADE_ERR_FULL 4      /* the device index has no free slot */
#define CASCADE_ERR_NODEVICE 5  /* no CUDA device: there is no CPU path */
#define CASCADE_ERR_UNSUPPORTED 6
#define CASCADE_ERR_TIMEOUT 7   /* a bounded device-side wait gave up */

/* Per-block status codes written by the batched put. */
#define CASCADE_PUT_STORED 0     /* stored as a new block */
#define CASCADE_PUT_DUP_KNOWN 1  /* key already stored: a dedup hit */
#define CASCADE_PUT_DUP_BATCH 2  /* an earlier block of this batch had the key */
#define CASCADE_PUT_FAILED 3     /* no tier had room */

const char *cascade_last_error(void);
int cascade_abi_version(void);

/* ------------------------------------------------------------------ */
/* Stateless batched kernels.                                           */

/* SHA-256 of n device-resident blocks; 32 digest bytes per block to
 * d_digests (4-byte aligned).  Replaces the per-block OpenSSL SHA256() of
 * compute_block_id, cascade_core.cpp:43-53 (bound at bindings.cpp:173-176);
 * the block id is the lowercase hex of digest bytes 0..15. */
int cascade_sha256_batch(const uint64_t *d_ptrs, const uint64_t *d_sizes,
                         size_t n, uint8_t *d_digests, void *stream);

/* KVCompressor::compress (cascade_core.cpp:818-849) of n blocks: block i
 * (d_sizes[i] bytes) -> d_dst[i] = 8-byte header + d_sizes[i]/2 codes, the
 * reference's byte layout.  max_size >= every size (sizes the launch). */
int cascade_kv_compress_batch(const uint64_t *d_src, const uint64_t *d_sizes,
                              const uint64_t *d_dst, size_t n,
                              uint64_t max_size, void *stream);

/* KVCompressor::decompress (cascade_core.cpp:851-872) as called by
 * CascadeStore::get (cascade_core.cpp:1149-1156): d_src[i] holds a
 * compressed block; d_out_sizes[i] (even) bytes are written to d_dst[i]. */
int cascade_kv_decompress_batch(const uint64_t *d_src,
                                const uint64_t *d_out_sizes,
                                const uint64_t *d_dst, size_t n,
                                uint64_t max_out_size, void *stream);

/* n device-to-device block copies in one launch (the pool copy that
 * GPUBackend::put/get do with cudaMemcpyAsync, gpu_backend.cu:298-308,
 * 362-377). */
int cascade_copy_batch(const uint64_t *d_src, const uint64_t *d_dst,
                       const uint64_t *d_sizes, size_t n, uint64_t max_size,
                       void *stream);

/* compute_block_id(np.uint8[]) (bindings.cpp:173-176 ->
 * cascade_core.cpp:43-53) for one host buffer, hashed on the current CUDA
 * device.  Writes 32 hex chars + NUL.  Synchronous. */
int cascade_compute_block_id(const uint8_t *data, uint64_t size,
                             char out_hex[33]);

/* Diagnostics: SHA-256 round-function throughput with every warp slot
 * occupied and no memory traffic (the integer-pipe ceiling used as the
 * SHA roofline denominator).  Synchronous. */
int cascade_diag_sha_peak(int device, uint32_t chunks_per_thread,
                          double *gbps, double *ms);

#ifdef __cplusplus
}
#endif

#endif /* CASCADE_B200_H */
