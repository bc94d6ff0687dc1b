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
 * the block id is the lowercase hex of digest bytes 0..15.
 * Each block is one serial chain, so large blocks need many blocks in one
 * call to fill the GPU.  The launch spreads its CTAs (32 blocks each)
 * evenly by reserving unused shared memory.  When n <= 32 x (SMs - 16) it
 * runs one CTA per SM and fills those SMs' shared memory to within 6 KiB,
 * so kernels the caller runs concurrently use the other SMs unless they
 * need almost no shared memory. */
int cascade_sha256_batch(const uint64_t *d_ptrs, const uint64_t *d_sizes,
                         size_t n, uint8_t *d_digests, void *stream);

/* KVCompressor::compress (cascade_core.cpp:818-849) of n blocks: block i
 * (d_sizes[i] bytes) -> d_dst[i] = 8-byte header + d_sizes[i]/2 codes, the
 * reference's byte layout.  max_size >= every size (sizes the launch). */
int cascade_kv_compress_batch(const uint64_t *d_src, const uint64_t *d_sizes,
                              const uint64_t *d_dst, size_t n,
                              uint64_t max_size, void *stream);

/* No counterpart in the reference.  The same compression as
 * cascade_kv_compress_batch (identical output bytes), for callers that
 * cannot let a library allocate device memory: for example an inference
 * engine that reserved nearly all of HBM for its own KV cache at start-up,
 * or an ingest loop that cannot risk an allocator call stalling or failing
 * mid-step.  It calls no cudaMalloc, cudaFree or other allocating routine;
 * its per-block scratch is a fixed 512 KiB array built into the library.
 * Limits and rules:
 *   - at most 65536 blocks per call; larger n fails with
 *     CASCADE_ERR_INVALID and an explanatory cascade_last_error();
 *   - CUDA places the array on a GPU lazily, at the first call on that GPU
 *     (which also looks up the array's device address, a one-time set-up),
 *     and it stays there until the process exits.  A call with n = 0 does
 *     only this set-up: make it on each GPU before reserving that GPU's
 *     memory and before any stream capture.  The set-up is redone by
 *     itself after the device's context changes (cudaDeviceReset);
 *   - all calls on a GPU share that one array, so calls whose work overlaps
 *     on the same GPU race: keep them on one stream;
 *   - `stream` must belong to the current device (else CASCADE_ERR_INVALID). */
int cascade_kv_compress_batch_noalloc(const uint64_t *d_src,
                                      const uint64_t *d_sizes,
                                      const uint64_t *d_dst, size_t n,
                                      uint64_t max_size, void *stream);

/* KVCompressor::decompress (cascade_core.cpp:851-872) as called by
 * CascadeStore::get (cascade_core.cpp:1149-1156): d_src[i] holds a
 * compressed block; d_out_sizes[i] (even) bytes are written to d_dst[i]. */
int cascade_kv_decompress_batch(const uint64_t *d_src,
                                const uint64_t *d_out_sizes,
                                const uint64_t *d_dst, size_t n,
                                uint64_t max_out_size, void *stream);

/* ------------------------------------------------------------------ */
/* KV-cache wire format on the device.                                  */

/* One layer's K or V tensor of one cache: element [h][s][d] is at
 * ptr + (h * stride_head + s * stride_seq + d) * element size.  head_dim
 * elements are contiguous; the strides (in elements) may be anything, so
 * a [1, heads, seq, dim] tensor, a slice of a longer static cache and a
 * [seq, heads, dim] tensor permuted to [heads, seq, dim] all describe
 * themselves without a copy. */
typedef struct {
  uint64_t ptr;
  int64_t stride_head;
  int64_t stride_seq;
} cascade_kv_tensor_t;

#define CASCADE_KV_FP16 0
#define CASCADE_KV_BF16 1
#define CASCADE_KV_FP32 2

/* Bytes of one wire block: the 18-byte "<IIIIH" header + 2 x layers x
 * heads x seq x head_dim FP16 values (kv_manager.py:11-12, 43-63). */
uint64_t cascade_kv_wire_bytes(uint32_t layers, uint32_t heads, uint32_t seq,
                               uint32_t head_dim);

/* kv_manager.serialize_kv_cache (inference_benchmark/kv_manager.py:43-63)
 * on the device, for n caches of one shape in one launch.  d_src holds
 * n x 2 x layers tensor descriptors (cache 0's K0, V0, K1, V1, ..., then
 * cache 1's), elements of src_dtype (CASCADE_KV_*; BF16 and FP32 round to
 * FP16 to nearest even, as the reference's .to(torch.float16) does).
 * d_dst[i] receives cache i's wire block, cascade_kv_wire_bytes() bytes:
 * the header (dtype id 0) then K0, V0, K1, ... as contiguous
 * [heads][seq][head_dim] FP16, the reference's bytes exactly.  16-byte
 * aligned outputs and head_dim a multiple of 8 take the vector path; any
 * other alignment is handled element by element. */
int cascade_kv_serialize_batch(const cascade_kv_tensor_t *d_src,
                               int src_dtype, uint32_t layers, uint32_t heads,
                               uint32_t seq, uint32_t head_dim,
                               const uint64_t *d_dst, size_t n, void *stream);

/* kv_manager.deserialize_kv_cache (kv_manager.py:66-95) on the device: n
 * wire blocks d_src[i] of one shape (the caller has read the header) into
 * n x 2 x layers FP16 tensors d_dst (same order as serialize). */
int cascade_kv_deserialize_batch(const uint64_t *d_src, uint32_t layers,
                                 uint32_t heads, uint32_t seq,
                                 uint32_t head_dim,
                                 const cascade_kv_tensor_t *d_dst, size_t n,
                                 void *stream);

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

/* Diagnostics: kernels this library has launched since it was loaded
 * (all devices, all threads). */
uint64_t cascade_diag_launch_count(void);

/* ------------------------------------------------------------------ */
/* The block store (CascadeStore, cascade.hpp:420-502).                 */

/* CascadeConfig (cascade.hpp:25-60; the 18 fields bound at
 * bindings.cpp:15-35, plus num_io_threads), followed by B200 extensions.
 * cascade_config_init() sets the reference defaults.  Fields the reference
 * never reads on this path (compression_enabled, num_io_threads) and the
 * cold-tier / prefetch fields (lustre_*, prefetch_*, aggregated_lustre,
 * agg_file_size) are accepted and ignored: the Lustre tier and the
 * prefetch pipeline are not part of this library. */
typedef struct cascade_config {
  uint64_t gpu_capacity_bytes;  /* 32 GiB: the HBM pool */
  int32_t gpu_device_id;        /* 0 */
  int32_t use_gpu;              /* 1: 0 = no HBM tier (kernels still run on
                                   the GPU; blocks live in the DRAM tier) */
  uint64_t shm_capacity_bytes;  /* 64 GiB: the pinned DRAM tier */
  const char *shm_path;         /* "/dev/shm/cascade" (unused: the DRAM tier
                                   is anonymous pinned memory) */
  const char *lustre_path;      /* "cascade_store" */
  uint64_t lustre_stripe_size;  /* 1 MiB */
  int32_t lustre_stripe_count;  /* 16 */
  int32_t dedup_enabled;        /* 1 */
  int32_t compression_enabled;  /* 1 */
  int32_t num_io_threads;       /* 8 */
  int32_t semantic_eviction;    /* 1: demote non-prefix blocks first */
  int32_t promotion_enabled;    /* 1: DRAM hits move back to HBM */
  int32_t prefetch_enabled;     /* 1 */
  int32_t prefetch_threads;     /* 2 */
  uint64_t prefetch_queue_size; /* 64 */
  int32_t kv_compression;       /* 0: 1 = DRAM tier holds KVCompressor's
                                   INT8 form of blocks >= 64 bytes */
  int32_t aggregated_lustre;    /* 0 */
  uint64_t agg_file_size;       /* 256 MiB */
  /* --- B200 extensions --- */
  int32_t gpu_q8;               /* 0: HBM holds raw bytes, as the
                                   reference's GPU tier; 1 = HBM also holds
                                   the INT8 form when kv_compression is on
                                   (gpu_used then counts those size/2
                                   bytes) */
  int32_t reserved0;
  uint64_t index_slots;         /* device index capacity, a power of two;
                                   0 = derived from the tier capacities */
  uint64_t dram_chunk_bytes;    /* pinned-arena growth unit; 0 = 1 GiB */
} cascade_config_t;

/* CascadeStore::Stats (cascade.hpp:439-456), field for field. */
typedef struct cascade_stats {
  uint64_t gpu_used, shm_used, gpu_hits, shm_hits, lustre_hits, misses,
      dedup_hits, gpu_evictions, shm_evictions, promotions_to_gpu,
      promotions_to_shm, prefetch_completed, compression_savings_bytes,
      shm_puts, lustre_puts;
} cascade_stats_t;

typedef struct cascade_store cascade_store_t;

void cascade_config_init(cascade_config_t *cfg);
/* sizeof(cascade_config_t) and sizeof(cascade_stats_t) as compiled, for
 * bindings that lay the structs out themselves (ctypes, cgo, JNA). */
void cascade_struct_sizes(size_t *config_bytes, size_t *stats_bytes);

/* CascadeStore(cfg) (bindings.cpp:72, cascade_core.cpp:960-989).
 * Fails with CASCADE_ERR_NODEVICE on a machine without a CUDA device. */
int cascade_store_create(const cascade_config_t *cfg, cascade_store_t **out);
int cascade_store_destroy(cascade_store_t *s);

/* CascadeStore.put(block_id, data, is_prefix) (bindings.cpp:73-76,
 * cascade_core.cpp:1074-1135) from a host buffer.  *stored = the
 * reference's bool result.  Synchronous. */
int cascade_store_put(cascade_store_t *s, const char *block_id,
                      const uint8_t *data, uint64_t size, int is_prefix,
                      int *stored);

/* CascadeStore.get(block_id, out) (bindings.cpp:77-82,
 * cascade_core.cpp:1138-1189) into a host buffer of out_capacity bytes.
 * *found / *size as the reference's (found, size) tuple.  When the block
 * is larger than out_capacity nothing is written, *found = 1 and *size is
 * the size needed (the reference writes past the buffer instead).
 * Synchronous. */
int cascade_store_get(cascade_store_t *s, const char *block_id, uint8_t *out,
                      uint64_t out_capacity, int *found, uint64_t *size);

/* CascadeStore::contains (cascade_core.cpp:1192-1200). */
int cascade_store_contains(cascade_store_t *s, const char *block_id,
                           int *present);
/* CascadeStore::get_stats (cascade_core.cpp:1238-1257). */
int cascade_store_get_stats(cascade_store_t *s, cascade_stats_t *out);
/* CascadeStore::clear (cascade_core.cpp:1259-1277). */
int cascade_store_clear(cascade_store_t *s);
/* CascadeStore::flush (cascade_core.cpp:1279-1282): waits for the store's
 * device work; there is no file tier to flush. */
int cascade_store_flush(cascade_store_t *s);

/* The 16-byte key a block id names: the id's bytes when it is 32
 * lowercase hex characters (compute_block_id's format), otherwise a key
 * this store assigned to that string on first use. */
int cascade_store_key_of(cascade_store_t *s, const char *block_id,
                         uint8_t key_out[16]);

/* Batched put of n device-resident blocks (the reference's OpenMP
 * put_batch, cascade_core.cpp:1203-1218, not bound to Python there).
 * h_ptrs/h_sizes: host arrays of device addresses and byte counts.
 * h_keys: n x 16 key bytes, or NULL to content-address every block by
 * SHA-256 (key = digest bytes 0..15, as compute_block_id).  h_prefix:
 * n is_prefix flags or NULL.  h_status: n CASCADE_PUT_* codes or NULL.
 * h_digests: n x 32 digest bytes (content-addressed only) or NULL.
 * `stream` is waited on before the inputs are read.  Synchronous. */
int cascade_store_put_batch(cascade_store_t *s, size_t n,
                            const uint64_t *h_ptrs, const uint64_t *h_sizes,
                            const uint8_t *h_keys, const uint8_t *h_prefix,
                            uint8_t *h_status, uint8_t *h_digests,
                            void *stream, uint64_t *n_stored);

/* Batched put of n HOST blocks (pinned or pageable), content-addressed
 * when h_keys is NULL.  The library moves the bytes to the GPU through its
 * own staging in pipelined chunks.  Synchronous. */
int cascade_store_put_batch_host(cascade_store_t *s, size_t n,
                                 const uint8_t *const *h_blocks,
                                 const uint64_t *h_sizes,
                                 const uint8_t *h_keys,
                                 const uint8_t *h_prefix, uint8_t *h_status,
                                 uint8_t *h_digests, uint64_t *n_stored);

/* Batched get (get_batch, cascade_core.cpp:1220-1235) into device
 * buffers: h_out_ptrs[i] (device address) of h_out_caps[i] bytes.
 * h_sizes[i] = stored size (also when it did not fit), h_found[i] = 1 when
 * the key is stored.  Synchronous. */
int cascade_store_get_batch(cascade_store_t *s, size_t n,
                            const uint8_t *h_keys, const uint64_t *h_out_ptrs,
                            const uint64_t *h_out_caps, uint64_t *h_sizes,
                            uint8_t *h_found, void *stream,
                            uint64_t *n_found);

/* KVCacheStore.store (inference_benchmark/kv_manager.py:116-127) for n
 * keyed KV caches of one shape (descriptors and src_dtype as
 * cascade_kv_serialize_batch), when every wire block fits the HBM pool as a
 * raw payload: each cache is serialised straight into its pool slot, with
 * the statuses, dedup and counters of cascade_store_put_batch.  A block
 * whose slot cannot be allocated (size-class rounding) is serialised into
 * a staging buffer and placed in the next tier, as put_batch places it.
 * Returns CASCADE_ERR_UNSUPPORTED, storing nothing, when the store has no
 * HBM tier, keeps INT8 payloads in HBM, or lacks room for the batch: the
 * caller then serialises and uses cascade_store_put_batch.  Synchronous. */
int cascade_store_put_kv_batch(cascade_store_t *s, size_t n,
                               const uint8_t *h_keys, uint32_t layers,
                               uint32_t heads, uint32_t seq, uint32_t head_dim,
                               const cascade_kv_tensor_t *d_src, int src_dtype,
                               const uint8_t *h_prefix, uint8_t *h_status,
                               void *stream, uint64_t *n_stored);

/* KVCacheStore.load (inference_benchmark/kv_manager.py:135-156) for n keys
 * whose blocks are kv_manager wire blocks of one shape: get_batch and
 * deserialize_kv_cache in one call, into the caller's 2 x layers FP16
 * tensors per key (d_dst, as cascade_kv_deserialize_batch).  Raw blocks in
 * HBM are split straight out of the pool, one pass over their bytes; DRAM
 * or INT8 blocks are decoded into a staging buffer first (and promoted as
 * get_batch promotes).  h_found[i] = 1 when key i holds a block of exactly
 * cascade_kv_wire_bytes(); a block of another size is left alone and
 * counts neither hit nor miss.  The split is ordered on `stream`; the
 * lookup is synchronous. */
int cascade_store_get_kv_batch(cascade_store_t *s, size_t n,
                               const uint8_t *h_keys, uint32_t layers,
                               uint32_t heads, uint32_t seq, uint32_t head_dim,
                               const cascade_kv_tensor_t *d_dst,
                               uint8_t *h_found, void *stream,
                               uint64_t *n_found);

/* ------------------------------------------------------------------ */
/* Sharded dedup across the GPUs of one box (one rank per GPU).         */
/* The reference keeps one replicated dedup set per node, synchronised  */
/* by MPI_Allgatherv (DistributedStore::put / sync_metadata,            */
/* distributed_backend.cpp:583-590, 1269-1324).  Here each key has one   */
/* owner rank (the top bits of digest byte 0) and a batch is four calls */
/* around two all-to-all exchanges the caller runs (NCCL):               */
/*   begin:   hash and store every block speculatively in this rank's   */
/*            HBM pool;                                                  */
/*   records: once the hash is done, one 64-byte record per block into  */
/*            the owner rank's segment of d_send;                        */
/*   resolve: as owner, decide each received record (the first put of a */
/*            new key in (rank, block) order stores; later ones and keys */
/*            already stored are dedup hits) and write 8-byte replies;   */
/*   end:     take the replies for this rank's blocks (in any order),    */
/*            free the slots of duplicates and report per-block status.  */
/* The exchange buffers are padded: world segments of cap entries each  */
/* (segment r goes to / comes from rank r), cap the same on every rank   */
/* and at least every rank's batch size plus its relocation records     */
/* (cascade_shard_put_prepare), so both all-to-alls have equal splits   */
/* and no rank needs the others' counts; a caller learns cap (one small */
/* all-gather) while the hash runs, between begin and records.  Entries */
/* that carry nothing are all 0xff bytes.  begin, records and resolve   */
/* do not wait for the device: their outputs are ready on `stream` when */
/* they return (the caller's exchange must be ordered after `stream`).  */
/* end is synchronous.  A rank must not run other operations on the     */
/* store between begin and end.  Blocks are content-addressed; HBM must */
/* hold the whole batch (cascade_shard_put_prepare makes room with a    */
/* DRAM tier). */
#define CASCADE_SHARD_RECORD_BYTES 64
#define CASCADE_SHARD_REPLY_BYTES 8

/* Before a put with a DRAM tier: makes room in this rank's HBM pool for a
 * batch of n blocks of h_sizes bytes by demoting its least recently used
 * payloads to its DRAM tier (prefix blocks last; GPUBackend::evict_for_space,
 * gpu_backend.cu:467-487, as called from CascadeStore::put,
 * cascade_core.cpp:1100-1103), and sets *n_moves to the relocation records
 * the next records call adds to d_send: one per demoted payload whose key
 * another rank owns, so that the owner's entry follows it.  Records that a
 * failed put never sent stay pending and count here too; when begin fails
 * after prepare, a records call still sends them (the batch carries no
 * blocks).  Without a DRAM tier it does nothing (*n_moves = 0). */
int cascade_shard_put_prepare(cascade_store_t *s, size_t n,
                              const uint64_t *h_sizes, int world, int rank,
                              uint64_t *n_moves);
int cascade_shard_put_begin(cascade_store_t *s, size_t n,
                            const uint64_t *h_ptrs, const uint64_t *h_sizes,
                            const uint8_t *h_prefix, int world, int rank,
                            void *stream);
/* begin for blocks in host memory (the sharded form of
 * cascade_store_put_batch_host): the blocks are copied to this rank's GPU
 * first.  Pinned blocks of one size at a constant pitch are copied in
 * stripes and hashed as each stripe lands. */
int cascade_shard_put_begin_host(cascade_store_t *s, size_t n,
                                 const uint8_t *const *h_blocks,
                                 const uint64_t *h_sizes,
                                 const uint8_t *h_prefix, int world, int rank,
                                 void *stream);
/* begin for blocks whose SHA-256 digests the caller already computed on
 * this GPU (d_digests: n x 32 bytes, 4-byte aligned, e.g. from
 * cascade_sha256_batch; ready on `stream`).  A batch larger than the HBM
 * pool is put in slices (cascade_shard_put_slices); hashing the whole batch
 * in one launch first runs all its chains at once, where slices hashed one
 * by one would each run only theirs.  The payload kernels then have the
 * whole GPU. */
int cascade_shard_put_begin_digests(cascade_store_t *s, size_t n,
                                    const uint64_t *h_ptrs,
                                    const uint64_t *h_sizes,
                                    const uint8_t *h_prefix,
                                    const uint8_t *d_digests, int world,
                                    int rank, void *stream);
/* How to cut a batch of n blocks of h_sizes bytes into sharded puts that
 * each fit this rank's HBM pool: consecutive blocks whose payloads fill at
 * most 4/5 of the pool form a slice, and each slice's prepare demotes older
 * payloads to the DRAM tier.  A batch that fits the pool's free space, or
 * any batch without a DRAM tier, is one slice.  h_cuts gets *n_slices + 1 ascending block indices from 0 to n (room for
 * max(n, 1) + 1).  Every slice is a collective put of its own: ranks that
 * have fewer slices put empty batches while the others finish. */
int cascade_shard_put_slices(cascade_store_t *s, size_t n,
                             const uint64_t *h_sizes, uint64_t *h_cuts,
                             uint64_t *n_slices);
/* d_send: world * cap records (16-byte aligned). */
int cascade_shard_put_records(cascade_store_t *s, size_t cap, uint8_t *d_send,
                              void *stream);
/* m = world * cap received records; d_reply: m replies. */
int cascade_shard_resolve(cascade_store_t *s, const uint8_t *d_recv,
                          size_t m, uint8_t *d_reply, void *stream);
/* d_back: the m = world * cap replies received; n: this rank's batch. */
int cascade_shard_put_end(cascade_store_t *s, const uint8_t *d_back,
                          size_t m, size_t n, uint8_t *h_status,
                          uint8_t *h_digests, uint64_t *n_stored,
                          void *stream);

/* Sharded get: any rank reads any block of the sharded store.  The
 * reference reads a block another node holds through DistributedStore::get
 * (distributed_backend.cpp:673-767: local tiers, then the global location
 * table and a read of the holder's DRAM shadow).
 * Here the payload never leaves the holder's HBM pool until it is read:
 * every rank maps the other ranks' pools once (CUDA IPC, peer access over
 * NVLink), and a get is three calls around two all-to-all exchanges, with
 * padded buffers as for a put (world segments of cap entries):
 *   get_begin: route each 16-byte key to its owner: one 32-byte query per
 *              key in the owner's segment of d_send;
 *   lookup:    as owner, look the received keys up in this rank's slice of
 *              the index (touching their LRU epochs) and write one 48-byte
 *              location per query (found, holder rank, offset, size, INT8
 *              header);
 *   get_end:   take the locations of this rank's keys (in any order) and
 *              copy or dequantise each block from its holder's pool (this
 *              GPU's own or a peer's) into h_out_ptrs[i]; sizes, found
 *              flags and gpu_hits / misses as in cascade_store_get_batch.
 * get_begin and lookup do not wait for the device; get_end is synchronous.
 * cascade_shard_attach_pools must have run on every rank first.  As for a
 * put, a rank must not run other operations on the store between get_begin
 * and get_end.  A block its holder demoted is read from the holder's DRAM
 * tier (a shared-memory arena every rank maps; the reference reads the
 * holder's DRAM shadow, distributed_backend.cpp:720-767); sharded reads do
 * not promote. */
#define CASCADE_SHARD_QUERY_BYTES 32
#define CASCADE_SHARD_LOCATION_BYTES 48
#define CASCADE_IPC_HANDLE_BYTES 64
#define CASCADE_SHARD_DRAM_NAME_BYTES 64

/* This store's HBM pool as a CUDA IPC handle (64 bytes). */
int cascade_shard_pool_handle(cascade_store_t *s, uint8_t *h_handle);
/* This store's DRAM tier as a named shared-memory arena: a 64-byte record
 * (name, and chunk size in bytes 56..63; all zero without a DRAM tier).
 * The first call shares the arena, so it must come before the first put. */
int cascade_shard_dram_name(cascade_store_t *s, uint8_t *h_record);
/* Maps the pools of the other ranks: h_handles holds world handles, one per
 * rank in rank order (this rank's own is not opened), and h_dram_names
 * (or NULL) the world records of cascade_shard_dram_name.  Mappings are
 * closed by cascade_shard_detach_pools or when the store is destroyed.  A
 * rank must not free its store while another rank can still read its pool:
 * have every rank detach, then synchronise the ranks, then destroy. */
int cascade_shard_attach_pools(cascade_store_t *s, int world, int rank,
                               const uint8_t *h_handles,
                               const uint8_t *h_dram_names);
int cascade_shard_detach_pools(cascade_store_t *s);
/* d_send: world * cap queries. */
int cascade_shard_get_begin(cascade_store_t *s, size_t n,
                            const uint8_t *h_keys, size_t cap,
                            uint8_t *d_send, void *stream);
/* m = world * cap received queries; d_reply: m locations. */
int cascade_shard_lookup(cascade_store_t *s, const uint8_t *d_recv, size_t m,
                         uint8_t *d_reply, void *stream);
/* d_back: the m = world * cap locations received; n: this rank's keys. */
int cascade_shard_get_end(cascade_store_t *s, const uint8_t *d_back,
                          size_t m, size_t n, const uint64_t *h_out_ptrs,
                          const uint64_t *h_out_caps, uint64_t *h_sizes,
                          uint8_t *h_found, uint64_t *n_found, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CASCADE_B200_H */
