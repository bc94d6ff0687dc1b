// Test-only harness around the UNMODIFIED reference sources (cascade_core.cpp,
// gpu_backend.cu of Cascade-HPC/Cascade), compiled by oracle/Makefile into
// oracle/_ref/libcascade_ref.so.  It exists so the tests can ask the reference
// itself for digests, INT8 codes and dedup counts, and so bench.py can time
// the reference's CPU put path.  Nothing in the product links or loads it.
//
// Every entry point is a plain C function so Python can reach it via ctypes.
#include "cascade.hpp"

#include <cstdint>
#include <cstring>
#ifdef _OPENMP
#include <omp.h>
#endif
#include <memory>
#include <string>
#include <vector>

namespace {

cascade::CascadeConfig cpu_only_config(const char *shm_path, size_t shm_bytes,
                                       int kv_compression, int dedup_enabled) {
  cascade::CascadeConfig cfg;
  cfg.use_gpu = false;              // the reference's "login node store"
  cfg.gpu_capacity_bytes = 0;
  cfg.shm_capacity_bytes = shm_bytes;
  cfg.shm_path = shm_path;
  cfg.lustre_path = "";             // no cold tier: no files written
  cfg.prefetch_enabled = false;     // the prefetch workers would zero 1 GiB
  cfg.kv_compression = kv_compression != 0;
  cfg.dedup_enabled = dedup_enabled != 0;
  return cfg;
}

}  // namespace

extern "C" {

// cascade_core.cpp:43-53: first 16 digest bytes as 32 lowercase hex chars.
void ref_compute_block_id(const uint8_t *data, size_t size, char *out_hex33) {
  std::string id = cascade::compute_block_id(data, size);
  std::memcpy(out_hex33, id.c_str(), 33);
}

// cascade_core.cpp:818-849.  Writes 8 + size/2 bytes; returns that count, or
// 0 when `cap` is too small.  Padding bytes 5..7 of the header are whatever
// the reference's stack struct held; a caller must not compare them.
size_t ref_kv_compress(const uint8_t *data, size_t size, uint8_t *out,
                       size_t cap) {
  cascade::CompressionMeta meta;
  std::memset(&meta, 0, sizeof(meta));
  std::vector<uint8_t> c = cascade::KVCompressor::compress(data, size, meta);
  if (c.size() > cap) return 0;
  std::memcpy(out, c.data(), c.size());
  return c.size();
}

// cascade_core.cpp:851-872, called the way CascadeStore::get calls it
// (cascade_core.cpp:1149-1156): meta read from the first 8 bytes.
int ref_kv_decompress(const uint8_t *comp, size_t comp_size, uint8_t *out,
                      size_t orig_size) {
  cascade::CompressionMeta meta;
  std::memcpy(&meta, comp, sizeof(meta));
  return cascade::KVCompressor::decompress(comp, comp_size, meta, out,
                                           orig_size)
             ? 1
             : 0;
}

size_t ref_compressed_size(size_t original) {
  return cascade::KVCompressor::compressed_size(original);
}

// A CPU-only reference CascadeStore (use_gpu=false) for semantic checks.
void *ref_store_create(const char *shm_path, size_t shm_bytes,
                       int kv_compression, int dedup_enabled) {
  auto cfg = cpu_only_config(shm_path, shm_bytes, kv_compression,
                             dedup_enabled);
  return new cascade::CascadeStore(cfg);
}

// The reference CascadeStore with its GPU tier on device 0 (GPUBackend:
// cudaMalloc'd pool, copies only, no kernels), to pin the store model's
// demotion counters.
void *ref_store_create_gpu(const char *shm_path, size_t shm_bytes,
                           size_t gpu_bytes, int kv_compression,
                           int dedup_enabled, int semantic_eviction) {
  auto cfg = cpu_only_config(shm_path, shm_bytes, kv_compression,
                             dedup_enabled);
  cfg.use_gpu = true;
  cfg.gpu_capacity_bytes = gpu_bytes;
  cfg.gpu_device_id = 0;
  cfg.semantic_eviction = semantic_eviction != 0;
  return new cascade::CascadeStore(cfg);
}

void ref_store_destroy(void *s) {
  delete static_cast<cascade::CascadeStore *>(s);
}

int ref_store_put(void *s, const char *id, const uint8_t *data, size_t size,
                  int is_prefix) {
  return static_cast<cascade::CascadeStore *>(s)->put(id, data, size,
                                                      is_prefix != 0)
             ? 1
             : 0;
}

int ref_store_get(void *s, const char *id, uint8_t *out, size_t *out_size) {
  return static_cast<cascade::CascadeStore *>(s)->get(id, out, out_size) ? 1
                                                                         : 0;
}

int ref_store_contains(void *s, const char *id) {
  return static_cast<cascade::CascadeStore *>(s)->contains(id) ? 1 : 0;
}

// Stats in declaration order of CascadeStore::Stats (cascade.hpp:439-456).
void ref_store_stats(void *s, uint64_t out[15]) {
  auto st = static_cast<cascade::CascadeStore *>(s)->get_stats();
  const size_t v[15] = {st.gpu_used,          st.shm_used,
                        st.gpu_hits,          st.shm_hits,
                        st.lustre_hits,       st.misses,
                        st.dedup_hits,        st.gpu_evictions,
                        st.shm_evictions,     st.promotions_to_gpu,
                        st.promotions_to_shm, st.prefetch_completed,
                        st.compression_savings_bytes, st.shm_puts,
                        st.lustre_puts};
  for (int i = 0; i < 15; ++i) out[i] = v[i];
}

// The reference's own multi-core PUT: CascadeStore::put_batch
// (cascade_core.cpp:1203-1218, OpenMP) with content-addressed ids.
size_t ref_store_put_batch(void *s, const uint8_t *const *blocks,
                           const size_t *sizes, size_t n,
                           const char *ids_hex33) {
  std::vector<cascade::BlockId> ids(n);
  std::vector<const uint8_t *> ptrs(blocks, blocks + n);
  std::vector<size_t> sz(sizes, sizes + n);
  for (size_t i = 0; i < n; ++i) ids[i] = std::string(ids_hex33 + 33 * i, 32);
  return static_cast<cascade::CascadeStore *>(s)->put_batch(ids, ptrs, sz);
}

// The whole reference CPU ingest path for a batch, on `nthreads` OpenMP
// threads: compute_block_id per block (cascade_core.cpp:43-53), then the
// reference's own put_batch (cascade_core.cpp:1203-1218), which runs
// KVCompressor::compress and ShmBackend::put per block when the store was
// created with kv_compression=1.  Returns the number of successful puts.
size_t ref_cpu_put_path(void *s, const uint8_t *const *blocks,
                        const size_t *sizes, size_t n, int nthreads) {
#ifdef _OPENMP
  omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  std::vector<cascade::BlockId> ids(n);
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic)
#endif
  for (long i = 0; i < static_cast<long>(n); ++i)
    ids[i] = cascade::compute_block_id(blocks[i], sizes[i]);
  std::vector<const uint8_t *> ptrs(blocks, blocks + n);
  std::vector<size_t> sz(sizes, sizes + n);
  return static_cast<cascade::CascadeStore *>(s)->put_batch(ids, ptrs, sz);
}

void ref_store_clear(void *s) {
  static_cast<cascade::CascadeStore *>(s)->clear();
}

int ref_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
