// cascade_kv_compress_batch_noalloc: KV INT8 compression that allocates no
// memory of its own.
//
// cascade_kv_compress_batch needs a little scratch (one int16 min/max pair
// per block) and takes it from the stream-ordered allocator.  Some callers
// cannot allow that: an inference engine that has reserved almost all of
// HBM for its own KV-cache pool at start-up has no room left to hand out,
// or must account for every byte it gives away; and a latency-critical
// ingest loop cannot afford an allocator call that may synchronise or fail
// part-way through a step.  This variant keeps its scratch in a fixed array
// that is part of the library image on each GPU instead.
//
// The scratch array (kNoAllocMaxBlocks pairs, 512 KiB) exists once per GPU
// that loads this library and stays there until the process exits.  Every
// call on a GPU uses the same array, so two calls whose work overlaps on
// that GPU (different streams, or threads enqueueing at the same time)
// corrupt each other's results: serialise them on one stream.  Each call
// first resets the pairs it uses, so leftovers from an earlier call do not
// matter.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace cb {

namespace {

constexpr size_t kNoAllocMaxBlocks = 65536;

// One (min, max) int16 pair per block of a call, widened to int32.
static __device__ __align__(256) int2 g_noalloc_minmax[kNoAllocMaxBlocks];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
int2 *g_noalloc_addr[kMaxDevices] = {};

// The device address of the scratch array on `dev`, looked up once per
// device with that device current.  Host code cannot use the array's name
// as a device pointer (it names a host-side stand-in), so kernels get the
// address found here.
int noalloc_scratch(int dev, int2 **out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_minmax);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    g_noalloc_addr[dev] = static_cast<int2 *>(p);
  }
  *out = g_noalloc_addr[dev];
  return CASCADE_OK;
}

}  // namespace

}  // namespace cb

extern "C" int cascade_kv_compress_batch_noalloc(const uint64_t *d_src,
                                                 const uint64_t *d_sizes,
                                                 const uint64_t *d_dst,
                                                 size_t n, uint64_t max_size,
                                                 void *stream) {
  cb::clear_error();
  if (n == 0) return CASCADE_OK;
  if (n > cb::kNoAllocMaxBlocks) {
    cb::set_error("cascade_kv_compress_batch_noalloc: " + std::to_string(n) +
                  " blocks requested; this entry point handles at most 65536 "
                  "blocks per call (use cascade_kv_compress_batch, or split "
                  "the batch)");
    return CASCADE_ERR_INVALID;
  }
  CB_CHECK(d_src && d_sizes && d_dst, CASCADE_ERR_INVALID,
           "null pointer argument");
  int dev = 0;
  CB_CUDA(cudaGetDevice(&dev));
  CB_CHECK(dev >= 0 && dev < cb::kMaxDevices, CASCADE_ERR_INVALID,
           "device ordinal out of range");
  int2 *mnmx = nullptr;
  int rc = cb::noalloc_scratch(dev, &mnmx);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // launch_minmax's first kernel resets the n pairs before they are used.
  rc = cb::launch_minmax(d_src, d_sizes, (int)n, max_size, mnmx, s);
  if (rc) return rc;
  return cb::launch_quantize(d_src, d_sizes, (int)n, max_size, mnmx, d_dst,
                             nullptr, 1, s);
}
