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
// that is part of the library's device image instead.
//
// Placement.  CUDA loads a library's device code onto a GPU lazily (the
// default since CUDA 12.2): the 512 KiB array is placed on a GPU the first
// time this file's set-up runs there, not when the library is loaded.  The
// set-up is the first call on each GPU, and a call with n = 0 does only the
// set-up, so a caller that is about to reserve HBM makes one n = 0 call per
// GPU first.  The array then stays on that GPU until the process exits.
// The set-up is redone automatically when the GPU's context changes (after
// a cudaDeviceReset), since the old address is gone with the old context.
//
// Sharing.  Every call on a GPU uses the same array, so two calls whose
// work overlaps on that GPU (different streams, or threads enqueueing at
// the same time) corrupt each other's results: serialise them on one
// stream.  Each call first resets the pairs it uses, so leftovers from an
// earlier call do not matter.
#include <cuda.h>

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
struct Scratch {
  int2 *addr = nullptr;
  unsigned long long ctx_id = 0;  // context the address belongs to
};
Scratch g_noalloc[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

// Unique id of the calling thread's current context (0 if unknown).  The
// driver entry points are fetched through the runtime, so the library does
// not link libcuda itself.
unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000,
                                         cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000,
                                         cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx &&
      get_id(ctx, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

// The set-up: the device address of the scratch array on `dev`, looked up
// with that device current.  Host code cannot use the array's name as a
// device pointer (it names a host-side stand-in), so kernels get the
// address found here.  The lookup also makes CUDA place the array on the
// GPU if this module was not loaded there yet.
int noalloc_scratch(int dev, int2 **out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  Scratch &sc = g_noalloc[dev];
  if (!sc.addr || sc.ctx_id == 0 || sc.ctx_id != current_ctx_id()) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_minmax);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    sc.addr = static_cast<int2 *>(p);
    sc.ctx_id = current_ctx_id();  // the lookup made a context current
  }
  *out = sc.addr;
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
  if (n > cb::kNoAllocMaxBlocks) {
    cb::set_error("cascade_kv_compress_batch_noalloc: " + std::to_string(n) +
                  " blocks requested; this entry point handles at most 65536 "
                  "blocks per call (use cascade_kv_compress_batch, or split "
                  "the batch)");
    return CASCADE_ERR_INVALID;
  }
  CB_CHECK(n == 0 || (d_src && d_sizes && d_dst), CASCADE_ERR_INVALID,
           "null pointer argument");
  int dev = 0;
  CB_CUDA(cudaGetDevice(&dev));
  CB_CHECK(dev >= 0 && dev < cb::kMaxDevices, CASCADE_ERR_INVALID,
           "device ordinal out of range");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int sdev = dev;
  CB_CUDA(cudaStreamGetDevice(s, &sdev));
  CB_CHECK(sdev == dev, CASCADE_ERR_INVALID,
           "cascade_kv_compress_batch_noalloc: the stream belongs to another "
           "device than the current one");
  int2 *mnmx = nullptr;
  int rc = cb::noalloc_scratch(dev, &mnmx);
  if (rc || n == 0) return rc;  // n == 0: the set-up alone
  // launch_minmax's first kernel resets the n pairs before they are used.
  rc = cb::launch_minmax(d_src, d_sizes, (int)n, max_size, mnmx, s);
  if (rc) return rc;
  return cb::launch_quantize(d_src, d_sizes, (int)n, max_size, mnmx, d_dst,
                             nullptr, 1, s);
}
