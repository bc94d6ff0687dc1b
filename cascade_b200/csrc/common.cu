// Error reporting, small utility kernels and the device diagnostics behind
// the C-ABI.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.cuh"
#include "sha256.cuh"

namespace cb {

namespace {
thread_local std::string g_error;
std::atomic<uint64_t> g_launches{0};

__global__ void offset_ptrs_kernel(const uint64_t *in, uint64_t delta,
                                   uint64_t *out, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = in[i] + delta;
}

// Chunks compressed back to back from registers only: the integer-pipe
// ceiling of the SHA-256 round function with every warp slot occupied.
__global__ void __launch_bounds__(256)
    sha_peak_kernel(uint32_t chunks, uint32_t *sink) {
  uint32_t st[8];
  sha::init(st);
  uint32_t w[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) w[j] = threadIdx.x * 16u + j + blockIdx.x;
  for (uint32_t c = 0; c < chunks; ++c) {
    sha::compress(st, w);
    w[0] ^= st[0];  // keep the chunks dependent on one another
  }
  uint32_t x = st[0] ^ st[1] ^ st[2] ^ st[3] ^ st[4] ^ st[5] ^ st[6] ^ st[7];
  if (x == 0x9e3779b9u) sink[0] = x;  // never true in practice; defeats DCE
}
}  // namespace

void count_launches(int k) { g_launches.fetch_add((uint64_t)k); }

int sm_count() {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cached[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    dev = 0;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) !=
          cudaSuccess || v <= 0)
    v = 1;  // the launch that follows reports the device error
  cached[dev].store(v, std::memory_order_relaxed);
  return v;
}

void set_error(const std::string &msg) { g_error = msg; }
void clear_error() { g_error.clear(); }
const char *last_error() { return g_error.c_str(); }

int cuda_fail(cudaError_t e, const char *what) {
  g_error = std::string(what) + ": " + cudaGetErrorString(e);
  return CASCADE_ERR_CUDA;
}

int launch_offset_ptrs(const uint64_t *d_in, uint64_t delta, uint64_t *d_out,
                       int n, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  offset_ptrs_kernel<<<(n + 255) / 256, 256, 0, s>>>(d_in, delta, d_out, n);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

}  // namespace cb

extern "C" const char *cascade_last_error(void) { return cb::last_error(); }

extern "C" int cascade_abi_version(void) { return CASCADE_ABI_VERSION; }

extern "C" uint64_t cascade_diag_launch_count(void) {
  return cb::g_launches.load();
}

extern "C" int cascade_diag_sha_peak(int device, uint32_t chunks_per_thread,
                                     double *gbps, double *ms) {
  cb::clear_error();
  CB_CHECK(gbps && ms && chunks_per_thread > 0, CASCADE_ERR_INVALID,
           "bad argument");
  CB_CUDA(cudaSetDevice(device));
  const int threads = 256, blocks = cb::sm_count() * 8;  // 64 warps per SM
  uint32_t *sink = nullptr;
  CB_CUDA(cudaMalloc(&sink, sizeof(uint32_t)));
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cb::sha_peak_kernel<<<blocks, threads>>>(8, sink);  // warm-up
  cudaEventRecord(a);
  cb::sha_peak_kernel<<<blocks, threads>>>(chunks_per_thread, sink);
  cudaEventRecord(b);
  cudaError_t e = cudaEventSynchronize(b);
  float t = 0.f;
  cudaEventElapsedTime(&t, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaFree(sink);
  if (e != cudaSuccess) return cb::cuda_fail(e, "sha_peak_kernel");
  const double bytes = 64.0 * chunks_per_thread * (double)threads * blocks;
  *ms = t;
  *gbps = bytes / (t * 1e-3) / 1e9;
  return CASCADE_OK;
}
