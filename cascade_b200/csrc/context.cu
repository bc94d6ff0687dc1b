// Per-device scratch for the host-pointer convenience entry points
// (compute_block_id on a host buffer).  Batched device entry points never
// touch it.
#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace cb {

namespace {

struct DeviceCtx {
  std::mutex mu;
  bool ready = false;
  cudaStream_t stream = nullptr;
  uint8_t *d_buf = nullptr;
  size_t d_cap = 0;
  uint64_t *d_desc = nullptr;  // [ptr, size]
  uint8_t *d_digest = nullptr;
};

DeviceCtx g_ctx[64];

int ensure(DeviceCtx &c, size_t bytes) {
  if (!c.ready) {
    CB_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    CB_CUDA(cudaMalloc(&c.d_desc, 2 * sizeof(uint64_t)));
    CB_CUDA(cudaMalloc(&c.d_digest, 32));
    c.ready = true;
  }
  if (bytes > c.d_cap) {
    if (c.d_buf) CB_CUDA(cudaFree(c.d_buf));
    c.d_buf = nullptr;
    c.d_cap = 0;
    size_t cap = bytes < 4096 ? 4096 : bytes;
    CB_CUDA(cudaMalloc(&c.d_buf, cap));
    c.d_cap = cap;
  }
  return CASCADE_OK;
}

}  // namespace

}  // namespace cb

extern "C" int cascade_compute_block_id(const uint8_t *data, uint64_t size,
                                        char out_hex[33]) {
  cb::clear_error();
  CB_CHECK(out_hex && (data || size == 0), CASCADE_ERR_INVALID,
           "null pointer argument");
  int dev = 0, count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cb::set_error("no CUDA device: compute_block_id runs only on the GPU");
    return CASCADE_ERR_NODEVICE;
  }
  CB_CUDA(cudaGetDevice(&dev));
  CB_CHECK(dev >= 0 && dev < 64, CASCADE_ERR_INVALID, "device id out of range");
  cb::DeviceCtx &c = cb::g_ctx[dev];
  std::lock_guard<std::mutex> lock(c.mu);
  int rc = cb::ensure(c, size);
  if (rc) return rc;
  if (size) CB_CUDA(cudaMemcpyAsync(c.d_buf, data, size, cudaMemcpyHostToDevice,
                                    c.stream));
  uint64_t desc[2] = {(uint64_t)(uintptr_t)c.d_buf, size};
  CB_CUDA(cudaMemcpyAsync(c.d_desc, desc, sizeof(desc), cudaMemcpyHostToDevice,
                          c.stream));
  rc = cb::launch_sha256(c.d_desc, c.d_desc + 1, 1, c.d_digest, c.stream);
  if (rc) return rc;
  uint8_t dig[32];
  CB_CUDA(cudaMemcpyAsync(dig, c.d_digest, 32, cudaMemcpyDeviceToHost,
                          c.stream));
  CB_CUDA(cudaStreamSynchronize(c.stream));
  static const char hexd[] = "0123456789abcdef";
  for (int i = 0; i < 16; ++i) {
    out_hex[2 * i] = hexd[dig[i] >> 4];
    out_hex[2 * i + 1] = hexd[dig[i] & 15];
  }
  out_hex[32] = '\0';
  return CASCADE_OK;
}
