// Shared definitions for the cascade_b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "cascade_b200.h"

namespace cb {

// Thread-local last-error text behind cascade_last_error().
void set_error(const std::string &msg);
void clear_error();
const char *last_error();

// Kernel launches made by this library since load (cascade_diag_launch_count).
void count_launches(int k);

// Records `what` + the CUDA error text and returns CASCADE_ERR_CUDA.
int cuda_fail(cudaError_t e, const char *what);

#define CB_CUDA(call)                                                         \
  do {                                                                        \
    cudaError_t _e = (call);                                                  \
    if (_e != cudaSuccess) return ::cb::cuda_fail(_e, #call);                 \
  } while (0)

#define CB_CHECK(cond, code, msg)                                             \
  do {                                                                        \
    if (!(cond)) {                                                            \
      ::cb::set_error(msg);                                                   \
      return (code);                                                          \
    }                                                                         \
  } while (0)

// Streaming multiprocessors of the current device (148 on a B200), read
// from the device once per device and cached.
int sm_count();

// Grid size for a grid-stride kernel: a multiple of the SM count.
inline int grid_for(uint64_t work_items, int per_block, int blocks_per_sm) {
  uint64_t want = (work_items + per_block - 1) / per_block;
  uint64_t cap = (uint64_t)sm_count() * blocks_per_sm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return (int)want;
}

__host__ __device__ inline uint64_t div_up(uint64_t a, uint64_t b) {
  return (a + b - 1) / b;
}

}  // namespace cb
