// Launchers shared between the library's translation units.  Every pointer
// is a device pointer; descriptor arrays hold device addresses as uint64.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cascade_b200.h"

namespace cb {

// Unused shared memory (bytes per CTA) that a kernel running beside a
// SHA-256 launch requests so that it cannot share an SM with the hash
// chains: when a launch of one CTA per SM leaves SMs idle, the SHA-256 CTAs
// fill their SMs' shared memory to within less than this.
constexpr size_t kHashNeighbourSmem = 16 * 1024;

// kHashNeighbourSmem when a SHA-256 launch over n blocks fills its SMs (one
// CTA per SM, at least 16 SMs spare), else 0: what a kernel launched beside
// that hash should request.
size_t sha256_neighbour_smem(int n);

int launch_sha256(const uint64_t *d_ptrs, const uint64_t *d_sizes, int n,
                  uint8_t *d_digests, cudaStream_t s);

// Chunks [c_begin, c_end) of each block (64-byte chunks of the padded
// message).  Blocks that end in the range get their digest; blocks that go
// on get their running state in d_state (8 words per block), from which a
// call starting at c_end resumes.  d_state may be null when c_begin == 0
// and c_end covers every block.
int launch_sha256_range(const uint64_t *d_ptrs, const uint64_t *d_sizes,
                        int n, uint8_t *d_digests, uint32_t *d_state,
                        uint64_t c_begin, uint64_t c_end, cudaStream_t s);

// smem_pad (bytes of unused dynamic shared memory per CTA) keeps the
// payload kernels off SMs whose shared memory a concurrent SHA-256 launch
// has filled; see launch_sha256_range.
int launch_minmax(const uint64_t *d_ptrs, const uint64_t *d_sizes, int n,
                  uint64_t max_size, int2 *d_mnmx, cudaStream_t s,
                  size_t smem_pad = 0);

// header_inline=1: the reference layout (8-byte header, then codes) at
// d_dsts[b]; header_inline=0: codes at d_dsts[b], header at d_headers+8*b.
int launch_quantize(const uint64_t *d_ptrs, const uint64_t *d_sizes, int n,
                    uint64_t max_size, const int2 *d_mnmx,
                    const uint64_t *d_dsts, uint8_t *d_headers,
                    int header_inline, cudaStream_t s, size_t smem_pad = 0);

// Single-pass compression (min/max and codes in one HBM read, clusters of
// CTAs exchanging their partial min/max through distributed shared memory).
// Returns CASCADE_ERR_UNSUPPORTED, launching nothing, when max_size is too
// large for the blocks in flight to stay in L2; the caller then uses
// launch_minmax + launch_quantize.
int launch_compress_fused(const uint64_t *d_ptrs, const uint64_t *d_sizes,
                          int n, uint64_t max_size, const uint64_t *d_dsts,
                          uint8_t *d_headers, int header_inline,
                          cudaStream_t s);

int launch_dequantize(const uint64_t *d_srcs, const uint8_t *d_headers,
                      int header_inline, const uint64_t *d_out_sizes, int n,
                      uint64_t max_out_size, const uint64_t *d_dsts,
                      cudaStream_t s);

int launch_copy(const uint64_t *d_srcs, const uint64_t *d_dsts,
                const uint64_t *d_sizes, int n, uint64_t max_size,
                cudaStream_t s, size_t smem_pad = 0);

// n caches' K/V tensors (2 x layers descriptors each) into kv_manager wire
// blocks d_dst[i] (null: skipped) (cascade_kv_serialize_batch).
int launch_kv_serialize(const cascade_kv_tensor_t *d_src, int src_dtype,
                        uint32_t layers, uint32_t heads, uint32_t seq,
                        uint32_t head_dim, const uint64_t *d_dst, int n,
                        cudaStream_t s);

// kv_manager wire blocks d_src[i] (null: skipped) into 2 x layers FP16
// tensors each (cascade_kv_deserialize_batch).
int launch_kv_deserialize(const uint64_t *d_src, uint32_t layers,
                          uint32_t heads, uint32_t seq, uint32_t head_dim,
                          const cascade_kv_tensor_t *d_dst, int n,
                          cudaStream_t s);

// out[i] = in[i] + delta
int launch_offset_ptrs(const uint64_t *d_in, uint64_t delta, uint64_t *d_out,
                       int n, cudaStream_t s);

}  // namespace cb
