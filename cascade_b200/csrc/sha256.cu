// Batched SHA-256 over device-resident blocks (one serial chain per block).
//
// Replaces the per-block OpenSSL call of compute_block_id
// (cascade_core.cpp:43-53) with one launch over a whole batch.  A lane owns
// one block; 32 blocks share a warp, and CTAs are sized so the warps spread
// over all 148 SMs before any SM gets a second warp (a chain is bound by its
// own warp's issue rate, so spreading beats packing).
#include "common.cuh"
#include "sha256.cuh"

namespace cb {

namespace {

__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ldg_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Full chunks of a 16-byte aligned block, with the next chunk's loads issued
// before the current chunk's rounds.
__device__ __forceinline__ void chunks_aligned16(uint32_t st[8],
                                                 const uint4 *q,
                                                 uint64_t nfull) {
  if (nfull == 0) return;
  uint4 n0 = ldg_stream(q), n1 = ldg_stream(q + 1), n2 = ldg_stream(q + 2),
        n3 = ldg_stream(q + 3);
  for (uint64_t c = 0; c < nfull; ++c) {
    uint32_t w[16] = {sha::bswap(n0.x), sha::bswap(n0.y), sha::bswap(n0.z),
                      sha::bswap(n0.w), sha::bswap(n1.x), sha::bswap(n1.y),
                      sha::bswap(n1.z), sha::bswap(n1.w), sha::bswap(n2.x),
                      sha::bswap(n2.y), sha::bswap(n2.z), sha::bswap(n2.w),
                      sha::bswap(n3.x), sha::bswap(n3.y), sha::bswap(n3.z),
                      sha::bswap(n3.w)};
    if (c + 1 < nfull) {
      const uint4 *nq = q + 4 * (c + 1);
      n0 = ldg_stream(nq);
      n1 = ldg_stream(nq + 1);
      n2 = ldg_stream(nq + 2);
      n3 = ldg_stream(nq + 3);
    }
    sha::compress(st, w);
  }
}

// Full chunks of a block at any address: aligned 32-bit loads of the words
// that cover the chunk, then one byte permute per message word.  The
// covering words stay inside the 4-byte-aligned span of the block, so no
// load leaves the allocation's granule.
__device__ __forceinline__ void chunks_unaligned(uint32_t st[8],
                                                 const uint8_t *p,
                                                 uint64_t nfull) {
  const uint32_t o = (uint32_t)((uintptr_t)p & 3u);
  const uint32_t *base = (const uint32_t *)(p - o);
  // Selector picking bytes o..o+3 of the pair (x, y) in big-endian order.
  const uint32_t sel = (o << 12) | ((o + 1) << 8) | ((o + 2) << 4) | (o + 3);
  for (uint64_t c = 0; c < nfull; ++c) {
    const uint32_t *cw = base + 16 * c;
    uint32_t raw[17];
#pragma unroll
    for (int j = 0; j < 16; ++j) raw[j] = ldg_u32(cw + j);
    // The 17th word is needed only when the chunk is misaligned.
    raw[16] = o ? ldg_u32(cw + 16) : 0u;
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = __byte_perm(raw[j], raw[j + 1], sel);
    sha::compress(st, w);
  }
}

__global__ void __launch_bounds__(256)
    sha256_lane_per_block(const uint64_t *__restrict__ ptrs,
                          const uint64_t *__restrict__ sizes, int n,
                          uint32_t *__restrict__ digests) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t *p = reinterpret_cast<const uint8_t *>(ptrs[i]);
  const uint64_t len = sizes[i];
  const uint64_t nfull = len >> 6;
  uint32_t st[8];
  sha::init(st);
  if (((uintptr_t)p & 15u) == 0)
    chunks_aligned16(st, reinterpret_cast<const uint4 *>(p), nfull);
  else
    chunks_unaligned(st, p, nfull);
  sha::finish(st, p + (nfull << 6), (uint32_t)(len & 63u), len);
  uint32_t *out = digests + 8 * (size_t)i;
#pragma unroll
  for (int k = 0; k < 8; ++k) out[k] = sha::bswap(st[k]);  // digest byte order
}

}  // namespace

// Threads per CTA so that ceil(n/32) warps land on distinct SMs first.
static int sha_cta_threads(int n) {
  int warps = (n + 31) / 32;
  int per_cta = (warps + kSmCount - 1) / kSmCount;
  if (per_cta < 1) per_cta = 1;
  if (per_cta > 8) per_cta = 8;
  return 32 * per_cta;
}

int launch_sha256(const uint64_t *d_ptrs, const uint64_t *d_sizes, int n,
                  uint8_t *d_digests, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  int threads = sha_cta_threads(n);
  int blocks = (n + threads - 1) / threads;
  sha256_lane_per_block<<<blocks, threads, 0, s>>>(
      d_ptrs, d_sizes, n, reinterpret_cast<uint32_t *>(d_digests));
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

}  // namespace cb

extern "C" int cascade_sha256_batch(const uint64_t *d_ptrs,
                                    const uint64_t *d_sizes, size_t n,
                                    uint8_t *d_digests, void *stream) {
  cb::clear_error();
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  CB_CHECK(n == 0 || (d_ptrs && d_sizes && d_digests), CASCADE_ERR_INVALID,
           "null pointer argument");
  CB_CHECK(((uintptr_t)d_digests & 3u) == 0, CASCADE_ERR_INVALID,
           "digest buffer must be 4-byte aligned");
  return cb::launch_sha256(d_ptrs, d_sizes, (int)n, d_digests,
                           static_cast<cudaStream_t>(stream));
}
