// Batched KV compression kernels: int16 min/max, INT8 quantise, dequantise,
// and the batched block copy used by the raw-format pool.
//
// All four are HBM-bound streaming kernels: 16-byte vector loads, 8- or
// 16-byte vector stores, grid-stride over (block, tile) work items with the
// grid a multiple of the SM count.  Arithmetic per element matches
// KVCompressor (cascade_core.cpp:818-872) bit for bit; see kvq8.cuh.
#include <algorithm>
#include <climits>

#include "common.cuh"
#include "kvq8.cuh"
#include "kernels.cuh"

namespace cb {

namespace {

constexpr int kThreads = 256;
constexpr int kVec = 8;                              // uint4 per thread
constexpr uint64_t kTileElems = kThreads * kVec * 8;  // 16384 int16 = 32 KiB

__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ int16_t ld_i16_bytes(const uint8_t *p) {
  return (int16_t)((uint16_t)p[0] | ((uint16_t)p[1] << 8));
}

__global__ void init_minmax_kernel(int2 *mnmx, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) mnmx[i] = make_int2(INT_MAX, INT_MIN);
}

__global__ void __launch_bounds__(kThreads)
    minmax_kernel(const uint64_t *__restrict__ ptrs,
                  const uint64_t *__restrict__ sizes, int n, int tiles,
                  int2 *__restrict__ mnmx) {
  __shared__ int smin[kThreads / 32], smax[kThreads / 32];
  const uint64_t items = (uint64_t)n * tiles;
  for (uint64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int b = (int)(w / tiles);
    const uint64_t t = w - (uint64_t)b * tiles;
    const uint64_t nelem = sizes[b] >> 1;
    const uint64_t e0 = t * kTileElems;
    if (e0 >= nelem) continue;  // uniform across the CTA
    const uint64_t e1 = min(e0 + kTileElems, nelem);
    const uint8_t *src = reinterpret_cast<const uint8_t *>(ptrs[b]);
    int lo = INT_MAX, hi = INT_MIN;
    if (((uintptr_t)src & 15u) == 0) {
      const uint64_t v0 = e0 >> 3, v1 = e1 >> 3;  // whole uint4 groups
      const uint4 *q = reinterpret_cast<const uint4 *>(src);
      uint32_t pmin = 0x7fff7fffu, pmax = 0x80008000u;
      uint64_t v = v0 + threadIdx.x;
#pragma unroll 1
      for (; v + (kVec - 1) * kThreads < v1; v += kVec * kThreads) {
        uint4 r[kVec];
#pragma unroll
        for (int k = 0; k < kVec; ++k) r[k] = ld_stream(q + v + k * kThreads);
#pragma unroll
        for (int k = 0; k < kVec; ++k) {
          pmin = __vmins2(pmin, __vmins2(__vmins2(r[k].x, r[k].y),
                                         __vmins2(r[k].z, r[k].w)));
          pmax = __vmaxs2(pmax, __vmaxs2(__vmaxs2(r[k].x, r[k].y),
                                         __vmaxs2(r[k].z, r[k].w)));
        }
      }
      for (; v < v1; v += kThreads) {
        uint4 r = ld_stream(q + v);
        pmin = __vmins2(pmin, __vmins2(__vmins2(r.x, r.y), __vmins2(r.z, r.w)));
        pmax = __vmaxs2(pmax, __vmaxs2(__vmaxs2(r.x, r.y), __vmaxs2(r.z, r.w)));
      }
      lo = min((int)(int16_t)(pmin & 0xffffu), (int)(int16_t)(pmin >> 16));
      hi = max((int)(int16_t)(pmax & 0xffffu), (int)(int16_t)(pmax >> 16));
      // Elements after the last whole group.
      for (uint64_t e = (v1 << 3) + threadIdx.x; e < e1; e += kThreads) {
        int x = ld_i16_bytes(src + 2 * e);
        lo = min(lo, x);
        hi = max(hi, x);
      }
    } else {
      for (uint64_t e = e0 + threadIdx.x; e < e1; e += kThreads) {
        int x = ld_i16_bytes(src + 2 * e);
        lo = min(lo, x);
        hi = max(hi, x);
      }
    }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { smin[warp] = lo; smax[warp] = hi; }
    __syncthreads();
    if (threadIdx.x < 32) {
      int a = threadIdx.x < kThreads / 32 ? smin[threadIdx.x] : INT_MAX;
      int c = threadIdx.x < kThreads / 32 ? smax[threadIdx.x] : INT_MIN;
      a = __reduce_min_sync(0xffffffffu, a);
      c = __reduce_max_sync(0xffffffffu, c);
      if (threadIdx.x == 0) {
        atomicMin(&mnmx[b].x, a);
        atomicMax(&mnmx[b].y, c);
      }
    }
    __syncthreads();
  }
}

__device__ __forceinline__ void write_header(uint8_t *h, const q8::Params &p) {
  uint32_t s = __float_as_uint(p.scale);
  h[0] = s & 0xff; h[1] = (s >> 8) & 0xff; h[2] = (s >> 16) & 0xff;
  h[3] = s >> 24;
  h[4] = (uint8_t)p.zp;
  h[5] = h[6] = h[7] = 0;
}

__global__ void __launch_bounds__(kThreads)
    quantize_kernel(const uint64_t *__restrict__ ptrs,
                    const uint64_t *__restrict__ sizes, int n, int tiles,
                    const int2 *__restrict__ mnmx,
                    const uint64_t *__restrict__ dsts,
                    uint8_t *__restrict__ headers, int header_inline) {
  const uint64_t items = (uint64_t)n * tiles;
  for (uint64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int b = (int)(w / tiles);
    const uint64_t t = w - (uint64_t)b * tiles;
    const uint64_t nelem = sizes[b] >> 1;
    const int2 m = mnmx[b];
    const q8::Params p = q8::params_from_minmax(m.x, m.y, nelem == 0);
    uint8_t *dst = reinterpret_cast<uint8_t *>(dsts[b]);
    uint8_t *codes = header_inline ? dst + 8 : dst;
    if (t == 0 && threadIdx.x == 0)
      write_header(header_inline ? dst : headers + 8 * (size_t)b, p);
    const uint64_t e0 = t * kTileElems;
    if (e0 >= nelem) continue;
    const uint64_t e1 = min(e0 + kTileElems, nelem);
    const uint8_t *src = reinterpret_cast<const uint8_t *>(ptrs[b]);
    uint64_t tail_from = e0;
    if (((uintptr_t)src & 15u) == 0 && ((uintptr_t)codes & 7u) == 0) {
      const uint64_t v0 = e0 >> 3, v1 = e1 >> 3;
      const uint4 *q = reinterpret_cast<const uint4 *>(src);
      uint2 *o = reinterpret_cast<uint2 *>(codes);
      uint64_t v = v0 + threadIdx.x;
#pragma unroll 1
      for (; v + (kVec - 1) * kThreads < v1; v += kVec * kThreads) {
        uint4 r[kVec];
#pragma unroll
        for (int k = 0; k < kVec; ++k) r[k] = ld_stream(q + v + k * kThreads);
#pragma unroll
        for (int k = 0; k < kVec; ++k) o[v + k * kThreads] = q8::codes8(r[k], p);
      }
      for (; v < v1; v += kThreads) o[v] = q8::codes8(ld_stream(q + v), p);
      tail_from = v1 << 3;
    }
    for (uint64_t e = tail_from + threadIdx.x; e < e1; e += kThreads)
      codes[e] = (uint8_t)q8::code(ld_i16_bytes(src + 2 * e), p);
  }
}

// src_codes[b]: the codes; headers: header per block (8 bytes each) when
// header_inline is 0, otherwise the header sits in the 8 bytes before the
// codes.  out_sizes[b]: bytes to produce (2 per code).
__global__ void __launch_bounds__(kThreads, 8)
    dequantize_kernel(const uint64_t *__restrict__ srcs,
                      const uint8_t *__restrict__ headers, int header_inline,
                      const uint64_t *__restrict__ out_sizes, int n,
                      int tiles, const uint64_t *__restrict__ dsts) {
  const uint64_t items = (uint64_t)n * tiles;
  for (uint64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int b = (int)(w / tiles);
    const uint64_t t = w - (uint64_t)b * tiles;
    const uint64_t nelem = out_sizes[b] >> 1;
    const uint64_t e0 = t * kTileElems;
    if (e0 >= nelem) continue;
    const uint64_t e1 = min(e0 + kTileElems, nelem);
    const uint8_t *codes = reinterpret_cast<const uint8_t *>(srcs[b]);
    const uint8_t *h = header_inline ? codes - 8 : headers + 8 * (size_t)b;
    const uint32_t sbits = (uint32_t)h[0] | ((uint32_t)h[1] << 8) |
                           ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
    const q8::DeParams d = q8::deparams(sbits, (int8_t)h[4]);
    uint8_t *dst = reinterpret_cast<uint8_t *>(dsts[b]);
    uint64_t tail_from = e0;
    if (((uintptr_t)codes & 7u) == 0 && ((uintptr_t)dst & 15u) == 0) {
      const uint64_t v0 = e0 >> 3, v1 = e1 >> 3;
      const uint2 *q = reinterpret_cast<const uint2 *>(codes);
      uint4 *o = reinterpret_cast<uint4 *>(dst);
      uint64_t v = v0 + threadIdx.x;
#pragma unroll 1
      for (; v + (kVec - 1) * kThreads < v1; v += kVec * kThreads) {
        uint2 r[kVec];
#pragma unroll
        for (int k = 0; k < kVec; ++k) r[k] = __ldg(q + v + k * kThreads);
#pragma unroll
        for (int k = 0; k < kVec; ++k) o[v + k * kThreads] = q8::values8(r[k], d);
      }
      for (; v < v1; v += kThreads) o[v] = q8::values8(__ldg(q + v), d);
      tail_from = v1 << 3;
    }
    for (uint64_t e = tail_from + threadIdx.x; e < e1; e += kThreads) {
      uint32_t x = q8::value(codes[e], d);
      dst[2 * e] = x & 0xff;
      dst[2 * e + 1] = x >> 8;
    }
  }
}

constexpr uint64_t kCopyTile = kThreads * kVec * 16;  // 32 KiB

__global__ void __launch_bounds__(kThreads)
    copy_kernel(const uint64_t *__restrict__ srcs,
                const uint64_t *__restrict__ dsts,
                const uint64_t *__restrict__ sizes, int n, int tiles) {
  const uint64_t items = (uint64_t)n * tiles;
  for (uint64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int b = (int)(w / tiles);
    const uint64_t t = w - (uint64_t)b * tiles;
    const uint64_t size = sizes[b];
    const uint64_t b0 = t * kCopyTile;
    if (b0 >= size) continue;
    const uint64_t b1 = min(b0 + kCopyTile, size);
    const uint8_t *src = reinterpret_cast<const uint8_t *>(srcs[b]);
    uint8_t *dst = reinterpret_cast<uint8_t *>(dsts[b]);
    uint64_t tail_from = b0;
    if ((((uintptr_t)src | (uintptr_t)dst) & 15u) == 0) {
      const uint64_t v0 = b0 >> 4, v1 = b1 >> 4;
      const uint4 *q = reinterpret_cast<const uint4 *>(src);
      uint4 *o = reinterpret_cast<uint4 *>(dst);
      uint64_t v = v0 + threadIdx.x;
#pragma unroll 1
      for (; v + (kVec - 1) * kThreads < v1; v += kVec * kThreads) {
        uint4 r[kVec];
#pragma unroll
        for (int k = 0; k < kVec; ++k) r[k] = ld_stream(q + v + k * kThreads);
#pragma unroll
        for (int k = 0; k < kVec; ++k) o[v + k * kThreads] = r[k];
      }
      for (; v < v1; v += kThreads) o[v] = ld_stream(q + v);
      tail_from = v1 << 4;
    }
    for (uint64_t e = tail_from + threadIdx.x; e < b1; e += kThreads)
      dst[e] = src[e];
  }
}

}  // namespace

// ------------------------------------------------------------- launchers
int launch_minmax(const uint64_t *d_ptrs, const uint64_t *d_sizes, int n,
                  uint64_t max_size, int2 *d_mnmx, cudaStream_t s,
                  size_t smem_pad) {
  if (n <= 0) return CASCADE_OK;
  init_minmax_kernel<<<(n + 255) / 256, 256, 0, s>>>(d_mnmx, n);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  const int tiles = (int)std::max<uint64_t>(1, div_up(max_size / 2, kTileElems));
  const int grid = grid_for((uint64_t)n * tiles, 1, 4);
  minmax_kernel<<<grid, kThreads, smem_pad, s>>>(d_ptrs, d_sizes, n, tiles,
                                                 d_mnmx);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_quantize(const uint64_t *d_ptrs, const uint64_t *d_sizes, int n,
                    uint64_t max_size, const int2 *d_mnmx,
                    const uint64_t *d_dsts, uint8_t *d_headers,
                    int header_inline, cudaStream_t s, size_t smem_pad) {
  if (n <= 0) return CASCADE_OK;
  const int tiles = (int)std::max<uint64_t>(1, div_up(max_size / 2, kTileElems));
  const int grid = grid_for((uint64_t)n * tiles, 1, 4);
  quantize_kernel<<<grid, kThreads, smem_pad, s>>>(
      d_ptrs, d_sizes, n, tiles, d_mnmx, d_dsts, d_headers, header_inline);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_dequantize(const uint64_t *d_srcs, const uint8_t *d_headers,
                      int header_inline, const uint64_t *d_out_sizes, int n,
                      uint64_t max_out_size, const uint64_t *d_dsts,
                      cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  const int tiles =
      (int)std::max<uint64_t>(1, div_up(max_out_size / 2, kTileElems));
  // 8 CTAs per SM (2048 threads at 32 registers): more loads in flight for
  // this latency-bound stream (5.7 vs 5.5 TB/s at 4 per SM).
  const int grid = grid_for((uint64_t)n * tiles, 1, 8);
  dequantize_kernel<<<grid, kThreads, 0, s>>>(d_srcs, d_headers, header_inline,
                                              d_out_sizes, n, tiles, d_dsts);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_copy(const uint64_t *d_srcs, const uint64_t *d_dsts,
                const uint64_t *d_sizes, int n, uint64_t max_size,
                cudaStream_t s, size_t smem_pad) {
  if (n <= 0) return CASCADE_OK;
  const int tiles = (int)std::max<uint64_t>(1, div_up(max_size, kCopyTile));
  const int grid = grid_for((uint64_t)n * tiles, 1, 4);
  copy_kernel<<<grid, kThreads, smem_pad, s>>>(d_srcs, d_dsts, d_sizes, n,
                                               tiles);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

}  // namespace cb

// ------------------------------------------------------------------ C-ABI
extern "C" int cascade_kv_compress_batch(const uint64_t *d_src,
                                         const uint64_t *d_sizes,
                                         const uint64_t *d_dst, size_t n,
                                         uint64_t max_size, void *stream) {
  cb::clear_error();
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (n == 0) return CASCADE_OK;
  CB_CHECK(d_src && d_sizes && d_dst, CASCADE_ERR_INVALID,
           "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int2 *mnmx = nullptr;
  CB_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&mnmx), n * sizeof(int2),
                          s));
  int rc = cb::launch_minmax(d_src, d_sizes, (int)n, max_size, mnmx, s);
  if (rc == CASCADE_OK)
    rc = cb::launch_quantize(d_src, d_sizes, (int)n, max_size, mnmx, d_dst,
                             nullptr, 1, s);
  cudaError_t e = cudaFreeAsync(mnmx, s);
  if (rc == CASCADE_OK && e != cudaSuccess)
    return cb::cuda_fail(e, "cudaFreeAsync");
  return rc;
}

extern "C" int cascade_kv_decompress_batch(const uint64_t *d_src,
                                           const uint64_t *d_out_sizes,
                                           const uint64_t *d_dst, size_t n,
                                           uint64_t max_out_size,
                                           void *stream) {
  cb::clear_error();
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (n == 0) return CASCADE_OK;
  CB_CHECK(d_src && d_out_sizes && d_dst, CASCADE_ERR_INVALID,
           "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The reference format keeps the header inline: codes start 8 bytes in.
  uint64_t *codes = nullptr;
  CB_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&codes),
                          n * sizeof(uint64_t), s));
  int rc = cb::launch_offset_ptrs(d_src, 8, codes, (int)n, s);
  if (rc == CASCADE_OK)
    rc = cb::launch_dequantize(codes, nullptr, 1, d_out_sizes, (int)n,
                               max_out_size, d_dst, s);
  cudaError_t e = cudaFreeAsync(codes, s);
  if (rc == CASCADE_OK && e != cudaSuccess)
    return cb::cuda_fail(e, "cudaFreeAsync");
  return rc;
}

extern "C" int cascade_copy_batch(const uint64_t *d_src,
                                  const uint64_t *d_dst,
                                  const uint64_t *d_sizes, size_t n,
                                  uint64_t max_size, void *stream) {
  cb::clear_error();
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (n == 0) return CASCADE_OK;
  CB_CHECK(d_src && d_dst && d_sizes, CASCADE_ERR_INVALID,
           "null pointer argument");
  return cb::launch_copy(d_src, d_dst, d_sizes, (int)n, max_size,
                         static_cast<cudaStream_t>(stream));
}
