// Batched KV compression kernels: int16 min/max, INT8 quantise, dequantise,
// and the batched block copy used by the raw-format pool.
//
// All four are HBM-bound streaming kernels: 16-byte vector loads, 8- or
// 16-byte vector stores, grid-stride over (block, tile) work items with the
// grid a multiple of the SM count.  Arithmetic per element matches
// KVCompressor (cascade_core.cpp:818-872) bit for bit; see kvq8.cuh.
#include <algorithm>
#include <atomic>
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

// ------------------------------------------------ single-pass compression
//
// One HBM read of each block and one write of its codes.  A cluster of C
// CTAs owns one block at a time and each CTA one C-th of it (its slice).
// The clusters walk the batch persistently: block j + 1 of a cluster is
// reduced (int16 min/max, HBM read, lines kept in L2) in the same loop
// that quantises block j from the same slice, which the reduction read one
// step earlier and which is still in L2, so the HBM reads, the L2 reads
// and the code stores are in flight together.  Between the two the
// cluster exchanges its per-CTA (min, max) pairs through distributed
// shared memory, as remote stores that complete an mbarrier in the
// receiving CTA (no cluster-wide barrier and no memory fence per block, so
// a block's outstanding code stores never hold up the exchange).  The L2
// holds two blocks per active cluster, which bounds the block sizes and
// cluster sizes this form takes (the launcher checks it).

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// ------------------------------------------------------------ mbarriers
constexpr uint32_t kWaitLimit = 1u << 26;            // polls before giving up

// Bounded waits that gave up (a peer's pair that never came):
// the kernel carries on without the data, so that no CTA of a cluster is
// left waiting, and counts the event here.
__device__ unsigned int g_pair_wait_timeouts;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *m) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_addr(m)));
}

__device__ __forceinline__ void mbar_expect(uint64_t *m, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
      :: "r"(smem_addr(m)), "r"(bytes) : "memory");
}

// Waits (at most kWaitLimit polls) for the phase of parity `ph` of a
// barrier that peers complete with remote stores: acquire at cluster scope.
__device__ __forceinline__ void mbar_wait_cluster(uint64_t *m, uint32_t ph) {
  uint32_t done = 0;
  for (uint32_t i = 0; i < kWaitLimit && !done; ++i) {
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done) : "r"(smem_addr(m)), "r"(ph) : "memory");
  }
  if (!done && threadIdx.x == 0) atomicAdd(&g_pair_wait_timeouts, 1u);
}

// Stores (a, b) at `slot` and completes 8 bytes of `bar`, both as mapped
// into the shared memory of CTA `rank` of this cluster (no fence: the
// receiver's barrier phase makes the data visible).
__device__ __forceinline__ void st_async_pair(const int2 *slot,
                                              const uint64_t *bar,
                                              uint32_t rank, int a, int b) {
  uint32_t dst, rb;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(dst) : "r"(smem_addr(slot)), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(rb) : "r"(smem_addr(bar)), "r"(rank));
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.s32 "
      "[%0], {%1, %2}, [%3];"
      :: "r"(dst), "r"(a), "r"(b), "r"(rb) : "memory");
}

// The first read keeps its lines in L2 for the second (evict_last); the
// second read and the code stores let theirs go first.
__device__ __forceinline__ uint64_t l2_policy_keep() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_drop() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ld_hint(const uint4 *p, uint64_t pol) {
  uint4 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ void st_hint(uint2 *p, uint2 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v2.u32 [%0], {%1, %2}, %3;"
               :: "l"(p), "r"(v.x), "r"(v.y), "l"(pol) : "memory");
}

// The element range [e0, e1) of a block of `nelem` int16 values that CTA
// `rank` of `csize` handles: whole groups of 8, the remainder to the last.
__device__ __forceinline__ void slice_of(uint64_t nelem, uint32_t rank,
                                         uint32_t csize, uint64_t *e0,
                                         uint64_t *e1) {
  const uint64_t groups = nelem >> 3;
  *e0 = (groups * rank / csize) << 3;
  *e1 = rank + 1 == csize ? nelem : (groups * (rank + 1) / csize) << 3;
}

__device__ __forceinline__ void minmax16(uint4 r, uint32_t &pmin,
                                         uint32_t &pmax) {
  pmin = __vmins2(pmin, __vmins2(__vmins2(r.x, r.y), __vmins2(r.z, r.w)));
  pmax = __vmaxs2(pmax, __vmaxs2(__vmaxs2(r.x, r.y), __vmaxs2(r.z, r.w)));
}

struct FusedArgs {
  const uint64_t *ptrs;
  const uint64_t *sizes;
  const uint64_t *dsts;
  uint8_t *headers;
  int n;
  int header_inline;
};

template <int T>
struct FusedSmem {
  uint64_t pmbar[2];   // the peers' pairs have landed, by block parity
  int2 pairs[2][16];   // exchange arrays, by block parity; [rank]
  int wmin[T / 32], wmax[T / 32];
};

// Thread-local int16 min/max of elements [e0, e1) of src (HBM read; the
// lines are kept in L2 for the second read when HINT).  U loads per thread
// are in flight at a time.
template <int T, bool HINT, int U = 1>
__device__ __forceinline__ void minmax_range(const uint8_t *src, uint64_t e0,
                                             uint64_t e1, int &lo, int &hi) {
  uint64_t tail = e0;
  if (((uintptr_t)src & 15u) == 0 && e1 > e0) {
    const uint4 *q = reinterpret_cast<const uint4 *>(src);
    uint32_t pmin = 0x7fff7fffu, pmax = 0x80008000u;
    const uint64_t pol = HINT ? l2_policy_keep() : 0;
    const uint64_t v1 = e1 >> 3;
    uint64_t v = (e0 >> 3) + threadIdx.x;
#pragma unroll 1
    for (; v + (U - 1) * T < v1; v += U * T) {
      const uint4 *qv = q + v;
      uint4 r[U];
#pragma unroll
      for (int k = 0; k < U; ++k)
        r[k] = HINT ? ld_hint(qv + k * T, pol) : ld_stream(qv + k * T);
#pragma unroll
      for (int k = 0; k < U; ++k) minmax16(r[k], pmin, pmax);
    }
    for (; v < v1; v += T)
      minmax16(HINT ? ld_hint(q + v, pol) : ld_stream(q + v), pmin, pmax);
    lo = min(lo, min((int)(int16_t)(pmin & 0xffffu), (int)(int16_t)(pmin >> 16)));
    hi = max(hi, max((int)(int16_t)(pmax & 0xffffu), (int)(int16_t)(pmax >> 16)));
    tail = v1 << 3;
  }
  for (uint64_t e = tail + threadIdx.x; e < e1; e += T) {
    const int x = ld_i16_bytes(src + 2 * e);
    lo = min(lo, x);
    hi = max(hi, x);
  }
}

// Codes of elements [e0, e1) of src into codes (the second read, from L2
// when HINT).  U loads per thread are in flight at a time.
template <int T, bool HINT, int U = 1>
__device__ __forceinline__ void quantize_range(const uint8_t *src,
                                               uint8_t *codes, uint64_t e0,
                                               uint64_t e1,
                                               const q8::Params &p) {
  uint64_t tail = e0;
  if (((uintptr_t)src & 15u) == 0 && ((uintptr_t)codes & 7u) == 0 && e1 > e0) {
    const uint4 *q = reinterpret_cast<const uint4 *>(src);
    uint2 *o = reinterpret_cast<uint2 *>(codes);
    const uint64_t pol = HINT ? l2_policy_drop() : 0;
    const uint64_t v1 = e1 >> 3;
    uint64_t v = (e0 >> 3) + threadIdx.x;
#pragma unroll 1
    for (; v + (U - 1) * T < v1; v += U * T) {
      const uint4 *qv = q + v;
      uint2 *ov = o + v;
      uint4 r[U];
#pragma unroll
      for (int k = 0; k < U; ++k)
        r[k] = HINT ? ld_hint(qv + k * T, pol) : ld_stream(qv + k * T);
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const uint2 c = q8::codes8(r[k], p);
        if (HINT) st_hint(ov + k * T, c, pol); else ov[k * T] = c;
      }
    }
    for (; v < v1; v += T) {
      const uint2 c = q8::codes8(HINT ? ld_hint(q + v, pol) : ld_stream(q + v), p);
      if (HINT) st_hint(o + v, c, pol); else o[v] = c;
    }
    tail = v1 << 3;
  }
  for (uint64_t e = tail + threadIdx.x; e < e1; e += T)
    codes[e] = (uint8_t)q8::code(ld_i16_bytes(src + 2 * e), p);
}

template <int T>
__device__ __forceinline__ int2 cta_reduce_pair(int lo, int hi,
                                                FusedSmem<T> &sm) {
  lo = __reduce_min_sync(0xffffffffu, lo);
  hi = __reduce_max_sync(0xffffffffu, hi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sm.wmin[warp] = lo; sm.wmax[warp] = hi; }
  __syncthreads();
  lo = lane < T / 32 ? sm.wmin[lane] : INT_MAX;
  hi = lane < T / 32 ? sm.wmax[lane] : INT_MIN;
  lo = __reduce_min_sync(0xffffffffu, lo);
  hi = __reduce_max_sync(0xffffffffu, hi);
  __syncthreads();  // wmin/wmax are reused by the next reduction
  return make_int2(lo, hi);
}

// One step of a cluster: quantise this CTA's slice of block bq (params p;
// bq < 0: none) while reducing its slice of block br (br < 0: none), in one
// loop when both are aligned, so the HBM reads of br, the L2 reads of bq
// and the code stores are in flight together.  Returns the CTA's (min, max)
// of br's slice.
template <int T, int U, bool HINT>
__device__ __forceinline__ int2 fused_step(const FusedArgs &a, int bq,
                                           const q8::Params &p, int br,
                                           uint32_t rank, uint32_t csize,
                                           FusedSmem<T> &sm) {
  int lo = INT_MAX, hi = INT_MIN;
  uint64_t qe0 = 0, qe1 = 0, re0 = 0, re1 = 0;
  const uint8_t *qs = nullptr, *rs = nullptr;
  uint8_t *qc = nullptr;
  if (bq >= 0) {
    slice_of(a.sizes[bq] >> 1, rank, csize, &qe0, &qe1);
    qs = reinterpret_cast<const uint8_t *>(a.ptrs[bq]);
    uint8_t *dst = reinterpret_cast<uint8_t *>(a.dsts[bq]);
    qc = a.header_inline ? dst + 8 : dst;
  }
  if (br >= 0) {
    slice_of(a.sizes[br] >> 1, rank, csize, &re0, &re1);
    rs = reinterpret_cast<const uint8_t *>(a.ptrs[br]);
  }
  if (bq >= 0 && br >= 0 && ((uintptr_t)qs & 15u) == 0 &&
      ((uintptr_t)qc & 7u) == 0 && ((uintptr_t)rs & 15u) == 0) {
    const uint4 *qq = reinterpret_cast<const uint4 *>(qs);
    const uint4 *rq = reinterpret_cast<const uint4 *>(rs);
    uint2 *o = reinterpret_cast<uint2 *>(qc);
    const uint64_t qv1 = qe1 >> 3, rv1 = re1 >> 3;
    uint64_t qv = (qe0 >> 3) + threadIdx.x, rv = (re0 >> 3) + threadIdx.x;
    uint32_t pmin = 0x7fff7fffu, pmax = 0x80008000u;
    const uint64_t keep = HINT ? l2_policy_keep() : 0;
    const uint64_t drop = HINT ? l2_policy_drop() : 0;
#pragma unroll 1
    for (; qv + (U - 1) * T < qv1 && rv + (U - 1) * T < rv1;
         qv += U * T, rv += U * T) {
      uint4 x[U], y[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        x[k] = HINT ? ld_hint(rq + rv + k * T, keep) : ld_stream(rq + rv + k * T);
        y[k] = HINT ? ld_hint(qq + qv + k * T, drop) : ld_stream(qq + qv + k * T);
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        minmax16(x[k], pmin, pmax);
        const uint2 c = q8::codes8(y[k], p);
        if (HINT) st_hint(o + qv + k * T, c, drop); else o[qv + k * T] = c;
      }
    }
    for (; rv < rv1; rv += T)
      minmax16(HINT ? ld_hint(rq + rv, keep) : ld_stream(rq + rv), pmin, pmax);
    for (; qv < qv1; qv += T) {
      const uint2 c = q8::codes8(HINT ? ld_hint(qq + qv, drop) : ld_stream(qq + qv), p);
      if (HINT) st_hint(o + qv, c, drop); else o[qv] = c;
    }
    lo = min((int)(int16_t)(pmin & 0xffffu), (int)(int16_t)(pmin >> 16));
    hi = max((int)(int16_t)(pmax & 0xffffu), (int)(int16_t)(pmax >> 16));
    minmax_range<T, false>(rs, re1 & ~7ull, re1, lo, hi);   // ragged ends
    quantize_range<T, false>(qs, qc, qe1 & ~7ull, qe1, p);
  } else {
    if (br >= 0) minmax_range<T, HINT>(rs, re0, re1, lo, hi);
    if (bq >= 0) quantize_range<T, HINT>(qs, qc, qe0, qe1, p);
  }
  return cta_reduce_pair<T>(lo, hi, sm);
}

// Blocks cid, cid + ncl, ... of the batch, LA = 1 or 2 blocks of
// look-ahead: in step j the CTA quantises block j and reduces block j + LA.
// The pairs of block j travel as remote stores that complete the
// receiver's pmbar[j & 1] (armed for C x 8 bytes before they can arrive),
// as in compress_staged_kernel; with LA = 2 the pair of block j + 1 is sent
// before step j, so its exchange completes under a whole step.
template <int T, int U, int LA, bool HINT>
__global__ void __launch_bounds__(T, 1) compress_fused_kernel(FusedArgs a) {
  static_assert(LA == 1 || LA == 2, "look-ahead of one or two blocks");
  __shared__ FusedSmem<T> sm;
  const uint32_t rank = cluster_rank(), csize = cluster_size();
  const int cid = (int)cluster_id(), ncl = (int)cluster_count();
  const int J = a.n > cid ? (a.n - cid + ncl - 1) / ncl : 0;
  auto block = [&](int j) { return j < J ? cid + j * ncl : -1; };
  if (threadIdx.x == 0) {
    mbar_init(&sm.pmbar[0]);
    mbar_init(&sm.pmbar[1]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (J > 0) mbar_expect(&sm.pmbar[0], csize * 8);
    if (J > 1) mbar_expect(&sm.pmbar[1], csize * 8);
  }
  __syncthreads();
  cluster_arrive();  // every CTA's barriers exist before any remote store
  cluster_wait();
  if (J == 0) return;
  auto send = [&](int j, int2 m) {
    if (threadIdx.x < csize)
      st_async_pair(&sm.pairs[j & 1][rank], &sm.pmbar[j & 1], threadIdx.x,
                    m.x, m.y);
  };
  const q8::Params none{};
  int2 held = fused_step<T, U, HINT>(a, -1, none, block(0), rank, csize, sm);
  send(0, held);
  if (LA == 2)
    held = fused_step<T, U, HINT>(a, -1, none, block(1), rank, csize, sm);
#pragma unroll 1
  for (int j = 0; j < J; ++j) {
    mbar_wait_cluster(&sm.pmbar[j & 1], (j >> 1) & 1);
    int lo = INT_MAX, hi = INT_MIN;
    for (uint32_t q = 0; q < csize; ++q) {
      const int2 v = sm.pairs[j & 1][q];
      lo = min(lo, v.x);
      hi = max(hi, v.y);
    }
    if (threadIdx.x == 0 && j + 2 < J) mbar_expect(&sm.pmbar[j & 1], csize * 8);
    __syncthreads();  // pairs read and the barrier re-armed before any send
    const int b = block(j);
    const q8::Params p = q8::params_from_minmax(lo, hi, (a.sizes[b] >> 1) == 0);
    if (rank == 0 && threadIdx.x == 0) {
      uint8_t *dst = reinterpret_cast<uint8_t *>(a.dsts[b]);
      write_header(a.header_inline ? dst : a.headers + 8 * (size_t)b, p);
    }
    if (LA == 2 && j + 1 < J) send(j + 1, held);
    held = fused_step<T, U, HINT>(a, b, p, block(j + LA), rank, csize, sm);
    if (LA == 1 && j + 1 < J) send(j + 1, held);
  }
  // No CTA leaves while a peer may still address its shared memory.
  cluster_arrive();
  cluster_wait();
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

// Launch configuration of the single-pass kernel with csize CTAs per
// cluster.
template <int T, int U, int LA, bool HINT>
cudaLaunchConfig_t fused_config(int csize, cudaStream_t s,
                                cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(T);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Clusters of csize CTAs the device keeps resident (cached per device and
// cluster size).
template <int T, int U, int LA, bool HINT>
int fused_active_clusters(int csize, int *active_out) {
  auto kernel = compress_fused_kernel<T, U, LA, HINT>;
  constexpr int kMaxDev = 64, kMaxCluster = 16;
  static std::atomic<int> cache[kMaxDev][kMaxCluster + 1];
  int dev = 0;
  CB_CUDA(cudaGetDevice(&dev));
  CB_CHECK(csize >= 1 && csize <= kMaxCluster, CASCADE_ERR_INVALID,
           "cluster size out of range");
  int active = dev < kMaxDev ? cache[dev][csize].load() : 0;
  if (active <= 0) {
    if (csize > 8)
      CB_CUDA(cudaFuncSetAttribute(
          kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = fused_config<T, U, LA, HINT>(csize, nullptr, attr);
    cfg.gridDim = dim3(csize * sm_count());
    CB_CUDA(cudaOccupancyMaxActiveClusters(&active, kernel, &cfg));
    CB_CHECK(active > 0, CASCADE_ERR_UNSUPPORTED,
             "no cluster of this size fits on the device");
    if (dev < kMaxDev) cache[dev][csize].store(active);
  }
  *active_out = active;
  return CASCADE_OK;
}

template <int T, int U, int LA, bool HINT>
int launch_fused_form(const FusedArgs &a, int csize, cudaStream_t s,
                      int *active_out) {
  int active = 0;
  int rc = fused_active_clusters<T, U, LA, HINT>(csize, &active);
  if (rc) return rc;
  if (active_out) *active_out = active;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = fused_config<T, U, LA, HINT>(csize, s, attr);
  cfg.gridDim = dim3(std::min(active, a.n) * csize);
  CB_CUDA(cudaLaunchKernelEx(&cfg, compress_fused_kernel<T, U, LA, HINT>, a));
  count_launches(1);
  return CASCADE_OK;
}

// The single-pass form that the batch sizes call for.  The L2 holds two
// blocks per active cluster (the one being quantised and the one being
// reduced); the cluster is the smallest whose blocks in flight fit 72 MiB.
// Measured on 4096 x 2 MiB and 1024 x 1 MiB: 8 and 4 CTAs per cluster, 3.03
// and 0.37 ms against 3.50 and 0.43 ms for min/max + quantise.  Smaller
// blocks gain nothing over the two kernels (and larger ones need clusters
// of 16, which only 7 of fit on the device, and lose), so they get
// CASCADE_ERR_UNSUPPORTED.
constexpr uint64_t kFusedL2Budget = 72ull << 20;
constexpr int kFusedThreads = 1024;
constexpr int kFusedUnroll = 4;
constexpr int kFusedLookahead = 1;

int launch_compress_fused(const uint64_t *d_ptrs, const uint64_t *d_sizes,
                          int n, uint64_t max_size, const uint64_t *d_dsts,
                          uint8_t *d_headers, int header_inline,
                          cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  if (max_size < (1ull << 20) || max_size > (2ull << 20) + 4096)
    return CASCADE_ERR_UNSUPPORTED;
  FusedArgs a{d_ptrs, d_sizes, d_dsts, d_headers, n, header_inline};
  auto launch = [&](int cs, int *active) {
    return launch_fused_form<kFusedThreads, kFusedUnroll, kFusedLookahead,
                             true>(a, cs, s, active);
  };
  for (int cs = 1; cs <= 8; cs *= 2) {
    int active = 0;
    int rc = fused_active_clusters<kFusedThreads, kFusedUnroll,
                                   kFusedLookahead, true>(cs, &active);
    if (rc) return rc;
    if ((uint64_t)active * (kFusedLookahead + 1) * max_size <= kFusedL2Budget)
      return launch(cs, nullptr);
  }
  return CASCADE_ERR_UNSUPPORTED;
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
  // One HBM pass when the blocks are small enough to stay in L2 between
  // the reduction and the quantise (the common KV block sizes); otherwise
  // the two-pass form with its per-block scratch.
  int rc0 = cb::launch_compress_fused(d_src, d_sizes, (int)n, max_size, d_dst,
                                      nullptr, 1, s);
  if (rc0 != CASCADE_ERR_UNSUPPORTED) return rc0;
  cb::clear_error();
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
