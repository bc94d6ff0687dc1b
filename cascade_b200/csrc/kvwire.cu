// The KV-cache wire format of kv_manager.serialize_kv_cache /
// deserialize_kv_cache (inference_benchmark/kv_manager.py:11-95), built and
// split on the device.
//
// A wire block is an 18-byte header struct.pack("<IIIIH", layers, kv_heads,
// seq_len, head_dim, 0) followed by, for each layer, the K tensor then the V
// tensor as contiguous [kv_heads][seq_len][head_dim] FP16 (dtype id 0: the
// reference always converts to float16, kv_manager.py:54-59).  The reference
// builds it with .cpu() + bytes joins and reads it back with numpy copies;
// here one launch serialises a batch of caches straight out of their
// (possibly strided) device tensors, and one launch splits a batch of wire
// blocks into per-layer device tensors, so a KV cache reaches the store
// without leaving HBM.
//
// Both kernels are HBM-bound streams: 2 x payload bytes per block.  The
// 18-byte header puts every payload byte 2 bytes off a 16-byte boundary, so
// each thread produces one ALIGNED 16-byte output vector from the matching
// 16-byte input unit and the neighbouring lane's edge word (warp shuffle,
// funnel shift by 16 bits): loads and stores both stay 16-byte vectors.
// Ragged shapes (head_dim not a multiple of 8, payloads that end inside a
// vector) and misaligned pointers take an element-wise path instead; no
// access ever leaves the tensors' and blocks' own bytes.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace cb {

namespace {

constexpr int kWThreads = 256;
constexpr int kWPer = 8;                          // vectors per thread per item
constexpr uint32_t kWTile = kWThreads * kWPer;    // 2048 vectors = 32 KiB
constexpr uint32_t kHeaderBytes = 18;

// n / d for n < 2^31 as one 64-bit multiply and shift: m = ceil(2^k / d),
// k = 32 + ceil(log2 d).  The error of m stays below d <= 2^(k-32), so
// floor(n m / 2^k) = floor(n / d) for every n < 2^32, and n m < 2^64.
struct FastDiv {
  uint64_t m;
  uint32_t k;
};

FastDiv make_div(uint32_t d) {
  FastDiv f;
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  f.k = 32 + l;
  f.m = (uint64_t)(((unsigned __int128)1 << f.k) + d - 1) / d;
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, FastDiv f) {
  return (uint32_t)(((uint64_t)n * f.m) >> f.k);
}

struct WireGeom {
  uint32_t L, H, S, D;
  uint32_t SD, E;     // elements per head, per tensor
  uint32_t N;         // payload elements per block (2 L E)
  uint32_t units;     // 8-element payload units per block, ceil(N / 8)
  uint32_t vecs;      // 16-byte vectors per wire block, ceil((18 + 2N) / 16)
  uint32_t tiles;     // work items per block
  FastDiv dE, dSD, dD;
  int vec_ok;         // D % 8 == 0: a unit never straddles two rows
};

struct Coord {
  uint32_t seg, h, s, d;
};

__device__ __forceinline__ Coord coord(uint32_t e, const WireGeom &g) {
  Coord c;
  c.seg = fdiv(e, g.dE);
  uint32_t r = e - c.seg * g.E;
  c.h = fdiv(r, g.dSD);
  r -= c.h * g.SD;
  c.s = fdiv(r, g.dD);
  c.d = r - c.s * g.D;
  return c;
}

__device__ __forceinline__ uint64_t elem_addr(const cascade_kv_tensor_t &t,
                                              const Coord &c, int es) {
  const int64_t idx = (int64_t)c.h * t.stride_head +
                      (int64_t)c.s * t.stride_seq + (int64_t)c.d;
  return t.ptr + (uint64_t)(idx * es);
}

// (lo >> 16) | (hi << 16): the 4 bytes that start 2 bytes into `lo`.
__device__ __forceinline__ uint32_t fs16(uint32_t lo, uint32_t hi) {
  return __funnelshift_r(lo, hi, 16);
}

__device__ __forceinline__ uint4 ld16_stream(uint64_t a) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(a));
  return v;
}

// Source element (SRC 0 = FP16, 1 = BF16, 2 = FP32) as FP16 bits.  The
// conversions round to nearest even, as torch's .to(torch.float16) does.
template <int SRC>
__device__ __forceinline__ uint32_t to_f16(uint32_t raw) {
  if (SRC == 0) return raw & 0xffffu;
  const float f = SRC == 1 ? __uint_as_float(raw << 16) : __uint_as_float(raw);
  return __half_as_ushort(__float2half_rn(f));
}

template <int SRC>
__device__ __forceinline__ uint32_t pack2(uint32_t a, uint32_t b) {
  return to_f16<SRC>(a) | (to_f16<SRC>(b) << 16);
}

template <int SRC>
__device__ __forceinline__ uint32_t load_raw(uint64_t a) {
  constexpr int es = SRC == 2 ? 4 : 2;
  if ((a & (es - 1)) == 0)
    return es == 4 ? *reinterpret_cast<const uint32_t *>(a)
                   : *reinterpret_cast<const uint16_t *>(a);
  const uint8_t *p = reinterpret_cast<const uint8_t *>(a);
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < es; ++i) r |= (uint32_t)p[i] << (8 * i);
  return r;
}

// Payload element e of this block's cache, as FP16 bits (0 past the end).
template <int SRC>
__device__ uint32_t load_elem(const cascade_kv_tensor_t *ts, uint32_t e,
                              const WireGeom &g) {
  if (e >= g.N) return 0;
  const Coord c = coord(e, g);
  const cascade_kv_tensor_t t = ts[c.seg];
  return to_f16<SRC>(load_raw<SRC>(elem_addr(t, c, SRC == 2 ? 4 : 2)));
}

// Address of payload element e, the first of a unit that lies inside one
// row (head_dim % 8 == 0 and e % 8 == 0).  A tensor laid out contiguously
// as [heads][seq][dim] needs one division; any other strides need three.
template <int ES>
__device__ __forceinline__ uint64_t unit_addr(const cascade_kv_tensor_t *ts,
                                              uint32_t e, const WireGeom &g) {
  const uint32_t seg = fdiv(e, g.dE);
  const uint32_t r = e - seg * g.E;
  const cascade_kv_tensor_t *t = ts + seg;
  const uint64_t ptr = __ldg(reinterpret_cast<const unsigned long long *>(&t->ptr));
  const int64_t sh = __ldg(reinterpret_cast<const long long *>(&t->stride_head));
  const int64_t ss = __ldg(reinterpret_cast<const long long *>(&t->stride_seq));
  if (ss == (int64_t)g.D && sh == (int64_t)g.SD) return ptr + (uint64_t)r * ES;
  const uint32_t h = fdiv(r, g.dSD);
  const uint32_t r2 = r - h * g.SD;
  const uint32_t s = fdiv(r2, g.dD);
  const uint32_t d = r2 - s * g.D;
  return ptr + (uint64_t)(((int64_t)h * sh + (int64_t)s * ss + (int64_t)d) * ES);
}

// Payload unit q (elements 8q .. 8q+7) as four words of FP16 pairs, from an
// address unit_addr gave (16-byte aligned).
template <int SRC>
__device__ __forceinline__ uint4 load_unit_at(uint64_t a) {
  if (SRC == 0) return ld16_stream(a);
  if (SRC == 1) {
    const uint4 r = ld16_stream(a);
    return make_uint4(pack2<1>(r.x, r.x >> 16), pack2<1>(r.y, r.y >> 16),
                      pack2<1>(r.z, r.z >> 16), pack2<1>(r.w, r.w >> 16));
  }
  const uint4 r0 = ld16_stream(a), r1 = ld16_stream(a + 16);
  return make_uint4(pack2<2>(r0.x, r0.y), pack2<2>(r0.z, r0.w),
                    pack2<2>(r1.x, r1.y), pack2<2>(r1.z, r1.w));
}

// Payload unit q element by element (0 past the end of the payload).
template <int SRC>
__device__ __noinline__ uint4 load_unit_slow(const cascade_kv_tensor_t *ts,
                                             uint32_t q, const WireGeom &g) {
  const uint32_t e = q * 8;
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = load_elem<SRC>(ts, e + 2 * j, g) |
           (load_elem<SRC>(ts, e + 2 * j + 1, g) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __noinline__ void store_bytes(uint8_t *p, uint4 v,
                                         uint32_t nbytes) {
  for (uint32_t i = 0; i < nbytes; ++i) {
    const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
    p[i] = (uint8_t)(w >> (8 * (i & 3)));
  }
}

// One work item = kWTile output vectors of one wire block; warp w of the
// CTA owns kWPer x 32 consecutive vectors, 32 per step.  Vector v = 0 is
// header bytes 0..15; vector v >= 1 is wire bytes 16v..16v+15 = the last 2
// bytes of payload unit v-2 (the header's dtype id for v = 1) and the first
// 14 of unit v-1.  A lane takes unit v-2's last word from the lane before
// it; lane 0 from lane 31 of the previous step, so only a warp's first
// vector loads it on its own.
template <int SRC>
__global__ void __launch_bounds__(kWThreads, 3)
    kv_serialize_kernel(const cascade_kv_tensor_t *__restrict__ src,
                        const uint64_t *__restrict__ dst, int n, WireGeom g) {
  constexpr int ES = SRC == 2 ? 4 : 2;
  const int lane = threadIdx.x & 31;
  const uint32_t wofs = (threadIdx.x >> 5) * (kWPer * 32);
  const uint64_t items = (uint64_t)n * g.tiles;
  const uint64_t wire = kHeaderBytes + 2ull * g.N;
  for (uint64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int b = (int)(w / g.tiles);
    const uint32_t wbase =
        (uint32_t)(w - (uint64_t)b * g.tiles) * kWTile + wofs;
    if (wbase >= g.vecs) continue;          // uniform across the warp
    const cascade_kv_tensor_t *ts = src + (uint64_t)b * 2 * g.L;
    uint8_t *out = reinterpret_cast<uint8_t *>(dst[b]);
    if (!out) continue;                     // a block this call skips
    const bool out_al = ((uintptr_t)out & 15u) == 0;
    uint64_t addr[kWPer];
#pragma unroll
    for (int k = 0; k < kWPer; ++k) {       // addresses, then loads
      const uint32_t q = wbase + k * 32 + lane - 1;   // unit of vector v
      addr[k] = 0;
      if (g.vec_ok && q < g.units && q * 8 + 8 <= g.N) {
        addr[k] = unit_addr<ES>(ts, q * 8, g);
        if (addr[k] & 15u) addr[k] = 0;
      }
    }
    uint4 cur[kWPer];
#pragma unroll
    for (int k = 0; k < kWPer; ++k) {
      const uint32_t q = wbase + k * 32 + lane - 1;
      cur[k] = make_uint4(0, 0, 0, 0);      // v = 0: unit -1 = the dtype id
      if (addr[k]) cur[k] = load_unit_at<SRC>(addr[k]);
      else if (q < g.units) cur[k] = load_unit_slow<SRC>(ts, q, g);
    }
    uint32_t carry = 0;                     // lane 0: word 3 of unit v-2
    if (lane == 0 && wbase >= 2 && wbase - 2 < g.units)
      carry = load_elem<SRC>(ts, (wbase - 2) * 8 + 6, g) |
              (load_elem<SRC>(ts, (wbase - 2) * 8 + 7, g) << 16);
#pragma unroll
    for (int k = 0; k < kWPer; ++k) {
      const uint32_t v = wbase + k * 32 + lane;
      const uint32_t up = __shfl_up_sync(0xffffffffu, cur[k].w, 1);
      const uint32_t last = __shfl_sync(0xffffffffu, cur[k].w, 31);
      const uint32_t prev = lane == 0 ? carry : up;
      carry = last;
      if (v >= g.vecs) continue;
      const uint4 o =
          v == 0 ? make_uint4(g.L, g.H, g.S, g.D)
                 : make_uint4(fs16(prev, cur[k].x), fs16(cur[k].x, cur[k].y),
                              fs16(cur[k].y, cur[k].z), fs16(cur[k].z, cur[k].w));
      const uint64_t off = (uint64_t)v * 16;
      if (out_al && off + 16 <= wire)
        *reinterpret_cast<uint4 *>(out + off) = o;
      else
        store_bytes(out + off, o, (uint32_t)(wire - off < 16 ? wire - off : 16));
    }
  }
}

// Element-wise store of payload unit q (its first `cnt` elements).
__device__ __noinline__ void store_unit_slow(const cascade_kv_tensor_t *ts,
                                             uint32_t e, uint32_t cnt,
                                             uint4 o, const WireGeom &g) {
  for (uint32_t j = 0; j < cnt; ++j) {
    const Coord cj = coord(e + j, g);
    const cascade_kv_tensor_t tj = ts[cj.seg];
    const uint64_t aj = elem_addr(tj, cj, 2);
    const uint32_t w = j < 2 ? o.x : j < 4 ? o.y : j < 6 ? o.z : o.w;
    const uint16_t h = (uint16_t)(w >> (16 * (j & 1)));
    if ((aj & 1u) == 0) {
      *reinterpret_cast<uint16_t *>(aj) = h;
    } else {
      reinterpret_cast<uint8_t *>(aj)[0] = (uint8_t)h;
      reinterpret_cast<uint8_t *>(aj)[1] = (uint8_t)(h >> 8);
    }
  }
}

// Payload unit q read byte by byte from a wire block (0 past the end).
__device__ __noinline__ uint4 wire_unit_slow(const uint8_t *in, uint32_t e,
                                             const WireGeom &g) {
  uint32_t wv[4] = {0, 0, 0, 0};
#pragma unroll
  for (uint32_t j = 0; j < 8; ++j) {
    if (e + j < g.N) {
      const uint8_t *p = in + kHeaderBytes + 2ull * (e + j);
      wv[j >> 1] |= ((uint32_t)p[0] | ((uint32_t)p[1] << 8)) << (16 * (j & 1));
    }
  }
  return make_uint4(wv[0], wv[1], wv[2], wv[3]);
}

// One work item = 256 x PER payload units of one wire block; warp w of the
// CTA owns PER x 32 consecutive units, 32 per step.  Unit q is wire bytes
// 18 + 16q .. 18 + 16q + 15 = bytes 2..15 of the block's 16-byte unit q+1
// and bytes 0..1 of unit q+2, which the next lane loaded (lane 31: lane 0
// of the next step; the warp's last unit loads it on its own).
template <int PER>
__global__ void __launch_bounds__(kWThreads, 3)
    kv_deserialize_kernel(const uint64_t *__restrict__ src,
                          const cascade_kv_tensor_t *__restrict__ dst, int n,
                          WireGeom g) {
  const int lane = threadIdx.x & 31;
  const uint32_t wofs = (threadIdx.x >> 5) * (PER * 32);
  const uint64_t items = (uint64_t)n * g.tiles;
  for (uint64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int b = (int)(w / g.tiles);
    const uint32_t qbase =
        (uint32_t)(w - (uint64_t)b * g.tiles) * (kWThreads * PER) + wofs;
    if (qbase >= g.units) continue;         // uniform across the warp
    const cascade_kv_tensor_t *ts = dst + (uint64_t)b * 2 * g.L;
    const uint8_t *in = reinterpret_cast<const uint8_t *>(src[b]);
    if (!in) continue;                      // a block this call skips
    const bool in_al = ((uintptr_t)in & 15u) == 0;
    uint4 a[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {         // source loads first
      const uint32_t q = qbase + k * 32 + lane;
      a[k] = make_uint4(0, 0, 0, 0);
      if (in_al && q < g.units && q * 8 + 8 <= g.N)
        a[k] = ld16_stream((uint64_t)(in + 16ull * (q + 1)));
    }
    uint64_t daddr[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {       // then destination addresses
      const uint32_t q = qbase + k * 32 + lane;
      daddr[k] = 0;
      if (g.vec_ok && q < g.units && q * 8 + 8 <= g.N) {
        daddr[k] = unit_addr<2>(ts, q * 8, g);
        if (daddr[k] & 15u) daddr[k] = 0;
      }
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const uint32_t q = qbase + k * 32 + lane;
      uint32_t nxt = __shfl_down_sync(0xffffffffu, a[k].x, 1);
      const uint32_t first_next =
          __shfl_sync(0xffffffffu, k + 1 < PER ? a[k + 1 < PER ? k + 1 : k].x : 0u, 0);
      if (lane == 31) nxt = first_next;
      if (q >= g.units) continue;
      const uint32_t e = q * 8;
      const bool full = e + 8 <= g.N;
      uint4 o;
      if (in_al && full) {
        // The neighbour loaded unit q+2 only if its own unit is full.
        if ((lane == 31 && k + 1 == PER) || (q + 1) * 8 + 8 > g.N)
          nxt = *reinterpret_cast<const uint16_t *>(in + 16ull * (q + 2));
        o = make_uint4(fs16(a[k].x, a[k].y), fs16(a[k].y, a[k].z),
                       fs16(a[k].z, a[k].w), fs16(a[k].w, nxt));
      } else {
        o = wire_unit_slow(in, e, g);
      }
      if (daddr[k])
        *reinterpret_cast<uint4 *>(daddr[k]) = o;
      else
        store_unit_slow(ts, e, full ? 8 : g.N - e, o, g);
    }
  }
}

int make_geom(uint32_t layers, uint32_t heads, uint32_t seq,
              uint32_t head_dim, WireGeom *g) {
  CB_CHECK(layers && heads && seq && head_dim, CASCADE_ERR_INVALID,
           "layers, heads, seq_len and head_dim must be positive");
  const uint64_t sd = (uint64_t)seq * head_dim;
  const uint64_t e = sd * heads;
  const uint64_t nel = 2ull * layers * e;
  CB_CHECK(nel < (1ull << 31), CASCADE_ERR_INVALID,
           "a KV cache of 2^31 or more elements is not supported");
  g->L = layers;
  g->H = heads;
  g->S = seq;
  g->D = head_dim;
  g->SD = (uint32_t)sd;
  g->E = (uint32_t)e;
  g->N = (uint32_t)nel;
  g->units = (uint32_t)div_up(nel, 8);
  g->vecs = (uint32_t)div_up(kHeaderBytes + 2 * nel, 16);
  g->dE = make_div(g->E);
  g->dSD = make_div(g->SD);
  g->dD = make_div(head_dim);
  g->vec_ok = head_dim % 8 == 0;
  return CASCADE_OK;
}

}  // namespace

}  // namespace cb

// ------------------------------------------------------------------ C-ABI
extern "C" uint64_t cascade_kv_wire_bytes(uint32_t layers, uint32_t heads,
                                          uint32_t seq, uint32_t head_dim) {
  return 18ull + 4ull * layers * heads * seq * head_dim;
}

namespace cb {

int launch_kv_serialize(const cascade_kv_tensor_t *d_src, int src_dtype,
                        uint32_t layers, uint32_t heads, uint32_t seq,
                        uint32_t head_dim, const uint64_t *d_dst, int n,
                        cudaStream_t s) {
  CB_CHECK(src_dtype >= CASCADE_KV_FP16 && src_dtype <= CASCADE_KV_FP32,
           CASCADE_ERR_INVALID, "src_dtype must be FP16, BF16 or FP32");
  WireGeom g;
  int rc = make_geom(layers, heads, seq, head_dim, &g);
  if (rc != CASCADE_OK || n <= 0) return rc;
  g.tiles = (uint32_t)div_up(g.vecs, kWTile);
  const int grid = grid_for((uint64_t)n * g.tiles, 1, 3);
  switch (src_dtype) {
    case CASCADE_KV_FP16:
      kv_serialize_kernel<0><<<grid, kWThreads, 0, s>>>(d_src, d_dst, n, g);
      break;
    case CASCADE_KV_BF16:
      kv_serialize_kernel<1><<<grid, kWThreads, 0, s>>>(d_src, d_dst, n, g);
      break;
    default:
      kv_serialize_kernel<2><<<grid, kWThreads, 0, s>>>(d_src, d_dst, n, g);
  }
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

}  // namespace cb

extern "C" int cascade_kv_serialize_batch(const cascade_kv_tensor_t *d_src,
                                          int src_dtype, uint32_t layers,
                                          uint32_t heads, uint32_t seq,
                                          uint32_t head_dim,
                                          const uint64_t *d_dst, size_t n,
                                          void *stream) {
  cb::clear_error();
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  CB_CHECK(src_dtype >= CASCADE_KV_FP16 && src_dtype <= CASCADE_KV_FP32,
           CASCADE_ERR_INVALID, "src_dtype must be FP16, BF16 or FP32");
  cb::WireGeom g;
  int rc = cb::make_geom(layers, heads, seq, head_dim, &g);
  if (rc != CASCADE_OK) return rc;
  if (n == 0) return CASCADE_OK;
  CB_CHECK(d_src && d_dst, CASCADE_ERR_INVALID, "null pointer argument");
  return cb::launch_kv_serialize(d_src, src_dtype, layers, heads, seq,
                                 head_dim, d_dst, (int)n,
                                 static_cast<cudaStream_t>(stream));
}

namespace cb {

int launch_kv_deserialize(const uint64_t *d_src, uint32_t layers,
                          uint32_t heads, uint32_t seq, uint32_t head_dim,
                          const cascade_kv_tensor_t *d_dst, int n,
                          cudaStream_t s) {
  WireGeom g;
  int rc = make_geom(layers, heads, seq, head_dim, &g);
  if (rc != CASCADE_OK || n <= 0) return rc;
  constexpr int kPer = 6;                 // units per thread per work item
  g.tiles = (uint32_t)div_up(g.units, kWThreads * kPer);
  const int grid = grid_for((uint64_t)n * g.tiles, 1, 3);
  kv_deserialize_kernel<kPer><<<grid, kWThreads, 0, s>>>(d_src, d_dst, n, g);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

}  // namespace cb

extern "C" int cascade_kv_deserialize_batch(const uint64_t *d_src,
                                            uint32_t layers, uint32_t heads,
                                            uint32_t seq, uint32_t head_dim,
                                            const cascade_kv_tensor_t *d_dst,
                                            size_t n, void *stream) {
  cb::clear_error();
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  cb::WireGeom g;
  int rc = cb::make_geom(layers, heads, seq, head_dim, &g);
  if (rc != CASCADE_OK) return rc;
  if (n == 0) return CASCADE_OK;
  CB_CHECK(d_src && d_dst, CASCADE_ERR_INVALID, "null pointer argument");
  return cb::launch_kv_deserialize(d_src, layers, heads, seq, head_dim, d_dst,
                                   (int)n, static_cast<cudaStream_t>(stream));
}
