// Batched SHA-256 over device-resident blocks (one serial chain per block).
//
// Replaces the per-block OpenSSL call of compute_block_id
// (cascade_core.cpp:43-53) with one launch over a whole batch.  A lane owns
// one block's chain; 32 blocks share a warp.  Merkle-Damgard chaining makes
// a block's 64-byte chunks strictly sequential, so a batch of large blocks
// is bound by how fast one warp can run the rounds of one chunk; the kernel
// below takes everything else (loads, byte swaps, the message schedule) off
// that warp.
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
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

// 16-byte global -> shared copy that completes asynchronously; each thread
// waits for its own copies with cp.async.wait_group.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const uint32_t dst = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

__device__ __forceinline__ uint32_t ldg_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// Producer/consumer SHA-256: a CTA of two warps hashes 32 blocks.  Warp 0
// (the consumer) runs only the 64 rounds of each chunk; warp 1 (the
// producer, on another scheduler) loads the message, expands the schedule
// and hands K[t]+W[t] to the consumer through a ring of kStages chunk slots
// in shared memory.  Named barriers order the ring: full[s] (producer ->
// consumer) and empty[s] (consumer -> producer).  Both warps run the same
// warp-uniform number of chunks, so every barrier is reached by all 64
// threads; lanes whose block needs fewer chunks process padding and discard
// the result.
__device__ __forceinline__ void bar_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}
__device__ __forceinline__ void bar_arrive(int id) {
  asm volatile("bar.arrive %0, 64;" ::"r"(id) : "memory");
}

struct Lane {
  const uint8_t *p;
  uint64_t len, nfull;
  uint32_t rem, nch;  // nch: chunks including padding
  bool aligned;
};

__device__ __forceinline__ Lane lane_of(const uint64_t *ptrs,
                                        const uint64_t *sizes, int n, int i) {
  Lane l;
  l.p = i < n ? reinterpret_cast<const uint8_t *>(ptrs[i]) : nullptr;
  l.len = i < n ? sizes[i] : 0;
  l.nfull = l.len >> 6;
  l.rem = (uint32_t)(l.len & 63u);
  l.nch = (uint32_t)l.nfull + (l.rem < 56 ? 1u : 2u);
  l.aligned = ((uintptr_t)l.p & 15u) == 0;
  return l;
}

// Big-endian message words of chunk c of a lane's padded message.
__device__ __forceinline__ void message_words(const Lane &l, uint64_t c,
                                              const uint4 *pre, uint32_t w[16]) {
  if (c < l.nfull) {
    if (l.aligned) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        w[4 * k] = sha::bswap(pre[k].x);
        w[4 * k + 1] = sha::bswap(pre[k].y);
        w[4 * k + 2] = sha::bswap(pre[k].z);
        w[4 * k + 3] = sha::bswap(pre[k].w);
      }
    } else {
      const uint32_t o = (uint32_t)((uintptr_t)l.p & 3u);
      const uint32_t *cw = (const uint32_t *)(l.p - o) + 16 * c;
      const uint32_t sel = (o << 12) | ((o + 1) << 8) | ((o + 2) << 4) | (o + 3);
      uint32_t raw[17];
#pragma unroll
      for (int j = 0; j < 16; ++j) raw[j] = ldg_u32(cw + j);
      raw[16] = o ? ldg_u32(cw + 16) : 0u;
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = __byte_perm(raw[j], raw[j + 1], sel);
    }
    return;
  }
  // Padding: the tail bytes, 0x80, zeros, and the bit length in the last
  // two words of the final chunk (FIPS 180-4 section 5.1.1).
  const uint64_t extra = c - l.nfull;   // 0 or 1 for real lanes
  const uint8_t *tail = l.p + (l.nfull << 6);
  const bool first = extra == 0;
  const bool last = c + 1 == l.nch;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t idx = 4 * j + k;
      uint32_t byte = 0;
      if (first && idx < l.rem) byte = tail[idx];
      else if (first && idx == l.rem) byte = 0x80u;
      word |= byte << (24 - 8 * k);
    }
    w[j] = word;
  }
  if (last) {
    const uint64_t bits = l.len * 8u;
    w[14] = (uint32_t)(bits >> 32);
    w[15] = (uint32_t)bits;
  }
}

// Producer side of one chunk: waits for ring slot it % kStages to be free,
// expands the message schedule and publishes K[t] + W[t] for t = 0..63.
template <int kStages>
__device__ __forceinline__ void publish_chunk(uint4 (*ring)[16][32], int lane,
                                              uint32_t it, uint32_t w[16],
                                              int full_bar, int empty_bar) {
  const int s = (int)(it % kStages);
  if (it >= kStages) bar_sync(empty_bar + s);
#pragma unroll
  for (int t = 0; t < 64; t += 4) {
    uint32_t kw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int tt = t + u;
      uint32_t wt;
      if (tt < 16) {
        wt = w[tt];
      } else {
        wt = w[tt & 15] + sha::sig0(w[(tt - 15) & 15]) + w[(tt - 7) & 15] +
             sha::sig1(w[(tt - 2) & 15]);
        w[tt & 15] = wt;
      }
      kw[u] = wt + sha::K(tt);
    }
    ring[s][t >> 2][lane] = make_uint4(kw[0], kw[1], kw[2], kw[3]);
  }
  bar_arrive(full_bar + s);
}

// kGroups (consumer, producer) warp pairs per CTA: warp 2g consumes and
// warp 2g+1 produces for group g.  kAhead > 0: the producer streams the
// chunks that every live lane of its warp has in full, at 16-byte-aligned
// addresses, through a ring of kAhead chunk slots in shared memory
// (cp.async, kAhead chunks in flight per lane), which hides DRAM latency
// when each scheduler holds a single warp pair; the other chunks (unaligned
// blocks, tails, padding), and every chunk when kAhead = 0, take the generic
// path that loads the next chunk into registers while this one is expanded
// (enough once several warps share a scheduler).  Named barrier ids per group:
// full = 1 + 2*kStages*g + s, empty = full + kStages (at most 15 ids).
// Chunks [c_begin, c_end) of every block are processed; a block whose last
// chunk falls in that range gets its digest written, a block that goes on
// beyond c_end gets its running state saved to `state` (and the next call
// with c_begin = this c_end resumes from it).  c_begin = 0 starts from the
// initial hash value.  One call with [0, ~0) hashes whole blocks.
template <int kGroups, int kStages, int kRound, int kUnroll, int kAhead>
__global__ void __launch_bounds__(64 * kGroups)
    sha256_pipelined(const uint64_t *__restrict__ ptrs,
                     const uint64_t *__restrict__ sizes, int n,
                     uint32_t *__restrict__ digests, uint32_t one,
                     uint32_t neg_one, uint32_t *__restrict__ state,
                     uint64_t c_begin, uint64_t c_end) {
  static_assert(2 * kGroups * kStages <= 15, "named barrier ids");
  // ring[g][s][t/4][lane] holds K[t..t+3] + W[t..t+3] of one chunk.
  __shared__ uint4 ring_all[kGroups][kStages][16][32];
  // raw[g][slot][k][lane]: bytes 16k..16k+15 of a lane's chunk in flight
  __shared__ uint4 raw_all[kGroups][kAhead > 0 ? kAhead : 1][4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = kGroups == 1 ? 0 : warp >> 1;
  uint4 (*ring)[16][32] = ring_all[grp];
  uint4 (*raw)[4][32] = raw_all[grp];
  const int full_bar = 1 + 2 * kStages * grp;
  const int empty_bar = full_bar + kStages;
  const int i = (blockIdx.x * kGroups + grp) * 32 + lane;
  const Lane l = lane_of(ptrs, sizes, n, i);
  const uint64_t nch_warp = __reduce_max_sync(0xffffffffu, l.nch);
  const uint64_t c_stop = nch_warp < c_end ? nch_warp : c_end;
  // iterations of this call (warp-uniform): chunks c_begin + 0 .. + iters-1
  const uint32_t iters = c_stop > c_begin ? (uint32_t)(c_stop - c_begin) : 0u;

  if (warp & 1) {  // -------------------------------------------- producer
    const uint4 *q = reinterpret_cast<const uint4 *>(l.p);
    uint32_t it = 0;
    // Loads never reach past this call's range: the bytes of later chunks
    // may not have arrived yet.
    if constexpr (kAhead > 0) {
      // Fast range (warp-uniform): chunks that every live lane has in full
      // at a 16-byte-aligned address.  Lanes without a block load nothing
      // and publish words that the consumer discards.
      const bool live = i < n;
      const uint64_t mine = !live ? ~0ull : (l.aligned ? l.nfull : 0ull);
      const uint32_t fast_end = __reduce_min_sync(
          0xffffffffu, (uint32_t)(mine < 0xffffffffull ? mine : 0xffffffffull));
      const uint64_t fast_stop = fast_end < c_stop ? fast_end : c_stop;
      const uint32_t it_fast =
          fast_stop > c_begin ? (uint32_t)(fast_stop - c_begin) : 0u;
#pragma unroll 1
      for (uint32_t j = 0; j < (uint32_t)kAhead; ++j) {
        if (live && j < it_fast) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            cp_async16(&raw[j][k][lane], q + 4 * (c_begin + j) + k);
        }
        cp_async_commit();
      }
#pragma unroll 1
      for (; it < it_fast; ++it) {
        const int slot = (int)(it % (uint32_t)kAhead);
        cp_async_wait<kAhead - 1>();  // this lane's copy of chunk it landed
        uint32_t w[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 v = raw[slot][k][lane];
          w[4 * k] = sha::bswap(v.x);
          w[4 * k + 1] = sha::bswap(v.y);
          w[4 * k + 2] = sha::bswap(v.z);
          w[4 * k + 3] = sha::bswap(v.w);
        }
        // The slot is refilled after its words are in registers.
        if (live && it + kAhead < it_fast) {
          const uint64_t cn = c_begin + it + kAhead;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            cp_async16(&raw[slot][k][lane], q + 4 * cn + k);
        }
        cp_async_commit();
        publish_chunk<kStages>(ring, lane, it, w, full_bar, empty_bar);
      }
      cp_async_wait<0>();
    }
    // Generic range: unaligned blocks, the tail and the padding chunks,
    // with the next chunk's loads in registers.
    uint4 pre[4] = {};
    if (l.aligned && c_begin + it < l.nfull && it < iters) {
#pragma unroll
      for (int k = 0; k < 4; ++k) pre[k] = ldg_stream(q + 4 * (c_begin + it) + k);
    }
#pragma unroll 1
    for (; it < iters; ++it) {
      const uint64_t c = c_begin + it;
      uint32_t w[16];
      message_words(l, c, pre, w);
      if (l.aligned && c + 1 < l.nfull && it + 1 < iters) {
#pragma unroll
        for (int k = 0; k < 4; ++k) pre[k] = ldg_stream(q + 4 * (c + 1) + k);
      }
      publish_chunk<kStages>(ring, lane, it, w, full_bar, empty_bar);
    }
    // Take the consumer's last releases so no arrival is left pending.
    for (uint32_t j = iters > kStages ? iters - kStages : 0; j < iters; ++j)
      bar_sync(empty_bar + (int)(j % kStages));
    return;
  }
  // -------------------------------------------------------------- consumer
  uint32_t st[8];
  if (c_begin == 0) {
    sha::init(st);
  } else if (i < n) {
#pragma unroll
    for (int k = 0; k < 8; ++k) st[k] = state[8 * (size_t)i + k];
  }
  for (uint32_t it = 0; it < iters; ++it) {
    const uint64_t c = c_begin + it;
    const int s = (int)(it % kStages);
    bar_sync(full_bar + s);
    uint32_t a = st[0], b = st[1], cc = st[2], d = st[3];
    uint32_t e = st[4], f = st[5], g = st[6], h = st[7];
    // Every round runs the same instructions (K[t] is folded into kw by the
    // producer), and the eight working variables come back to their
    // registers every 8 rounds, so kUnroll rounds (a multiple of 8) form a
    // loop body small enough for the instruction cache.
#pragma unroll 1
    for (int t0 = 0; t0 < 64; t0 += kUnroll) {
#pragma unroll
      for (int t = t0; t < t0 + kUnroll; t += 4) {
        const uint4 kw = ring[s][t >> 2][lane];
        const uint32_t kv[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (kRound == 0)
            sha::round_kw(a, b, cc, d, e, f, g, h, kv[u], one, neg_one);
          else if (kRound == 1)
            sha::round_kw3(a, b, cc, d, e, f, g, h, kv[u], one, neg_one);
          else
            sha::round_kw9(a, b, cc, d, e, f, g, h, kv[u], one, neg_one);
        }
      }
    }
    bar_arrive(empty_bar + s);
    if (c < l.nch) {
      st[0] += a; st[1] += b; st[2] += cc; st[3] += d;
      st[4] += e; st[5] += f; st[6] += g; st[7] += h;
    }
  }
  if (i < n && l.nch > c_begin) {
    if (l.nch <= c_end) {  // finished in this call: the digest
      uint32_t *out = digests + 8 * (size_t)i;
#pragma unroll
      for (int k = 0; k < 8; ++k) out[k] = sha::bswap(st[k]);
    } else {               // continues in the next call
#pragma unroll
      for (int k = 0; k < 8; ++k) state[8 * (size_t)i + k] = st[k];
    }
  }
}

}  // namespace

// Unused dynamic shared memory that keeps at most `want` CTAs of a kernel
// with `static_smem` bytes of its own on one SM.
struct SmemLimits {
  int per_sm = 0, optin = 0, reserved = 0, sms = 0;
};

static int smem_limits(SmemLimits *out) {
  static std::mutex mu;
  static std::map<int, SmemLimits> cache;
  int dev = 0;
  CB_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it == cache.end()) {
    SmemLimits l;
    CB_CUDA(cudaDeviceGetAttribute(
        &l.per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    CB_CUDA(cudaDeviceGetAttribute(
        &l.optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    CB_CUDA(cudaDeviceGetAttribute(
        &l.reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev));
    CB_CUDA(cudaDeviceGetAttribute(&l.sms, cudaDevAttrMultiProcessorCount,
                                   dev));
    it = cache.emplace(dev, l).first;
  }
  *out = it->second;
  return CASCADE_OK;
}

// One CTA per SM and at least 16 SMs spare: the launch fills its SMs'
// shared memory so that neighbours run on the spare SMs only.
static bool fills_sms(const SmemLimits &lim, int blocks) {
  return blocks <= lim.sms && lim.sms - blocks >= 16;
}

template <int G, int S, int R, int U, int A>
int launch_sha256_pipelined(const uint64_t *d_ptrs, const uint64_t *d_sizes,
                            int n, uint8_t *d_digests, uint32_t *d_state,
                            uint64_t c_begin, uint64_t c_end, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  const int blocks = (n + 32 * G - 1) / (32 * G);
  auto kernel = sha256_pipelined<G, S, R, U, A>;
  // Each chain's speed is its consumer warp's issue rate, so the CTAs must
  // spread evenly: two consumers on one scheduler halve their chains' speed
  // and the launch ends with the slowest chain.  A CTA is small enough that
  // four fit on an SM, and when other kernels are resident as the launch
  // dispatches (the speculative payload kernels of a put), some SMs took 3-4
  // CTAs: 8192 chains of 2 MiB ran 54 ms instead of 28.  Unused dynamic
  // shared memory caps each SM at ceil(blocks / SMs) CTAs.
  SmemLimits lim;
  int rc = smem_limits(&lim);
  if (rc) return rc;
  cudaFuncAttributes attr;
  CB_CUDA(cudaFuncGetAttributes(&attr, kernel));
  const size_t own = attr.sharedSizeBytes + (size_t)lim.reserved;
  const int want = (blocks + lim.sms - 1) / lim.sms;
  size_t pad = 0;
  const size_t slice = (size_t)lim.per_sm / (want + 1) + 1;  // want+1 cannot fit
  if (slice > own && (size_t)want * slice <= (size_t)lim.per_sm &&
      attr.sharedSizeBytes + (slice - own) <= (size_t)lim.optin)
    pad = slice - own;
  // One CTA per SM with >= 16 SMs spare: the CTAs also fill their SMs'
  // shared memory to within 6 KiB.  Kernels launched beside the hash with
  // kHashNeighbourSmem of shared memory then run only on the spare SMs and
  // take no issue slots from the chains (when the hash ends they may use
  // every SM).  4096 chains of 2 MiB with the put's INT8 payload beside
  // them: 28.0 ms per step, the hash's own time, against 29.7 sharing SMs.
  // With two CTAs per SM the payload is twice as large per unit of hash
  // time and the spare SMs fall behind (8192 chains: 36 against 32 ms).
  if (fills_sms(lim, blocks)) {
    const size_t fill = ((size_t)lim.per_sm - own - 6 * 1024) & ~size_t(1023);
    static_assert(6 * 1024 < kHashNeighbourSmem + 1024,
                  "the leftover must not fit a neighbour CTA");
    if (fill > pad && attr.sharedSizeBytes + fill <= (size_t)lim.optin)
      pad = fill;
  }
  if (pad > (size_t)attr.maxDynamicSharedSizeBytes)
    CB_CUDA(cudaFuncSetAttribute(kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 lim.optin - (int)attr.sharedSizeBytes));
  kernel<<<blocks, 64 * G, pad, s>>>(
      d_ptrs, d_sizes, n, reinterpret_cast<uint32_t *>(d_digests), 1u,
      0xffffffffu, d_state, c_begin, c_end);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_sha256_range(const uint64_t *d_ptrs, const uint64_t *d_sizes,
                        int n, uint8_t *d_digests, uint32_t *d_state,
                        uint64_t c_begin, uint64_t c_end, cudaStream_t s) {
  // Up to two producer/consumer pairs per SM, each warp has a scheduler to
  // itself: the latency-tuned round (one IMAD on the e-recurrence), all 64
  // rounds unrolled, and 8 chunks of loads in flight per lane (8192 chains:
  // 610 GB/s against 523 for the other form).  Beyond that, warps share
  // schedulers, the ALU pipe is the limit and the round with the fewest ALU
  // instructions wins (12288 chains: 526 against 490).
  if (n <= 2 * 32 * sm_count())
    return launch_sha256_pipelined<1, 4, 2, 64, 8>(
        d_ptrs, d_sizes, n, d_digests, d_state, c_begin, c_end, s);
  return launch_sha256_pipelined<2, 3, 0, 16, 0>(d_ptrs, d_sizes, n, d_digests,
                                                 d_state, c_begin, c_end, s);
}

size_t sha256_neighbour_smem(int n) {
  SmemLimits lim;
  if (n <= 0 || smem_limits(&lim) != CASCADE_OK) return 0;
  const int per_cta = n <= 2 * 32 * lim.sms ? 32 : 64;  // chains per CTA
  return fills_sms(lim, (n + per_cta - 1) / per_cta) ? kHashNeighbourSmem : 0;
}

int launch_sha256(const uint64_t *d_ptrs, const uint64_t *d_sizes, int n,
                  uint8_t *d_digests, cudaStream_t s) {
  return launch_sha256_range(d_ptrs, d_sizes, n, d_digests, nullptr, 0, ~0ull,
                             s);
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
