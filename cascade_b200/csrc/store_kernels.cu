// Batched kernels over the device block index and the HBM pool allocator.
//
// Put protocol for a batch (each step one launch, stream-ordered):
//   claim    every request finds or inserts its key (128-bit CAS on the key)
//            and lowers the slot's claim to its own sequence number;
//   resolve  the request holding the slot's smallest sequence number wins
//            (the reference's "first put stores, later puts are dedup hits",
//            CascadeStore::put, cascade_core.cpp:1077-1080), a live slot
//            means the key is already stored;
//   (alloc + payload kernels for the winners)
//   commit   winners publish location/size/header and turn the slot live;
//   finalize duplicates of a winner that failed fail too.
// No kernel here waits on another thread: every conflict is settled by one
// atomic, so nothing can spin.
#include "common.cuh"
#include "store_dev.cuh"

namespace cb {

namespace {

__device__ __forceinline__ void ld_key(const Slot *s, uint64_t &a,
                                       uint64_t &b) {
  asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];"
               : "=l"(a), "=l"(b)
               : "l"(&s->k0));
}

__global__ void claim_kernel(Slot *slots, uint64_t mask,
                             const uint64_t *__restrict__ keys, int stride,
                             const uint64_t *__restrict__ seqs, int n,
                             uint32_t *__restrict__ slot_idx, int *err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (seqs[i] == kNoSeq) {  // an unused entry: no key, status FAILED
    slot_idx[i] = kNoSlot;
    return;
  }
  const uint64_t s0 = keys[(size_t)i * stride] ^ kKeyMask0;
  const uint64_t s1 = keys[(size_t)i * stride + 1] ^ kKeyMask1;
  const uint64_t h = slot_hash(s0, s1);
  for (int p = 0; p < kMaxProbe; ++p) {
    const uint64_t idx = (h + (uint64_t)p) & mask;
    Slot *sl = slots + idx;
    uint64_t a, b;
    ld_key(sl, a, b);
    if ((a | b) != 0) {  // keys are never rewritten: a non-empty read is final
      if (a != s0 || b != s1) continue;
    } else {
      cas128(&sl->k0, 0, 0, s0, s1, a, b);
      if (!((a == 0 && b == 0) || (a == s0 && b == s1))) continue;
    }
    atomicMax(reinterpret_cast<unsigned long long *>(&sl->claim),
              (unsigned long long)~seqs[i]);
    slot_idx[i] = (uint32_t)idx;
    return;
  }
  slot_idx[i] = kNoSlot;
  atomicExch(err, CASCADE_ERR_FULL);
}

__global__ void resolve_kernel(const Slot *__restrict__ slots,
                               const uint32_t *__restrict__ slot_idx,
                               const uint64_t *__restrict__ seqs, int n,
                               uint8_t *__restrict__ status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t idx = slot_idx[i];
  if (idx == kNoSlot) { status[i] = CASCADE_PUT_FAILED; return; }
  const Slot &sl = slots[idx];
  if (sl.state == kLive) status[i] = CASCADE_PUT_DUP_KNOWN;
  else if (sl.claim == ~seqs[i]) status[i] = CASCADE_PUT_STORED;
  else status[i] = CASCADE_PUT_DUP_BATCH;
}

__global__ void commit_kernel(Slot *slots, const uint32_t *__restrict__ slot_idx,
                              const uint8_t *__restrict__ status,
                              const uint64_t *__restrict__ offsets,
                              const uint64_t *__restrict__ sizes,
                              const uint32_t *__restrict__ flags,
                              const uint8_t *__restrict__ headers,
                              uint64_t epoch_base, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || status[i] != CASCADE_PUT_STORED) return;
  Slot &sl = slots[slot_idx[i]];
  if (offsets[i] != kInvalidOffset) {
    const uint8_t *h = headers + 8 * (size_t)i;
    sl.offset = offsets[i];
    sl.size = sizes[i];
    sl.flags = flags[i];
    sl.hdr_scale = (uint32_t)h[0] | ((uint32_t)h[1] << 8) |
                   ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
    sl.hdr_zp = h[4];
    sl.epoch = epoch_base + (uint64_t)i;
    sl.state = kLive;
  }
  sl.claim = 0;
}

__global__ void finalize_kernel(const Slot *__restrict__ slots,
                                const uint32_t *__restrict__ slot_idx,
                                const uint64_t *__restrict__ offsets,
                                uint8_t *__restrict__ status, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t st = status[i];
  if (st == CASCADE_PUT_STORED && offsets[i] == kInvalidOffset)
    status[i] = CASCADE_PUT_FAILED;
  else if (st == CASCADE_PUT_DUP_BATCH && slots[slot_idx[i]].state != kLive)
    status[i] = CASCADE_PUT_FAILED;
}

__global__ void lookup_kernel(Slot *slots, uint64_t mask,
                              const uint64_t *__restrict__ keys, int stride,
                              int n, int touch, uint64_t epoch_base,
                              LookupInfo *__restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t s0 = keys[(size_t)i * stride] ^ kKeyMask0;
  const uint64_t s1 = keys[(size_t)i * stride + 1] ^ kKeyMask1;
  const uint64_t h = slot_hash(s0, s1);
  LookupInfo r = {};
  r.slot = kNoSlot;
  for (int p = 0; p < kMaxProbe; ++p) {
    const uint64_t idx = (h + (uint64_t)p) & mask;
    Slot *sl = slots + idx;
    uint64_t a, b;
    ld_key(sl, a, b);
    if ((a | b) == 0) break;
    if (a != s0 || b != s1) continue;
    if (sl->state == kLive) {
      r.found = 1;
      r.flags = sl->flags;
      r.offset = sl->offset;
      r.size = sl->size;
      r.hdr_scale = sl->hdr_scale;
      r.hdr_zp = sl->hdr_zp;
      r.slot = (uint32_t)idx;
      if (touch) sl->epoch = epoch_base + (uint64_t)i;
    }
    break;
  }
  out[i] = r;
}

__global__ void relocate_kernel(Slot *slots, const uint32_t *__restrict__ idx,
                                const uint64_t *__restrict__ offsets,
                                const uint32_t *__restrict__ flags,
                                const uint8_t *__restrict__ headers, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  Slot &sl = slots[idx[i]];
  const uint8_t *h = headers + 8 * (size_t)i;
  sl.offset = offsets[i];
  sl.flags = flags[i];
  sl.hdr_scale = (uint32_t)h[0] | ((uint32_t)h[1] << 8) |
                 ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
  sl.hdr_zp = h[4];
}

// Demotion candidates.  A live HBM slot belongs to class 1 when it is a
// prefix block and prefix protection is on, else to class 0; within a class
// the least recent epoch goes first.  Epochs are bucketed linearly over
// [0, span) into kVictimBuckets buckets per class; the histogram sums each
// bucket's HBM payload bytes and slot count, the host picks per class the
// last bucket it needs, and the collect pass writes out every candidate up
// to that bucket.  Only those few are sorted on the host.
__device__ __forceinline__ bool victim_of(const Slot &sl, int semantic,
                                          uint64_t span, int &cls, int &bucket,
                                          uint64_t &pay) {
  if (sl.state != kLive || !(sl.flags & kTierHbm) ||
      (sl.flags & kFlagRemote))
    return false;
  cls = (semantic && (sl.flags & kFlagPrefix)) ? 1 : 0;
  const uint64_t e = sl.epoch < span ? sl.epoch : span - 1;
  bucket = (int)((e * (uint64_t)kVictimBuckets) / span);
  pay = (sl.flags & kFlagQ8) ? sl.size / 2 : sl.size;
  return true;
}

__global__ void victim_hist_kernel(const Slot *__restrict__ slots,
                                   uint64_t nslots, int semantic,
                                   uint64_t span,
                                   unsigned long long *__restrict__ bytes,
                                   uint32_t *__restrict__ count) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
       i < nslots; i += (uint64_t)gridDim.x * blockDim.x) {
    int cls, b;
    uint64_t pay;
    if (!victim_of(slots[i], semantic, span, cls, b, pay)) continue;
    atomicAdd(&bytes[cls * kVictimBuckets + b], (unsigned long long)pay);
    atomicAdd(&count[cls * kVictimBuckets + b], 1u);
  }
}

__global__ void victim_collect_kernel(const Slot *__restrict__ slots,
                                      uint64_t nslots, int semantic,
                                      uint64_t span, int cut0, int cut1,
                                      uint32_t *__restrict__ n_out,
                                      ScanRec *__restrict__ out,
                                      uint32_t max_out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
       i < nslots; i += (uint64_t)gridDim.x * blockDim.x) {
    int cls, b;
    uint64_t pay;
    const Slot &sl = slots[i];
    if (!victim_of(sl, semantic, span, cls, b, pay)) continue;
    if (b > (cls ? cut1 : cut0)) continue;
    const uint32_t k = atomicAdd(n_out, 1u);
    if (k >= max_out) continue;
    ScanRec r;
    r.slot = (uint32_t)i;
    r.flags = sl.flags;
    r.size = sl.size;
    r.offset = sl.offset;
    r.epoch = sl.epoch;
    r.hdr_scale = sl.hdr_scale;
    r.hdr_zp = sl.hdr_zp;
    r.k0 = sl.k0 ^ kKeyMask0;
    r.k1 = sl.k1 ^ kKeyMask1;
    out[k] = r;
  }
}

// An owner's entry follows its payload to the holder's DRAM tier.
__global__ void apply_moves_kernel(Slot *slots, uint64_t mask,
                                   const ShardRecord *__restrict__ in, int m,
                                   uint32_t rank) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  const ShardRecord r = in[j];
  if (r.src_idx != kMoveIdx) return;
  const uint64_t s0 = r.k0 ^ kKeyMask0, s1 = r.k1 ^ kKeyMask1;
  const uint64_t h = slot_hash(s0, s1);
  for (int p = 0; p < kMaxProbe; ++p) {
    Slot *sl = slots + ((h + (uint64_t)p) & mask);
    uint64_t a, b;
    ld_key(sl, a, b);
    if ((a | b) == 0) return;
    if (a != s0 || b != s1) continue;
    if (sl->state != kLive) return;
    sl->offset = r.offset;
    sl->flags = (r.flags & 0xffffu & ~(uint32_t)kFlagRelocate) |
                ((r.holder & 0xffu) << 16) |
                (r.holder != rank ? (uint32_t)kFlagRemote : 0u);
    sl->hdr_scale = r.hdr_scale;
    sl->hdr_zp = r.hdr_zp;
    return;
  }
}

// Bump space is claimed with compare-and-swap, advancing only when the
// request fits, so a request that fails never moves the bump offset and
// cannot make a smaller concurrent request fail.  Each warp claims its
// lanes' total in one CAS loop; if the total does not fit, the lanes try
// one at a time in lane order.  Every failed CAS means another warp
// advanced the offset, so the loops end.
__device__ __forceinline__ uint64_t claim_bump(PoolDev *pool, uint64_t bytes) {
  unsigned long long *bp = reinterpret_cast<unsigned long long *>(&pool->bump);
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long *>(bp);
  while (cur + bytes <= pool->capacity) {
    const unsigned long long prev = atomicCAS(bp, cur, cur + bytes);
    if (prev == cur) return cur;
    cur = prev;
  }
  return kInvalidOffset;
}

__global__ void pool_alloc_kernel(PoolDev *pool, const uint64_t *__restrict__ req,
                                  int n, uint64_t *__restrict__ offsets) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const uint64_t want = i < n ? req[i] : kNoRequest;
  bool need_bump = false;
  uint64_t bytes = 0;
  if (want != kNoRequest) {
    const int c = size_class(want);
    bytes = class_bytes(c);
    const uint32_t k = atomicAdd(&pool->taken[c], 1u);
    const uint32_t top = pool->top[c];  // not written by this kernel
    if (k < top)
      offsets[i] = pool->stack[c][top - 1 - k];
    else
      need_bump = true;
  } else if (i < n) {
    offsets[i] = kInvalidOffset;
  }
  const unsigned m = __ballot_sync(0xffffffffu, need_bump);
  if (!m) return;
  // Inclusive prefix of the bump requests' bytes in lane order.
  uint64_t incl = need_bump ? bytes : 0;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint64_t up = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += up;
  }
  const uint64_t total = __shfl_sync(0xffffffffu, incl, 31);
  const int leader = __ffs(m) - 1;
  uint64_t base = 0;
  if (lane == leader) base = claim_bump(pool, total);
  base = __shfl_sync(0xffffffffu, base, leader);
  if (base != kInvalidOffset) {
    if (need_bump) offsets[i] = base + incl - bytes;
    return;
  }
  for (int l = 0; l < 32; ++l) {
    if (lane == l && need_bump) offsets[i] = claim_bump(pool, bytes);
    __syncwarp();
  }
}

__global__ void pool_alloc_finish_kernel(PoolDev *pool) {
  for (int c = threadIdx.x; c < kNumClasses; c += blockDim.x) {
    const uint32_t t = pool->taken[c];
    if (t) {
      const uint32_t top = pool->top[c];
      pool->top[c] = top - (t < top ? t : top);
      pool->taken[c] = 0;
    }
  }
}

__global__ void pool_free_kernel(PoolDev *pool, const uint64_t *__restrict__ req,
                                 const uint64_t *__restrict__ offsets,
                                 const uint8_t *__restrict__ status, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n || status[i] == CASCADE_PUT_STORED) return;
  const uint64_t off = offsets[i];
  if (off == kInvalidOffset || req[i] == kNoRequest) return;
  const int c = size_class(req[i]);
  const uint32_t k = atomicAdd(&pool->top[c], 1u);
  if (k < pool->cap[c] && pool->stack[c] != nullptr) {
    pool->stack[c][k] = off;
  } else {
    atomicSub(&pool->top[c], 1u);
    atomicAdd(reinterpret_cast<unsigned long long *>(&pool->overflow), 1ull);
  }
}

inline int blocks_for(int n) { return (n + 255) / 256; }

}  // namespace

int launch_index_claim(Slot *slots, uint64_t mask, const uint64_t *keys,
                       int key_stride_u64, const uint64_t *seqs, int n,
                       uint32_t *slot_idx, int *err, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  claim_kernel<<<blocks_for(n), 256, 0, s>>>(slots, mask, keys, key_stride_u64,
                                             seqs, n, slot_idx, err);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_index_resolve(const Slot *slots, const uint32_t *slot_idx,
                         const uint64_t *seqs, int n, uint8_t *status,
                         cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  resolve_kernel<<<blocks_for(n), 256, 0, s>>>(slots, slot_idx, seqs, n,
                                               status);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_index_commit(Slot *slots, const uint32_t *slot_idx,
                        const uint8_t *status, const uint64_t *offsets,
                        const uint64_t *sizes, const uint32_t *flags,
                        const uint8_t *headers, uint64_t epoch_base, int n,
                        cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  commit_kernel<<<blocks_for(n), 256, 0, s>>>(slots, slot_idx, status, offsets,
                                              sizes, flags, headers,
                                              epoch_base, n);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_index_finalize(const Slot *slots, const uint32_t *slot_idx,
                          const uint64_t *offsets, uint8_t *status, int n,
                          cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  finalize_kernel<<<blocks_for(n), 256, 0, s>>>(slots, slot_idx, offsets,
                                                status, n);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_index_lookup(Slot *slots, uint64_t mask, const uint64_t *keys,
                        int key_stride_u64, int n, int touch,
                        uint64_t epoch_base, LookupInfo *out, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  lookup_kernel<<<blocks_for(n), 256, 0, s>>>(slots, mask, keys, key_stride_u64,
                                              n, touch, epoch_base, out);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_index_relocate(Slot *slots, const uint32_t *slot_idx,
                          const uint64_t *offsets, const uint32_t *flags,
                          const uint8_t *headers, int n, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  relocate_kernel<<<blocks_for(n), 256, 0, s>>>(slots, slot_idx, offsets,
                                                flags, headers, n);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_index_apply_moves(Slot *slots, uint64_t mask, const void *records,
                             int m, uint32_t rank, cudaStream_t s) {
  if (m <= 0) return CASCADE_OK;
  apply_moves_kernel<<<blocks_for(m), 256, 0, s>>>(
      slots, mask, static_cast<const ShardRecord *>(records), m, rank);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_victim_hist(const Slot *slots, uint64_t nslots, int semantic,
                       uint64_t span, unsigned long long *bytes,
                       uint32_t *count, cudaStream_t s) {
  CB_CUDA(cudaMemsetAsync(bytes, 0, 2 * kVictimBuckets * sizeof(*bytes), s));
  CB_CUDA(cudaMemsetAsync(count, 0, 2 * kVictimBuckets * sizeof(*count), s));
  const int grid = grid_for(nslots, 256, 8);
  victim_hist_kernel<<<grid, 256, 0, s>>>(slots, nslots, semantic, span,
                                          bytes, count);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_victim_collect(const Slot *slots, uint64_t nslots, int semantic,
                          uint64_t span, int cut0, int cut1, uint32_t *n_out,
                          ScanRec *out, uint32_t max_out, cudaStream_t s) {
  CB_CUDA(cudaMemsetAsync(n_out, 0, sizeof(uint32_t), s));
  const int grid = grid_for(nslots, 256, 8);
  victim_collect_kernel<<<grid, 256, 0, s>>>(slots, nslots, semantic, span,
                                             cut0, cut1, n_out, out, max_out);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_pool_alloc(PoolDev *pool, const uint64_t *req, int n,
                      uint64_t *offsets, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  pool_alloc_kernel<<<blocks_for(n), 256, 0, s>>>(pool, req, n, offsets);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  pool_alloc_finish_kernel<<<1, 256, 0, s>>>(pool);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

int launch_pool_free_unstored(PoolDev *pool, const uint64_t *req,
                              const uint64_t *offsets, const uint8_t *status,
                              int n, cudaStream_t s) {
  if (n <= 0) return CASCADE_OK;
  pool_free_kernel<<<blocks_for(n), 256, 0, s>>>(pool, req, offsets, status,
                                                 n);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

}  // namespace cb
