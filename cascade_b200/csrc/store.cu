// CascadeStore on a B200: host orchestration over the device index, the HBM
// pool and the pinned DRAM tier.  Block bytes never pass through host code
// except when a caller hands over host buffers (staged through pinned
// memory) or a block lives in the DRAM tier.
//
// Reference: CascadeStore (cascade.hpp:420-502, cascade_core.cpp:960-1303),
// GPUBackend (gpu_backend.cu:166-528), ShmBackend (cascade_core.cpp:237-569).
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "dram.cuh"
#include "kernels.cuh"
#include "store_dev.cuh"

namespace cb {

namespace {

// ------------------------------------------------------------ helpers
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

inline uint64_t pow2_at_least(uint64_t x) {
  uint64_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

inline bool is_hex_id(const char *s, size_t len) {
  if (len != 32) return false;
  for (size_t i = 0; i < 32; ++i) {
    char c = s[i];
    if (!((c >= '0' && c <= '9') || (c >= 'a' && c <= 'f'))) return false;
  }
  return true;
}

inline int hexval(char c) { return c <= '9' ? c - '0' : c - 'a' + 10; }

// Little-endian load of 8 key bytes.
inline uint64_t le64(const uint8_t *b) {
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | b[i];
  return v;
}

// After the pool allocation: final offsets, payload destinations and the
// per-format byte counts the payload kernels consume (0 = skip block).
__global__ void prepare_kernel(int n, const uint64_t *__restrict__ req,
                               uint64_t *__restrict__ off,
                               const uint64_t *__restrict__ off_host,
                               const uint64_t *__restrict__ dst_host,
                               const uint32_t *__restrict__ flags,
                               const uint64_t *__restrict__ sizes,
                               uint64_t pool_base, uint64_t *__restrict__ dst,
                               uint64_t *__restrict__ eff_raw,
                               uint64_t *__restrict__ eff_q8) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint64_t d = 0, o;
  if (req[i] != kNoRequest) {  // an HBM placement
    o = off[i];
    if (o != kInvalidOffset) d = pool_base + o;
  } else {  // a DRAM placement (offset chosen on the host) or nothing
    o = off_host[i];
    d = dst_host[i];
  }
  off[i] = o;
  dst[i] = d;
  const bool q8 = (flags[i] & kFlagQ8) != 0;
  eff_q8[i] = (d && q8) ? sizes[i] : 0;
  eff_raw[i] = (d && !q8) ? sizes[i] : 0;
}

}  // namespace

// ------------------------------------------------------------- scratch
// Per-batch device arrays and their pinned host mirrors, carved from two
// blobs with the same layout.
struct Scratch {
  size_t cap = 0;
  uint8_t *dblob = nullptr, *hblob = nullptr;
  // arrays: device pointer, host mirror
  uint64_t *ptrs, *h_ptrs, *sizes, *h_sizes, *seqs, *h_seqs, *keys, *h_keys;
  uint64_t *req, *h_req, *off, *h_off, *dst, *h_dst, *eff_raw, *eff_q8;
  uint64_t *hoff, *hdst;  // device copies of h_off / h_dst
  uint8_t *digests, *h_digests, *status, *h_status, *hdr, *h_hdr;
  uint32_t *slot, *h_slot, *flags, *h_flags;
  int2 *mnmx;
  LookupInfo *info, *h_info;
  int *err, *h_err;
};

constexpr int kDmaStreams = 4;  // copy streams per direction

struct Store {
  cascade_config_t cfg;
  std::string shm_path, lustre_path;
  int dev = 0;
  bool hbm = false, dram_tier = false;
  cudaStream_t s = nullptr;   // main: index, allocation, payload kernels
  cudaStream_t s2 = nullptr;  // hashing, overlapped with the main stream
  cudaStream_t s3 = nullptr;  // host-to-device copies of host blocks
  cudaEvent_t ev = nullptr, ev2 = nullptr, ev3 = nullptr;
  uint32_t *sha_state = nullptr;  // running SHA-256 states (striped hashing)
  size_t sha_state_cap = 0;       // blocks
  uint8_t *pool = nullptr;
  uint64_t pool_cap = 0;
  PoolDev *d_pool = nullptr;
  uint64_t *stack_ptr[kNumClasses] = {};
  Slot *slots = nullptr;
  uint64_t nslots = 0;
  uint64_t claimed = 0;  // keys that own a slot (upper bound)
  std::unique_ptr<DramArena> dram;
  Scratch sc;
  Scratch oc;                  // owner-side records of a sharded batch
  uint8_t *shard_aux = nullptr;  // staged records + per-owner counters
  size_t oc_aux_cap = 0;
  int shard_rank = 0;            // this store's rank in the open batch
  int shard_world = 1;           // and the number of ranks
  size_t shard_open = 0;         // blocks of the open sharded batch
  size_t shard_get_open = 0;     // keys of the open sharded get
  size_t resolve_pending = 0;    // records of a resolve not yet counted
  // Pools of the other ranks mapped into this process (CUDA IPC); entry
  // peer_rank is this store's own pool.
  std::vector<uint8_t *> peer_base;
  int peer_rank = -1;
  // The other ranks' DRAM tiers (shared arenas), by rank; null for this
  // rank and for ranks without one.
  std::vector<std::unique_ptr<DramView>> peer_dram;
  // Relocation records for the next sharded begin: blocks this rank holds
  // for other owners that it demoted to its DRAM tier.
  std::vector<ShardRecord> shard_moves;
  uint8_t *h_moves = nullptr;  // pinned copy of them on the way to d_send
  size_t h_moves_cap = 0;
  uint8_t *d_stage = nullptr;  // device staging for host buffers
  size_t d_stage_cap = 0;
  uint8_t *h_stage = nullptr;  // pinned staging for host buffers
  size_t h_stage_cap = 0;
  uint8_t *d_q8stage = nullptr;  // INT8 payloads on their way to DRAM
  size_t d_q8stage_cap = 0;
  uint8_t *d_evstage = nullptr;  // INT8 forms of blocks being demoted
  size_t d_evstage_cap = 0;
  uint8_t *d_kvstage = nullptr;  // wire blocks a KV-cache get decodes first
  size_t d_kvstage_cap = 0;
  uint8_t *d_kvsrc = nullptr;    // wire-block addresses of a KV-cache get
  size_t d_kvsrc_cap = 0;
  uint8_t *scan_d = nullptr;     // demotion-candidate histogram and list
  size_t scan_cap = 0;           // bytes
  // Copy streams between the device and the DRAM tier: [0] device to
  // host, [1] host to device.
  cudaStream_t dma[2][kDmaStreams] = {};
  cudaEvent_t dma_done[2][kDmaStreams] = {};
  cudaEvent_t dma_start = nullptr;
  // Per block of the batch being placed: 1 when serial puts would have
  // stored it in HBM and demoted it again within the batch (it goes to the
  // DRAM tier directly and counts as a GPU eviction).
  std::vector<uint8_t> demoted;
  std::mutex mu;
  uint64_t next_seq = 1, next_epoch = 1, next_name = 1;
  std::unordered_map<std::string, Key> names;
  // CascadeStore::Stats counters (cascade.hpp:439-456)
  uint64_t gpu_used = 0, shm_used = 0, gpu_hits = 0, shm_hits = 0,
           misses = 0, dedup_hits = 0, gpu_evictions = 0,
           promotions_to_gpu = 0, compression_savings = 0, shm_puts = 0;
};

namespace {

template <typename T>
T *carve(uint8_t *&p, size_t count) {
  T *r = reinterpret_cast<T *>(p);
  p += (count * sizeof(T) + 255) & ~size_t(255);
  return r;
}

size_t scratch_bytes(size_t c) {
  uint8_t *p = nullptr;
  carve<uint64_t>(p, c); carve<uint64_t>(p, c); carve<uint64_t>(p, c);
  carve<uint64_t>(p, 2 * c); carve<uint64_t>(p, c); carve<uint64_t>(p, c);
  carve<uint64_t>(p, c); carve<uint64_t>(p, c); carve<uint64_t>(p, c);
  carve<uint64_t>(p, c); carve<uint64_t>(p, c);
  carve<uint8_t>(p, 32 * c); carve<uint8_t>(p, c); carve<uint8_t>(p, 8 * c);
  carve<uint32_t>(p, c); carve<uint32_t>(p, c); carve<int2>(p, c);
  carve<LookupInfo>(p, c); carve<int>(p, 1);
  return (size_t)(p - (uint8_t *)nullptr);
}

void carve_all(Scratch &S, uint8_t *base, bool host) {
  uint8_t *p = base;
  uint64_t *ptrs = carve<uint64_t>(p, S.cap);
  uint64_t *sizes = carve<uint64_t>(p, S.cap);
  uint64_t *seqs = carve<uint64_t>(p, S.cap);
  uint64_t *keys = carve<uint64_t>(p, 2 * S.cap);
  uint64_t *req = carve<uint64_t>(p, S.cap);
  uint64_t *off = carve<uint64_t>(p, S.cap);
  uint64_t *dst = carve<uint64_t>(p, S.cap);
  uint64_t *eff_raw = carve<uint64_t>(p, S.cap);
  uint64_t *eff_q8 = carve<uint64_t>(p, S.cap);
  uint64_t *hoff = carve<uint64_t>(p, S.cap);
  uint64_t *hdst = carve<uint64_t>(p, S.cap);
  uint8_t *digests = carve<uint8_t>(p, 32 * S.cap);
  uint8_t *status = carve<uint8_t>(p, S.cap);
  uint8_t *hdr = carve<uint8_t>(p, 8 * S.cap);
  uint32_t *slot = carve<uint32_t>(p, S.cap);
  uint32_t *flags = carve<uint32_t>(p, S.cap);
  int2 *mnmx = carve<int2>(p, S.cap);
  LookupInfo *info = carve<LookupInfo>(p, S.cap);
  int *err = carve<int>(p, 1);
  if (host) {
    S.h_ptrs = ptrs; S.h_sizes = sizes; S.h_seqs = seqs; S.h_keys = keys;
    S.h_req = req; S.h_off = off; S.h_dst = dst; S.h_digests = digests;
    S.h_status = status; S.h_hdr = hdr; S.h_slot = slot; S.h_flags = flags;
    S.h_info = info; S.h_err = err;
    (void)eff_raw; (void)eff_q8; (void)mnmx; (void)hoff; (void)hdst;
  } else {
    S.ptrs = ptrs; S.sizes = sizes; S.seqs = seqs; S.keys = keys;
    S.req = req; S.off = off; S.dst = dst; S.eff_raw = eff_raw;
    S.eff_q8 = eff_q8; S.hoff = hoff; S.hdst = hdst; S.digests = digests; S.status = status; S.hdr = hdr;
    S.slot = slot; S.flags = flags; S.mnmx = mnmx; S.info = info;
    S.err = err;
  }
}

int ensure_scratch_of(Store &st, Scratch &sc, size_t n) {
  if (n <= sc.cap) return CASCADE_OK;
  size_t cap = std::max<size_t>(n, std::max<size_t>(1024, 2 * sc.cap));
  CB_CUDA(cudaStreamSynchronize(st.s));
  if (sc.dblob) cudaFree(sc.dblob);
  if (sc.hblob) cudaFreeHost(sc.hblob);
  sc = Scratch();
  size_t bytes = scratch_bytes(cap);
  CB_CUDA(cudaMalloc(&sc.dblob, bytes));
  CB_CUDA(cudaHostAlloc(&sc.hblob, bytes, cudaHostAllocDefault));
  sc.cap = cap;
  carve_all(sc, sc.dblob, false);
  carve_all(sc, sc.hblob, true);
  return CASCADE_OK;
}

int ensure_scratch(Store &st, size_t n) { return ensure_scratch_of(st, st.sc, n); }

int ensure_device_buf(uint8_t *&buf, size_t &cap, size_t need,
                      cudaStream_t s) {
  if (need <= cap) return CASCADE_OK;
  CB_CUDA(cudaStreamSynchronize(s));
  if (buf) CB_CUDA(cudaFree(buf));
  buf = nullptr;
  cap = 0;
  size_t c = std::max<size_t>(need, 1 << 20);
  CB_CUDA(cudaMalloc(&buf, c));
  cap = c;
  return CASCADE_OK;
}

int ensure_host_stage(Store &st, size_t need) {
  if (need <= st.h_stage_cap) return CASCADE_OK;
  CB_CUDA(cudaStreamSynchronize(st.s));
  if (st.h_stage) CB_CUDA(cudaFreeHost(st.h_stage));
  st.h_stage = nullptr;
  st.h_stage_cap = 0;
  size_t c = std::max<size_t>(need, 1 << 20);
  CB_CUDA(cudaHostAlloc(&st.h_stage, c, cudaHostAllocDefault));
  st.h_stage_cap = c;
  return CASCADE_OK;
}

// Free stacks exist for every class an allocation may use.
int ensure_stack(Store &st, int c) {
  if (st.stack_ptr[c]) return CASCADE_OK;
  uint64_t by_pool = st.pool_cap / class_bytes(c) + 1;
  uint64_t by_index = 2 * st.nslots;
  uint64_t cap = std::min(by_pool, by_index);
  if (cap > 0xffffffffull) cap = 0xffffffffull;
  uint64_t *d = nullptr;
  CB_CUDA(cudaMalloc(&d, cap * sizeof(uint64_t)));
  uint32_t cap32 = (uint32_t)cap;
  CB_CUDA(cudaMemcpyAsync(&st.d_pool->stack[c], &d, sizeof(d),
                          cudaMemcpyHostToDevice, st.s));
  CB_CUDA(cudaMemcpyAsync(&st.d_pool->cap[c], &cap32, sizeof(cap32),
                          cudaMemcpyHostToDevice, st.s));
  CB_CUDA(cudaStreamSynchronize(st.s));  // the sources live on this stack
  st.stack_ptr[c] = d;
  return CASCADE_OK;
}

int reset_pool(Store &st) {
  if (!st.hbm) return CASCADE_OK;
  PoolDev h;
  std::memset(&h, 0, sizeof(h));
  h.capacity = st.pool_cap;
  for (int c = 0; c < kNumClasses; ++c) {
    h.stack[c] = st.stack_ptr[c];
    if (st.stack_ptr[c]) {
      uint64_t cap = std::min(st.pool_cap / class_bytes(c) + 1, 2 * st.nslots);
      h.cap[c] = (uint32_t)std::min<uint64_t>(cap, 0xffffffffull);
    }
  }
  CB_CUDA(cudaMemcpyAsync(st.d_pool, &h, sizeof(h), cudaMemcpyHostToDevice,
                          st.s));
  CB_CUDA(cudaStreamSynchronize(st.s));
  return CASCADE_OK;
}

// Key of a block-id string (see cascade_store_key_of).  Synthetic keys live
// in the region k1 == ~0; a hex id falling there (or on the one unstorable
// key) is mapped through the name table as well, so no two ids share a key.
int key_of(Store &st, const char *id, bool create, Key *out, bool *known) {
  size_t len = std::strlen(id);
  *known = true;
  if (is_hex_id(id, len)) {
    uint8_t b[16];
    for (int i = 0; i < 16; ++i)
      b[i] = (uint8_t)(hexval(id[2 * i]) << 4 | hexval(id[2 * i + 1]));
    Key k{le64(b), le64(b + 8)};
    bool reserved = (k.k1 == ~0ull) || (k.k0 == kKeyMask0 && k.k1 == kKeyMask1);
    if (!reserved) { *out = k; return CASCADE_OK; }
  }
  std::string sid(id, len);
  auto it = st.names.find(sid);
  if (it != st.names.end()) { *out = it->second; return CASCADE_OK; }
  if (!create) { *known = false; return CASCADE_OK; }
  Key k{st.next_name++, ~0ull};
  st.names.emplace(std::move(sid), k);
  *out = k;
  return CASCADE_OK;
}

// Copies the kernel-side error word; non-zero aborts the operation.
int check_device_err(Store &st) {
  if (*st.sc.h_err) {
    set_error("device index is full: raise index_slots");
    return CASCADE_ERR_FULL;
  }
  return CASCADE_OK;
}

inline bool q8_eligible(const Store &st, uint64_t size, bool to_dram) {
  if (!st.cfg.kv_compression || size < 64) return false;
  return to_dram || st.cfg.gpu_q8;
}

inline uint64_t payload_bytes(uint64_t size, bool q8) {
  return q8 ? size / 2 : size;
}

// What the reference's ShmBackend accounts for a stored block: the
// compressed form is 8 + size/2 bytes (KVCompressor::compressed_size,
// cascade.hpp:357-359).
inline uint64_t dram_accounted(uint64_t size, bool q8) {
  return q8 ? 8 + size / 2 : size;
}

// Doubles the index and re-inserts every live slot.
int grow_index(Store &st);

}  // namespace

// Statistics and tier accounting for a finished put batch (sc.h_status,
// h_sizes, h_flags, h_off on the host), per CascadeStore::put.
constexpr uint8_t kRetry = 0xff;  // internal: placed again by a later pass

static void tally_put(Store &st, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const uint8_t r = st.sc.h_status[i];
    if (r == kRetry) continue;
    const uint64_t size = st.sc.h_sizes[i];
    const bool hit = (r == CASCADE_PUT_DUP_KNOWN || r == CASCADE_PUT_DUP_BATCH);
    if (hit && st.cfg.dedup_enabled) ++st.dedup_hits;
    // With dedup off a repeated id reaches the tier, whose put answers true
    // for an id it holds; the reference counts that as an SHM put when the
    // DRAM tier is the only tier (cascade_core.cpp:1108-1111).
    if (hit && !st.cfg.dedup_enabled && !st.hbm) ++st.shm_puts;
    // The reference compresses every block that passes the dedup check,
    // whatever tier then takes it (cascade_core.cpp:1086-1092).
    if (st.cfg.kv_compression && size >= 64 && !(hit && st.cfg.dedup_enabled))
      st.compression_savings += size - (8 + size / 2);
    if (r != CASCADE_PUT_STORED) {
      // A DRAM placement that did not become live gives its space back.
      if ((st.sc.h_flags[i] & kTierDram) && st.sc.h_off[i] != kInvalidOffset) {
        bool q8 = (st.sc.h_flags[i] & kFlagQ8) != 0;
        st.dram->free(st.sc.h_off[i], payload_bytes(size, q8));
      }
      continue;
    }
    ++st.claimed;
    if (st.sc.h_flags[i] & kTierHbm) {
      st.gpu_used += payload_bytes(size, (st.sc.h_flags[i] & kFlagQ8) != 0);
    } else {
      bool q8 = (st.sc.h_flags[i] & kFlagQ8) != 0;
      st.shm_used += dram_accounted(size, q8);
      if (i < st.demoted.size() && st.demoted[i])
        ++st.gpu_evictions;  // stored in HBM, then demoted, by serial puts
      else
        ++st.shm_puts;
    }
  }
  st.demoted.clear();
}


// ------------------------------------------------------------ DMA fan-out
// One copy between the device and the pinned DRAM arena.
struct Dma {
  void *dst;
  const void *src;
  uint64_t bytes;
};

// Spreads copies between the device and the DRAM tier over the store's copy
// streams of one direction (0: device to host, 1: host to device), as the
// reference spreads its transfers over a ring of streams
// (gpu_backend.cu:191-225): each copy goes to the stream with the fewest
// bytes queued.  The copies start after the work already on the main stream,
// and the main stream waits for all of them.
static int dma_fanout(Store &st, const std::vector<Dma> &jobs, int dir) {
  if (jobs.empty()) return CASCADE_OK;
  const cudaMemcpyKind kind =
      dir == 0 ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
  const int k = (int)std::min<size_t>(kDmaStreams, jobs.size());
  CB_CUDA(cudaEventRecord(st.dma_start, st.s));
  uint64_t load[kDmaStreams] = {};
  for (int q = 0; q < k; ++q)
    CB_CUDA(cudaStreamWaitEvent(st.dma[dir][q], st.dma_start, 0));
  for (const Dma &j : jobs) {
    if (!j.bytes) continue;
    int q = 0;
    for (int r = 1; r < k; ++r)
      if (load[r] < load[q]) q = r;
    CB_CUDA(cudaMemcpyAsync(j.dst, j.src, j.bytes, kind, st.dma[dir][q]));
    load[q] += j.bytes;
  }
  for (int q = 0; q < k; ++q) {
    CB_CUDA(cudaEventRecord(st.dma_done[dir][q], st.dma[dir][q]));
    CB_CUDA(cudaStreamWaitEvent(st.s, st.dma_done[dir][q], 0));
  }
  return CASCADE_OK;
}

// ------------------------------------------------------------- demotion
// HBM blocks leave for the DRAM tier least recently used first, prefix
// blocks last when semantic_eviction is on (GPUBackend::evict_for_space +
// evict_lru_semantic, gpu_backend.cu:432-487, called by
// CascadeStore::evict_gpu_to_shm, cascade_core.cpp:998-1018).  The
// reference takes the LRU tail of its largest index shard; here the order
// is by LRU epoch over the whole pool.  A demoted block keeps its index
// slot, which then points into the DRAM arena, and goes to DRAM in the DRAM
// tier's format (INT8 when kv_compression applies, compressed on the
// device; the reference demotes raw bytes).

// Demotion candidates per class (0: unprotected, 1: prefix), least recent
// first: the leading part of each class that the device selected.
struct Candidates {
  std::vector<ScanRec> c[2];
  bool complete[2] = {true, true};  // the whole class is listed
};

inline int victim_class(const Store &st, uint32_t flags) {
  return (st.cfg.semantic_eviction && st.cfg.dedup_enabled &&
          (flags & kFlagPrefix)) ? 1 : 0;
}

// The least recent candidates of each class whose HBM payloads add up to
// at least `budget` bytes (whole epoch buckets; every candidate when the
// class holds less): an epoch histogram on the device picks the buckets,
// and only their slots come back to the host.
static int select_candidates(Store &st, uint64_t budget, Candidates &out) {
  cudaStream_t s = st.s;
  constexpr size_t kHistBytes = 2 * kVictimBuckets * 8;
  constexpr size_t kCountBytes = 2 * kVictimBuckets * 4;
  constexpr size_t kRecBase = kHistBytes + kCountBytes + 256;
  int rc = ensure_device_buf(st.scan_d, st.scan_cap, kRecBase + 4096, s);
  if (rc) return rc;
  auto *d_bytes = reinterpret_cast<unsigned long long *>(st.scan_d);
  auto *d_count = reinterpret_cast<uint32_t *>(st.scan_d + kHistBytes);
  auto *d_n = reinterpret_cast<uint32_t *>(st.scan_d + kHistBytes + kCountBytes);
  const int semantic = st.cfg.semantic_eviction && st.cfg.dedup_enabled;
  const uint64_t span = std::max<uint64_t>(st.next_epoch, 1);
  if ((rc = launch_victim_hist(st.slots, st.nslots, semantic, span, d_bytes,
                               d_count, s)))
    return rc;
  std::vector<uint64_t> hb(2 * kVictimBuckets);
  std::vector<uint32_t> hc(2 * kVictimBuckets);
  CB_CUDA(cudaMemcpyAsync(hb.data(), d_bytes, kHistBytes, cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(hc.data(), d_count, kCountBytes, cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  int cut[2] = {-1, -1};
  size_t total = 0;
  for (int c = 0; c < 2; ++c) {
    uint64_t cum = 0;
    int last = -1;
    for (int b = 0; b < kVictimBuckets; ++b)
      if (hc[c * kVictimBuckets + b]) last = b;
    for (int b = 0; b <= last; ++b) {
      cum += hb[c * kVictimBuckets + b];
      total += hc[c * kVictimBuckets + b];
      cut[c] = b;
      if (cum >= budget) break;
    }
    out.complete[c] = cut[c] == last;
    out.c[c].clear();
  }
  if (total == 0) return CASCADE_OK;
  if ((rc = ensure_device_buf(st.scan_d, st.scan_cap,
                              kRecBase + total * sizeof(ScanRec), s)))
    return rc;
  d_n = reinterpret_cast<uint32_t *>(st.scan_d + kHistBytes + kCountBytes);
  ScanRec *d_recs = reinterpret_cast<ScanRec *>(st.scan_d + kRecBase);
  if ((rc = launch_victim_collect(st.slots, st.nslots, semantic, span, cut[0],
                                  cut[1], d_n, d_recs, (uint32_t)total, s)))
    return rc;
  std::vector<ScanRec> recs(total);
  uint32_t got = 0;
  CB_CUDA(cudaMemcpyAsync(&got, d_n, 4, cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(recs.data(), d_recs, total * sizeof(ScanRec),
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  CB_CHECK(got == total, CASCADE_ERR_CUDA,
           "demotion candidates changed between histogram and collection");
  for (const ScanRec &r : recs) out.c[victim_class(st, r.flags)].push_back(r);
  for (int c = 0; c < 2; ++c)
    std::sort(out.c[c].begin(), out.c[c].end(),
              [](const ScanRec &a, const ScanRec &b) {
                return a.epoch != b.epoch ? a.epoch < b.epoch : a.slot < b.slot;
              });
  return CASCADE_OK;
}

// A block that leaves HBM, with its DRAM space already allocated.
struct Demotion {
  ScanRec r;
  uint64_t dram_off;
  bool dq8;  // DRAM format: INT8
};

// Returns arena space on every path that does not hand it to the index.
struct ArenaGuard {
  DramArena *arena;
  std::vector<std::pair<uint64_t, uint64_t>> held;  // offset, bytes
  ~ArenaGuard() {
    for (auto &h : held) arena->free(h.first, h.second);
  }
  void keep() { held.clear(); }
};

// Moves `vic` from HBM to their DRAM places: INT8 forms of raw victims on
// the device, payloads to the arena over the copy streams, slots relocated,
// pool space returned.  Counts them as gpu_evictions.  On return `vic` is
// reordered and carries each block's DRAM-format header.
static int demote(Store &st, std::vector<Demotion> &vic) {
  if (vic.empty()) return CASCADE_OK;
  ArenaGuard guard{st.dram.get(), {}};
  for (const Demotion &v : vic)
    guard.held.emplace_back(v.dram_off, payload_bytes(v.r.size, v.dq8));
  cudaStream_t s = st.s;
  // raw blocks that become INT8 first: their quantise outputs index 0..nq-1
  std::stable_partition(vic.begin(), vic.end(), [](const Demotion &v) {
    return v.dq8 && !(v.r.flags & kFlagQ8);
  });
  size_t nq = 0;
  while (nq < vic.size() && vic[nq].dq8 && !(vic[nq].r.flags & kFlagQ8)) ++nq;
  const size_t k = vic.size();
  Scratch &oc = st.oc;
  int rc = ensure_scratch_of(st, oc, k);
  if (rc) return rc;
  const uint64_t pool = (uint64_t)(uintptr_t)st.pool;
  std::vector<uint64_t> so(nq);
  uint64_t stage_bytes = 0, max_size = 0;
  for (size_t j = 0; j < nq; ++j) {
    so[j] = stage_bytes;
    stage_bytes += (payload_bytes(vic[j].r.size, true) + 255) & ~uint64_t(255);
    max_size = std::max<uint64_t>(max_size, vic[j].r.size);
  }
  if (nq) {
    if ((rc = ensure_device_buf(st.d_evstage, st.d_evstage_cap, stage_bytes, s)))
      return rc;
    for (size_t j = 0; j < nq; ++j) {
      oc.h_ptrs[j] = pool + vic[j].r.offset;
      oc.h_sizes[j] = vic[j].r.size;
      oc.h_dst[j] = (uint64_t)(uintptr_t)(st.d_evstage + so[j]);
    }
    CB_CUDA(cudaMemcpyAsync(oc.ptrs, oc.h_ptrs, nq * 8, cudaMemcpyHostToDevice, s));
    CB_CUDA(cudaMemcpyAsync(oc.sizes, oc.h_sizes, nq * 8, cudaMemcpyHostToDevice, s));
    CB_CUDA(cudaMemcpyAsync(oc.dst, oc.h_dst, nq * 8, cudaMemcpyHostToDevice, s));
    rc = launch_minmax(oc.ptrs, oc.sizes, (int)nq, max_size, oc.mnmx, s);
    if (!rc) rc = launch_quantize(oc.ptrs, oc.sizes, (int)nq, max_size, oc.mnmx,
                                  oc.dst, oc.hdr, 0, s);
    if (rc) return rc;
  }
  std::vector<Dma> jobs;
  jobs.reserve(k);
  for (size_t j = 0; j < k; ++j) {
    const Demotion &v = vic[j];
    const void *src = j < nq ? (const void *)(st.d_evstage + so[j])
                             : (const void *)(uintptr_t)(pool + v.r.offset);
    jobs.push_back({st.dram->ptr(v.dram_off), src,
                    payload_bytes(v.r.size, v.dq8)});
  }
  if ((rc = dma_fanout(st, jobs, 0))) return rc;
  uint64_t freed = 0, acc_total = 0;
  for (size_t j = 0; j < k; ++j) {
    const Demotion &v = vic[j];
    const bool hq8 = (v.r.flags & kFlagQ8) != 0;
    oc.h_slot[j] = v.r.slot;
    oc.h_off[j] = v.dram_off;
    oc.h_flags[j] = (v.r.flags & (kFlagPrefix | kFlagHeld | 0xff0000u)) |
                    kTierDram | (v.dq8 ? kFlagQ8 : 0);
    oc.h_req[j] = payload_bytes(v.r.size, hq8);
    oc.h_seqs[j] = v.r.offset;
    uint8_t *h = oc.h_hdr + 8 * j;
    std::memcpy(h, &v.r.hdr_scale, 4);
    h[4] = (uint8_t)v.r.hdr_zp;
    h[5] = h[6] = h[7] = 0;
    freed += payload_bytes(v.r.size, hq8);
    acc_total += dram_accounted(v.r.size, v.dq8);
  }
  CB_CUDA(cudaMemcpyAsync(oc.slot, oc.h_slot, k * 4, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(oc.off, oc.h_off, k * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(oc.flags, oc.h_flags, k * 4, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(oc.req, oc.h_req, k * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(oc.seqs, oc.h_seqs, k * 8, cudaMemcpyHostToDevice, s));
  if (k > nq)  // headers of blocks already INT8 (the others come from quantise)
    CB_CUDA(cudaMemcpyAsync(oc.hdr + 8 * nq, oc.h_hdr + 8 * nq, (k - nq) * 8,
                            cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemsetAsync(oc.status, CASCADE_PUT_FAILED, k, s));
  rc = launch_index_relocate(st.slots, oc.slot, oc.off, oc.flags, oc.hdr,
                             (int)k, s);
  if (!rc) rc = launch_pool_free_unstored(st.d_pool, oc.req, oc.seqs,
                                          oc.status, (int)k, s);
  if (rc) return rc;
  if (nq)  // the headers the quantise wrote, for the caller's records
    CB_CUDA(cudaMemcpyAsync(oc.h_hdr, oc.hdr, nq * 8, cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  for (size_t j = 0; j < nq; ++j) {
    std::memcpy(&vic[j].r.hdr_scale, oc.h_hdr + 8 * j, 4);
    vic[j].r.hdr_zp = oc.h_hdr[8 * j + 4];
  }
  guard.keep();
  st.gpu_used -= freed;
  st.shm_used += acc_total;
  st.gpu_evictions += k;
  return CASCADE_OK;
}

// A block entering HBM within a batch, in the order of the serial calls.
struct Arrival {
  uint64_t size;  // logical size
  uint64_t pay;   // HBM payload bytes
  int cls;        // demotion class
  bool put;       // a put (else the promotion of a DRAM block)
  uint64_t acc;   // promotion: the DRAM bytes accounted to the block now
};

// Where an arrival ends after the batch.
enum Fate : uint8_t {
  kFateHbm = 0,      // in HBM
  kFateEvicted = 1,  // entered HBM, then left for DRAM within the batch
  kFateDram = 2,     // a put that went to the DRAM tier directly
  kFateNone = 3,     // no HBM and (put) no DRAM room: the put fails;
                     // a promotion leaves the block where it is
};

struct Replay {
  std::vector<uint8_t> fate;
  std::vector<uint64_t> off;  // DRAM offset (kFateEvicted puts, kFateDram)
  std::vector<uint8_t> dq8;   // DRAM format of those
  std::vector<Demotion> old;  // older blocks demoted, in order
  bool need_more = false;     // a class ran past its selected candidates
};

// Replays the serial puts / promotions of a batch (CascadeStore::put,
// cascade_core.cpp:1097-1118, and promote_to_gpu, 1039-1056): an arrival
// that does not fit demotes blocks until it has freed its own size -- older
// blocks of class 0, then the batch's own class-0 arrivals already in HBM
// in arrival order, then the same for class 1 -- and takes HBM if it then
// fits; a put that gets no HBM goes to the DRAM tier while it has room.
// Every demotion needs DRAM room (accounted bytes and arena space); a
// demotion that finds none ends that arrival's demotions (the block stays
// in HBM; nothing is dropped).  DRAM space is allocated here, in the serial
// order; with need_more set, all of it is given back.
static void replay(Store &st, const std::vector<Arrival> &arr,
                   const Candidates &cand, bool allow_hbm, Replay &out) {
  const size_t n = arr.size();
  out.fate.assign(n, kFateNone);
  out.off.assign(n, kInvalidOffset);
  out.dq8.assign(n, 0);
  out.old.clear();
  out.need_more = false;
  uint64_t used = st.gpu_used, shm = st.shm_used;
  const uint64_t cap = st.pool_cap;
  const uint64_t dcap = st.dram_tier ? st.dram->capacity() : 0;
  std::vector<std::pair<uint64_t, uint64_t>> allocs;
  auto alloc = [&](uint64_t size, bool q8) {
    const uint64_t off = st.dram->alloc(payload_bytes(size, q8));
    if (off != DramArena::kNone) allocs.emplace_back(off, payload_bytes(size, q8));
    return off;
  };
  size_t oi[2] = {0, 0};
  std::deque<size_t> fresh[2];
  const bool hbm = allow_hbm && st.hbm;
  for (size_t j = 0; j < n; ++j) {
    const Arrival &a = arr[j];
    if (hbm && st.dram_tier && used + a.pay > cap) {
      uint64_t freed = 0;
      while (freed < a.pay) {
        int cls = -1;
        bool old = false;
        for (int c = 0; c < 2 && cls < 0; ++c) {
          if (oi[c] < cand.c[c].size()) {
            cls = c;
            old = true;
          } else if (!cand.complete[c]) {
            out.need_more = true;
            for (auto &h : allocs) st.dram->free(h.first, h.second);
            return;
          } else if (!fresh[c].empty()) {
            cls = c;
          }
        }
        if (cls < 0) break;
        if (old) {
          const ScanRec &r = cand.c[cls][oi[cls]];
          const bool hq8 = (r.flags & kFlagQ8) != 0;
          const bool dq8 = hq8 || q8_eligible(st, r.size, true);
          const uint64_t acc = dram_accounted(r.size, dq8);
          if (shm + acc > dcap) break;
          const uint64_t off = alloc(r.size, dq8);
          if (off == DramArena::kNone) break;
          out.old.push_back({r, off, dq8});
          ++oi[cls];
          used -= payload_bytes(r.size, hq8);
          freed += payload_bytes(r.size, hq8);
          shm += acc;
        } else {
          const size_t k = fresh[cls].front();
          const Arrival &b = arr[k];
          uint64_t acc = b.acc;
          if (b.put) {
            const bool dq8 = q8_eligible(st, b.size, true);
            acc = dram_accounted(b.size, dq8);
            if (shm + acc > dcap) break;
            const uint64_t off = alloc(b.size, dq8);
            if (off == DramArena::kNone) break;
            out.off[k] = off;
            out.dq8[k] = dq8;
          } else if (shm + acc > dcap) {
            break;
          }
          fresh[cls].pop_front();
          out.fate[k] = kFateEvicted;
          used -= b.pay;
          freed += b.pay;
          shm += acc;
        }
      }
    }
    if (hbm && used + a.pay <= cap) {
      out.fate[j] = kFateHbm;
      used += a.pay;
      fresh[a.cls].push_back(j);
      if (!a.put) shm -= a.acc;
      continue;
    }
    if (a.put && st.dram_tier) {
      const bool dq8 = q8_eligible(st, a.size, true);
      const uint64_t acc = dram_accounted(a.size, dq8);
      if (shm + acc <= dcap) {
        const uint64_t off = alloc(a.size, dq8);
        if (off != DramArena::kNone) {
          out.fate[j] = kFateDram;
          out.off[j] = off;
          out.dq8[j] = dq8;
          shm += acc;
        }
      }
    }
  }
}

// Candidates enough for the batch, then the replay (more candidates if the
// replay ran past them).  `deficit`: the HBM bytes the batch needs beyond
// the free room if every arrival took HBM.
static int plan_batch(Store &st, const std::vector<Arrival> &arr,
                      bool allow_hbm, Replay &out) {
  Candidates cand;
  uint64_t need = 0;
  for (const Arrival &a : arr) need += a.pay;
  const bool may_demote = allow_hbm && st.hbm && st.dram_tier &&
                          st.gpu_used + need > st.pool_cap;
  uint64_t budget = 0;
  if (may_demote) {
    const uint64_t deficit = st.gpu_used + need - st.pool_cap;
    budget = deficit + deficit / 2 + (16ull << 20);
  }
  for (;;) {
    if (may_demote) {
      int rc = select_candidates(st, budget, cand);
      if (rc) return rc;
    }
    replay(st, arr, cand, allow_hbm, out);
    if (!out.need_more) return CASCADE_OK;
    budget = ~0ull;  // every candidate
  }
}

// ----------------------------------------------------------------- put
// Core of every put: the inputs (device addresses, sizes, sequence numbers,
// keys or digests) are already in st.sc on the device.
//   use_digests: keys are sc.digests (stride 4) instead of sc.keys.
//   h_prefix: per-block is_prefix or null.
// On return st.sc.h_status holds the final per-block status.
static int put_placed(Store &st, size_t n, bool use_digests,
                      const uint8_t *h_prefix, uint64_t max_size,
                      bool allow_hbm) {
  cudaStream_t s = st.s;
  const uint64_t *keys = use_digests
                             ? reinterpret_cast<const uint64_t *>(st.sc.digests)
                             : st.sc.keys;
  const int stride = use_digests ? 4 : 2;
  if (st.claimed + n > st.nslots / 2) {
    int rc = grow_index(st);
    if (rc) return rc;
  }
  CB_CUDA(cudaMemsetAsync(st.sc.err, 0, sizeof(int), s));
  int rc = launch_index_claim(st.slots, st.nslots - 1, keys, stride,
                              st.sc.seqs, (int)n, st.sc.slot, st.sc.err, s);
  if (!rc) rc = launch_index_resolve(st.slots, st.sc.slot, st.sc.seqs, (int)n,
                                     st.sc.status, s);
  if (rc) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_status, st.sc.status, n,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_err, st.sc.err, sizeof(int),
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  if ((rc = check_device_err(st))) return rc;

  // Placement: the batch's serial puts replayed (plan_batch): HBM first,
  // older blocks demoted to make room (cascade_core.cpp:1097-1105), the
  // DRAM tier for the rest while its capacity holds (1108-1118), FAILED
  // when neither has room (the Lustre tier of 1121-1124 is not part of this
  // library).  Only the end state is written: a block that serial puts
  // would store in HBM and demote within the batch goes to DRAM directly.
  std::vector<Arrival> arr;
  for (size_t i = 0; i < n; ++i) {
    if (st.sc.h_status[i] != CASCADE_PUT_STORED) continue;
    const uint64_t size = st.sc.h_sizes[i];
    const bool pre = h_prefix && h_prefix[i] && st.cfg.dedup_enabled;
    arr.push_back({size, payload_bytes(size, st.hbm && q8_eligible(st, size, false)),
                   victim_class(st, pre ? kFlagPrefix : 0u), true, 0});
  }
  Replay plan;
  if ((rc = plan_batch(st, arr, allow_hbm, plan))) return rc;
  ArenaGuard arena{st.dram.get(), {}};  // the batch's DRAM space, until placed
  for (size_t j = 0; j < arr.size(); ++j)
    if (plan.fate[j] == kFateEvicted || plan.fate[j] == kFateDram)
      arena.held.emplace_back(plan.off[j],
                              payload_bytes(arr[j].size, plan.dq8[j]));
  if ((rc = demote(st, plan.old))) return rc;
  uint64_t q8stage_bytes = 0;
  std::vector<size_t> dram_raw, dram_q8;
  std::vector<uint64_t> q8stage_off;
  bool any_hbm = false, any_hbm_raw = false, any_q8 = false;
  st.demoted.assign(n, 0);
  for (size_t i = 0, j = 0; i < n; ++i) {
    st.sc.h_req[i] = kNoRequest;
    st.sc.h_off[i] = kInvalidOffset;
    st.sc.h_dst[i] = 0;
    const uint64_t size = st.sc.h_sizes[i];
    uint32_t prefix =
        (h_prefix && h_prefix[i] && st.cfg.dedup_enabled) ? kFlagPrefix : 0;
    st.sc.h_flags[i] = prefix;
    if (st.sc.h_status[i] != CASCADE_PUT_STORED) continue;
    const size_t k = j++;
    const uint8_t fate = plan.fate[k];
    if (fate == kFateHbm) {
      const bool q8 = st.hbm && q8_eligible(st, size, false);
      st.sc.h_req[i] = payload_bytes(size, q8);
      st.sc.h_flags[i] |= kTierHbm | (q8 ? kFlagQ8 : 0);
      any_hbm = true;
      any_q8 |= q8;
      any_hbm_raw |= !q8;
    } else if (fate == kFateEvicted || fate == kFateDram) {
      const bool q8 = plan.dq8[k] != 0;
      st.sc.h_off[i] = plan.off[k];
      st.sc.h_flags[i] |= kTierDram | (q8 ? kFlagQ8 : 0);
      st.demoted[i] = fate == kFateEvicted;
      if (q8) {
        any_q8 = true;
        dram_q8.push_back(i);
        q8stage_off.push_back(q8stage_bytes);
        q8stage_bytes += (payload_bytes(size, true) + 255) & ~uint64_t(255);
      } else {
        dram_raw.push_back(i);
      }
    }
    // kFateNone: req = none and no offset -> FAILED.
  }
  if (!dram_q8.empty()) {
    if ((rc = ensure_device_buf(st.d_q8stage, st.d_q8stage_cap, q8stage_bytes,
                                s)))
      return rc;
    for (size_t k = 0; k < dram_q8.size(); ++k)
      st.sc.h_dst[dram_q8[k]] = (uint64_t)(uintptr_t)(st.d_q8stage + q8stage_off[k]);
  }
  if (any_hbm) {
    for (size_t i = 0; i < n; ++i)
      if (st.sc.h_req[i] != kNoRequest)
        if ((rc = ensure_stack(st, size_class(std::max<uint64_t>(st.sc.h_req[i], 1)))))
          return rc;
  }
  // Host decisions to the device: requests, DRAM offsets, staging
  // destinations and flags.
  CB_CUDA(cudaMemcpyAsync(st.sc.req, st.sc.h_req, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.hoff, st.sc.h_off, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.hdst, st.sc.h_dst, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.flags, st.sc.h_flags, n * 4, cudaMemcpyHostToDevice, s));
  const int nb = (int)((n + 255) / 256);
  if (any_hbm) {
    rc = launch_pool_alloc(st.d_pool, st.sc.req, (int)n, st.sc.off, s);
    if (rc) return rc;
  }
  prepare_kernel<<<nb, 256, 0, s>>>((int)n, st.sc.req, st.sc.off, st.sc.hoff,
                                    st.sc.hdst, st.sc.flags, st.sc.sizes,
                                    (uint64_t)(uintptr_t)st.pool, st.sc.dst,
                                    st.sc.eff_raw, st.sc.eff_q8);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  // Payloads.  INT8: min/max then quantise with the header kept apart (it
  // goes into the index slot).  Raw HBM: one batched copy.
  if (any_q8) {
    rc = launch_minmax(st.sc.ptrs, st.sc.eff_q8, (int)n, max_size, st.sc.mnmx, s);
    if (!rc) rc = launch_quantize(st.sc.ptrs, st.sc.eff_q8, (int)n, max_size,
                                  st.sc.mnmx, st.sc.dst, st.sc.hdr, 0, s);
  }
  if (!rc && any_hbm_raw)
    rc = launch_copy(st.sc.ptrs, st.sc.dst, st.sc.eff_raw, (int)n, max_size, s);
  if (rc) return rc;
  // DRAM placements leave the device by DMA into the pinned arena.
  std::vector<Dma> jobs;
  for (size_t k = 0; k < dram_q8.size(); ++k) {
    const size_t i = dram_q8[k];
    jobs.push_back({st.dram->ptr(st.sc.h_off[i]), st.d_q8stage + q8stage_off[k],
                    payload_bytes(st.sc.h_sizes[i], true)});
  }
  for (size_t i : dram_raw)
    jobs.push_back({st.dram->ptr(st.sc.h_off[i]),
                    reinterpret_cast<const void *>(st.sc.h_ptrs[i]),
                    st.sc.h_sizes[i]});
  if ((rc = dma_fanout(st, jobs, 0))) return rc;
  const uint64_t epoch = st.next_epoch;
  st.next_epoch += n;
  rc = launch_index_commit(st.slots, st.sc.slot, st.sc.status, st.sc.off,
                           st.sc.sizes, st.sc.flags, st.sc.hdr, epoch, (int)n, s);
  if (!rc) rc = launch_index_finalize(st.slots, st.sc.slot, st.sc.off,
                                      st.sc.status, (int)n, s);
  if (rc) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_status, st.sc.status, n,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_off, st.sc.off, n * 8,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  arena.keep();  // the index (or tally_put, for blocks that failed) owns it
  return CASCADE_OK;
}

// Hands a finished batch's statuses (and digests) to the caller.
static int finish_put(Store &st, size_t n, bool content_addressed,
                      uint8_t *h_status, uint8_t *h_digests,
                      uint64_t *n_stored) {
  if (h_digests && content_addressed) {
    CB_CUDA(cudaMemcpyAsync(st.sc.h_digests, st.sc.digests, 32 * n,
                            cudaMemcpyDeviceToHost, st.s));
    CB_CUDA(cudaStreamSynchronize(st.s));
    std::memcpy(h_digests, st.sc.h_digests, 32 * n);
  }
  uint64_t ok = 0;
  for (size_t i = 0; i < n; ++i) {
    if (st.sc.h_status[i] != CASCADE_PUT_FAILED) ++ok;
    if (h_status) h_status[i] = st.sc.h_status[i];
  }
  if (n_stored) *n_stored = ok;
  return CASCADE_OK;
}

// Copies the batch description into the scratch arrays and to the device
// (main stream): addresses, sizes, sequence numbers and, when given, keys.
static int upload_batch(Store &st, size_t n, const uint64_t *h_ptrs,
                        const uint64_t *h_sizes, const uint8_t *h_keys,
                        uint64_t *max_size) {
  int rc = ensure_scratch(st, n);
  if (rc) return rc;
  cudaStream_t s = st.s;
  uint64_t mx = 0;
  for (size_t i = 0; i < n; ++i) {
    st.sc.h_ptrs[i] = h_ptrs[i];
    st.sc.h_sizes[i] = h_sizes[i];
    st.sc.h_seqs[i] = st.next_seq + i;
    mx = std::max(mx, h_sizes[i]);
    if (h_keys) {
      uint64_t k0 = le64(h_keys + 16 * i), k1 = le64(h_keys + 16 * i + 8);
      CB_CHECK(!(k0 == kKeyMask0 && k1 == kKeyMask1), CASCADE_ERR_INVALID,
               "key equals the index's reserved mask value");
      st.sc.h_keys[2 * i] = k0;
      st.sc.h_keys[2 * i + 1] = k1;
    }
  }
  st.next_seq += n;
  CB_CUDA(cudaMemcpyAsync(st.sc.ptrs, st.sc.h_ptrs, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.sizes, st.sc.h_sizes, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.seqs, st.sc.h_seqs, n * 8, cudaMemcpyHostToDevice, s));
  if (h_keys)
    CB_CUDA(cudaMemcpyAsync(st.sc.keys, st.sc.h_keys, n * 16, cudaMemcpyHostToDevice, s));
  *max_size = mx;
  return CASCADE_OK;
}

// True when every block of a content-addressed batch can be given an HBM
// slot before its digest is known (the HBM tier takes all of them even if
// none is a duplicate).
static bool can_speculate(const Store &st, size_t n) {
  if (!st.hbm) return false;
  uint64_t need = 0;
  for (size_t i = 0; i < n; ++i) {
    const uint64_t size = st.sc.h_sizes[i];
    need += payload_bytes(size, q8_eligible(st, size, false));
  }
  return st.gpu_used + need <= st.pool_cap;
}

// Content-addressed put with the hash off the critical path: every block
// gets an HBM slot and its payload (INT8 codes or a copy) on the main
// stream while SHA-256 runs on the hash stream; when the digests are in,
// the index decides winners and the slots of duplicates are freed.  The
// result is the same as hashing first (the index sees the same keys in the
// same sequence order); only the order of device work differs.
// `digests_ready`: the caller already hashed on s2 and recorded ev2.
// First half of the speculative put: plan every block into HBM, start the
// hash on s2 (unless the caller did, `digests_ready`), allocate the slots
// and write the payloads on the main stream.  ev2 marks the digests.
static int speculate_local(Store &st, size_t n, const uint8_t *h_prefix,
                           uint64_t max_size, bool digests_ready,
                           bool beside_hash = true) {
  cudaStream_t s = st.s;
  bool any_q8 = false, any_raw = false;
  for (size_t i = 0; i < n; ++i) {
    const uint64_t size = st.sc.h_sizes[i];
    const bool q8 = q8_eligible(st, size, false);
    st.sc.h_req[i] = payload_bytes(size, q8);
    st.sc.h_off[i] = kInvalidOffset;
    st.sc.h_dst[i] = 0;
    st.sc.h_flags[i] = kTierHbm | (q8 ? kFlagQ8 : 0) |
                       ((h_prefix && h_prefix[i] && st.cfg.dedup_enabled)
                            ? kFlagPrefix : 0);
    any_q8 |= q8;
    any_raw |= !q8;
    int rc = ensure_stack(st, size_class(std::max<uint64_t>(st.sc.h_req[i], 1)));
    if (rc) return rc;
  }
  if (st.claimed + n > st.nslots / 2) {
    int rc = grow_index(st);
    if (rc) return rc;
  }
  CB_CUDA(cudaMemcpyAsync(st.sc.req, st.sc.h_req, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.hoff, st.sc.h_off, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.hdst, st.sc.h_dst, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.flags, st.sc.h_flags, n * 4, cudaMemcpyHostToDevice, s));
  int rc;
  if (!digests_ready) {  // hash on s2 as soon as the descriptors are there
    CB_CUDA(cudaEventRecord(st.ev, s));
    CB_CUDA(cudaStreamWaitEvent(st.s2, st.ev, 0));
    rc = launch_sha256(st.sc.ptrs, st.sc.sizes, (int)n, st.sc.digests, st.s2);
    if (rc) return rc;
    CB_CUDA(cudaEventRecord(st.ev2, st.s2));
  }
  rc = launch_pool_alloc(st.d_pool, st.sc.req, (int)n, st.sc.off, s);
  if (rc) return rc;
  const int nb = (int)((n + 255) / 256);
  prepare_kernel<<<nb, 256, 0, s>>>((int)n, st.sc.req, st.sc.off, st.sc.hoff,
                                    st.sc.hdst, st.sc.flags, st.sc.sizes,
                                    (uint64_t)(uintptr_t)st.pool, st.sc.dst,
                                    st.sc.eff_raw, st.sc.eff_q8);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  // These run while the hash is still running.  When the hash launch fills
  // its SMs, an unused shared-memory request keeps them on the spare SMs,
  // so they take no issue slots from the serial chains.  With two hash
  // CTAs per SM they share the SMs (the spare SMs alone fall behind).
  const size_t pad = beside_hash ? sha256_neighbour_smem((int)n) : 0;
  if (any_q8) {
    rc = launch_minmax(st.sc.ptrs, st.sc.eff_q8, (int)n, max_size, st.sc.mnmx,
                       s, pad);
    if (!rc) rc = launch_quantize(st.sc.ptrs, st.sc.eff_q8, (int)n, max_size,
                                  st.sc.mnmx, st.sc.dst, st.sc.hdr, 0, s, pad);
  }
  if (!rc && any_raw)
    rc = launch_copy(st.sc.ptrs, st.sc.dst, st.sc.eff_raw, (int)n, max_size, s,
                     pad);
  return rc;
}

static int put_speculative(Store &st, size_t n, const uint8_t *h_prefix,
                           uint64_t max_size, bool digests_ready) {
  cudaStream_t s = st.s;
  int rc = speculate_local(st, n, h_prefix, max_size, digests_ready);
  if (rc) return rc;
  // The digests decide who stores.
  CB_CUDA(cudaStreamWaitEvent(s, st.ev2, 0));
  CB_CUDA(cudaMemsetAsync(st.sc.err, 0, sizeof(int), s));
  const uint64_t *keys = reinterpret_cast<const uint64_t *>(st.sc.digests);
  const uint64_t epoch = st.next_epoch;
  st.next_epoch += n;
  rc = launch_index_claim(st.slots, st.nslots - 1, keys, 4, st.sc.seqs, (int)n,
                          st.sc.slot, st.sc.err, s);
  if (!rc) rc = launch_index_resolve(st.slots, st.sc.slot, st.sc.seqs, (int)n,
                                     st.sc.status, s);
  if (!rc) rc = launch_index_commit(st.slots, st.sc.slot, st.sc.status,
                                    st.sc.off, st.sc.sizes, st.sc.flags,
                                    st.sc.hdr, epoch, (int)n, s);
  if (!rc) rc = launch_index_finalize(st.slots, st.sc.slot, st.sc.off,
                                      st.sc.status, (int)n, s);
  if (!rc) rc = launch_pool_free_unstored(st.d_pool, st.sc.req, st.sc.off,
                                          st.sc.status, (int)n, s);
  if (rc) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_status, st.sc.status, n,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_off, st.sc.off, n * 8,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_err, st.sc.err, sizeof(int),
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  return check_device_err(st);
}

// Runs a put batch whose description upload_batch() has placed on the
// device, then accounts for it.
//   mode 0: content-addressed with HBM room for every block: speculative
//           (the hash overlaps the payload work);
//   mode 1: tiered placement (HBM while it has room, then DRAM);
//   mode 2: tiered placement without HBM.
// Blocks whose HBM slot could not be allocated (the size classes are
// fuller than the byte count says) are placed again by the next mode, as
// the reference falls back to the SHM tier when the GPU put fails
// (cascade_core.cpp:1097-1118).  On return sc.h_status holds the final
// per-block status.
static int put_uploaded(Store &st, size_t n, bool content_addressed,
                        const uint8_t *h_prefix, uint64_t max_size,
                        bool digests_ready, int mode = -1) {
  int rc;
  st.demoted.clear();
  if (mode < 0) mode = (content_addressed && can_speculate(st, n)) ? 0 : 1;
  if (mode == 0) {
    if ((rc = put_speculative(st, n, h_prefix, max_size, digests_ready)))
      return rc;
  } else {
    if (content_addressed) {
      if (digests_ready) {
        CB_CUDA(cudaStreamWaitEvent(st.s, st.ev2, 0));
      } else {
        rc = launch_sha256(st.sc.ptrs, st.sc.sizes, (int)n, st.sc.digests, st.s);
        if (rc) return rc;
      }
    }
    if ((rc = put_placed(st, n, content_addressed, h_prefix, max_size,
                         mode == 1)))
      return rc;
  }
  // A failed HBM allocation sends every failed block of the batch to the
  // next mode, duplicates of a failed block included (they follow it).
  std::vector<size_t> retry;
  bool hbm_alloc_failed = false;
  for (size_t i = 0; i < n; ++i)
    hbm_alloc_failed |= st.sc.h_status[i] == CASCADE_PUT_FAILED &&
                        (st.sc.h_flags[i] & kTierHbm) &&
                        st.sc.h_off[i] == kInvalidOffset;
  const bool can_retry =
      hbm_alloc_failed && (mode == 0 || (mode == 1 && st.dram_tier));
  for (size_t i = 0; can_retry && i < n; ++i)
    if (st.sc.h_status[i] == CASCADE_PUT_FAILED) retry.push_back(i);
  if (retry.empty()) {
    tally_put(st, n);
    return CASCADE_OK;
  }
  // Keys of the blocks to place again: digest bytes 0..15 or the given keys.
  std::vector<uint8_t> keys;
  if (content_addressed) {
    CB_CUDA(cudaMemcpyAsync(st.sc.h_digests, st.sc.digests, 32 * n,
                            cudaMemcpyDeviceToHost, st.s));
    CB_CUDA(cudaStreamSynchronize(st.s));
  }
  std::vector<uint64_t> ptrs, sizes;
  std::vector<uint8_t> pre;
  for (size_t i : retry) {
    uint8_t k[16];
    if (content_addressed) {
      std::memcpy(k, st.sc.h_digests + 32 * i, 16);
    } else {
      for (int b = 0; b < 8; ++b) {
        k[b] = (uint8_t)(st.sc.h_keys[2 * i] >> (8 * b));
        k[8 + b] = (uint8_t)(st.sc.h_keys[2 * i + 1] >> (8 * b));
      }
    }
    keys.insert(keys.end(), k, k + 16);
    ptrs.push_back(st.sc.h_ptrs[i]);
    sizes.push_back(st.sc.h_sizes[i]);
    pre.push_back(h_prefix ? h_prefix[i] : 0);
    st.sc.h_status[i] = kRetry;
  }
  tally_put(st, n);
  // The sub-batch overwrites the scratch arrays; keep this batch's view.
  std::vector<uint8_t> status(st.sc.h_status, st.sc.h_status + n);
  std::vector<uint64_t> all_ptrs(st.sc.h_ptrs, st.sc.h_ptrs + n);
  std::vector<uint64_t> all_sizes(st.sc.h_sizes, st.sc.h_sizes + n);
  const size_t m = retry.size();
  uint64_t mx = 0;
  if ((rc = upload_batch(st, m, ptrs.data(), sizes.data(), keys.data(), &mx)))
    return rc;
  if ((rc = put_uploaded(st, m, false, pre.data(), mx, false, mode + 1)))
    return rc;
  for (size_t k = 0; k < m; ++k) status[retry[k]] = st.sc.h_status[k];
  std::memcpy(st.sc.h_status, status.data(), n);
  std::memcpy(st.sc.h_ptrs, all_ptrs.data(), 8 * n);
  std::memcpy(st.sc.h_sizes, all_sizes.data(), 8 * n);
  return CASCADE_OK;
}

// Uploads the batch description and runs the put.  When h_keys is null the
// blocks are content-addressed: the SHA-256 digests are the keys.  h_ptrs
// are device addresses.
static int put_batch_locked(Store &st, size_t n, const uint64_t *h_ptrs,
                            const uint64_t *h_sizes, const uint8_t *h_keys,
                            const uint8_t *h_prefix, uint8_t *h_status,
                            uint8_t *h_digests, uint64_t *n_stored) {
  uint64_t max_size = 0;
  int rc = upload_batch(st, n, h_ptrs, h_sizes, h_keys, &max_size);
  if (!rc) rc = put_uploaded(st, n, h_keys == nullptr, h_prefix, max_size, false);
  if (rc) return rc;
  return finish_put(st, n, h_keys == nullptr, h_status, h_digests, n_stored);
}

// KVCacheStore.store for a batch of keyed KV caches whose wire blocks all
// fit the HBM pool as raw payloads: the speculative put's allocation and
// index steps with the serialise kernel as the payload writer, so each
// cache is written once, straight into its pool slot.  Blocks whose slot
// could not be allocated (size-class rounding) are serialised into the
// KV staging buffer and placed again by the tiered path, as put_uploaded
// places them.  Returns CASCADE_ERR_UNSUPPORTED, having done nothing, when
// the batch does not qualify (no HBM tier, INT8 payloads, or no room).
static int put_kv_locked(Store &st, size_t n, const uint8_t *h_keys,
                         const uint32_t shape[4],
                         const cascade_kv_tensor_t *d_src, int src_dtype,
                         const uint8_t *h_prefix, uint8_t *h_status,
                         uint64_t *n_stored) {
  const uint64_t wb = cascade_kv_wire_bytes(shape[0], shape[1], shape[2],
                                            shape[3]);
  CB_CHECK(st.hbm && !q8_eligible(st, wb, false), CASCADE_ERR_UNSUPPORTED,
           "a fused KV put needs raw payloads in an HBM tier");
  CB_CHECK(st.gpu_used + n * payload_bytes(wb, false) <= st.pool_cap,
           CASCADE_ERR_UNSUPPORTED, "the HBM pool cannot take the whole batch");
  cudaStream_t s = st.s;
  std::vector<uint64_t> zeros(n, 0), sizes(n, wb);
  uint64_t mx = 0;
  int rc = upload_batch(st, n, zeros.data(), sizes.data(), h_keys, &mx);
  if (rc) return rc;
  st.demoted.clear();
  for (size_t i = 0; i < n; ++i) {
    st.sc.h_req[i] = payload_bytes(wb, false);
    st.sc.h_off[i] = kInvalidOffset;
    st.sc.h_dst[i] = 0;
    st.sc.h_flags[i] = kTierHbm | ((h_prefix && h_prefix[i] &&
                                    st.cfg.dedup_enabled) ? kFlagPrefix : 0);
  }
  if ((rc = ensure_stack(st, size_class(std::max<uint64_t>(st.sc.h_req[0], 1)))))
    return rc;
  if (st.claimed + n > st.nslots / 2 && (rc = grow_index(st))) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.req, st.sc.h_req, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.hoff, st.sc.h_off, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.hdst, st.sc.h_dst, n * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.flags, st.sc.h_flags, n * 4, cudaMemcpyHostToDevice, s));
  if ((rc = launch_pool_alloc(st.d_pool, st.sc.req, (int)n, st.sc.off, s)))
    return rc;
  prepare_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(
      (int)n, st.sc.req, st.sc.off, st.sc.hoff, st.sc.hdst, st.sc.flags,
      st.sc.sizes, (uint64_t)(uintptr_t)st.pool, st.sc.dst, st.sc.eff_raw,
      st.sc.eff_q8);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  // The payloads: every cache serialised into its slot (dst 0: no slot).
  if ((rc = launch_kv_serialize(d_src, src_dtype, shape[0], shape[1],
                                shape[2], shape[3], st.sc.dst, (int)n, s)))
    return rc;
  // The keys decide who stores, first in the batch winning.
  CB_CUDA(cudaMemsetAsync(st.sc.err, 0, sizeof(int), s));
  const uint64_t epoch = st.next_epoch;
  st.next_epoch += n;
  rc = launch_index_claim(st.slots, st.nslots - 1, st.sc.keys, 2, st.sc.seqs,
                          (int)n, st.sc.slot, st.sc.err, s);
  if (!rc) rc = launch_index_resolve(st.slots, st.sc.slot, st.sc.seqs, (int)n,
                                     st.sc.status, s);
  if (!rc) rc = launch_index_commit(st.slots, st.sc.slot, st.sc.status,
                                    st.sc.off, st.sc.sizes, st.sc.flags,
                                    st.sc.hdr, epoch, (int)n, s);
  if (!rc) rc = launch_index_finalize(st.slots, st.sc.slot, st.sc.off,
                                      st.sc.status, (int)n, s);
  if (!rc) rc = launch_pool_free_unstored(st.d_pool, st.sc.req, st.sc.off,
                                          st.sc.status, (int)n, s);
  if (rc) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_status, st.sc.status, n,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_off, st.sc.off, n * 8,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_err, st.sc.err, sizeof(int),
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  if ((rc = check_device_err(st))) return rc;
  // Blocks that got no slot: serialised into staging, then placed again.
  std::vector<size_t> retry;
  for (size_t i = 0; i < n; ++i)
    if (st.sc.h_status[i] == CASCADE_PUT_FAILED &&
        st.sc.h_off[i] == kInvalidOffset)
      retry.push_back(i);
  if (retry.empty()) {
    tally_put(st, n);
    return finish_put(st, n, false, h_status, nullptr, n_stored);
  }
  const uint64_t pitch = (wb + 255) & ~uint64_t(255);
  const size_t m = retry.size();
  if ((rc = ensure_device_buf(st.d_kvstage, st.d_kvstage_cap, m * pitch, s)) ||
      (rc = ensure_device_buf(st.d_kvsrc, st.d_kvsrc_cap, n * 8, s)))
    return rc;
  std::vector<uint64_t> stage_dst(n, 0), ptrs(m), msizes(m, wb);
  std::vector<uint8_t> keys(16 * m), pre(m);
  for (size_t k = 0; k < m; ++k) {
    const size_t i = retry[k];
    stage_dst[i] = (uint64_t)(uintptr_t)st.d_kvstage + k * pitch;
    ptrs[k] = stage_dst[i];
    std::memcpy(keys.data() + 16 * k, h_keys + 16 * i, 16);
    pre[k] = h_prefix ? h_prefix[i] : 0;
    st.sc.h_status[i] = kRetry;
  }
  uint64_t *d_stage_dst = reinterpret_cast<uint64_t *>(st.d_kvsrc);
  CB_CUDA(cudaMemcpyAsync(d_stage_dst, stage_dst.data(), n * 8,
                          cudaMemcpyHostToDevice, s));
  if ((rc = launch_kv_serialize(d_src, src_dtype, shape[0], shape[1],
                                shape[2], shape[3], d_stage_dst, (int)n, s)))
    return rc;
  tally_put(st, n);
  std::vector<uint8_t> status(st.sc.h_status, st.sc.h_status + n);
  if ((rc = upload_batch(st, m, ptrs.data(), msizes.data(), keys.data(), &mx)))
    return rc;
  if ((rc = put_uploaded(st, m, false, pre.data(), mx, false, 1))) return rc;
  for (size_t k = 0; k < m; ++k) status[retry[k]] = st.sc.h_status[k];
  // Report the whole batch: statuses and the stored count.
  uint64_t stored = 0;
  for (size_t i = 0; i < n; ++i) {
    if (h_status) h_status[i] = status[i];
    stored += status[i] != CASCADE_PUT_FAILED ? 1 : 0;
  }
  if (n_stored) *n_stored = stored;
  return CASCADE_OK;
}

// ----------------------------------------------------------------- get
// Looks the keys up (touching LRU epochs when `touch`); infos land in
// st.sc.h_info.  Keys must already be in st.sc.keys on the device.
static int lookup_locked(Store &st, size_t n, bool touch) {
  cudaStream_t s = st.s;
  const uint64_t epoch = st.next_epoch;
  if (touch) st.next_epoch += n;
  int rc = launch_index_lookup(st.slots, st.nslots - 1, st.sc.keys, 2, (int)n,
                               touch ? 1 : 0, epoch, st.sc.info, s);
  if (rc) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_info, st.sc.info, n * sizeof(LookupInfo),
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  return CASCADE_OK;
}

static int upload_keys(Store &st, size_t n, const uint8_t *h_keys) {
  for (size_t i = 0; i < n; ++i) {
    st.sc.h_keys[2 * i] = le64(h_keys + 16 * i);
    st.sc.h_keys[2 * i + 1] = le64(h_keys + 16 * i + 8);
  }
  CB_CUDA(cudaMemcpyAsync(st.sc.keys, st.sc.h_keys, n * 16,
                          cudaMemcpyHostToDevice, st.s));
  return CASCADE_OK;
}

// Moves the found blocks (h_info) into device buffers out[i], decoding INT8
// payloads.  deliver[i] = 0 skips a block.  Updates hit/miss counters and
// promotes DRAM hits to HBM when the configuration asks for it.  HBM
// payloads are read at pool + offset, or at bases[i] + offset when `bases`
// is given (another rank's pool mapped into this process).
static int deliver_locked(Store &st, size_t n, const uint64_t *out,
                          const uint8_t *deliver,
                          const uint64_t *bases = nullptr,
                          const uint64_t *dram_src = nullptr) {
  cudaStream_t s = st.s;
  // Copy jobs and dequantise jobs, packed into the scratch arrays:
  //   copies:  ptrs (src) / dst / eff_raw (bytes)
  //   decodes: req (src codes) / off (dst) / eff_q8 (out bytes) / hdr
  size_t nc = 0, nd = 0;
  uint64_t max_c = 0, max_d = 0, stage_bytes = 0;
  std::vector<size_t> dram_q8;
  for (size_t i = 0; i < n; ++i) {
    const LookupInfo &f = st.sc.h_info[i];
    if (!f.found || !deliver[i]) continue;
    const bool q8 = (f.flags & kFlagQ8) != 0;
    if ((f.flags & kTierDram) && q8) {
      dram_q8.push_back(i);
      stage_bytes += (payload_bytes(f.size, true) + 255) & ~uint64_t(255);
    }
  }
  if (stage_bytes) {
    int rc = ensure_device_buf(st.d_q8stage, st.d_q8stage_cap, stage_bytes, s);
    if (rc) return rc;
  }
  uint64_t stage_off = 0;
  std::vector<Dma> jobs;  // DRAM payloads up to the device
  for (size_t i = 0; i < n; ++i) {
    const LookupInfo &f = st.sc.h_info[i];
    if (!f.found || !deliver[i]) continue;
    const bool q8 = (f.flags & kFlagQ8) != 0;
    uint64_t src;
    if (f.flags & kTierHbm) {
      src = (bases ? bases[i] : (uint64_t)(uintptr_t)st.pool) + f.offset;
    } else {  // DRAM: bring the payload up first
      uint64_t pay = payload_bytes(f.size, q8);
      const void *from = dram_src ? reinterpret_cast<const void *>(dram_src[i])
                                  : st.dram->ptr(f.offset);
      if (!q8) {
        jobs.push_back({reinterpret_cast<void *>(out[i]), from, f.size});
        continue;
      }
      src = (uint64_t)(uintptr_t)(st.d_q8stage + stage_off);
      jobs.push_back({st.d_q8stage + stage_off, from, pay});
      stage_off += (pay + 255) & ~uint64_t(255);
    }
    if (q8) {
      st.sc.h_req[nd] = src;
      st.sc.h_off[nd] = out[i];
      st.sc.h_seqs[nd] = 2 * (f.size / 2);  // decoded bytes (2 per code)
      uint8_t *h = st.sc.h_hdr + 8 * nd;
      std::memcpy(h, &f.hdr_scale, 4);
      h[4] = (uint8_t)f.hdr_zp;
      h[5] = h[6] = h[7] = 0;
      max_d = std::max<uint64_t>(max_d, f.size);
      ++nd;
    } else {
      st.sc.h_ptrs[nc] = src;
      st.sc.h_dst[nc] = out[i];
      st.sc.h_sizes[nc] = f.size;
      max_c = std::max<uint64_t>(max_c, f.size);
      ++nc;
    }
  }
  if (int rc = dma_fanout(st, jobs, 1)) return rc;
  if (nc) {
    CB_CUDA(cudaMemcpyAsync(st.sc.ptrs, st.sc.h_ptrs, nc * 8, cudaMemcpyHostToDevice, s));
    CB_CUDA(cudaMemcpyAsync(st.sc.dst, st.sc.h_dst, nc * 8, cudaMemcpyHostToDevice, s));
    CB_CUDA(cudaMemcpyAsync(st.sc.eff_raw, st.sc.h_sizes, nc * 8, cudaMemcpyHostToDevice, s));
    int rc = launch_copy(st.sc.ptrs, st.sc.dst, st.sc.eff_raw, (int)nc, max_c, s);
    if (rc) return rc;
  }
  if (nd) {
    CB_CUDA(cudaMemcpyAsync(st.sc.req, st.sc.h_req, nd * 8, cudaMemcpyHostToDevice, s));
    CB_CUDA(cudaMemcpyAsync(st.sc.off, st.sc.h_off, nd * 8, cudaMemcpyHostToDevice, s));
    CB_CUDA(cudaMemcpyAsync(st.sc.eff_q8, st.sc.h_seqs, nd * 8, cudaMemcpyHostToDevice, s));
    CB_CUDA(cudaMemcpyAsync(st.sc.hdr, st.sc.h_hdr, nd * 8, cudaMemcpyHostToDevice, s));
    int rc = launch_dequantize(st.sc.req, st.sc.hdr, 0, st.sc.eff_q8, (int)nd,
                               max_d, st.sc.off, s);
    if (rc) return rc;
  }
  // Counters: CascadeStore::get (cascade_core.cpp:1138-1189).
  for (size_t i = 0; i < n; ++i) {
    const LookupInfo &f = st.sc.h_info[i];
    if (!deliver[i]) continue;
    if (!f.found) ++st.misses;
    else if (f.flags & kTierHbm) ++st.gpu_hits;
    else ++st.shm_hits;
  }
  CB_CUDA(cudaStreamSynchronize(s));
  // Promotion of DRAM hits (promote_to_gpu, cascade_core.cpp:1039-1056):
  // the decoded block, now in out[i], is stored in HBM and its DRAM space
  // released.
  // A sharded read (bases given) carries no index slot of this rank, so its
  // DRAM hits are not promoted.
  if (!(st.cfg.promotion_enabled && st.hbm) || bases) return CASCADE_OK;
  // The promotions replayed in get order (promote_to_gpu demotes older
  // blocks when HBM is full): a block that serial gets would promote and
  // demote again within the batch stays in DRAM and counts both ways.
  std::vector<size_t> promo, want;
  std::vector<Arrival> arr;
  for (size_t i = 0; i < n; ++i) {
    const LookupInfo &f = st.sc.h_info[i];
    if (!f.found || !deliver[i] || !(f.flags & kTierDram)) continue;
    const bool was_q8 = (f.flags & kFlagQ8) != 0;
    const uint64_t size = was_q8 ? 2 * (f.size / 2) : f.size;
    want.push_back(i);
    arr.push_back({size, payload_bytes(size, q8_eligible(st, size, false)),
                   victim_class(st, f.flags), false,
                   dram_accounted(f.size, was_q8)});
  }
  if (arr.empty()) return CASCADE_OK;
  Replay plan;
  int prc = plan_batch(st, arr, true, plan);
  if (!prc) prc = demote(st, plan.old);
  if (prc) return prc;
  for (size_t k = 0; k < arr.size(); ++k) {
    if (plan.fate[k] == kFateHbm) promo.push_back(want[k]);
    if (plan.fate[k] == kFateEvicted) {
      ++st.promotions_to_gpu;
      ++st.gpu_evictions;
    }
  }
  if (promo.empty()) return CASCADE_OK;
  // Build a placement batch over the scratch arrays: one request each.
  const size_t m = promo.size();
  std::vector<LookupInfo> infos(m);
  uint64_t max_size = 0;
  for (size_t k = 0; k < m; ++k) {
    const size_t i = promo[k];
    const LookupInfo &f = st.sc.h_info[i];
    infos[k] = f;
    const bool was_q8 = (f.flags & kFlagQ8) != 0;
    const uint64_t size = was_q8 ? 2 * (f.size / 2) : f.size;
    const bool q8 = q8_eligible(st, size, false);
    st.sc.h_ptrs[k] = out[i];
    st.sc.h_sizes[k] = size;
    st.sc.h_req[k] = payload_bytes(size, q8);
    st.sc.h_flags[k] = (f.flags & kFlagPrefix) | kTierHbm | (q8 ? kFlagQ8 : 0);
    st.sc.h_slot[k] = f.slot;
    max_size = std::max(max_size, size);
    int rc = ensure_stack(st, size_class(std::max<uint64_t>(st.sc.h_req[k], 1)));
    if (rc) return rc;
  }
  CB_CUDA(cudaMemcpyAsync(st.sc.ptrs, st.sc.h_ptrs, m * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.sizes, st.sc.h_sizes, m * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.req, st.sc.h_req, m * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.flags, st.sc.h_flags, m * 4, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.slot, st.sc.h_slot, m * 4, cudaMemcpyHostToDevice, s));
  int rc = launch_pool_alloc(st.d_pool, st.sc.req, (int)m, st.sc.off, s);
  if (rc) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_off, st.sc.off, m * 8, cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaStreamSynchronize(s));
  // Only the allocations that succeeded move.
  size_t good = 0;
  for (size_t k = 0; k < m; ++k) {
    if (st.sc.h_off[k] == kInvalidOffset) continue;
    st.sc.h_ptrs[good] = st.sc.h_ptrs[k];
    st.sc.h_sizes[good] = st.sc.h_sizes[k];
    st.sc.h_flags[good] = st.sc.h_flags[k];
    st.sc.h_slot[good] = st.sc.h_slot[k];
    st.sc.h_dst[good] = (uint64_t)(uintptr_t)st.pool + st.sc.h_off[k];
    st.sc.h_req[good] = st.sc.h_off[k];  // keep the offset for relocate
    infos[good] = infos[k];
    ++good;
  }
  if (!good) return CASCADE_OK;
  std::vector<uint64_t> eff_q8(good), eff_raw(good);
  for (size_t k = 0; k < good; ++k) {
    bool q8 = (st.sc.h_flags[k] & kFlagQ8) != 0;
    eff_q8[k] = q8 ? st.sc.h_sizes[k] : 0;
    eff_raw[k] = q8 ? 0 : st.sc.h_sizes[k];
  }
  std::memcpy(st.sc.h_seqs, eff_q8.data(), good * 8);
  CB_CUDA(cudaMemcpyAsync(st.sc.ptrs, st.sc.h_ptrs, good * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.dst, st.sc.h_dst, good * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.eff_q8, st.sc.h_seqs, good * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaStreamSynchronize(s));
  std::memcpy(st.sc.h_seqs, eff_raw.data(), good * 8);
  CB_CUDA(cudaMemcpyAsync(st.sc.eff_raw, st.sc.h_seqs, good * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.off, st.sc.h_req, good * 8, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.flags, st.sc.h_flags, good * 4, cudaMemcpyHostToDevice, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.slot, st.sc.h_slot, good * 4, cudaMemcpyHostToDevice, s));
  rc = launch_minmax(st.sc.ptrs, st.sc.eff_q8, (int)good, max_size, st.sc.mnmx, s);
  if (!rc) rc = launch_quantize(st.sc.ptrs, st.sc.eff_q8, (int)good, max_size,
                                st.sc.mnmx, st.sc.dst, st.sc.hdr, 0, s);
  if (!rc) rc = launch_copy(st.sc.ptrs, st.sc.dst, st.sc.eff_raw, (int)good,
                            max_size, s);
  if (!rc) rc = launch_index_relocate(st.slots, st.sc.slot, st.sc.off,
                                      st.sc.flags, st.sc.hdr, (int)good, s);
  if (rc) return rc;
  CB_CUDA(cudaStreamSynchronize(s));
  for (size_t k = 0; k < good; ++k) {
    const LookupInfo &f = infos[k];
    const bool was_q8 = (f.flags & kFlagQ8) != 0;
    st.dram->free(f.offset, payload_bytes(f.size, was_q8));
    st.shm_used -= dram_accounted(f.size, was_q8);
    st.gpu_used += payload_bytes(st.sc.h_sizes[k],
                                 (st.sc.h_flags[k] & kFlagQ8) != 0);
    ++st.promotions_to_gpu;
  }
  return CASCADE_OK;
}

static int get_batch_locked(Store &st, size_t n, const uint8_t *h_keys,
                            const uint64_t *h_out, const uint64_t *h_caps,
                            uint64_t *h_sizes, uint8_t *h_found,
                            uint64_t *n_found) {
  int rc = ensure_scratch(st, n);
  if (!rc) rc = upload_keys(st, n, h_keys);
  if (!rc) rc = lookup_locked(st, n, true);
  if (rc) return rc;
  std::vector<uint8_t> deliver(n);
  std::vector<uint64_t> out(h_out, h_out + n);
  uint64_t found = 0;
  for (size_t i = 0; i < n; ++i)
    CB_CHECK(!(st.sc.h_info[i].found && (st.sc.h_info[i].flags & kFlagRemote)),
             CASCADE_ERR_UNSUPPORTED,
             "block is held by another rank of a sharded store: read it on "
             "its holder");
  for (size_t i = 0; i < n; ++i) {
    const LookupInfo &f = st.sc.h_info[i];
    uint64_t size = f.found ? ((f.flags & kFlagQ8) ? 2 * (f.size / 2) : f.size) : 0;
    if (h_sizes) h_sizes[i] = size;
    if (h_found) h_found[i] = f.found ? 1 : 0;
    found += f.found ? 1 : 0;
    deliver[i] = (!f.found || size <= h_caps[i]) ? 1 : 0;
  }
  if (n_found) *n_found = found;
  return deliver_locked(st, n, out.data(), deliver.data());
}

// get_batch of blocks that hold kv_manager wire blocks of one shape, split
// into the caller's K/V tensors.  Raw HBM hits are split straight out of
// the pool (one pass over their bytes), before deliver_locked's promotions
// can move anything; other hits (DRAM tier, INT8) are delivered into a
// staging buffer first and split from there.  Blocks of another size are
// reported not found and count neither hit nor miss, as a get into a
// buffer too small for them does.
static int get_kv_batch_locked(Store &st, size_t n, const uint8_t *h_keys,
                               const uint32_t shape[4],
                               const cascade_kv_tensor_t *d_dst,
                               uint8_t *h_found, uint64_t *n_found) {
  const uint64_t wb = cascade_kv_wire_bytes(shape[0], shape[1], shape[2],
                                            shape[3]);
  int rc = ensure_scratch(st, n);
  if (!rc) rc = upload_keys(st, n, h_keys);
  if (!rc) rc = lookup_locked(st, n, true);
  if (rc) return rc;
  for (size_t i = 0; i < n; ++i)
    CB_CHECK(!(st.sc.h_info[i].found && (st.sc.h_info[i].flags & kFlagRemote)),
             CASCADE_ERR_UNSUPPORTED,
             "block is held by another rank of a sharded store: read it on "
             "its holder");
  const uint64_t pitch = (wb + 255) & ~uint64_t(255);
  std::vector<uint64_t> direct(n, 0), staged(n, 0), out(n, 0);
  std::vector<uint8_t> deliver(n, 0);
  size_t nstage = 0, ndirect = 0;
  uint64_t found = 0;
  for (size_t i = 0; i < n; ++i) {
    const LookupInfo &f = st.sc.h_info[i];
    if (!f.found) {               // counted as a miss by deliver_locked
      deliver[i] = 1;
      h_found[i] = 0;
      continue;
    }
    const bool q8 = (f.flags & kFlagQ8) != 0;
    const uint64_t size = q8 ? 2 * (f.size / 2) : f.size;
    h_found[i] = size == wb ? 1 : 0;
    if (size != wb) continue;
    ++found;
    if ((f.flags & kTierHbm) && !q8) {
      direct[i] = (uint64_t)(uintptr_t)st.pool + f.offset;
      ++ndirect;
      ++st.gpu_hits;
    } else {
      deliver[i] = 1;
      out[i] = nstage++;          // staging slot, made an address below
    }
  }
  if (n_found) *n_found = found;
  cudaStream_t s = st.s;
  if ((rc = ensure_device_buf(st.d_kvsrc, st.d_kvsrc_cap, 2 * n * 8, s)))
    return rc;
  uint64_t *d_direct = reinterpret_cast<uint64_t *>(st.d_kvsrc);
  uint64_t *d_staged = d_direct + n;
  if (ndirect) {
    // Pageable source: the copy has read `direct` when the call returns.
    CB_CUDA(cudaMemcpyAsync(d_direct, direct.data(), n * 8,
                            cudaMemcpyHostToDevice, s));
    if ((rc = launch_kv_deserialize(d_direct, shape[0], shape[1], shape[2],
                                    shape[3], d_dst, (int)n, s)))
      return rc;
  }
  if (nstage) {
    if ((rc = ensure_device_buf(st.d_kvstage, st.d_kvstage_cap,
                                nstage * pitch, s)))
      return rc;
    for (size_t i = 0; i < n; ++i)
      if (deliver[i] && st.sc.h_info[i].found) {
        out[i] = (uint64_t)(uintptr_t)st.d_kvstage + out[i] * pitch;
        staged[i] = out[i];
      }
  }
  // Misses and staged hits: counters, copies / decodes, promotions.
  if ((rc = deliver_locked(st, n, out.data(), deliver.data()))) return rc;
  if (nstage) {
    CB_CUDA(cudaMemcpyAsync(d_staged, staged.data(), n * 8,
                            cudaMemcpyHostToDevice, s));
    if ((rc = launch_kv_deserialize(d_staged, shape[0], shape[1], shape[2],
                                    shape[3], d_dst, (int)n, s)))
      return rc;
  }
  return CASCADE_OK;
}

// ---------------------------------------------------------- index growth
namespace {

__global__ void rehash_kernel(const Slot *__restrict__ old_slots,
                              uint64_t old_n, Slot *new_slots,
                              uint64_t new_mask, int *err) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
       i < old_n; i += (uint64_t)gridDim.x * blockDim.x) {
    const Slot &o = old_slots[i];
    if (o.state != kLive) continue;
    const uint64_t z = slot_hash(o.k0, o.k1);
    bool placed = false;
    for (int p = 0; p < kMaxProbe && !placed; ++p) {
      Slot *t = new_slots + ((z + (uint64_t)p) & new_mask);
      uint64_t a, b;
      cas128(&t->k0, 0, 0, o.k0, o.k1, a, b);
      if (a == 0 && b == 0) {  // the key is unique: the slot is ours
        t->claim = 0;
        t->state = o.state;
        t->flags = o.flags;
        t->offset = o.offset;
        t->size = o.size;
        t->hdr_scale = o.hdr_scale;
        t->hdr_zp = o.hdr_zp;
        t->epoch = o.epoch;
        placed = true;
      }
    }
    if (!placed) atomicExch(err, CASCADE_ERR_FULL);
  }
}

int grow_index(Store &st) {
  uint64_t want = pow2_at_least(2 * (st.claimed + st.sc.cap) + 1);
  if (want <= st.nslots) want = st.nslots * 2;
  Slot *fresh = nullptr;
  CB_CUDA(cudaMalloc(&fresh, want * sizeof(Slot)));
  CB_CUDA(cudaMemsetAsync(fresh, 0, want * sizeof(Slot), st.s));
  CB_CUDA(cudaMemsetAsync(st.sc.err, 0, sizeof(int), st.s));
  const int grid = grid_for(st.nslots, 256, 8);
  rehash_kernel<<<grid, 256, 0, st.s>>>(st.slots, st.nslots, fresh, want - 1,
                                        st.sc.err);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  CB_CUDA(cudaMemcpyAsync(st.sc.h_err, st.sc.err, sizeof(int),
                          cudaMemcpyDeviceToHost, st.s));
  CB_CUDA(cudaStreamSynchronize(st.s));
  if (*st.sc.h_err) {
    cudaFree(fresh);
    set_error("index rehash failed");
    return CASCADE_ERR_FULL;
  }
  CB_CUDA(cudaFree(st.slots));
  st.slots = fresh;
  st.nslots = want;
  return CASCADE_OK;
}

}  // namespace

// ------------------------------------------------------------- lifecycle
static int create_store(const cascade_config_t *cfg, Store **out) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    set_error("no CUDA device: the block store runs only on the GPU");
    return CASCADE_ERR_NODEVICE;
  }
  CB_CHECK(cfg->gpu_device_id >= 0 && cfg->gpu_device_id < count,
           CASCADE_ERR_INVALID, "gpu_device_id out of range");
  std::unique_ptr<Store> st(new Store());
  st->cfg = *cfg;
  st->shm_path = cfg->shm_path ? cfg->shm_path : "";
  st->lustre_path = cfg->lustre_path ? cfg->lustre_path : "";
  st->cfg.shm_path = st->shm_path.c_str();
  st->cfg.lustre_path = st->lustre_path.c_str();
  st->dev = cfg->gpu_device_id;
  DeviceGuard g(st->dev);
  CB_CUDA(cudaStreamCreateWithFlags(&st->s, cudaStreamNonBlocking));
  CB_CUDA(cudaStreamCreateWithFlags(&st->s2, cudaStreamNonBlocking));
  CB_CUDA(cudaStreamCreateWithFlags(&st->s3, cudaStreamNonBlocking));
  CB_CUDA(cudaEventCreateWithFlags(&st->ev, cudaEventDisableTiming));
  CB_CUDA(cudaEventCreateWithFlags(&st->ev2, cudaEventDisableTiming));
  CB_CUDA(cudaEventCreateWithFlags(&st->ev3, cudaEventDisableTiming));
  CB_CUDA(cudaEventCreateWithFlags(&st->dma_start, cudaEventDisableTiming));
  for (int d = 0; d < 2; ++d)
    for (int q = 0; q < kDmaStreams; ++q) {
      CB_CUDA(cudaStreamCreateWithFlags(&st->dma[d][q], cudaStreamNonBlocking));
      CB_CUDA(cudaEventCreateWithFlags(&st->dma_done[d][q],
                                       cudaEventDisableTiming));
    }
  st->hbm = cfg->use_gpu && cfg->gpu_capacity_bytes > 0;
  st->dram_tier = cfg->shm_capacity_bytes > 0;
  if (st->hbm) {
    st->pool_cap = cfg->gpu_capacity_bytes;
    cudaError_t e = cudaMalloc(&st->pool, st->pool_cap);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error("cannot allocate the HBM pool of gpu_capacity_bytes");
      return CASCADE_ERR_NOMEM;
    }
    CB_CUDA(cudaMalloc(&st->d_pool, sizeof(PoolDev)));
  }
  uint64_t slots = cfg->index_slots;
  if (!slots) {
    uint64_t blocks = (cfg->gpu_capacity_bytes * (st->hbm ? 1 : 0) +
                       cfg->shm_capacity_bytes) / (256ull << 10);
    slots = std::min<uint64_t>(std::max<uint64_t>(2 * blocks, 1ull << 16),
                               1ull << 22);
  }
  st->nslots = pow2_at_least(std::max<uint64_t>(slots, 1024));
  CB_CUDA(cudaMalloc(&st->slots, st->nslots * sizeof(Slot)));
  CB_CUDA(cudaMemsetAsync(st->slots, 0, st->nslots * sizeof(Slot), st->s));
  if (st->dram_tier) {
    uint64_t chunk = cfg->dram_chunk_bytes ? cfg->dram_chunk_bytes : (1ull << 30);
    st->dram.reset(new DramArena(cfg->shm_capacity_bytes, chunk));
  }
  int rc = ensure_scratch(*st, 1024);
  if (!rc) rc = reset_pool(*st);
  if (rc) return rc;
  CB_CUDA(cudaStreamSynchronize(st->s));
  *out = st.release();
  return CASCADE_OK;
}

static void close_peer_pools(Store &st) {
  for (size_t r = 0; r < st.peer_base.size(); ++r)
    if ((int)r != st.peer_rank && st.peer_base[r])
      cudaIpcCloseMemHandle(st.peer_base[r]);
  st.peer_base.clear();
  st.peer_rank = -1;
  st.peer_dram.clear();
}

static void destroy_store(Store *st) {
  DeviceGuard g(st->dev);
  for (cudaStream_t q : {st->s, st->s2, st->s3})
    if (q) cudaStreamSynchronize(q);
  st->dram.reset();
  close_peer_pools(*st);
  for (int c = 0; c < kNumClasses; ++c)
    if (st->stack_ptr[c]) cudaFree(st->stack_ptr[c]);
  if (st->pool) cudaFree(st->pool);
  if (st->d_pool) cudaFree(st->d_pool);
  if (st->slots) cudaFree(st->slots);
  for (Scratch *sc : {&st->sc, &st->oc}) {
    if (sc->dblob) cudaFree(sc->dblob);
    if (sc->hblob) cudaFreeHost(sc->hblob);
  }
  if (st->shard_aux) cudaFree(st->shard_aux);
  if (st->h_moves) cudaFreeHost(st->h_moves);
  if (st->d_stage) cudaFree(st->d_stage);
  if (st->h_stage) cudaFreeHost(st->h_stage);
  if (st->d_q8stage) cudaFree(st->d_q8stage);
  if (st->d_evstage) cudaFree(st->d_evstage);
  if (st->d_kvstage) cudaFree(st->d_kvstage);
  if (st->d_kvsrc) cudaFree(st->d_kvsrc);
  if (st->scan_d) cudaFree(st->scan_d);
  if (st->sha_state) cudaFree(st->sha_state);
  for (cudaEvent_t e : {st->ev, st->ev2, st->ev3, st->dma_start})
    if (e) cudaEventDestroy(e);
  for (cudaStream_t q : {st->s, st->s2, st->s3})
    if (q) cudaStreamDestroy(q);
  for (int d = 0; d < 2; ++d)
    for (int q = 0; q < kDmaStreams; ++q) {
      if (st->dma_done[d][q]) cudaEventDestroy(st->dma_done[d][q]);
      if (st->dma[d][q]) cudaStreamDestroy(st->dma[d][q]);
    }
  delete st;
}

static int clear_store(Store &st) {
  CB_CUDA(cudaStreamSynchronize(st.s));
  CB_CUDA(cudaMemsetAsync(st.slots, 0, st.nslots * sizeof(Slot), st.s));
  int rc = reset_pool(st);
  if (rc) return rc;
  if (st.dram) st.dram->reset();
  st.names.clear();
  st.shard_moves.clear();
  st.claimed = 0;
  st.gpu_used = st.shm_used = st.gpu_hits = st.shm_hits = st.misses = 0;
  st.dedup_hits = st.gpu_evictions = st.promotions_to_gpu = 0;
  st.compression_savings = st.shm_puts = 0;
  CB_CUDA(cudaStreamSynchronize(st.s));
  return CASCADE_OK;
}

// Host-buffer put of one block: staged to the device, then the batch path.
static int put_host_locked(Store &st, const Key &k, const uint8_t *data,
                           uint64_t size, int is_prefix, int *stored) {
  int rc = ensure_device_buf(st.d_stage, st.d_stage_cap, size, st.s);
  if (!rc) rc = ensure_host_stage(st, size);
  if (rc) return rc;
  if (size) {
    std::memcpy(st.h_stage, data, size);
    CB_CUDA(cudaMemcpyAsync(st.d_stage, st.h_stage, size,
                            cudaMemcpyHostToDevice, st.s));
  }
  uint8_t key[16];
  for (int i = 0; i < 8; ++i) {
    key[i] = (uint8_t)(k.k0 >> (8 * i));
    key[8 + i] = (uint8_t)(k.k1 >> (8 * i));
  }
  uint64_t ptr = (uint64_t)(uintptr_t)st.d_stage;
  uint8_t pf = is_prefix ? 1 : 0, status = 0;
  uint64_t ok = 0;
  rc = put_batch_locked(st, 1, &ptr, &size, key, &pf, &status, nullptr, &ok);
  if (rc) return rc;
  *stored = ok ? 1 : 0;
  return CASCADE_OK;
}

static int get_host_locked(Store &st, const Key &k, uint8_t *out,
                           uint64_t cap, int *found, uint64_t *size) {
  int rc = ensure_scratch(st, 1);
  if (rc) return rc;
  st.sc.h_keys[0] = k.k0;
  st.sc.h_keys[1] = k.k1;
  CB_CUDA(cudaMemcpyAsync(st.sc.keys, st.sc.h_keys, 16, cudaMemcpyHostToDevice,
                          st.s));
  if ((rc = lookup_locked(st, 1, true))) return rc;
  LookupInfo f = st.sc.h_info[0];
  if (!f.found) {
    ++st.misses;
    *found = 0;
    *size = 0;
    return CASCADE_OK;
  }
  CB_CHECK(!(f.flags & kFlagRemote), CASCADE_ERR_UNSUPPORTED,
           "block is held by another rank of a sharded store: read it on its "
           "holder");
  const uint64_t bytes = (f.flags & kFlagQ8) ? 2 * (f.size / 2) : f.size;
  *found = 1;
  *size = bytes;
  if (bytes > cap) return CASCADE_OK;  // caller retries with a larger buffer
  if ((f.flags & kTierDram) && !(f.flags & kFlagQ8) &&
      !(st.cfg.promotion_enabled && st.hbm)) {
    // A raw DRAM block goes straight from the arena to the caller.
    if (bytes) std::memcpy(out, st.dram->ptr(f.offset), bytes);
    ++st.shm_hits;
    return CASCADE_OK;
  }
  if ((rc = ensure_device_buf(st.d_stage, st.d_stage_cap, bytes, st.s)) ||
      (rc = ensure_host_stage(st, bytes)))
    return rc;
  uint64_t dst = (uint64_t)(uintptr_t)st.d_stage;
  uint8_t deliver = 1;
  if ((rc = deliver_locked(st, 1, &dst, &deliver))) return rc;
  if (bytes) {
    CB_CUDA(cudaMemcpyAsync(st.h_stage, st.d_stage, bytes,
                            cudaMemcpyDeviceToHost, st.s));
    CB_CUDA(cudaStreamSynchronize(st.s));
    std::memcpy(out, st.h_stage, bytes);
  }
  return CASCADE_OK;
}

// Host blocks for the batched put.
//
// Uniform batches (equal sizes, equally spaced, in pinned memory) stream to
// the GPU in stripes: stripe k holds bytes [k*B, (k+1)*B) of every block and
// is one strided copy; as each stripe lands, the hash stream advances every
// block's SHA-256 over that stripe's chunks (the running states are kept
// between stripes).  Hashing thus hides under the host-to-device transfer,
// and when the last stripe lands only its chunks, the INT8 compression and
// the index work remain.
//
// Other batches are copied block by block (directly from pinned memory,
// through the pinned stage otherwise) and then put like device blocks.
// Host blocks of one size at a constant pitch, in pinned memory: copied to
// the device staging area in ~16 stripes on the copy stream while the hash
// stream hashes each stripe as it lands (launch_sha256_range keeps the
// running states).  On return the descriptors are uploaded, the digests are
// being computed (st.ev2 marks the end) and the main stream waits for the
// last stripe.  *taken = false when the layout does not qualify.
static int stage_host_striped(Store &st, size_t n,
                              const uint8_t *const *blocks,
                              const uint64_t *sizes, bool *taken,
                              uint64_t *max_size) {
  *taken = false;
  const uint64_t S = sizes[0];
  const intptr_t pitch = n > 1 ? (intptr_t)(blocks[1] - blocks[0]) : (intptr_t)S;
  bool uniform = S > 0 && pitch >= (intptr_t)S;
  for (size_t i = 0; uniform && i < n; ++i)
    uniform = sizes[i] == S && blocks[i] == blocks[0] + (intptr_t)i * pitch;
  if (uniform) {
    cudaPointerAttributes a0, a1;
    bool p0 = cudaPointerGetAttributes(&a0, blocks[0]) == cudaSuccess &&
              a0.type == cudaMemoryTypeHost;
    cudaGetLastError();
    bool p1 = cudaPointerGetAttributes(&a1, blocks[n - 1] + S - 1) == cudaSuccess &&
              a1.type == cudaMemoryTypeHost;
    cudaGetLastError();
    uniform = p0 && p1;
  }
  if (!uniform) return CASCADE_OK;
  int rc;
  const uint64_t Pd = (S + 255) & ~uint64_t(255);
  if ((rc = ensure_device_buf(st.d_stage, st.d_stage_cap, n * Pd, st.s)))
    return rc;
  if (n > st.sha_state_cap) {
    CB_CUDA(cudaStreamSynchronize(st.s2));
    if (st.sha_state) CB_CUDA(cudaFree(st.sha_state));
    st.sha_state = nullptr;
    st.sha_state_cap = 0;
    CB_CUDA(cudaMalloc(&st.sha_state, n * 32));
    st.sha_state_cap = n;
  }
  std::vector<uint64_t> ptrs(n);
  for (size_t i = 0; i < n; ++i)
    ptrs[i] = (uint64_t)(uintptr_t)(st.d_stage + i * Pd);
  if ((rc = upload_batch(st, n, ptrs.data(), sizes, nullptr, max_size)))
    return rc;
  CB_CUDA(cudaEventRecord(st.ev, st.s));
  CB_CUDA(cudaStreamWaitEvent(st.s2, st.ev, 0));
  // ~16 stripes for large blocks, each a whole number of 64-byte chunks.
  uint64_t K = std::min<uint64_t>(16, (S + 65535) / 65536);
  if (K < 1) K = 1;
  const uint64_t B = ((S + K - 1) / K + 63) & ~uint64_t(63);
  K = (S + B - 1) / B;
  for (uint64_t k = 0; k < K; ++k) {
    const uint64_t off = k * B, w = std::min<uint64_t>(B, S - off);
    CB_CUDA(cudaMemcpy2DAsync(st.d_stage + off, Pd, blocks[0] + off,
                              (size_t)pitch, w, n, cudaMemcpyHostToDevice,
                              st.s3));
    CB_CUDA(cudaEventRecord(st.ev3, st.s3));
    CB_CUDA(cudaStreamWaitEvent(st.s2, st.ev3, 0));
    const uint64_t c0 = off / 64;
    const uint64_t c1 = (k + 1 == K) ? ~0ull : (off + B) / 64;
    rc = launch_sha256_range(st.sc.ptrs, st.sc.sizes, (int)n, st.sc.digests,
                             st.sha_state, c0, c1, st.s2);
    if (rc) return rc;
  }
  CB_CUDA(cudaEventRecord(st.ev2, st.s2));
  CB_CUDA(cudaStreamWaitEvent(st.s, st.ev3, 0));  // every stripe is in
  *taken = true;
  return CASCADE_OK;
}

// Any other host blocks: one copy each into the device staging area (pinned
// blocks directly, pageable ones through the pinned stage); device
// addresses to ptrs.
static int stage_host_blocks(Store &st, size_t n, const uint8_t *const *blocks,
                             const uint64_t *sizes, std::vector<uint64_t> &ptrs) {
  uint64_t total = 0;
  std::vector<uint64_t> offs(n);
  for (size_t i = 0; i < n; ++i) {
    offs[i] = total;
    total += (sizes[i] + 255) & ~uint64_t(255);
  }
  int rc = ensure_device_buf(st.d_stage, st.d_stage_cap, total, st.s);
  if (rc) return rc;
  size_t pinned_need = 0;
  std::vector<uint8_t> pinned(n);
  for (size_t i = 0; i < n; ++i) {
    cudaPointerAttributes a;
    pinned[i] = (sizes[i] && cudaPointerGetAttributes(&a, blocks[i]) == cudaSuccess &&
                 a.type == cudaMemoryTypeHost) ? 1 : 0;
    cudaGetLastError();
    if (!pinned[i]) pinned_need = std::max<size_t>(pinned_need, sizes[i]);
  }
  if (pinned_need && (rc = ensure_host_stage(st, pinned_need))) return rc;
  ptrs.assign(n, 0);
  for (size_t i = 0; i < n; ++i) {
    ptrs[i] = (uint64_t)(uintptr_t)(st.d_stage + offs[i]);
    if (!sizes[i]) continue;
    if (pinned[i]) {
      CB_CUDA(cudaMemcpyAsync(st.d_stage + offs[i], blocks[i], sizes[i],
                              cudaMemcpyHostToDevice, st.s));
    } else {  // through the pinned stage, one block at a time
      CB_CUDA(cudaStreamSynchronize(st.s));
      std::memcpy(st.h_stage, blocks[i], sizes[i]);
      CB_CUDA(cudaMemcpyAsync(st.d_stage + offs[i], st.h_stage, sizes[i],
                              cudaMemcpyHostToDevice, st.s));
    }
  }
  return CASCADE_OK;
}

static int put_batch_host_locked(Store &st, size_t n,
                                 const uint8_t *const *blocks,
                                 const uint64_t *sizes, const uint8_t *keys,
                                 const uint8_t *prefix, uint8_t *status,
                                 uint8_t *digests, uint64_t *n_stored) {
  int rc;
  if (keys == nullptr) {
    bool taken = false;
    uint64_t max_size = 0;
    if ((rc = stage_host_striped(st, n, blocks, sizes, &taken, &max_size)))
      return rc;
    if (taken) {
      rc = put_uploaded(st, n, true, prefix, max_size, true);
      if (rc) return rc;
      return finish_put(st, n, true, status, digests, n_stored);
    }
  }
  std::vector<uint64_t> ptrs;
  if ((rc = stage_host_blocks(st, n, blocks, sizes, ptrs))) return rc;
  return put_batch_locked(st, n, ptrs.data(), sizes, keys, prefix, status,
                          digests, n_stored);
}

// ------------------------------------------------------- sharded dedup
// Exchange buffers are padded: `world` segments of `cap` entries, segment r
// for rank r, so that both all-to-alls move equal splits and no rank needs
// to learn the others' counts.  An entry whose src_idx is kUnused (the
// buffers are filled with 0xff bytes) carries nothing.
namespace {

// One record per block, written into its owner's segment.  A segment that
// overflows `cap` is an error (the caller's cap is below the batch size).
__global__ void shard_records_kernel(int n, int world, uint32_t rank,
                                     uint64_t seq_base, uint32_t cap,
                                     const uint64_t *__restrict__ digests,
                                     const uint64_t *__restrict__ off,
                                     const uint64_t *__restrict__ sizes,
                                     const uint32_t *__restrict__ flags,
                                     const uint8_t *__restrict__ hdr,
                                     uint32_t *__restrict__ cursor,
                                     ShardRecord *__restrict__ out,
                                     int *__restrict__ err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  ShardRecord r;
  r.k0 = digests[4 * (size_t)i];
  r.k1 = digests[4 * (size_t)i + 1];
  r.seq = seq_base + (uint64_t)i;
  r.offset = off[i];
  r.size = sizes[i];
  r.flags = flags[i];
  r.holder = rank;
  r.src_idx = (uint32_t)i;
  const uint8_t *h = hdr + 8 * (size_t)i;
  r.hdr_scale = (uint32_t)h[0] | ((uint32_t)h[1] << 8) |
                ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
  r.hdr_zp = h[4];
  r.pad = 0;
  const int o = owner_of(r.k0, world);
  const uint32_t k = atomicAdd(&cursor[o], 1u);
  if (k < cap)
    out[(size_t)o * cap + k] = r;
  else
    atomicExch(err, CASCADE_ERR_INVALID);
}

// Unused records get no key and the sequence number kNoSeq, which the
// claim step skips (their status becomes FAILED and is never sent back).
__global__ void shard_unpack_kernel(int m, uint32_t rank,
                                    const ShardRecord *__restrict__ in,
                                    uint64_t *__restrict__ keys,
                                    uint64_t *__restrict__ seqs,
                                    uint64_t *__restrict__ off,
                                    uint64_t *__restrict__ sizes,
                                    uint32_t *__restrict__ flags,
                                    uint8_t *__restrict__ hdr) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  const ShardRecord r = in[j];
  const bool used = r.src_idx != kUnused && r.src_idx != kMoveIdx;
  keys[2 * (size_t)j] = r.k0;
  keys[2 * (size_t)j + 1] = r.k1;
  seqs[j] = used ? r.seq : kNoSeq;
  off[j] = used ? r.offset : kInvalidOffset;
  sizes[j] = used ? r.size : 0;
  flags[j] = used ? ((r.flags & 0xffffu) | ((r.holder & 0xffu) << 16) |
                     (r.holder != rank ? (uint32_t)kFlagRemote : 0u))
                  : 0u;
  uint8_t *h = hdr + 8 * (size_t)j;
  h[0] = r.hdr_scale & 0xff; h[1] = (r.hdr_scale >> 8) & 0xff;
  h[2] = (r.hdr_scale >> 16) & 0xff; h[3] = r.hdr_scale >> 24;
  h[4] = (uint8_t)r.hdr_zp; h[5] = h[6] = h[7] = 0;
}

__global__ void shard_reply_kernel(int m, const ShardRecord *__restrict__ in,
                                   const uint8_t *__restrict__ status,
                                   ShardReply *__restrict__ out) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  ShardReply r;
  r.src_idx = in[j].src_idx;
  if (r.src_idx == kMoveIdx) r.src_idx = kUnused;  // moves get no reply
  r.status = r.src_idx == kUnused ? kUnused : status[j];
  out[j] = r;
}

__global__ void shard_apply_kernel(int m, int n,
                                   const ShardReply *__restrict__ back,
                                   uint8_t *__restrict__ status,
                                   int *__restrict__ err) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  const ShardReply r = back[j];
  if (r.src_idx == kUnused) return;
  if (r.src_idx < (uint32_t)n && r.status <= CASCADE_PUT_FAILED)
    status[r.src_idx] = (uint8_t)r.status;
  else
    atomicExch(err, CASCADE_ERR_INVALID);
}

// Held-slot requests: entry i claims digest i's key when block i stored
// here and another rank owns the key, else takes no part (kNoSeq).
__global__ void shard_held_kernel(int n, int world, uint32_t rank,
                                  const uint64_t *__restrict__ digests,
                                  const uint8_t *__restrict__ status,
                                  const uint32_t *__restrict__ flags,
                                  uint64_t *__restrict__ keys,
                                  uint64_t *__restrict__ seqs,
                                  uint32_t *__restrict__ hflags,
                                  uint32_t *__restrict__ count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t k0 = digests[4 * (size_t)i], k1 = digests[4 * (size_t)i + 1];
  const bool held = status[i] == CASCADE_PUT_STORED && (flags[i] & kTierHbm) &&
                    owner_of(k0, world) != (int)rank;
  keys[2 * (size_t)i] = k0;
  keys[2 * (size_t)i + 1] = k1;
  seqs[i] = held ? (uint64_t)i + 1 : kNoSeq;
  hflags[i] = (flags[i] & 0xffffu) | kFlagHeld | (rank << 16);
  if (held) atomicAdd(count, 1u);
}

// Relocation records into their owners' segments, after the batch's own.
__global__ void shard_moves_kernel(int k, int world, uint32_t cap,
                                   const ShardRecord *__restrict__ moves,
                                   uint32_t *__restrict__ cursor,
                                   ShardRecord *__restrict__ out,
                                   int *__restrict__ err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= k) return;
  const ShardRecord r = moves[i];
  const int o = owner_of(r.k0, world);
  const uint32_t c = atomicAdd(&cursor[o], 1u);
  if (c < cap)
    out[(size_t)o * cap + c] = r;
  else
    atomicExch(err, CASCADE_ERR_INVALID);
}

inline int nblocks(size_t n) { return (int)((n + 255) / 256); }

}  // namespace

// Makes room in this rank's HBM pool for a batch of n blocks of h_sizes by
// demoting its least recently used payloads to its DRAM tier (prefix blocks
// last), and prepares a relocation record for each demoted payload whose
// key another rank owns, for the next begin to send.  A sharded put keeps
// its whole batch in HBM until the keys resolve, so the room is made first.
static int shard_prepare(Store &st, size_t n, const uint64_t *h_sizes,
                         int world, int rank, uint64_t *n_moves) {
  // Relocation records that a failed put never sent stay pending: the
  // owners' entries must still learn where those payloads went.  A records
  // step after a begin that failed sends them alone.
  *n_moves = st.shard_moves.size();
  st.shard_open = 0;
  st.shard_world = world;
  st.shard_rank = rank;
  if (!st.hbm || !st.dram_tier || n == 0) return CASCADE_OK;
  uint64_t need = 0;
  for (size_t i = 0; i < n; ++i)
    need += payload_bytes(h_sizes[i], q8_eligible(st, h_sizes[i], false));
  if (st.gpu_used + need <= st.pool_cap) return CASCADE_OK;
  const uint64_t deficit = st.gpu_used + need - st.pool_cap;
  Candidates cand;
  int rc = select_candidates(st, deficit, cand);
  if (rc) return rc;
  std::vector<Demotion> vic;
  {
    ArenaGuard guard{st.dram.get(), {}};
    uint64_t freed = 0, shm = st.shm_used;
    for (int c = 0; c < 2 && freed < deficit; ++c)
      for (const ScanRec &r : cand.c[c]) {
        if (freed >= deficit) break;
        const bool hq8 = (r.flags & kFlagQ8) != 0;
        const bool dq8 = hq8 || q8_eligible(st, r.size, true);
        const uint64_t acc = dram_accounted(r.size, dq8);
        if (shm + acc > st.dram->capacity()) break;
        const uint64_t off = st.dram->alloc(payload_bytes(r.size, dq8));
        if (off == DramArena::kNone) break;
        guard.held.emplace_back(off, payload_bytes(r.size, dq8));
        vic.push_back({r, off, dq8});
        freed += payload_bytes(r.size, hq8);
        shm += acc;
      }
    guard.keep();  // demote() owns the space now
  }
  if ((rc = demote(st, vic))) return rc;
  for (const Demotion &v : vic) {
    if (!(v.r.flags & kFlagHeld)) continue;  // this rank's own entry moved
    ShardRecord m;
    m.k0 = v.r.k0;
    m.k1 = v.r.k1;
    m.seq = kNoSeq;
    m.offset = v.dram_off;
    m.size = v.r.size;
    m.flags = (v.r.flags & kFlagPrefix) | kTierDram | (v.dq8 ? kFlagQ8 : 0) |
              kFlagRelocate;
    m.holder = (uint32_t)rank;
    m.src_idx = kMoveIdx;
    m.hdr_scale = v.r.hdr_scale;
    m.hdr_zp = v.r.hdr_zp;
    m.pad = 0;
    if (owner_of(m.k0, world) != rank) st.shard_moves.push_back(m);
  }
  *n_moves = st.shard_moves.size();
  return CASCADE_OK;
}

// Counts the keys the last cascade_shard_resolve stored, once its device
// work is done (it returns without waiting), and reports an index that ran
// out of probes there.
static int settle_resolve(Store &st) {
  if (!st.resolve_pending) return CASCADE_OK;
  const size_t m = st.resolve_pending;
  st.resolve_pending = 0;
  CB_CUDA(cudaStreamSynchronize(st.s));
  for (size_t j = 0; j < m; ++j)
    st.claimed += st.oc.h_status[j] == CASCADE_PUT_STORED;
  if (*st.oc.h_err) {
    set_error("device index is full: raise index_slots");
    return CASCADE_ERR_FULL;
  }
  return CASCADE_OK;
}

// The caller's stream waits for the store's main stream: outputs written
// there (exchange buffers) are ready on `stream` when an ABI call returns
// without synchronising.
static int join_back(Store &st, void *stream) {
  CB_CUDA(cudaEventRecord(st.ev, st.s));
  CB_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), st.ev, 0));
  return CASCADE_OK;
}

// The relocation records shard_prepare made, into the send buffer after
// the batch's records (cursor: the per-owner fill, on the device).
static int shard_send_moves(Store &st, int world, size_t cap,
                            uint32_t *cursor, uint8_t *d_send) {
  const size_t k = st.shard_moves.size();
  if (!k) return CASCADE_OK;
  const size_t bytes = k * sizeof(ShardRecord);
  if (bytes > st.h_moves_cap) {
    CB_CUDA(cudaStreamSynchronize(st.s));  // the old buffer may be in flight
    if (st.h_moves) CB_CUDA(cudaFreeHost(st.h_moves));
    st.h_moves = nullptr;
    st.h_moves_cap = 0;
    CB_CUDA(cudaHostAlloc(&st.h_moves, bytes, cudaHostAllocDefault));
    st.h_moves_cap = bytes;
  }
  std::memcpy(st.h_moves, st.shard_moves.data(), bytes);
  // shard_aux holds the cursors, then room for the moves (begin sized it)
  ShardRecord *d_moves = reinterpret_cast<ShardRecord *>(st.shard_aux + 2048);
  CB_CUDA(cudaMemcpyAsync(d_moves, st.h_moves, bytes, cudaMemcpyHostToDevice,
                          st.s));
  shard_moves_kernel<<<nblocks(k), 256, 0, st.s>>>(
      (int)k, world, (uint32_t)cap, d_moves, cursor,
      reinterpret_cast<ShardRecord *>(d_send), st.sc.err);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  st.shard_moves.clear();
  return CASCADE_OK;
}

// The batch's descriptors are uploaded (and, with digests_ready, its hash is
// under way on the hash stream): store it speculatively.  The records are
// written by shard_records once the caller knows the exchange's segment
// size.  Does not wait for the device.
static int shard_begin_staged(Store &st, size_t n, uint64_t max_size,
                              bool digests_ready, const uint8_t *h_prefix,
                              bool beside_hash = true) {
  CB_CHECK(can_speculate(st, n), CASCADE_ERR_NOMEM,
           "sharded put: the HBM pool cannot hold the whole batch");
  int rc = speculate_local(st, n, h_prefix, max_size, digests_ready,
                           beside_hash);
  if (rc) return rc;
  st.shard_open = n;
  return CASCADE_OK;
}

static int shard_check(const Store &st, int world, int rank) {
  CB_CHECK(world >= 1 && world <= 256 && rank >= 0 && rank < world,
           CASCADE_ERR_INVALID, "bad world/rank");
  CB_CHECK(st.hbm, CASCADE_ERR_UNSUPPORTED,
           "sharded puts need the HBM tier (use_gpu)");
  return CASCADE_OK;
}

static int shard_begin(Store &st, size_t n, const uint64_t *h_ptrs,
                       const uint64_t *h_sizes, const uint8_t *h_prefix,
                       int world, int rank) {
  st.shard_open = 0;
  int rc = shard_check(st, world, rank);
  if (rc) return rc;
  st.shard_rank = rank;
  st.shard_world = world;
  if (n == 0) return CASCADE_OK;
  uint64_t max_size = 0;
  if ((rc = upload_batch(st, n, h_ptrs, h_sizes, nullptr, &max_size)))
    return rc;
  return shard_begin_staged(st, n, max_size, false, h_prefix);
}

// begin for a slice of a batch whose digests the caller already computed
// on the device (one hash launch over the whole batch runs all its chains
// at once; slices hashed one by one would each run only theirs).
static int shard_begin_digests(Store &st, size_t n, const uint64_t *h_ptrs,
                               const uint64_t *h_sizes,
                               const uint8_t *h_prefix,
                               const uint8_t *d_digests, int world, int rank) {
  st.shard_open = 0;
  int rc = shard_check(st, world, rank);
  if (rc) return rc;
  st.shard_rank = rank;
  st.shard_world = world;
  if (n == 0) return CASCADE_OK;
  uint64_t max_size = 0;
  if ((rc = upload_batch(st, n, h_ptrs, h_sizes, nullptr, &max_size)))
    return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.digests, d_digests, n * 32,
                          cudaMemcpyDeviceToDevice, st.s));
  CB_CUDA(cudaEventRecord(st.ev2, st.s));
  return shard_begin_staged(st, n, max_size, true, h_prefix, false);
}

// Cut points of a sharded put: consecutive blocks whose payloads fill at
// most 4/5 of the HBM pool form a slice (a sharded put holds its batch in
// HBM until the keys resolve, and prepare demotes older payloads to the
// DRAM tier to make room for each slice).  Without a DRAM tier nothing can
// make room, so the batch stays one slice.  h_cuts gets n_slices + 1
// entries (at most max(n, 1) + 1).
static void shard_slices(const Store &st, size_t n, const uint64_t *h_sizes,
                         uint64_t *h_cuts, uint64_t *n_slices) {
  size_t k = 0;
  h_cuts[k++] = 0;
  uint64_t need = 0;
  for (size_t i = 0; i < n; ++i)
    need += payload_bytes(h_sizes[i], q8_eligible(st, h_sizes[i], false));
  // A batch that fits the pool's free space goes in one round: its payload
  // kernels then run beside its own hash instead of after a whole-batch one.
  if (st.hbm && st.dram_tier && st.gpu_used + need > st.pool_cap) {
    const uint64_t budget = st.pool_cap / 5 * 4;
    uint64_t acc = 0;
    for (size_t i = 0; i < n; ++i) {
      const uint64_t b =
          payload_bytes(h_sizes[i], q8_eligible(st, h_sizes[i], false));
      if (acc > 0 && acc + b > budget) {
        h_cuts[k++] = i;
        acc = 0;
      }
      acc += b;
    }
  }
  h_cuts[k++] = n;
  *n_slices = k - 1;
}

// Host blocks: staged to the device first.  Uniform pinned batches are
// hashed stripe by stripe while they cross PCIe, as put_batch_host does.
static int shard_begin_host(Store &st, size_t n, const uint8_t *const *blocks,
                            const uint64_t *sizes, const uint8_t *h_prefix,
                            int world, int rank) {
  st.shard_open = 0;
  int rc = shard_check(st, world, rank);
  if (rc) return rc;
  st.shard_rank = rank;
  st.shard_world = world;
  if (n == 0) return CASCADE_OK;
  uint64_t need = 0;
  for (size_t i = 0; i < n; ++i)
    need += payload_bytes(sizes[i], q8_eligible(st, sizes[i], false));
  CB_CHECK(st.gpu_used + need <= st.pool_cap, CASCADE_ERR_NOMEM,
           "sharded put: the HBM pool cannot hold the whole batch");
  bool taken = false;
  uint64_t max_size = 0;
  if ((rc = stage_host_striped(st, n, blocks, sizes, &taken, &max_size)))
    return rc;
  if (taken) return shard_begin_staged(st, n, max_size, true, h_prefix);
  std::vector<uint64_t> ptrs;
  if ((rc = stage_host_blocks(st, n, blocks, sizes, ptrs))) return rc;
  if ((rc = upload_batch(st, n, ptrs.data(), sizes, nullptr, &max_size)))
    return rc;
  return shard_begin_staged(st, n, max_size, false, h_prefix);
}

// The open batch's records (and shard_prepare's relocation records) into
// d_send, `world` segments of `cap` entries, once its digests are done.
// Sequence numbers order the batch as serial puts in (rank, block) order:
// rank in the high half, block + 1 in the low half (claims last one batch).
// Does not wait for the device.
static int shard_records(Store &st, size_t cap, uint8_t *d_send) {
  const size_t n = st.shard_open;
  const int world = st.shard_world, rank = st.shard_rank;
  CB_CHECK(cap >= n + st.shard_moves.size() &&
               cap <= (size_t)INT32_MAX / (size_t)world,
           CASCADE_ERR_INVALID,
           "cap must cover the batch and its relocation records "
           "(and world * cap < 2^31)");
  cudaStream_t s = st.s;
  CB_CUDA(cudaMemsetAsync(d_send, 0xff,
                          (size_t)world * cap * sizeof(ShardRecord), s));
  if (n == 0 && st.shard_moves.empty()) return CASCADE_OK;
  int rc = ensure_device_buf(st.shard_aux, st.oc_aux_cap,
                             2048 + st.shard_moves.size() * sizeof(ShardRecord),
                             s);
  if (rc) return rc;
  uint32_t *cursor = reinterpret_cast<uint32_t *>(st.shard_aux);
  CB_CUDA(cudaMemsetAsync(cursor, 0, 256 * sizeof(uint32_t), s));
  CB_CUDA(cudaMemsetAsync(st.sc.err, 0, sizeof(int), s));
  if (n > 0) {
    CB_CUDA(cudaStreamWaitEvent(s, st.ev2, 0));
    shard_records_kernel<<<nblocks(n), 256, 0, s>>>(
        (int)n, world, (uint32_t)rank, ((uint64_t)rank << 32) + 1,
        (uint32_t)cap, reinterpret_cast<const uint64_t *>(st.sc.digests),
        st.sc.off, st.sc.sizes, st.sc.flags, st.sc.hdr, cursor,
        reinterpret_cast<ShardRecord *>(d_send), st.sc.err);
    count_launches(1);
    CB_CUDA(cudaGetLastError());
  }
  if ((rc = shard_send_moves(st, world, cap, cursor, d_send))) return rc;
  if (n == 0) return CASCADE_OK;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_off, st.sc.off, n * 8,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_err, st.sc.err, sizeof(int),
                          cudaMemcpyDeviceToHost, s));
  return CASCADE_OK;
}

// As owner: decides the received records and writes one reply per record.
// Does not wait for the device; the keys it stored are counted by the next
// call on the store (settle_resolve).
static int shard_resolve(Store &st, const uint8_t *d_recv, size_t m,
                         uint8_t *d_reply) {
  if (m == 0) return CASCADE_OK;
  Scratch &oc = st.oc;
  int rc = ensure_scratch_of(st, oc, m);
  if (rc) return rc;
  if (st.claimed + m > st.nslots / 2 && (rc = grow_index(st))) return rc;
  cudaStream_t s = st.s;
  const ShardRecord *in = reinterpret_cast<const ShardRecord *>(d_recv);
  shard_unpack_kernel<<<nblocks(m), 256, 0, s>>>(
      (int)m, (uint32_t)st.shard_rank, in, oc.keys, oc.seqs, oc.off,
      oc.sizes, oc.flags, oc.hdr);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  // Entries whose holders demoted the payload follow it first.
  if ((rc = launch_index_apply_moves(st.slots, st.nslots - 1, d_recv, (int)m,
                                     (uint32_t)st.shard_rank, s)))
    return rc;
  CB_CUDA(cudaMemsetAsync(oc.err, 0, sizeof(int), s));
  const uint64_t epoch = st.next_epoch;
  st.next_epoch += m;
  rc = launch_index_claim(st.slots, st.nslots - 1, oc.keys, 2, oc.seqs,
                          (int)m, oc.slot, oc.err, s);
  if (!rc) rc = launch_index_resolve(st.slots, oc.slot, oc.seqs, (int)m,
                                     oc.status, s);
  if (!rc) rc = launch_index_commit(st.slots, oc.slot, oc.status, oc.off,
                                    oc.sizes, oc.flags, oc.hdr, epoch,
                                    (int)m, s);
  if (!rc) rc = launch_index_finalize(st.slots, oc.slot, oc.off, oc.status,
                                      (int)m, s);
  if (rc) return rc;
  shard_reply_kernel<<<nblocks(m), 256, 0, s>>>(
      (int)m, in, oc.status, reinterpret_cast<ShardReply *>(d_reply));
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  CB_CUDA(cudaMemcpyAsync(oc.h_status, oc.status, m, cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(oc.h_err, oc.err, sizeof(int), cudaMemcpyDeviceToHost, s));
  st.resolve_pending = m;
  return CASCADE_OK;
}

// With a DRAM tier, the blocks this rank stored for keys that other ranks
// own get a held slot in this rank's index (kFlagHeld), so that demotion
// here sees every payload in this rank's pool, in put order.  Queued on the
// main stream after the batch's statuses are final; *d_count receives how
// many (read after the caller's synchronisation, with oc.err).
static int shard_hold(Store &st, size_t n, uint32_t *d_count) {
  Scratch &oc = st.oc;
  int rc = ensure_scratch_of(st, oc, n);
  if (!rc && st.claimed + n > st.nslots / 2) rc = grow_index(st);
  if (rc) return rc;
  cudaStream_t s = st.s;
  CB_CUDA(cudaMemsetAsync(d_count, 0, sizeof(uint32_t), s));
  CB_CUDA(cudaMemsetAsync(oc.err, 0, sizeof(int), s));
  shard_held_kernel<<<nblocks(n), 256, 0, s>>>(
      (int)n, st.shard_world, (uint32_t)st.shard_rank,
      reinterpret_cast<const uint64_t *>(st.sc.digests), st.sc.status,
      st.sc.flags, oc.keys, oc.seqs, oc.flags, d_count);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  const uint64_t epoch = st.next_epoch;
  st.next_epoch += n;
  rc = launch_index_claim(st.slots, st.nslots - 1, oc.keys, 2, oc.seqs, (int)n,
                          oc.slot, oc.err, s);
  if (!rc) rc = launch_index_resolve(st.slots, oc.slot, oc.seqs, (int)n,
                                     oc.status, s);
  if (!rc) rc = launch_index_commit(st.slots, oc.slot, oc.status, st.sc.off,
                                    st.sc.sizes, oc.flags, st.sc.hdr, epoch,
                                    (int)n, s);
  return rc;
}

static int shard_end(Store &st, const uint8_t *d_back, size_t m, size_t n,
                     uint8_t *h_status, uint8_t *h_digests,
                     uint64_t *n_stored) {
  CB_CHECK(st.shard_open == n, CASCADE_ERR_INVALID,
           "shard_put_end: no open batch of this size");
  if (n == 0) return CASCADE_OK;
  cudaStream_t s = st.s;
  // The records kernel's error word (a segment over cap) is already on its
  // way to sc.h_err; read it once the stream is done.
  CB_CUDA(cudaStreamSynchronize(s));
  if (*st.sc.h_err) {
    st.shard_open = 0;
    set_error("shard_put_begin: a segment of the send buffer overflowed cap");
    return CASCADE_ERR_INVALID;
  }
  // 0xff marks "no reply yet"; every block must get exactly one reply.
  CB_CUDA(cudaMemsetAsync(st.sc.status, 0xff, n, s));
  CB_CUDA(cudaMemsetAsync(st.sc.err, 0, sizeof(int), s));
  shard_apply_kernel<<<nblocks(m), 256, 0, s>>>(
      (int)m, (int)n, reinterpret_cast<const ShardReply *>(d_back),
      st.sc.status, st.sc.err);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  int rc = launch_pool_free_unstored(st.d_pool, st.sc.req, st.sc.off,
                                     st.sc.status, (int)n, s);
  if (rc) return rc;
  uint32_t *d_held = reinterpret_cast<uint32_t *>(st.shard_aux) + 256;  // after the cursors
  if (st.dram_tier && (rc = shard_hold(st, n, d_held))) return rc;
  CB_CUDA(cudaMemcpyAsync(st.sc.h_status, st.sc.status, n,
                          cudaMemcpyDeviceToHost, s));
  CB_CUDA(cudaMemcpyAsync(st.sc.h_err, st.sc.err, sizeof(int),
                          cudaMemcpyDeviceToHost, s));
  uint32_t held = 0;
  if (st.dram_tier) {
    CB_CUDA(cudaMemcpyAsync(&held, d_held, sizeof(held),
                            cudaMemcpyDeviceToHost, s));
    CB_CUDA(cudaMemcpyAsync(st.oc.h_err, st.oc.err, sizeof(int),
                            cudaMemcpyDeviceToHost, s));
  }
  CB_CUDA(cudaStreamSynchronize(s));
  st.shard_open = 0;
  if (st.dram_tier && *st.oc.h_err) {
    set_error("device index is full: raise index_slots");
    return CASCADE_ERR_FULL;
  }
  st.claimed += held;
  CB_CHECK(*st.sc.h_err == 0, CASCADE_ERR_INVALID,
           "shard_put_end: a reply names no block of this batch");
  size_t missing = 0;
  for (size_t i = 0; i < n; ++i) missing += st.sc.h_status[i] == 0xff;
  CB_CHECK(missing == 0, CASCADE_ERR_INVALID,
           "shard_put_end: " + std::to_string(missing) +
               " blocks of this batch got no reply");
  // Index load is counted by the owners; the rest is this rank's.
  const uint64_t claimed = st.claimed;
  tally_put(st, n);
  st.claimed = claimed;
  return finish_put(st, n, true, h_status, h_digests, n_stored);
}

// ------------------------------------------------------------ sharded get
namespace {

// Unused queries look up the one unstorable key (kKeyMask), which is never
// found, so they touch no entry.
__global__ void shard_query_keys_kernel(int m,
                                        const ShardQuery *__restrict__ in,
                                        uint64_t *__restrict__ keys) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  const ShardQuery q = in[j];
  const bool used = q.src_idx != kUnused;
  keys[2 * (size_t)j] = used ? q.k0 : kKeyMask0;
  keys[2 * (size_t)j + 1] = used ? q.k1 : kKeyMask1;
}

// Holder of a live entry: the rank recorded at put time when the payload
// sits in another rank's pool, this rank otherwise.
__global__ void shard_locate_kernel(int m, uint32_t rank,
                                    const ShardQuery *__restrict__ in,
                                    const LookupInfo *__restrict__ info,
                                    ShardLocation *__restrict__ out) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  const LookupInfo f = info[j];
  ShardLocation r;
  r.src_idx = in[j].src_idx;
  r.found = r.src_idx == kUnused ? 0 : f.found;
  r.flags = f.flags;
  r.holder = (f.flags & kFlagRemote) ? ((f.flags >> 16) & 0xffu) : rank;
  r.offset = f.offset;
  r.size = f.size;
  r.hdr_scale = f.hdr_scale;
  r.hdr_zp = f.hdr_zp;
  r.pad = 0;
  out[j] = r;
}

}  // namespace

static int shard_attach(Store &st, int world, int rank,
                        const uint8_t *h_handles, const uint8_t *h_dram) {
  CB_CHECK(world >= 1 && world <= 256 && rank >= 0 && rank < world,
           CASCADE_ERR_INVALID, "bad world/rank");
  CB_CHECK(st.hbm && st.pool, CASCADE_ERR_UNSUPPORTED,
           "sharded gets need the HBM tier (use_gpu)");
  close_peer_pools(st);
  std::vector<uint8_t *> bases(world, nullptr);
  for (int r = 0; r < world; ++r) {
    if (r == rank) {
      bases[r] = st.pool;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, h_handles + (size_t)CASCADE_IPC_HANDLE_BYTES * r,
                sizeof(h));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != rank && bases[q]) cudaIpcCloseMemHandle(bases[q]);
      return cuda_fail(e, "cudaIpcOpenMemHandle (peer pool)");
    }
    bases[r] = static_cast<uint8_t *>(p);
  }
  st.peer_base = std::move(bases);
  st.peer_rank = rank;
  st.peer_dram.clear();
  st.peer_dram.resize(world);
  for (int r = 0; h_dram && r < world; ++r) {
    const uint8_t *rec = h_dram + (size_t)CASCADE_SHARD_DRAM_NAME_BYTES * r;
    if (r == rank || rec[0] == 0) continue;
    const std::string name(reinterpret_cast<const char *>(rec),
                           strnlen(reinterpret_cast<const char *>(rec), 55));
    uint64_t chunk = 0;
    std::memcpy(&chunk, rec + 56, 8);
    CB_CHECK(chunk > 0, CASCADE_ERR_INVALID, "bad DRAM tier record");
    st.peer_dram[r].reset(new DramView(name, chunk));
  }
  return CASCADE_OK;
}

// This store's DRAM tier as a shared arena others can map: its name and
// chunk size in a 64-byte record (all zero without a DRAM tier).  Shares
// the arena on the first call, which must come before the tier holds data.
static int shard_dram_name(Store &st, uint8_t *rec) {
  std::memset(rec, 0, CASCADE_SHARD_DRAM_NAME_BYTES);
  if (!st.dram_tier) return CASCADE_OK;
  if (st.dram->shared_name().empty()) {
    char name[56];
    std::snprintf(name, sizeof(name), "/cascade_b200_%d_%llx", (int)getpid(),
                  (unsigned long long)(uintptr_t)&st);
    CB_CHECK(st.dram->share(name), CASCADE_ERR_INVALID,
             "the DRAM tier already holds data; share it before the first put");
  }
  const std::string &nm = st.dram->shared_name();
  CB_CHECK(nm.size() < 56, CASCADE_ERR_INVALID, "DRAM tier name too long");
  std::memcpy(rec, nm.data(), nm.size());
  const uint64_t chunk = st.dram->chunk_bytes();
  std::memcpy(rec + 56, &chunk, 8);
  return CASCADE_OK;
}

// Routes each key to its owner: the padded query buffer is built in pinned
// memory and copied to d_send on the main stream.  Does not wait for it.
static int shard_get_begin(Store &st, size_t n, const uint8_t *h_keys,
                           size_t cap, uint8_t *d_send) {
  const int world = (int)st.peer_base.size();
  CB_CHECK(world > 0, CASCADE_ERR_INVALID,
           "sharded get: attach the ranks' pools first");
  CB_CHECK(cap >= n && cap <= (size_t)INT32_MAX / (size_t)world,
           CASCADE_ERR_INVALID,
           "cap must be at least the batch size (and world * cap < 2^31)");
  const size_t m = (size_t)world * cap;
  int rc = ensure_host_stage(st, m * std::max(sizeof(ShardQuery),
                                              sizeof(ShardLocation)));
  if (rc) return rc;
  // The stage may still be the source of the last get's copy.
  CB_CUDA(cudaStreamSynchronize(st.s));
  ShardQuery *q = reinterpret_cast<ShardQuery *>(st.h_stage);
  std::memset(q, 0xff, m * sizeof(ShardQuery));
  std::vector<size_t> cursor(world, 0);
  for (size_t i = 0; i < n; ++i) {
    const int o = owner_of(le64(h_keys + 16 * i), world);
    ShardQuery &r = q[(size_t)o * cap + cursor[o]++];
    r.k0 = le64(h_keys + 16 * i);
    r.k1 = le64(h_keys + 16 * i + 8);
    r.src_idx = (uint32_t)i;
    r.pad0 = 0;
    r.pad1 = 0;
  }
  CB_CUDA(cudaMemcpyAsync(d_send, st.h_stage, m * sizeof(ShardQuery),
                          cudaMemcpyHostToDevice, st.s));
  st.shard_get_open = n;
  return CASCADE_OK;
}

// As owner: one location per received query.  Does not wait for the device.
static int shard_lookup(Store &st, const uint8_t *d_recv, size_t m,
                        uint8_t *d_reply) {
  CB_CHECK(st.peer_rank >= 0, CASCADE_ERR_INVALID,
           "sharded get: attach the ranks' pools first");
  if (m == 0) return CASCADE_OK;
  Scratch &oc = st.oc;
  int rc = ensure_scratch_of(st, oc, m);
  if (rc) return rc;
  cudaStream_t s = st.s;
  const ShardQuery *in = reinterpret_cast<const ShardQuery *>(d_recv);
  shard_query_keys_kernel<<<nblocks(m), 256, 0, s>>>((int)m, in, oc.keys);
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  const uint64_t epoch = st.next_epoch;
  st.next_epoch += m;
  rc = launch_index_lookup(st.slots, st.nslots - 1, oc.keys, 2, (int)m, 1,
                           epoch, oc.info, s);
  if (rc) return rc;
  shard_locate_kernel<<<nblocks(m), 256, 0, s>>>(
      (int)m, (uint32_t)st.peer_rank, in, oc.info,
      reinterpret_cast<ShardLocation *>(d_reply));
  count_launches(1);
  CB_CUDA(cudaGetLastError());
  return CASCADE_OK;
}

static int shard_get_end(Store &st, const uint8_t *d_back, size_t m, size_t n,
                         const uint64_t *h_out, const uint64_t *h_caps,
                         uint64_t *h_sizes, uint8_t *h_found,
                         uint64_t *n_found) {
  CB_CHECK(st.shard_get_open == n, CASCADE_ERR_INVALID,
           "shard_get_end: no open get of this size");
  st.shard_get_open = 0;
  if (n == 0) return CASCADE_OK;
  int rc = ensure_scratch(st, n);
  if (!rc) rc = ensure_host_stage(st, m * sizeof(ShardLocation));
  if (rc) return rc;
  CB_CUDA(cudaMemcpyAsync(st.h_stage, d_back, m * sizeof(ShardLocation),
                          cudaMemcpyDeviceToHost, st.s));
  CB_CUDA(cudaStreamSynchronize(st.s));
  const ShardLocation *loc = reinterpret_cast<const ShardLocation *>(st.h_stage);
  const int world = (int)st.peer_base.size();
  std::vector<uint8_t> seen(n, 0), deliver(n, 0);
  std::vector<uint64_t> bases(n, 0), dram_src(n, 0);
  uint64_t found = 0;
  size_t named = 0;
  for (size_t j = 0; j < m; ++j) {
    const ShardLocation &r = loc[j];
    if (r.src_idx == kUnused) continue;
    CB_CHECK(r.src_idx < n && !seen[r.src_idx], CASCADE_ERR_INVALID,
             "shard_get_end: the locations do not name each key once");
    seen[r.src_idx] = 1;
    ++named;
    LookupInfo &f = st.sc.h_info[r.src_idx];
    f.found = r.found;
    f.flags = r.flags;
    f.offset = r.offset;
    f.size = r.size;
    f.hdr_scale = r.hdr_scale;
    f.hdr_zp = r.hdr_zp;
    f.slot = kNoSlot;
    f.pad = 0;
    if (!r.found) continue;
    CB_CHECK((int)r.holder < world, CASCADE_ERR_INVALID,
             "shard_get_end: holder rank out of range");
    if (r.flags & kTierHbm) {
      bases[r.src_idx] = (uint64_t)(uintptr_t)st.peer_base[r.holder];
      continue;
    }
    // In the holder's DRAM tier: this rank's own arena, or the holder's
    // shared arena mapped here.  (Not promoted: a location carries no index
    // slot of this rank.)
    const uint64_t pay = payload_bytes(r.size, (r.flags & kFlagQ8) != 0);
    const uint8_t *p = nullptr;
    if ((int)r.holder == st.peer_rank)
      p = st.dram ? st.dram->ptr(r.offset) : nullptr;
    else if (r.holder < st.peer_dram.size() && st.peer_dram[r.holder])
      p = st.peer_dram[r.holder]->ptr(r.offset, pay);
    CB_CHECK(p != nullptr, CASCADE_ERR_UNSUPPORTED,
             "sharded get: the holder's DRAM tier is not mapped here");
    dram_src[r.src_idx] = (uint64_t)(uintptr_t)p;
  }
  CB_CHECK(named == n, CASCADE_ERR_INVALID,
           "shard_get_end: the locations do not name each key once");
  for (size_t i = 0; i < n; ++i) {
    const LookupInfo &f = st.sc.h_info[i];
    const uint64_t size =
        f.found ? ((f.flags & kFlagQ8) ? 2 * (f.size / 2) : f.size) : 0;
    if (h_sizes) h_sizes[i] = size;
    if (h_found) h_found[i] = f.found ? 1 : 0;
    found += f.found ? 1 : 0;
    deliver[i] = (!f.found || size <= h_caps[i]) ? 1 : 0;
  }
  if (n_found) *n_found = found;
  return deliver_locked(st, n, h_out, deliver.data(), bases.data(),
                        dram_src.data());
}

}  // namespace cb

// ------------------------------------------------------------------ C-ABI
struct cascade_store {
  cb::Store *impl;
};

namespace {
// The store's streams are non-blocking, so they do not wait for the legacy
// default stream by themselves: the caller's stream (NULL = the legacy
// default stream, which is also torch's default) is always joined with an
// event before the inputs are read.
int join_caller(cb::Store &st, void *stream) {
  CB_CUDA(cudaEventRecord(st.ev, static_cast<cudaStream_t>(stream)));
  CB_CUDA(cudaStreamWaitEvent(st.s, st.ev, 0));
  return CASCADE_OK;
}
}  // namespace

#define STORE_ENTRY(s)                                                       \
  cb::clear_error();                                                         \
  CB_CHECK((s) && (s)->impl, CASCADE_ERR_INVALID, "null store");             \
  cb::Store &st = *(s)->impl;                                                \
  std::lock_guard<std::mutex> lock(st.mu);                                   \
  cb::DeviceGuard guard(st.dev);                                             \
  if (int settle_rc = cb::settle_resolve(st)) return settle_rc

extern "C" void cascade_struct_sizes(size_t *config_bytes,
                                     size_t *stats_bytes) {
  if (config_bytes) *config_bytes = sizeof(cascade_config_t);
  if (stats_bytes) *stats_bytes = sizeof(cascade_stats_t);
}

extern "C" void cascade_config_init(cascade_config_t *c) {
  if (!c) return;
  std::memset(c, 0, sizeof(*c));
  c->gpu_capacity_bytes = 32ull << 30;
  c->gpu_device_id = 0;
  c->use_gpu = 1;
  c->shm_capacity_bytes = 64ull << 30;
  c->shm_path = "/dev/shm/cascade";
  c->lustre_path = "cascade_store";
  c->lustre_stripe_size = 1ull << 20;
  c->lustre_stripe_count = 16;
  c->dedup_enabled = 1;
  c->compression_enabled = 1;
  c->num_io_threads = 8;
  c->semantic_eviction = 1;
  c->promotion_enabled = 1;
  c->prefetch_enabled = 1;
  c->prefetch_threads = 2;
  c->prefetch_queue_size = 64;
  c->kv_compression = 0;
  c->aggregated_lustre = 0;
  c->agg_file_size = 256ull << 20;
}

extern "C" int cascade_store_create(const cascade_config_t *cfg,
                                    cascade_store_t **out) {
  cb::clear_error();
  CB_CHECK(cfg && out, CASCADE_ERR_INVALID, "null argument");
  cb::Store *impl = nullptr;
  int rc = cb::create_store(cfg, &impl);
  if (rc) return rc;
  *out = new cascade_store{impl};
  return CASCADE_OK;
}

extern "C" int cascade_store_destroy(cascade_store_t *s) {
  cb::clear_error();
  if (!s) return CASCADE_OK;
  if (s->impl) cb::destroy_store(s->impl);
  delete s;
  return CASCADE_OK;
}

extern "C" int cascade_store_put(cascade_store_t *s, const char *block_id,
                                 const uint8_t *data, uint64_t size,
                                 int is_prefix, int *stored) {
  STORE_ENTRY(s);
  CB_CHECK(block_id && stored && (data || !size), CASCADE_ERR_INVALID,
           "null argument");
  cb::Key k;
  bool known;
  int rc = cb::key_of(st, block_id, true, &k, &known);
  if (rc) return rc;
  return cb::put_host_locked(st, k, data, size, is_prefix, stored);
}

extern "C" int cascade_store_get(cascade_store_t *s, const char *block_id,
                                 uint8_t *out, uint64_t out_capacity,
                                 int *found, uint64_t *size) {
  STORE_ENTRY(s);
  CB_CHECK(block_id && found && size && (out || !out_capacity),
           CASCADE_ERR_INVALID, "null argument");
  cb::Key k;
  bool known;
  int rc = cb::key_of(st, block_id, false, &k, &known);
  if (rc) return rc;
  if (!known) {
    ++st.misses;
    *found = 0;
    *size = 0;
    return CASCADE_OK;
  }
  return cb::get_host_locked(st, k, out, out_capacity, found, size);
}

extern "C" int cascade_store_contains(cascade_store_t *s, const char *block_id,
                                      int *present) {
  STORE_ENTRY(s);
  CB_CHECK(block_id && present, CASCADE_ERR_INVALID, "null argument");
  cb::Key k;
  bool known;
  int rc = cb::key_of(st, block_id, false, &k, &known);
  if (rc) return rc;
  *present = 0;
  if (!known) return CASCADE_OK;
  if ((rc = cb::ensure_scratch(st, 1))) return rc;
  st.sc.h_keys[0] = k.k0;
  st.sc.h_keys[1] = k.k1;
  CB_CUDA(cudaMemcpyAsync(st.sc.keys, st.sc.h_keys, 16, cudaMemcpyHostToDevice,
                          st.s));
  if ((rc = cb::lookup_locked(st, 1, false))) return rc;
  *present = st.sc.h_info[0].found ? 1 : 0;
  return CASCADE_OK;
}

extern "C" int cascade_store_get_stats(cascade_store_t *s,
                                       cascade_stats_t *o) {
  STORE_ENTRY(s);
  CB_CHECK(o, CASCADE_ERR_INVALID, "null argument");
  std::memset(o, 0, sizeof(*o));
  o->gpu_used = st.gpu_used;
  o->shm_used = st.shm_used;
  o->gpu_hits = st.gpu_hits;
  o->shm_hits = st.shm_hits;
  o->misses = st.misses;
  o->dedup_hits = st.dedup_hits;
  o->gpu_evictions = st.gpu_evictions;
  o->promotions_to_gpu = st.promotions_to_gpu;
  o->compression_savings_bytes = st.compression_savings;
  o->shm_puts = st.shm_puts;
  return CASCADE_OK;
}

extern "C" int cascade_store_clear(cascade_store_t *s) {
  STORE_ENTRY(s);
  return cb::clear_store(st);
}

extern "C" int cascade_store_flush(cascade_store_t *s) {
  STORE_ENTRY(s);
  CB_CUDA(cudaStreamSynchronize(st.s));
  return CASCADE_OK;
}

extern "C" int cascade_store_key_of(cascade_store_t *s, const char *block_id,
                                    uint8_t key_out[16]) {
  STORE_ENTRY(s);
  CB_CHECK(block_id && key_out, CASCADE_ERR_INVALID, "null argument");
  cb::Key k;
  bool known;
  int rc = cb::key_of(st, block_id, true, &k, &known);
  if (rc) return rc;
  for (int i = 0; i < 8; ++i) {
    key_out[i] = (uint8_t)(k.k0 >> (8 * i));
    key_out[8 + i] = (uint8_t)(k.k1 >> (8 * i));
  }
  return CASCADE_OK;
}

extern "C" int cascade_store_put_batch(cascade_store_t *s, size_t n,
                                       const uint64_t *h_ptrs,
                                       const uint64_t *h_sizes,
                                       const uint8_t *h_keys,
                                       const uint8_t *h_prefix,
                                       uint8_t *h_status, uint8_t *h_digests,
                                       void *stream, uint64_t *n_stored) {
  STORE_ENTRY(s);
  if (n_stored) *n_stored = 0;
  if (n == 0) return CASCADE_OK;
  CB_CHECK(h_ptrs && h_sizes, CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  return cb::put_batch_locked(st, n, h_ptrs, h_sizes, h_keys, h_prefix,
                              h_status, h_digests, n_stored);
}

extern "C" int cascade_store_put_batch_host(
    cascade_store_t *s, size_t n, const uint8_t *const *h_blocks,
    const uint64_t *h_sizes, const uint8_t *h_keys, const uint8_t *h_prefix,
    uint8_t *h_status, uint8_t *h_digests, uint64_t *n_stored) {
  STORE_ENTRY(s);
  if (n_stored) *n_stored = 0;
  if (n == 0) return CASCADE_OK;
  CB_CHECK(h_blocks && h_sizes, CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  return cb::put_batch_host_locked(st, n, h_blocks, h_sizes, h_keys, h_prefix,
                                   h_status, h_digests, n_stored);
}

extern "C" int cascade_store_get_batch(cascade_store_t *s, size_t n,
                                       const uint8_t *h_keys,
                                       const uint64_t *h_out_ptrs,
                                       const uint64_t *h_out_caps,
                                       uint64_t *h_sizes, uint8_t *h_found,
                                       void *stream, uint64_t *n_found) {
  STORE_ENTRY(s);
  if (n_found) *n_found = 0;
  if (n == 0) return CASCADE_OK;
  CB_CHECK(h_keys && h_out_ptrs && h_out_caps, CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  return cb::get_batch_locked(st, n, h_keys, h_out_ptrs, h_out_caps, h_sizes,
                              h_found, n_found);
}

extern "C" int cascade_store_put_kv_batch(
    cascade_store_t *s, size_t n, const uint8_t *h_keys, uint32_t layers,
    uint32_t heads, uint32_t seq, uint32_t head_dim,
    const cascade_kv_tensor_t *d_src, int src_dtype, const uint8_t *h_prefix,
    uint8_t *h_status, void *stream, uint64_t *n_stored) {
  STORE_ENTRY(s);
  if (n_stored) *n_stored = 0;
  if (n == 0) return CASCADE_OK;
  CB_CHECK(h_keys && d_src, CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  CB_CHECK(layers && heads && seq && head_dim, CASCADE_ERR_INVALID,
           "layers, heads, seq_len and head_dim must be positive");
  CB_CHECK(src_dtype >= CASCADE_KV_FP16 && src_dtype <= CASCADE_KV_FP32,
           CASCADE_ERR_INVALID, "src_dtype must be FP16, BF16 or FP32");
  if (int rc = join_caller(st, stream)) return rc;
  const uint32_t shape[4] = {layers, heads, seq, head_dim};
  return cb::put_kv_locked(st, n, h_keys, shape, d_src, src_dtype, h_prefix,
                           h_status, n_stored);
}

extern "C" int cascade_store_get_kv_batch(
    cascade_store_t *s, size_t n, const uint8_t *h_keys, uint32_t layers,
    uint32_t heads, uint32_t seq, uint32_t head_dim,
    const cascade_kv_tensor_t *d_dst, uint8_t *h_found, void *stream,
    uint64_t *n_found) {
  STORE_ENTRY(s);
  if (n_found) *n_found = 0;
  if (n == 0) return CASCADE_OK;
  CB_CHECK(h_keys && d_dst && h_found, CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  CB_CHECK(layers && heads && seq && head_dim, CASCADE_ERR_INVALID,
           "layers, heads, seq_len and head_dim must be positive");
  if (int rc = join_caller(st, stream)) return rc;
  const uint32_t shape[4] = {layers, heads, seq, head_dim};
  int rc = cb::get_kv_batch_locked(st, n, h_keys, shape, d_dst, h_found,
                                   n_found);
  if (rc) return rc;
  return cb::join_back(st, stream);
}

extern "C" int cascade_shard_put_begin(cascade_store_t *s, size_t n,
                                       const uint64_t *h_ptrs,
                                       const uint64_t *h_sizes,
                                       const uint8_t *h_prefix, int world,
                                       int rank, void *stream) {
  STORE_ENTRY(s);
  CB_CHECK(n == 0 || (h_ptrs && h_sizes), CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(n <= (size_t)UINT32_MAX - 1, CASCADE_ERR_INVALID,
           "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  return cb::shard_begin(st, n, h_ptrs, h_sizes, h_prefix, world, rank);
}

extern "C" int cascade_shard_put_begin_digests(
    cascade_store_t *s, size_t n, const uint64_t *h_ptrs,
    const uint64_t *h_sizes, const uint8_t *h_prefix,
    const uint8_t *d_digests, int world, int rank, void *stream) {
  STORE_ENTRY(s);
  CB_CHECK(n == 0 || (h_ptrs && h_sizes && d_digests), CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(((uintptr_t)d_digests & 3u) == 0, CASCADE_ERR_INVALID,
           "d_digests must be 4-byte aligned");
  CB_CHECK(n <= (size_t)UINT32_MAX - 1, CASCADE_ERR_INVALID,
           "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  return cb::shard_begin_digests(st, n, h_ptrs, h_sizes, h_prefix, d_digests,
                                 world, rank);
}

extern "C" int cascade_shard_put_slices(cascade_store_t *s, size_t n,
                                        const uint64_t *h_sizes,
                                        uint64_t *h_cuts, uint64_t *n_slices) {
  STORE_ENTRY(s);
  CB_CHECK((n == 0 || h_sizes) && h_cuts && n_slices, CASCADE_ERR_INVALID,
           "null argument");
  cb::shard_slices(st, n, h_sizes, h_cuts, n_slices);
  return CASCADE_OK;
}

extern "C" int cascade_shard_put_begin_host(
    cascade_store_t *s, size_t n, const uint8_t *const *h_blocks,
    const uint64_t *h_sizes, const uint8_t *h_prefix, int world, int rank,
    void *stream) {
  STORE_ENTRY(s);
  CB_CHECK(n == 0 || (h_blocks && h_sizes), CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(n <= (size_t)UINT32_MAX - 1, CASCADE_ERR_INVALID,
           "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  return cb::shard_begin_host(st, n, h_blocks, h_sizes, h_prefix, world, rank);
}

extern "C" int cascade_shard_put_records(cascade_store_t *s, size_t cap,
                                         uint8_t *d_send, void *stream) {
  STORE_ENTRY(s);
  CB_CHECK(d_send, CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(((uintptr_t)d_send & 15u) == 0, CASCADE_ERR_INVALID,
           "d_send must be 16-byte aligned");
  if (int rc = join_caller(st, stream)) return rc;
  int rc = cb::shard_records(st, cap, d_send);
  if (rc) return rc;
  return cb::join_back(st, stream);
}

extern "C" int cascade_shard_resolve(cascade_store_t *s, const uint8_t *d_recv,
                                     size_t m, uint8_t *d_reply, void *stream) {
  STORE_ENTRY(s);
  CB_CHECK(m == 0 || (d_recv && d_reply), CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(m <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  int rc = cb::shard_resolve(st, d_recv, m, d_reply);
  if (rc) return rc;
  return cb::join_back(st, stream);
}

extern "C" int cascade_shard_put_end(cascade_store_t *s, const uint8_t *d_back,
                                     size_t m, size_t n, uint8_t *h_status,
                                     uint8_t *h_digests, uint64_t *n_stored,
                                     void *stream) {
  STORE_ENTRY(s);
  if (n_stored) *n_stored = 0;
  CB_CHECK(n == 0 || d_back, CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(m >= n && m <= (size_t)INT32_MAX, CASCADE_ERR_INVALID,
           "m: the padded reply count (world * cap)");
  if (int rc = join_caller(st, stream)) return rc;
  return cb::shard_end(st, d_back, m, n, h_status, h_digests, n_stored);
}

extern "C" int cascade_shard_pool_handle(cascade_store_t *s,
                                         uint8_t *h_handle) {
  STORE_ENTRY(s);
  CB_CHECK(h_handle, CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(st.hbm && st.pool, CASCADE_ERR_UNSUPPORTED,
           "sharded gets need the HBM tier (use_gpu)");
  static_assert(sizeof(cudaIpcMemHandle_t) == CASCADE_IPC_HANDLE_BYTES,
                "IPC handle size");
  cudaIpcMemHandle_t h;
  CB_CUDA(cudaIpcGetMemHandle(&h, st.pool));
  std::memcpy(h_handle, &h, sizeof(h));
  return CASCADE_OK;
}

extern "C" int cascade_shard_attach_pools(cascade_store_t *s, int world,
                                          int rank, const uint8_t *h_handles,
                                          const uint8_t *h_dram_names) {
  STORE_ENTRY(s);
  CB_CHECK(h_handles, CASCADE_ERR_INVALID, "null argument");
  return cb::shard_attach(st, world, rank, h_handles, h_dram_names);
}

extern "C" int cascade_shard_dram_name(cascade_store_t *s, uint8_t *h_record) {
  STORE_ENTRY(s);
  CB_CHECK(h_record, CASCADE_ERR_INVALID, "null argument");
  return cb::shard_dram_name(st, h_record);
}

extern "C" int cascade_shard_put_prepare(cascade_store_t *s, size_t n,
                                         const uint64_t *h_sizes, int world,
                                         int rank, uint64_t *n_moves) {
  STORE_ENTRY(s);
  CB_CHECK(n_moves && (n == 0 || h_sizes), CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(world >= 1 && world <= 256 && rank >= 0 && rank < world,
           CASCADE_ERR_INVALID, "bad world/rank");
  return cb::shard_prepare(st, n, h_sizes, world, rank, n_moves);
}

extern "C" int cascade_shard_detach_pools(cascade_store_t *s) {
  STORE_ENTRY(s);
  CB_CUDA(cudaStreamSynchronize(st.s));
  cb::close_peer_pools(st);
  return CASCADE_OK;
}

extern "C" int cascade_shard_get_begin(cascade_store_t *s, size_t n,
                                       const uint8_t *h_keys, size_t cap,
                                       uint8_t *d_send, void *stream) {
  STORE_ENTRY(s);
  CB_CHECK(d_send && (n == 0 || h_keys), CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(n <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  int rc = cb::shard_get_begin(st, n, h_keys, cap, d_send);
  if (rc) return rc;
  return cb::join_back(st, stream);
}

extern "C" int cascade_shard_lookup(cascade_store_t *s, const uint8_t *d_recv,
                                    size_t m, uint8_t *d_reply, void *stream) {
  STORE_ENTRY(s);
  CB_CHECK(m == 0 || (d_recv && d_reply), CASCADE_ERR_INVALID,
           "null argument");
  CB_CHECK(m <= (size_t)INT32_MAX, CASCADE_ERR_INVALID, "batch too large");
  if (int rc = join_caller(st, stream)) return rc;
  int rc = cb::shard_lookup(st, d_recv, m, d_reply);
  if (rc) return rc;
  return cb::join_back(st, stream);
}

extern "C" int cascade_shard_get_end(cascade_store_t *s, const uint8_t *d_back,
                                     size_t m, size_t n,
                                     const uint64_t *h_out_ptrs,
                                     const uint64_t *h_out_caps,
                                     uint64_t *h_sizes, uint8_t *h_found,
                                     uint64_t *n_found, void *stream) {
  STORE_ENTRY(s);
  if (n_found) *n_found = 0;
  CB_CHECK(n == 0 || (d_back && h_out_ptrs && h_out_caps),
           CASCADE_ERR_INVALID, "null argument");
  CB_CHECK(m >= n && m <= (size_t)INT32_MAX, CASCADE_ERR_INVALID,
           "m: the padded location count (world * cap)");
  if (int rc = join_caller(st, stream)) return rc;
  return cb::shard_get_end(st, d_back, m, n, h_out_ptrs, h_out_caps, h_sizes,
                           h_found, n_found);
}
