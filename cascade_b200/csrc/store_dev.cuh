// Device-resident metadata of the block store: the block index (an
// open-addressing hash table keyed by 16-byte block keys) and the HBM pool's
// size-class allocator.  Both live entirely in device memory and are updated
// by batched kernels, so a batch of puts or gets costs a few launches rather
// than a host round trip per block.
//
// Reference counterparts: ShardedIndex<V> (cascade.hpp:69-124,
// cascade_core.cpp:56-234) for the index and LRU metadata; GPUMemoryPool
// (gpu_backend.cu:34-163) for the allocator.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cb {

// ------------------------------------------------------------------ keys
// A block key is the 16 bytes a reference block id names: for content
// addressed blocks, SHA-256 digest bytes 0..15 (compute_block_id,
// cascade_core.cpp:43-53).  In the table a key is stored XOR-ed with
// kKeyMask so that the all-zero key (block id "000...0") is storable; the
// one unstorable key is kKeyMask itself.
constexpr uint64_t kKeyMask0 = 0x9e3779b97f4a7c15ull;
constexpr uint64_t kKeyMask1 = 0xc2b2ae3d27d4eb4full;

struct Key {
  uint64_t k0, k1;  // bytes 0..7 and 8..15, little-endian
};

// ----------------------------------------------------------------- index
enum SlotState : uint32_t { kReserved = 0, kLive = 1 };

enum SlotFlags : uint32_t {
  kFlagPrefix = 1u << 0,  // is_prefix at put (semantic eviction)
  kFlagQ8 = 1u << 1,      // payload is INT8 codes; header in hdr_*
  kTierHbm = 1u << 2,     // payload in the HBM pool
  kTierDram = 1u << 3,    // payload in the pinned DRAM arena
  kFlagRemote = 1u << 4,  // payload held by another rank (bits 16..23)
  // Sharded store: this rank holds the payload of a key another rank owns
  // (the slot tracks the payload for demotion; the owner's slot answers
  // lookups).
  kFlagHeld = 1u << 5,
  // Sharded exchange: the record moves an owner's entry (its holder demoted
  // the payload) instead of claiming the key.
  kFlagRelocate = 1u << 6,
};

// Sharded dedup exchange (one box, one rank per GPU).  A rank sends one
// record per block of its batch to the rank that owns the block's key;
// the owner answers with a reply per record.  The exchange buffers are
// padded to a fixed number of entries per rank; an entry whose src_idx is
// kUnused (all bytes 0xff) carries nothing.
constexpr uint32_t kUnused = 0xffffffffu;
// src_idx of a record that relocates an owner's entry (kFlagRelocate).
constexpr uint32_t kMoveIdx = 0xfffffffeu;
// Sequence number of a request that takes part in no claim.
constexpr uint64_t kNoSeq = ~0ull;
struct ShardRecord {
  uint64_t k0, k1;     // key: digest bytes 0..15, little-endian
  uint64_t seq;        // global sequence number: the smallest stores
  uint64_t offset;     // payload offset in the holder's pool (or invalid)
  uint64_t size;       // logical block size
  uint32_t flags;      // SlotFlags of the holder's copy
  uint32_t holder;     // rank whose pool holds the payload
  uint32_t src_idx;    // position of the block in the holder's batch
  uint32_t hdr_scale;  // INT8 header
  uint32_t hdr_zp;
  uint32_t pad;
};
static_assert(sizeof(ShardRecord) == 64, "shard record layout");

// Sharded get: a key routed to its owner rank.
struct ShardQuery {
  uint64_t k0, k1;     // key: digest bytes 0..15, little-endian
  uint32_t src_idx;    // position of the key in the requester's batch
  uint32_t pad0;
  uint64_t pad1;
};
static_assert(sizeof(ShardQuery) == 32, "shard query layout");

// The owner's answer to a query: where the block lives.
struct ShardLocation {
  uint32_t src_idx;
  uint32_t found;      // 1 when the key is live
  uint32_t flags;      // SlotFlags of the stored copy
  uint32_t holder;     // rank whose pool holds the payload
  uint64_t offset;     // payload offset in the holder's pool
  uint64_t size;       // logical block size
  uint32_t hdr_scale;  // INT8 header
  uint32_t hdr_zp;
  uint64_t pad;
};
static_assert(sizeof(ShardLocation) == 48, "shard location layout");

struct ShardReply {
  uint32_t src_idx;
  uint32_t status;     // CASCADE_PUT_*
};
static_assert(sizeof(ShardReply) == 8, "shard reply layout");

// Owner rank of a key among `world` ranks: the top bits of digest byte 0
// (the low byte of k0), scaled to the rank count.
__host__ __device__ inline int owner_of(uint64_t k0, int world) {
  return (int)(((k0 & 0xffu) * (uint64_t)world) >> 8);
}

struct __align__(16) Slot {
  uint64_t k0, k1;     // stored key (key ^ mask); (0,0) = empty slot
  uint64_t claim;      // ~(smallest claimant sequence number); 0 = idle
  uint32_t state;      // SlotState
  uint32_t flags;      // SlotFlags
  uint64_t offset;     // payload offset in its tier
  uint64_t size;       // logical size: the byte count get() returns
  uint32_t hdr_scale;  // Q8 header: float scale bits
  uint32_t hdr_zp;     // Q8 header: zero point (low byte)
  uint64_t epoch;      // last put/get, for LRU victim choice
};
static_assert(sizeof(Slot) == 64, "slot is one 64-byte line half");

constexpr uint64_t kInvalidOffset = ~0ull;
constexpr uint32_t kNoSlot = 0xffffffffu;
constexpr int kMaxProbe = 1 << 14;

// What a lookup returns for one key.
struct LookupInfo {
  uint32_t found;   // 1 when the key is live
  uint32_t flags;
  uint64_t offset;
  uint64_t size;
  uint32_t hdr_scale;
  uint32_t hdr_zp;
  uint32_t slot;
  uint32_t pad;
};
static_assert(sizeof(LookupInfo) == 40, "lookup record layout");

// ------------------------------------------------------------------ pool
constexpr uint64_t kPoolAlign = 256;
constexpr int kNumClasses = 16 + 8 * 40;

// Size classes: 256-byte units; 1..16 units exact, then 8 classes per
// power of two (at most 12.5 % rounding).  Sizes that are a power of two
// times 1..15/8 (2 MiB, 2.5 MiB, 5 MiB ...) are exact.
__host__ __device__ inline int log2_floor(uint64_t u) {
#ifdef __CUDA_ARCH__
  return 63 - __clzll((long long)u);
#else
  return 63 - __builtin_clzll(u);
#endif
}

__host__ __device__ inline int size_class(uint64_t bytes) {
  uint64_t u = (bytes + kPoolAlign - 1) / kPoolAlign;
  if (u == 0) u = 1;
  if (u <= 16) return (int)(u - 1);
  int e = log2_floor(u);
  uint64_t step = 1ull << (e - 3);
  uint64_t m = (u + step - 1) / step - 8;  // 0..8
  if (m == 8) { e += 1; m = 0; }
  return 16 + (e - 4) * 8 + (int)m;
}

__host__ __device__ inline uint64_t class_bytes(int c) {
  if (c < 16) return (uint64_t)(c + 1) * kPoolAlign;
  int e = (c - 16) / 8 + 4;
  uint64_t m = (uint64_t)((c - 16) % 8);
  return (8 + m) * (1ull << (e - 3)) * kPoolAlign;
}

struct PoolDev {
  uint64_t bump;       // first never-allocated byte
  uint64_t capacity;   // pool bytes
  uint64_t overflow;   // frees dropped because a stack was full (a bug)
  uint64_t pad;
  uint64_t *stack[kNumClasses];  // free offsets per class (device arrays)
  uint32_t top[kNumClasses];     // entries in stack[c]
  uint32_t cap[kNumClasses];     // capacity of stack[c]
  uint32_t taken[kNumClasses];   // pops claimed by the running alloc batch
};

// Epoch buckets per class of the demotion-candidate histogram.
constexpr int kVictimBuckets = 1024;

// One live slot as reported by a scan (victim selection for demotion).
struct ScanRec {
  uint32_t slot;
  uint32_t flags;
  uint64_t size;
  uint64_t offset;
  uint64_t epoch;
  uint32_t hdr_scale;
  uint32_t hdr_zp;
  uint64_t k0, k1;  // the key (unmasked)
};
static_assert(sizeof(ScanRec) == 56, "scan record layout");

constexpr uint64_t kNoRequest = ~0ull;  // pool request: allocate nothing

#ifdef __CUDACC__
// splitmix64 finaliser over both halves of a stored key: the home slot.
__device__ __forceinline__ uint64_t slot_hash(uint64_t s0, uint64_t s1) {
  uint64_t z = s0 ^ (s1 * 0xbf58476d1ce4e5b9ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// 128-bit compare-and-swap (sm_90+): *addr == {c0,c1} ? {n0,n1} : keep;
// returns the previous value.
__device__ __forceinline__ void cas128(uint64_t *addr, uint64_t c0,
                                       uint64_t c1, uint64_t n0, uint64_t n1,
                                       uint64_t &o0, uint64_t &o1) {
  asm volatile(
      "{\n\t.reg .b128 cmp, swp, old;\n\t"
      "mov.b128 cmp, {%2, %3};\n\t"
      "mov.b128 swp, {%4, %5};\n\t"
      "atom.global.cas.b128 old, [%6], cmp, swp;\n\t"
      "mov.b128 {%0, %1}, old;\n\t}"
      : "=l"(o0), "=l"(o1)
      : "l"(c0), "l"(c1), "l"(n0), "l"(n1), "l"(addr)
      : "memory");
}
#endif

// --------------------------------------------------------------- launchers
// Keys are read at keys + i * key_stride_u64 (2 for packed 16-byte keys,
// 4 for 32-byte SHA-256 digests whose first 16 bytes are the key).
int launch_index_claim(Slot *slots, uint64_t mask, const uint64_t *keys,
                       int key_stride_u64, const uint64_t *seqs, int n,
                       uint32_t *slot_idx, int *err, cudaStream_t s);
// status[i] = CASCADE_PUT_STORED for the first claimant (smallest seq) of a
// key that is not live yet, DUP_KNOWN when live, DUP_BATCH otherwise.
int launch_index_resolve(const Slot *slots, const uint32_t *slot_idx,
                         const uint64_t *seqs, int n, uint8_t *status,
                         cudaStream_t s);
// Winners with a valid offset become live; every winner closes its slot's
// claim.  headers: 8 bytes per request (Q8 scale, zero point).
int launch_index_commit(Slot *slots, const uint32_t *slot_idx,
                        const uint8_t *status, const uint64_t *offsets,
                        const uint64_t *sizes, const uint32_t *flags,
                        const uint8_t *headers, uint64_t epoch_base, int n,
                        cudaStream_t s);
// Winners without an offset, and DUP_BATCH entries whose winner did not
// become live, turn into FAILED.
int launch_index_finalize(const Slot *slots, const uint32_t *slot_idx,
                          const uint64_t *offsets, uint8_t *status, int n,
                          cudaStream_t s);
int launch_index_lookup(Slot *slots, uint64_t mask, const uint64_t *keys,
                        int key_stride_u64, int n, int touch,
                        uint64_t epoch_base, LookupInfo *out, cudaStream_t s);
// Rewrites the location of live slots (demotion / promotion).
int launch_index_relocate(Slot *slots, const uint32_t *slot_idx,
                          const uint64_t *offsets, const uint32_t *flags,
                          const uint8_t *headers, int n, cudaStream_t s);
// Applies the relocation records (src_idx == kMoveIdx) among `m` received
// shard records to this rank's live entries of their keys.
int launch_index_apply_moves(Slot *slots, uint64_t mask, const void *records,
                             int m, uint32_t rank, cudaStream_t s);
// Demotion candidates (live HBM slots whose payload this rank holds; class
// 1 = prefix blocks when
// `semantic`, else class 0), by epoch bucket over [0, span):
// bytes / count[cls * kVictimBuckets + b] = HBM payload bytes and slots.
int launch_victim_hist(const Slot *slots, uint64_t nslots, int semantic,
                       uint64_t span, unsigned long long *bytes,
                       uint32_t *count, cudaStream_t s);
// Every candidate of class c in buckets 0..cut_c (cut -1: none), in no
// particular order; *n_out = how many (at most max_out are written).
int launch_victim_collect(const Slot *slots, uint64_t nslots, int semantic,
                          uint64_t span, int cut0, int cut1, uint32_t *n_out,
                          ScanRec *out, uint32_t max_out, cudaStream_t s);

// Pool: req[i] = payload bytes to allocate, or kNoRequest.  offsets[i] =
// the allocation, or kInvalidOffset (no request, or the pool is full).
int launch_pool_alloc(PoolDev *pool, const uint64_t *req, int n,
                      uint64_t *offsets, cudaStream_t s);
// Returns offsets[i] (allocated for req[i] bytes) to the free stacks for
// every request whose status is not CASCADE_PUT_STORED (speculative
// allocations of blocks that turned out to be duplicates).
int launch_pool_free_unstored(PoolDev *pool, const uint64_t *req,
                              const uint64_t *offsets, const uint8_t *status,
                              int n, cudaStream_t s);

}  // namespace cb
