// The DRAM tier: a pinned host arena the copy engines read and write
// directly.  It stands where the reference's ShmBackend (an mmap'd
// /dev/shm file with a 64-byte best-fit allocator, cascade_core.cpp:237-569)
// stands: blocks that do not go to HBM, and blocks demoted from HBM.
//
// The arena grows in pinned chunks (cudaHostAlloc, portable) up to its
// capacity, so a 64 GiB tier costs nothing until it is used.  Allocation is
// best-fit per chunk with coalescing frees, as in ShmBackend::allocate /
// deallocate (cascade_core.cpp:285-350); a block never straddles chunks.
#pragma once

#include <stdint.h>

#include <map>
#include <vector>

namespace cb {

class DramArena {
 public:
  static constexpr uint64_t kAlign = 64;
  static constexpr uint64_t kNone = ~0ull;

  DramArena(uint64_t capacity, uint64_t chunk_bytes)
      : capacity_(capacity), chunk_bytes_(chunk_bytes) {}
  ~DramArena();
  DramArena(const DramArena &) = delete;
  DramArena &operator=(const DramArena &) = delete;

  // Offset of `bytes` of arena space, or kNone when the arena is full or a
  // pinned chunk cannot be allocated.
  uint64_t alloc(uint64_t bytes);
  void free(uint64_t offset, uint64_t bytes);
  uint8_t *ptr(uint64_t offset) const;
  // Forgets every allocation; chunks stay pinned for reuse.
  void reset();
  uint64_t capacity() const { return capacity_; }
  uint64_t pinned_bytes() const { return next_base_; }

 private:
  struct Chunk {
    uint64_t base = 0, size = 0, bump = 0;
    uint8_t *host = nullptr;
    std::map<uint64_t, uint64_t> free;  // offset within chunk -> bytes
  };
  uint64_t capacity_, chunk_bytes_;
  uint64_t next_base_ = 0;
  std::vector<Chunk> chunks_;
  const Chunk *chunk_of(uint64_t offset) const;
  Chunk *chunk_of(uint64_t offset);
};

}  // namespace cb
