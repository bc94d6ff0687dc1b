// The DRAM tier: a pinned host arena the copy engines read and write
// directly.  It stands where the reference's ShmBackend (an mmap'd
// /dev/shm file with a 64-byte best-fit allocator, cascade_core.cpp:237-569)
// stands: blocks that do not go to HBM, and blocks demoted from HBM.
//
// The arena grows in pinned chunks (cudaHostAlloc, portable) up to its
// capacity, so a 64 GiB tier costs nothing until it is used.  Allocation is
// best-fit per chunk with coalescing frees, as in ShmBackend::allocate /
// deallocate (cascade_core.cpp:285-350); a block never straddles chunks.
//
// A shared arena (share()) makes every chunk a named POSIX shared-memory
// object ("<name>.<k>", chunk k at offset k * chunk_bytes), mapped and
// registered with CUDA, so the other ranks of a sharded store can map it
// (DramView) and copy blocks out of it.  The reference's ShmBackend
// is likewise an mmap'd /dev/shm file.
#pragma once

#include <stdint.h>

#include <map>
#include <string>
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

  // Turns an arena that has no chunk yet into a shared one whose chunks are
  // the shared-memory objects "<name>.<k>" (fixed chunk size; a block larger
  // than a chunk then does not fit).  False when chunks exist already.
  bool share(const std::string &name);
  const std::string &shared_name() const { return name_; }
  uint64_t chunk_bytes() const { return chunk_bytes_; }

 private:
  struct Chunk {
    uint64_t base = 0, size = 0, bump = 0;
    uint8_t *host = nullptr;
    bool mapped = false;  // a shared-memory mapping (else cudaHostAlloc)
    std::map<uint64_t, uint64_t> free;  // offset within chunk -> bytes
  };
  uint64_t capacity_, chunk_bytes_;
  uint64_t next_base_ = 0;
  std::string name_;  // shared mode when not empty
  std::vector<Chunk> chunks_;
  const Chunk *chunk_of(uint64_t offset) const;
  Chunk *chunk_of(uint64_t offset);
  uint8_t *new_chunk(uint64_t size, bool *mapped);
};

// Another rank's shared arena, mapped chunk by chunk on first use (and
// registered with CUDA, so copies read it by DMA).  Never written.
class DramView {
 public:
  DramView(const std::string &name, uint64_t chunk_bytes)
      : name_(name), chunk_bytes_(chunk_bytes) {}
  ~DramView();
  DramView(const DramView &) = delete;
  DramView &operator=(const DramView &) = delete;
  // Host address of [offset, offset + bytes) in the arena, or null when that
  // chunk cannot be mapped or the range leaves it.
  const uint8_t *ptr(uint64_t offset, uint64_t bytes);

 private:
  struct Map {
    uint8_t *host = nullptr;
    uint64_t size = 0;
  };
  std::string name_;
  uint64_t chunk_bytes_;
  std::vector<Map> maps_;
};

}  // namespace cb
