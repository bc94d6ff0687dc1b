// Pinned DRAM arena (host code).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "dram.cuh"

namespace cb {

namespace {

std::string chunk_name(const std::string &base, size_t k) {
  return base + "." + std::to_string(k);
}

// Maps a shared-memory object of `size` bytes (created when `create`) and
// registers it with CUDA; null on any failure, with nothing left behind.
uint8_t *map_shared(const std::string &name, uint64_t size, bool create) {
  const int fd = create ? shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600)
                        : shm_open(name.c_str(), O_RDWR, 0);
  if (fd < 0) return nullptr;
  if (create && ftruncate(fd, (off_t)size) != 0) {
    close(fd);
    shm_unlink(name.c_str());
    return nullptr;
  }
  void *p = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    if (create) shm_unlink(name.c_str());
    return nullptr;
  }
  if (cudaHostRegister(p, size, cudaHostRegisterPortable) != cudaSuccess) {
    cudaGetLastError();  // reset the runtime's last-error state
    munmap(p, size);
    if (create) shm_unlink(name.c_str());
    return nullptr;
  }
  return static_cast<uint8_t *>(p);
}

void unmap_shared(uint8_t *p, uint64_t size) {
  cudaHostUnregister(p);
  munmap(p, size);
}

}  // namespace

DramArena::~DramArena() {
  for (size_t k = 0; k < chunks_.size(); ++k) {
    Chunk &c = chunks_[k];
    if (!c.host) continue;
    if (c.mapped) {
      unmap_shared(c.host, c.size);
      shm_unlink(chunk_name(name_, k).c_str());
    } else {
      cudaFreeHost(c.host);
    }
  }
}

bool DramArena::share(const std::string &name) {
  if (!chunks_.empty() || name.empty()) return name_ == name && !name.empty();
  name_ = name;
  return true;
}

uint8_t *DramArena::new_chunk(uint64_t size, bool *mapped) {
  *mapped = !name_.empty();
  if (*mapped) return map_shared(chunk_name(name_, chunks_.size()), size, true);
  void *host = nullptr;
  if (cudaHostAlloc(&host, size, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();  // reset the runtime's last-error state
    return nullptr;
  }
  return static_cast<uint8_t *>(host);
}

DramView::~DramView() {
  for (Map &m : maps_)
    if (m.host) unmap_shared(m.host, m.size);
}

const uint8_t *DramView::ptr(uint64_t offset, uint64_t bytes) {
  const size_t k = (size_t)(offset / chunk_bytes_);
  if (k >= maps_.size()) maps_.resize(k + 1);
  Map &m = maps_[k];
  if (!m.host) {
    const std::string name = chunk_name(name_, k);
    const int fd = shm_open(name.c_str(), O_RDONLY, 0);
    if (fd < 0) return nullptr;
    struct stat sb;
    const bool ok = fstat(fd, &sb) == 0 && sb.st_size > 0;
    close(fd);
    if (!ok) return nullptr;
    m.host = map_shared(name, (uint64_t)sb.st_size, false);
    if (!m.host) return nullptr;
    m.size = (uint64_t)sb.st_size;
  }
  const uint64_t in = offset - (uint64_t)k * chunk_bytes_;
  if (in + bytes > m.size) return nullptr;
  return m.host + in;
}

uint64_t DramArena::alloc(uint64_t bytes) {
  const uint64_t need = (bytes + kAlign - 1) & ~(kAlign - 1);
  const uint64_t want = need ? need : kAlign;
  // Best fit over every chunk's free list (ShmBackend::allocate's rule).
  Chunk *best_c = nullptr;
  std::map<uint64_t, uint64_t>::iterator best_it;
  uint64_t best_waste = ~0ull;
  for (auto &c : chunks_) {
    for (auto it = c.free.begin(); it != c.free.end(); ++it) {
      if (it->second >= want && it->second - want < best_waste) {
        best_waste = it->second - want;
        best_c = &c;
        best_it = it;
        if (best_waste == 0) break;
      }
    }
    if (best_waste == 0) break;
  }
  if (best_c) {
    uint64_t off = best_it->first, size = best_it->second;
    best_c->free.erase(best_it);
    if (size > want) best_c->free.emplace(off + want, size - want);
    return best_c->base + off;
  }
  for (auto &c : chunks_) {
    if (c.size - c.bump >= want) {
      uint64_t off = c.bump;
      c.bump += want;
      return c.base + off;
    }
  }
  // A new pinned chunk: the default growth unit, or (not shared) the
  // block's own size.  Shared chunks sit at multiples of chunk_bytes_.
  uint64_t size = chunk_bytes_;
  if (size < want) {
    if (!name_.empty()) return kNone;
    size = (want + (2ull << 20) - 1) & ~((2ull << 20) - 1);
  }
  if (next_base_ + size > capacity_) {
    if (next_base_ + want > capacity_) return kNone;
    size = capacity_ - next_base_;
  }
  bool mapped = false;
  uint8_t *host = new_chunk(size, &mapped);
  if (!host) return kNone;
  Chunk c;
  c.base = next_base_;
  c.size = size;
  c.bump = want;
  c.host = host;
  c.mapped = mapped;
  next_base_ += size;
  chunks_.push_back(std::move(c));
  return chunks_.back().base;
}

const DramArena::Chunk *DramArena::chunk_of(uint64_t offset) const {
  for (const auto &c : chunks_)
    if (offset >= c.base && offset < c.base + c.size) return &c;
  return nullptr;
}

DramArena::Chunk *DramArena::chunk_of(uint64_t offset) {
  for (auto &c : chunks_)
    if (offset >= c.base && offset < c.base + c.size) return &c;
  return nullptr;
}

void DramArena::free(uint64_t offset, uint64_t bytes) {
  Chunk *c = chunk_of(offset);
  if (!c) return;
  uint64_t size = (bytes + kAlign - 1) & ~(kAlign - 1);
  if (!size) size = kAlign;
  uint64_t off = offset - c->base;
  auto next = c->free.lower_bound(off);
  if (next != c->free.end() && off + size == next->first) {
    size += next->second;
    next = c->free.erase(next);
  }
  if (next != c->free.begin()) {
    auto prev = std::prev(next);
    if (prev->first + prev->second == off) {
      prev->second += size;
      return;
    }
  }
  c->free.emplace(off, size);
}

uint8_t *DramArena::ptr(uint64_t offset) const {
  const Chunk *c = chunk_of(offset);
  return c ? c->host + (offset - c->base) : nullptr;
}

void DramArena::reset() {
  for (auto &c : chunks_) {
    c.bump = 0;
    c.free.clear();
  }
}

}  // namespace cb
