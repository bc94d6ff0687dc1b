// Pinned DRAM arena (host code).
#include <cuda_runtime.h>

#include "dram.cuh"

namespace cb {

DramArena::~DramArena() {
  for (auto &c : chunks_)
    if (c.host) cudaFreeHost(c.host);
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
  // A new pinned chunk: the default growth unit, or the block's own size.
  uint64_t size = chunk_bytes_;
  if (size < want) size = (want + (2ull << 20) - 1) & ~((2ull << 20) - 1);
  if (next_base_ + size > capacity_) {
    if (next_base_ + want > capacity_) return kNone;
    size = capacity_ - next_base_;
  }
  void *host = nullptr;
  if (cudaHostAlloc(&host, size, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();  // reset the runtime's last-error state
    return kNone;
  }
  Chunk c;
  c.base = next_base_;
  c.size = size;
  c.bump = want;
  c.host = static_cast<uint8_t *>(host);
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
