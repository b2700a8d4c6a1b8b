// KV-cache page pool and per-sequence cache state.
//
// Mirrors tensor::runtime::KVPagePool / KVCacheState (reference
// src/runtime/KVCacheState.hpp:19-147, KVCacheState.cpp:30-446):
//   * KVPagePool: a LIFO free list of physical page ids with peak / allocation
//     / release counters (KVCacheState.cpp:30-86);
//   * KVCacheState: one sequence's logical->physical page list and committed
//     length, with stageLength (all-or-nothing page allocation, unwound on
//     exhaustion, KVCacheState.cpp:170-202,355-379), rollbackLength, commitLength,
//     reset and pageTable.
// Differences from the reference, by design for B200:
//   * page storage is owned by the executor as one [pages][Hkv][page][D] fp16
//     pool per layer in HBM; every layer of a sequence uses the same physical
//     page ids, so one block table row serves all layers;
//   * the block table is one device array [slots][maxPagesPerSequence] that
//     decode kernels index; stageLength writes this sequence's row through a
//     BlockTableSink instead of a per-request Metal buffer;
//   * a contiguous (non-paged) cache is the pool with page size = capacity.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

namespace tensor::runtime {

class KVPagePool {
 public:
  KVPagePool(std::size_t pageSize, std::size_t physicalPageCount);
  KVPagePool(const KVPagePool &) = delete;
  KVPagePool &operator=(const KVPagePool &) = delete;

  [[nodiscard]] std::size_t pageSize() const noexcept { return pageSize_; }
  [[nodiscard]] std::size_t capacityPages() const noexcept { return allocated_.size(); }
  [[nodiscard]] std::size_t usedPages() const noexcept { return allocated_.size() - freePages_.size(); }
  [[nodiscard]] std::size_t availablePages() const noexcept { return freePages_.size(); }
  [[nodiscard]] std::size_t peakUsedPages() const noexcept { return peakUsedPages_; }
  [[nodiscard]] std::size_t allocationCount() const noexcept { return allocationCount_; }
  [[nodiscard]] std::size_t releaseCount() const noexcept { return releaseCount_; }
  [[nodiscard]] bool isAllocated(std::int32_t page) const noexcept;

  // -1 when the pool is exhausted.
  [[nodiscard]] std::int32_t allocatePage();
  // Throws std::invalid_argument for a page that is not allocated.
  void releasePage(std::int32_t page);

  // Test hook: the next `n` allocations fail as if the pool were exhausted
  // (host-side failure injection; no device involvement).
  void failNextAllocations(std::size_t n) { injectedFailures_ = n; }

 private:
  std::size_t pageSize_;
  std::vector<std::int32_t> freePages_;
  std::vector<bool> allocated_;
  std::size_t peakUsedPages_ = 0;
  std::size_t allocationCount_ = 0;
  std::size_t releaseCount_ = 0;
  std::size_t injectedFailures_ = 0;
};

// Receives a sequence's block-table row whenever its page list changes.
using BlockTableSink = std::function<std::string(int slot, const std::vector<std::int32_t> &row)>;

class KVCacheState {
 public:
  KVCacheState(std::shared_ptr<KVPagePool> pool, std::size_t capacity, int slot,
               BlockTableSink sink);
  ~KVCacheState();
  KVCacheState(const KVCacheState &) = delete;
  KVCacheState &operator=(const KVCacheState &) = delete;

  [[nodiscard]] std::size_t currentLength() const noexcept { return currentLength_; }
  [[nodiscard]] std::size_t capacity() const noexcept { return capacity_; }
  [[nodiscard]] int slot() const noexcept { return slot_; }
  [[nodiscard]] std::size_t pageSize() const noexcept { return pool_->pageSize(); }
  [[nodiscard]] std::size_t maxPages() const noexcept { return logicalToPhysical_.size(); }
  [[nodiscard]] std::size_t allocatedPageCount() const noexcept;
  [[nodiscard]] std::vector<std::int32_t> pageTable() const;
  [[nodiscard]] const std::vector<std::int32_t> &blockTableRow() const { return logicalToPhysical_; }

  // Make `length` positions addressable (allocating pages as needed, all or
  // nothing). The committed length is unchanged until commitLength.
  [[nodiscard]] std::string stageLength(std::size_t length);
  // Release pages beyond `length` (length may be 0).
  [[nodiscard]] std::string rollbackLength(std::size_t length);
  // Throws std::invalid_argument for 0 or > capacity (KVCacheState.cpp:242-247).
  void commitLength(std::size_t length);
  // Release every page and set the length to 0.
  [[nodiscard]] std::string reset();

 private:
  [[nodiscard]] std::string resizePageAllocation(std::size_t pageCount);

  std::shared_ptr<KVPagePool> pool_;
  std::size_t capacity_;
  int slot_;
  BlockTableSink sink_;
  std::size_t currentLength_ = 0;
  std::vector<std::int32_t> logicalToPhysical_;
};

}  // namespace tensor::runtime
