// KV page pool and per-sequence cache state (see KVCacheState.hpp).
#include "KVCacheState.hpp"

#include <algorithm>
#include <limits>
#include <stdexcept>

namespace tensor::runtime {

KVPagePool::KVPagePool(std::size_t pageSize, std::size_t physicalPageCount)
    : pageSize_(pageSize), allocated_(physicalPageCount, false) {
  if (pageSize == 0 || physicalPageCount == 0 ||
      physicalPageCount > static_cast<std::size_t>(std::numeric_limits<std::int32_t>::max()))
    throw std::invalid_argument("KV page pool dimensions are invalid.");
  // LIFO free list seeded in ascending order: the first allocation returns the
  // highest page id, as the reference pool does (KVCacheState.cpp:36-41,70-78).
  freePages_.reserve(physicalPageCount);
  for (std::size_t page = 0; page < physicalPageCount; ++page)
    freePages_.push_back(static_cast<std::int32_t>(page));
}

bool KVPagePool::isAllocated(std::int32_t page) const noexcept {
  return page >= 0 && static_cast<std::size_t>(page) < allocated_.size() &&
         allocated_[static_cast<std::size_t>(page)];
}

std::int32_t KVPagePool::allocatePage() {
  if (injectedFailures_ > 0) {
    --injectedFailures_;
    return -1;
  }
  if (freePages_.empty()) return -1;
  const auto page = freePages_.back();
  freePages_.pop_back();
  allocated_[static_cast<std::size_t>(page)] = true;
  ++allocationCount_;
  peakUsedPages_ = std::max(peakUsedPages_, usedPages());
  return page;
}

void KVPagePool::releasePage(std::int32_t page) {
  if (!isAllocated(page)) throw std::invalid_argument("Paged KV attempted to release an invalid page.");
  allocated_[static_cast<std::size_t>(page)] = false;
  freePages_.push_back(page);
  ++releaseCount_;
}

KVCacheState::KVCacheState(std::shared_ptr<KVPagePool> pool, std::size_t capacity, int slot,
                           BlockTableSink sink)
    : pool_(std::move(pool)), capacity_(capacity), slot_(slot), sink_(std::move(sink)) {
  if (!pool_ || capacity_ == 0) throw std::invalid_argument("KV cache state needs a pool and a capacity.");
  const auto pages = (capacity_ + pool_->pageSize() - 1) / pool_->pageSize();
  if (pages > pool_->capacityPages())
    throw std::invalid_argument("Paged KV pool cannot hold one request at full capacity.");
  logicalToPhysical_.assign(pages, -1);
}

KVCacheState::~KVCacheState() {
  for (auto &page : logicalToPhysical_) {
    if (page < 0) continue;
    try {
      pool_->releasePage(page);
    } catch (...) {
    }
    page = -1;
  }
}

std::size_t KVCacheState::allocatedPageCount() const noexcept {
  std::size_t count = 0;
  while (count < logicalToPhysical_.size() && logicalToPhysical_[count] >= 0) ++count;
  return count;
}

std::vector<std::int32_t> KVCacheState::pageTable() const {
  return {logicalToPhysical_.begin(),
          logicalToPhysical_.begin() + static_cast<std::ptrdiff_t>(allocatedPageCount())};
}

std::string KVCacheState::resizePageAllocation(std::size_t pageCount) {
  const auto allocated = allocatedPageCount();
  if (pageCount > allocated) {
    std::size_t logical = allocated;
    for (; logical < pageCount; ++logical) {
      const auto physical = pool_->allocatePage();
      if (physical < 0) break;
      logicalToPhysical_[logical] = physical;
    }
    if (logical != pageCount) {
      while (logical > allocated) {  // unwind: all or nothing
        --logical;
        pool_->releasePage(logicalToPhysical_[logical]);
        logicalToPhysical_[logical] = -1;
      }
      return "Paged KV cache physical page pool is exhausted.";
    }
    return {};
  }
  for (std::size_t logical = allocated; logical > pageCount; --logical) {
    pool_->releasePage(logicalToPhysical_[logical - 1]);
    logicalToPhysical_[logical - 1] = -1;
  }
  return {};
}

std::string KVCacheState::stageLength(std::size_t length) {
  if (length == 0 || length > capacity_) return "KV cache valid length is outside the configured capacity.";
  const auto previous = allocatedPageCount();
  const auto required = (length + pool_->pageSize() - 1) / pool_->pageSize();
  if (required > logicalToPhysical_.size())
    return "Paged KV cache has no block-table capacity for this length.";
  if (required > previous) {
    auto error = resizePageAllocation(required);
    if (!error.empty()) return error;
    if (sink_) {
      error = sink_(slot_, logicalToPhysical_);
      if (!error.empty()) {
        (void)resizePageAllocation(previous);
        (void)sink_(slot_, logicalToPhysical_);
        return error;
      }
    }
  }
  return {};
}

std::string KVCacheState::rollbackLength(std::size_t length) {
  if (length > capacity_) return "Cannot roll back KV cache beyond its configured capacity.";
  const auto required = length == 0 ? 0 : (length + pool_->pageSize() - 1) / pool_->pageSize();
  const auto previous = allocatedPageCount();
  if (required < previous) {
    auto error = resizePageAllocation(required);
    if (!error.empty()) return error;
    if (sink_) {
      error = sink_(slot_, logicalToPhysical_);
      if (!error.empty()) return error;
    }
  }
  if (currentLength_ > length) currentLength_ = length;
  return {};
}

void KVCacheState::commitLength(std::size_t length) {
  if (length == 0 || length > capacity_) throw std::invalid_argument("Cannot commit an invalid KV cache length.");
  currentLength_ = length;
}

std::string KVCacheState::reset() {
  auto error = rollbackLength(0);
  currentLength_ = 0;
  return error;
}

}  // namespace tensor::runtime
