#include "dram_tier.h"

#include <algorithm>
#include <cmath>

namespace zs {
namespace kv {

DramTier::DramTier(uint32_t num_blocks, uint32_t block_tokens, uint32_t hbm_pages, double ratio)
    : capacity_(num_blocks), block_tokens_(block_tokens) {
  if (!(ratio > 0.0) || ratio > 0.5) ratio = 0.10;
  uint32_t la = hbm_pages > 1 ? uint32_t(std::ceil(double(hbm_pages) * ratio)) : 0;
  loading_area_ = std::min(std::max<uint32_t>(la, hbm_pages > 1 ? 1 : 0), std::max<uint32_t>(hbm_pages / 2, 1));
  for (int32_t s = int32_t(num_blocks) - 1; s >= 0; --s) free_.push_back(s);
}

std::optional<KvTransferOp> DramTier::admit(const Hash& key, int32_t hbm_page) {
  ++tick_;
  auto it = entries_.find(key);
  if (it != entries_.end()) {
    it->second.last_use = tick_;
    return std::nullopt;
  }
  int32_t slot;
  if (!free_.empty()) {
    slot = free_.back();
    free_.pop_back();
  } else {
    if (entries_.empty()) return std::nullopt;  // zero capacity
    auto lru = entries_.begin();
    for (auto e = entries_.begin(); e != entries_.end(); ++e)
      if (e->second.last_use < lru->second.last_use) lru = e;
    slot = lru->second.slot;
    entries_.erase(lru);
    ++evictions_;
  }
  entries_[key] = Entry{slot, tick_};
  ++offloads_;
  return KvTransferOp{hbm_page, slot, false};
}

void DramTier::rollback(const Hash& key) {
  auto it = entries_.find(key);
  if (it == entries_.end()) return;
  free_.push_back(it->second.slot);
  entries_.erase(it);
}

size_t DramTier::continuation(const std::vector<Hash>& keys, size_t first) const {
  size_t n = 0;
  for (size_t i = first; i < keys.size() && entries_.count(keys[i]); ++i) ++n;
  return n;
}

std::vector<int32_t> DramTier::take(const std::vector<Hash>& keys, size_t first, size_t max_blocks) {
  std::vector<int32_t> slots;
  for (size_t i = first; i < keys.size() && slots.size() < max_blocks; ++i) {
    auto it = entries_.find(keys[i]);
    if (it == entries_.end()) break;
    slots.push_back(it->second.slot);
    entries_.erase(it);
    ++reloads_;
    hit_tokens_ += block_tokens_;
  }
  return slots;
}

void DramTier::release(const std::vector<int32_t>& slots) { free_.insert(free_.end(), slots.begin(), slots.end()); }

DramTierStats DramTier::stats() const {
  DramTierStats s;
  s.capacity_blocks = capacity_;
  s.occupied_blocks = entries_.size();
  s.loading_area_pages = loading_area_;
  s.offloads = offloads_;
  s.reloads = reloads_;
  s.evictions = evictions_;
  s.hit_tokens = hit_tokens_;
  return s;
}

}  // namespace kv
}  // namespace zs
