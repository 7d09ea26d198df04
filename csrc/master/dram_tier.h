// Host DRAM tier of the prefix cache: an exclusive second level for evicted prefix
// blocks.  A block lives either in HBM (the prefix tree) or here, never in both.
//
//  * Demotion: when admission needs HBM pages, the engine evicts LRU prefix leaves and
//    admits each victim block here (D2H copy of its page into a pinned host slot)
//    before the freed pages are handed out again.  A full tier drops its own LRU entry.
//  * Reload: when a prompt's HBM match stops at block i and blocks i, i+1, ... are
//    resident here, the engine copies them back (H2D) into fresh pages, inserts them
//    into the tree and matches again.  Reloaded entries leave the tier (exclusive).
//  * Loading area: a share of the HBM pages (default 10%) is kept free for reloads, so
//    a reload never has to evict the prefix it is about to extend.
// Blocks are keyed by their chained block hash (one page per prefix node), which names
// the whole token path from the root.
//
// Reference parity: crates/zs-kv/src/dram_tier.rs (DramTierConfig :25, KvTransferOp :81,
// DramPrefixCache::admit_victim :219, take_continuation_for_reload), engine hooks
// crates/zs-scheduler/src/serving.rs:1236-1506.
#pragma once

#include <stdint.h>

#include <map>
#include <optional>
#include <vector>

#include "kv.h"

namespace zs {
namespace kv {

struct KvTransferOp {
  int32_t hbm_page = 0;
  int32_t dram_slot = 0;
  bool h2d = false;  // false: HBM -> DRAM (demote); true: DRAM -> HBM (reload)
};

struct DramTierStats {
  uint64_t capacity_blocks = 0, occupied_blocks = 0, loading_area_pages = 0;
  uint64_t offloads = 0, reloads = 0, evictions = 0, hit_tokens = 0;
};

class DramTier {
 public:
  // loading_area_ratio in (0, 0.5]: share of `hbm_pages` kept free for reloads.
  DramTier(uint32_t num_blocks, uint32_t block_tokens, uint32_t hbm_pages, double loading_area_ratio);
  uint32_t loading_area_pages() const { return loading_area_; }
  uint32_t capacity() const { return capacity_; }
  size_t occupied() const { return entries_.size(); }

  // Admit an evicted block; returns the D2H copy to run, or nothing if already resident.
  std::optional<KvTransferOp> admit(const Hash& key, int32_t hbm_page);
  // Undo an admission whose copy failed.
  void rollback(const Hash& key);
  // Resident blocks continuing a prefix: how many of keys[first], keys[first+1], ...
  size_t continuation(const std::vector<Hash>& keys, size_t first) const;
  // Remove up to max_blocks continuation blocks for reload; returns their slots in order.
  std::vector<int32_t> take(const std::vector<Hash>& keys, size_t first, size_t max_blocks);
  // Return slots after their reload copies ran.
  void release(const std::vector<int32_t>& slots);
  DramTierStats stats() const;

 private:
  struct Entry {
    int32_t slot;
    uint64_t last_use;
  };
  uint32_t capacity_, block_tokens_, loading_area_;
  std::map<Hash, Entry> entries_;
  std::vector<int32_t> free_;
  uint64_t tick_ = 0;
  uint64_t offloads_ = 0, reloads_ = 0, evictions_ = 0, hit_tokens_ = 0;
};

}  // namespace kv
}  // namespace zs
