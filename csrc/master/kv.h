// Paged-KV bookkeeping of the master: block pools with RAII leases, chained prefix
// block hashes, the automatic-prefix-caching (APC) radix tree with recurrent-state
// checkpoint slots, and the hybrid page <-> checkpoint alias table.
//
// Everything here is plain host code owned by the engine thread; leases are RAII so a
// request that is cancelled, fails or finishes returns exactly the pages it holds
// (conservation is checked by the tests).
//
// Reference parity: crates/zs-kv/src/lib.rs (BlockPool/BlockLease :68-196),
// prefix_cache.rs (PrefixTree :256, match_prefix_bounded :473, extend_prefix_with_aux
// :572, evict_lru_victims :806, PrefixLease :829, KvCacheEvent :36), kv_hash.rs
// (sha256 over canonical CBOR [parent, tokens, null], 8-byte external key),
// hybrid_alias.rs (HybridBlockAliasTable :37, SubPageAllocator :132).
#pragma once

#include <stdint.h>

#include <array>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

namespace zs {
namespace kv {

using Hash = std::array<uint8_t, 32>;

// ---------------------------------------------------------------------------- pools
class BlockLease;

class BlockPool {
 public:
  // Block ids [first_id, first_id + num_blocks).
  explicit BlockPool(int32_t num_blocks, int32_t first_id = 0);
  std::optional<BlockLease> allocate(size_t n);
  size_t available() const;
  size_t capacity() const { return capacity_; }

  struct State {
    std::mutex mu;
    std::vector<int32_t> free;
  };

 private:
  std::shared_ptr<State> st_;
  size_t capacity_;
};

class BlockLease {
 public:
  BlockLease() = default;
  BlockLease(std::shared_ptr<BlockPool::State> st, std::vector<int32_t> ids) : st_(std::move(st)), ids_(std::move(ids)) {}
  BlockLease(const BlockLease&) = delete;
  BlockLease& operator=(const BlockLease&) = delete;
  BlockLease(BlockLease&& o) noexcept : st_(std::move(o.st_)), ids_(std::move(o.ids_)) { o.ids_.clear(); }
  BlockLease& operator=(BlockLease&& o) noexcept;
  ~BlockLease() { release(); }

  const std::vector<int32_t>& ids() const { return ids_; }
  size_t size() const { return ids_.size(); }
  bool empty() const { return ids_.empty(); }
  // Split off the first n ids into a new lease.
  BlockLease take_front(size_t n);
  // Append another lease of the same pool.
  void absorb(BlockLease&& other);
  // Return all ids to the pool now.
  void release();

 private:
  std::shared_ptr<BlockPool::State> st_;
  std::vector<int32_t> ids_;
};

// ---------------------------------------------------------------------------- hashing
// Root hash: sha256(canonical CBOR text string of `seed`).
Hash none_hash(const std::string& seed);
// sha256(canonical CBOR [parent(bytes 32), [tokens...], null]); negative tokens clamp to 0.
Hash block_hash(const Hash& parent, const int32_t* tokens, size_t n);
// Chained hashes of every full `block_size` chunk of `tokens` (partial tail ignored).
std::vector<Hash> compute_block_hashes(const std::vector<int32_t>& tokens, size_t block_size, const std::string& seed);
// External 8-byte key: the trailing 8 bytes read big-endian.
uint64_t external_key(const Hash& h);
std::string kv_hash_seed_from_env();

// ---------------------------------------------------------------------------- events
struct KvEvent {
  enum Kind { kStored, kRemoved, kAllCleared } kind;
  std::vector<uint64_t> block_keys;      // external keys (one per page of the node)
  uint64_t parent_key = 0;               // stored: external key of the parent block (0 = root)
  std::vector<int32_t> tokens;           // stored: tokens of the node
  uint32_t block_tokens = 0;
};
using KvEventSink = std::function<void(const KvEvent&)>;

// ---------------------------------------------------------------------------- prefix tree
class PrefixTree;

struct PrefixVictim {
  std::vector<int32_t> pages;  // device pages freed by the eviction
  std::vector<int32_t> tokens;
  int32_t aux_slot = -1;
  Hash hash{};
  uint64_t node_id = 0;
};

// A pinned, matched prefix.  While alive, its nodes cannot be evicted.
class PrefixLease {
 public:
  PrefixLease() = default;
  PrefixLease(const PrefixLease&) = delete;
  PrefixLease& operator=(const PrefixLease&) = delete;
  PrefixLease(PrefixLease&& o) noexcept;
  PrefixLease& operator=(PrefixLease&& o) noexcept;
  ~PrefixLease() { release(); }
  const std::vector<int32_t>& pages() const { return pages_; }
  size_t matched_nodes() const { return nodes_.size(); }
  uint32_t matched_tokens() const { return matched_tokens_; }
  int32_t leaf_aux() const { return leaf_aux_; }
  uint64_t leaf_node() const { return nodes_.empty() ? 0 : nodes_.back(); }
  void release();

 private:
  friend class PrefixTree;
  std::shared_ptr<struct TreeState> st_;
  std::vector<uint64_t> nodes_;
  std::vector<int32_t> pages_;
  uint32_t matched_tokens_ = 0;
  int32_t leaf_aux_ = -1;
};

struct TreeNode {
  uint64_t id = 0;
  uint64_t parent = 0;  // 0 = root
  std::vector<int32_t> tokens;
  BlockLease pages;
  BlockLease aux;  // optional recurrent-state checkpoint slot
  Hash hash{};
  uint32_t pins = 0;
  uint64_t last_use = 0;
  std::map<std::vector<int32_t>, uint64_t> children;
};

struct TreeState {
  std::mutex mu;
  std::unordered_map<uint64_t, TreeNode> nodes;
  std::map<std::vector<int32_t>, uint64_t> roots;
  uint64_t next_id = 1;
  uint64_t tick = 0;
  uint32_t block_tokens = 16;
  uint32_t pages_per_node = 1;
  Hash root_hash{};
  KvEventSink sink;
  uint64_t queries = 0, hit_tokens = 0, query_tokens = 0, evictions = 0;
};

class PrefixTree {
 public:
  PrefixTree(uint32_t block_tokens, uint32_t pages_per_node, const std::string& seed = "42");
  uint32_t node_tokens() const { return st_->block_tokens * st_->pages_per_node; }
  uint32_t block_tokens() const { return st_->block_tokens; }
  uint32_t pages_per_node() const { return st_->pages_per_node; }
  void set_event_sink(KvEventSink sink);

  // Longest cached prefix of full nodes (at most max_nodes), pinned.
  PrefixLease match(const std::vector<int32_t>& tokens, size_t max_nodes = SIZE_MAX);
  // Match without pinning: (matched nodes, matched tokens).
  std::pair<size_t, size_t> peek(const std::vector<int32_t>& tokens, size_t max_nodes = SIZE_MAX) const;
  // Insert the node covering `node_tokens` tokens below `parent_node` (0 = root),
  // taking ownership of `pages` (pages_per_node ids) and `aux` only when a new node is
  // created (*created = true).  If the node already exists (concurrent promotion of
  // the same chunk) the leases are left with the caller and the existing node id is
  // returned.  Returns 0 if the parent no longer exists.
  uint64_t insert(uint64_t parent_node, const int32_t* tokens, BlockLease& pages, BlockLease& aux,
                  bool* created = nullptr);
  // Pin an existing node chain ending at `node` (used to keep promoted nodes alive).
  PrefixLease pin_chain(uint64_t node);
  // Evict least-recently-used unpinned leaves until `target_pages` device pages were
  // freed (or nothing is evictable); returns the victims (pages already returned).
  std::vector<PrefixVictim> evict_lru(size_t target_pages);
  int32_t aux_of(uint64_t node) const;

  size_t cached_nodes() const;
  size_t cached_pages() const;
  size_t evictable_pages() const;
  void clear();
  struct Stats {
    uint64_t queries, query_tokens, hit_tokens, evictions;
  };
  Stats stats() const;

 private:
  std::shared_ptr<TreeState> st_;
};

// ---------------------------------------------------------------------------- hybrid alias
// Bidirectional map: anchor KV page of an APC node <-> recurrent checkpoint slot.
class HybridAliasTable {
 public:
  bool insert(int32_t anchor_page, int32_t slot, const std::vector<int32_t>& pages);
  bool remove_by_anchor(int32_t anchor_page);
  std::optional<int32_t> slot_for_anchor(int32_t anchor_page) const;
  std::optional<int32_t> anchor_for_slot(int32_t slot) const;
  size_t size() const { return by_anchor_.size(); }

 private:
  std::unordered_map<int32_t, int32_t> by_anchor_;
  std::unordered_map<int32_t, int32_t> by_slot_;
  std::unordered_map<int32_t, std::vector<int32_t>> pages_;
};

// Best-fit allocator of fixed-size token slices (e.g. 128-token GDN checkpoint
// granularity) inside larger backing pages.
class SubPageAllocator {
 public:
  SubPageAllocator(uint32_t slice_tokens, uint32_t page_tokens, uint32_t num_pages);
  // Returns (page, slice index) or nullopt when full.
  std::optional<std::pair<int32_t, int32_t>> allocate();
  void release(int32_t page, int32_t slice);
  size_t active() const { return active_; }
  uint32_t slices_per_page() const { return per_page_; }

 private:
  uint32_t per_page_;
  std::vector<uint32_t> used_;   // per page bitmask of used slices (<= 32 slices)
  size_t active_ = 0;
};

}  // namespace kv
}  // namespace zs
