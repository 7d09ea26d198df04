#include "kv.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "sha256.h"

namespace zs {
namespace kv {

// ---------------------------------------------------------------------------- pools
BlockPool::BlockPool(int32_t num_blocks, int32_t first_id) : st_(std::make_shared<State>()), capacity_(num_blocks) {
  st_->free.reserve(num_blocks);
  // Free list as a stack; hand out low ids first.
  for (int32_t i = num_blocks - 1; i >= 0; --i) st_->free.push_back(first_id + i);
}

std::optional<BlockLease> BlockPool::allocate(size_t n) {
  std::lock_guard<std::mutex> g(st_->mu);
  if (st_->free.size() < n) return std::nullopt;
  std::vector<int32_t> ids(st_->free.end() - n, st_->free.end());
  std::reverse(ids.begin(), ids.end());
  st_->free.resize(st_->free.size() - n);
  return BlockLease(st_, std::move(ids));
}

size_t BlockPool::available() const {
  std::lock_guard<std::mutex> g(st_->mu);
  return st_->free.size();
}

BlockLease& BlockLease::operator=(BlockLease&& o) noexcept {
  if (this != &o) {
    release();
    st_ = std::move(o.st_);
    ids_ = std::move(o.ids_);
    o.ids_.clear();
  }
  return *this;
}

BlockLease BlockLease::take_front(size_t n) {
  n = std::min(n, ids_.size());
  std::vector<int32_t> front(ids_.begin(), ids_.begin() + n);
  ids_.erase(ids_.begin(), ids_.begin() + n);
  return BlockLease(st_, std::move(front));
}

void BlockLease::absorb(BlockLease&& other) {
  if (other.ids_.empty()) return;
  if (!st_) st_ = other.st_;
  ids_.insert(ids_.end(), other.ids_.begin(), other.ids_.end());
  other.ids_.clear();
  other.st_.reset();
}

void BlockLease::release() {
  if (st_ && !ids_.empty()) {
    std::lock_guard<std::mutex> g(st_->mu);
    for (auto it = ids_.rbegin(); it != ids_.rend(); ++it) st_->free.push_back(*it);
  }
  ids_.clear();
}

// ---------------------------------------------------------------------------- hashing
namespace {

void cbor_uint(std::vector<uint8_t>& out, uint8_t major, uint64_t n) {
  const uint8_t m = uint8_t(major << 5);
  if (n <= 23) {
    out.push_back(m | uint8_t(n));
  } else if (n <= 0xff) {
    out.push_back(m | 24);
    out.push_back(uint8_t(n));
  } else if (n <= 0xffff) {
    out.push_back(m | 25);
    out.push_back(uint8_t(n >> 8));
    out.push_back(uint8_t(n));
  } else if (n <= 0xffffffffull) {
    out.push_back(m | 26);
    for (int s = 24; s >= 0; s -= 8) out.push_back(uint8_t(n >> s));
  } else {
    out.push_back(m | 27);
    for (int s = 56; s >= 0; s -= 8) out.push_back(uint8_t(n >> s));
  }
}

}  // namespace

Hash none_hash(const std::string& seed) {
  std::vector<uint8_t> buf;
  cbor_uint(buf, 3, seed.size());  // text string
  buf.insert(buf.end(), seed.begin(), seed.end());
  return sha256(buf.data(), buf.size());
}

Hash block_hash(const Hash& parent, const int32_t* tokens, size_t n) {
  std::vector<uint8_t> buf;
  buf.reserve(8 + 34 + n * 5);
  cbor_uint(buf, 4, 3);         // array(3)
  cbor_uint(buf, 2, 32);        // bytes(32)
  buf.insert(buf.end(), parent.begin(), parent.end());
  cbor_uint(buf, 4, n);         // array(n)
  for (size_t i = 0; i < n; ++i) cbor_uint(buf, 0, tokens[i] > 0 ? uint64_t(tokens[i]) : 0);
  buf.push_back(0xf6);          // null
  return sha256(buf.data(), buf.size());
}

std::vector<Hash> compute_block_hashes(const std::vector<int32_t>& tokens, size_t block_size, const std::string& seed) {
  block_size = std::max<size_t>(1, block_size);
  std::vector<Hash> out;
  Hash parent = none_hash(seed);
  for (size_t i = 0; i + block_size <= tokens.size(); i += block_size) {
    parent = block_hash(parent, tokens.data() + i, block_size);
    out.push_back(parent);
  }
  return out;
}

uint64_t external_key(const Hash& h) {
  uint64_t v = 0;
  for (int i = 24; i < 32; ++i) v = (v << 8) | h[i];
  return v;
}

std::string kv_hash_seed_from_env() {
  const char* s = std::getenv("NEBULA_KV_HASH_SEED");
  std::string v = s ? s : "";
  while (!v.empty() && isspace((unsigned char)v.back())) v.pop_back();
  while (!v.empty() && isspace((unsigned char)v.front())) v.erase(v.begin());
  return v.empty() ? "42" : v;
}

// ---------------------------------------------------------------------------- prefix lease
PrefixLease::PrefixLease(PrefixLease&& o) noexcept
    : st_(std::move(o.st_)), nodes_(std::move(o.nodes_)), pages_(std::move(o.pages_)),
      matched_tokens_(o.matched_tokens_), leaf_aux_(o.leaf_aux_) {
  o.nodes_.clear();
}

PrefixLease& PrefixLease::operator=(PrefixLease&& o) noexcept {
  if (this != &o) {
    release();
    st_ = std::move(o.st_);
    nodes_ = std::move(o.nodes_);
    pages_ = std::move(o.pages_);
    matched_tokens_ = o.matched_tokens_;
    leaf_aux_ = o.leaf_aux_;
    o.nodes_.clear();
  }
  return *this;
}

void PrefixLease::release() {
  if (st_ && !nodes_.empty()) {
    std::lock_guard<std::mutex> g(st_->mu);
    for (uint64_t id : nodes_) {
      auto it = st_->nodes.find(id);
      if (it != st_->nodes.end() && it->second.pins > 0) --it->second.pins;
    }
  }
  nodes_.clear();
  pages_.clear();
}

// ---------------------------------------------------------------------------- prefix tree
PrefixTree::PrefixTree(uint32_t block_tokens, uint32_t pages_per_node, const std::string& seed)
    : st_(std::make_shared<TreeState>()) {
  st_->block_tokens = std::max<uint32_t>(1, block_tokens);
  st_->pages_per_node = std::max<uint32_t>(1, pages_per_node);
  st_->root_hash = none_hash(seed);
}

void PrefixTree::set_event_sink(KvEventSink sink) {
  std::lock_guard<std::mutex> g(st_->mu);
  st_->sink = std::move(sink);
}

namespace {

std::map<std::vector<int32_t>, uint64_t>& children_of(TreeState& s, uint64_t parent) {
  if (parent == 0) return s.roots;
  return s.nodes.at(parent).children;
}

std::vector<uint64_t> page_keys(const TreeState& s, uint64_t parent, const int32_t* tokens, Hash* out_last) {
  // One external key per page of the node, chained from the parent's last page.
  Hash h = parent == 0 ? s.root_hash : s.nodes.at(parent).hash;
  std::vector<uint64_t> keys;
  for (uint32_t p = 0; p < s.pages_per_node; ++p) {
    h = block_hash(h, tokens + p * s.block_tokens, s.block_tokens);
    keys.push_back(external_key(h));
  }
  if (out_last) *out_last = h;
  return keys;
}

}  // namespace

PrefixLease PrefixTree::match(const std::vector<int32_t>& tokens, size_t max_nodes) {
  std::lock_guard<std::mutex> g(st_->mu);
  PrefixLease lease;
  lease.st_ = st_;
  const size_t nt = node_tokens();
  uint64_t parent = 0;
  ++st_->queries;
  st_->query_tokens += tokens.size();
  const uint64_t tick = ++st_->tick;
  for (size_t off = 0; off + nt <= tokens.size() && lease.nodes_.size() < max_nodes; off += nt) {
    std::vector<int32_t> key(tokens.begin() + off, tokens.begin() + off + nt);
    auto& ch = children_of(*st_, parent);
    auto it = ch.find(key);
    if (it == ch.end()) break;
    TreeNode& n = st_->nodes.at(it->second);
    ++n.pins;
    n.last_use = tick;
    lease.nodes_.push_back(n.id);
    lease.pages_.insert(lease.pages_.end(), n.pages.ids().begin(), n.pages.ids().end());
    lease.matched_tokens_ += nt;
    lease.leaf_aux_ = n.aux.empty() ? -1 : n.aux.ids()[0];
    parent = n.id;
  }
  st_->hit_tokens += lease.matched_tokens_;
  return lease;
}

std::pair<size_t, size_t> PrefixTree::peek(const std::vector<int32_t>& tokens, size_t max_nodes) const {
  std::lock_guard<std::mutex> g(st_->mu);
  const size_t nt = node_tokens();
  uint64_t parent = 0;
  size_t n = 0;
  for (size_t off = 0; off + nt <= tokens.size() && n < max_nodes; off += nt) {
    std::vector<int32_t> key(tokens.begin() + off, tokens.begin() + off + nt);
    const auto& ch = children_of(*st_, parent);
    auto it = ch.find(key);
    if (it == ch.end()) break;
    parent = it->second;
    ++n;
  }
  return {n, n * nt};
}

uint64_t PrefixTree::insert(uint64_t parent_node, const int32_t* tokens, BlockLease& pages, BlockLease& aux,
                            bool* created) {
  KvEvent ev;
  KvEventSink sink;
  uint64_t id;
  if (created) *created = false;
  {
    std::lock_guard<std::mutex> g(st_->mu);
    const size_t nt = node_tokens();
    if (parent_node != 0 && st_->nodes.find(parent_node) == st_->nodes.end()) return 0;
    std::vector<int32_t> key(tokens, tokens + nt);
    auto& ch = children_of(*st_, parent_node);
    auto it = ch.find(key);
    if (it != ch.end()) {
      // Concurrent promotion of the same chunk: keep the existing node; the caller
      // keeps its leases.
      st_->nodes.at(it->second).last_use = ++st_->tick;
      return it->second;
    }
    if (created) *created = true;
    id = st_->next_id++;
    TreeNode n;
    n.id = id;
    n.parent = parent_node;
    n.tokens = key;
    Hash last;
    ev.block_keys = page_keys(*st_, parent_node, tokens, &last);
    n.hash = last;
    n.pages = std::move(pages);
    n.aux = std::move(aux);
    n.last_use = ++st_->tick;
    ev.kind = KvEvent::kStored;
    ev.parent_key = parent_node == 0 ? 0 : external_key(st_->nodes.at(parent_node).hash);
    ev.tokens = key;
    ev.block_tokens = st_->block_tokens;
    ch.emplace(std::move(key), id);
    st_->nodes.emplace(id, std::move(n));
    sink = st_->sink;
  }
  if (sink) sink(ev);
  return id;
}

PrefixLease PrefixTree::pin_chain(uint64_t node) {
  std::lock_guard<std::mutex> g(st_->mu);
  PrefixLease lease;
  lease.st_ = st_;
  std::vector<uint64_t> chain;
  for (uint64_t id = node; id != 0; id = st_->nodes.at(id).parent) chain.push_back(id);
  std::reverse(chain.begin(), chain.end());
  for (uint64_t id : chain) {
    TreeNode& n = st_->nodes.at(id);
    ++n.pins;
    lease.nodes_.push_back(id);
    lease.pages_.insert(lease.pages_.end(), n.pages.ids().begin(), n.pages.ids().end());
    lease.matched_tokens_ += node_tokens();
    lease.leaf_aux_ = n.aux.empty() ? -1 : n.aux.ids()[0];
  }
  return lease;
}

std::vector<PrefixVictim> PrefixTree::evict_lru(size_t target_pages) {
  std::vector<PrefixVictim> victims;
  std::vector<KvEvent> events;
  KvEventSink sink;
  {
    std::lock_guard<std::mutex> g(st_->mu);
    size_t freed = 0;
    while (freed < target_pages) {
      // Least recently used unpinned leaf.
      uint64_t best = 0, best_use = UINT64_MAX;
      for (auto& kvp : st_->nodes) {
        const TreeNode& n = kvp.second;
        if (n.pins == 0 && n.children.empty() && n.last_use < best_use) {
          best = n.id;
          best_use = n.last_use;
        }
      }
      if (best == 0) break;
      TreeNode& n = st_->nodes.at(best);
      PrefixVictim v;
      v.pages = n.pages.ids();
      v.tokens = n.tokens;
      v.aux_slot = n.aux.empty() ? -1 : n.aux.ids()[0];
      v.hash = n.hash;
      v.node_id = n.id;
      KvEvent ev;
      ev.kind = KvEvent::kRemoved;
      ev.block_keys = page_keys(*st_, n.parent, n.tokens.data(), nullptr);
      events.push_back(std::move(ev));
      freed += n.pages.size();
      children_of(*st_, n.parent).erase(n.tokens);
      st_->nodes.erase(best);  // releases pages + aux to their pools
      ++st_->evictions;
      victims.push_back(std::move(v));
    }
    sink = st_->sink;
  }
  if (sink)
    for (auto& e : events) sink(e);
  return victims;
}

int32_t PrefixTree::aux_of(uint64_t node) const {
  std::lock_guard<std::mutex> g(st_->mu);
  auto it = st_->nodes.find(node);
  if (it == st_->nodes.end() || it->second.aux.empty()) return -1;
  return it->second.aux.ids()[0];
}

size_t PrefixTree::cached_nodes() const {
  std::lock_guard<std::mutex> g(st_->mu);
  return st_->nodes.size();
}

size_t PrefixTree::cached_pages() const {
  std::lock_guard<std::mutex> g(st_->mu);
  size_t n = 0;
  for (auto& kvp : st_->nodes) n += kvp.second.pages.size();
  return n;
}

size_t PrefixTree::evictable_pages() const {
  // Pages reachable by repeated leaf eviction: nodes whose whole subtree is unpinned.
  std::lock_guard<std::mutex> g(st_->mu);
  std::unordered_map<uint64_t, bool> pinned_below;
  std::function<bool(uint64_t)> any_pinned = [&](uint64_t id) -> bool {
    auto f = pinned_below.find(id);
    if (f != pinned_below.end()) return f->second;
    const TreeNode& n = st_->nodes.at(id);
    bool p = n.pins > 0;
    for (auto& c : n.children) p = any_pinned(c.second) || p;
    pinned_below[id] = p;
    return p;
  };
  size_t pages = 0;
  for (auto& kvp : st_->nodes)
    if (!any_pinned(kvp.first)) pages += kvp.second.pages.size();
  return pages;
}

void PrefixTree::clear() {
  KvEventSink sink;
  {
    std::lock_guard<std::mutex> g(st_->mu);
    st_->nodes.clear();
    st_->roots.clear();
    sink = st_->sink;
  }
  if (sink) {
    KvEvent ev;
    ev.kind = KvEvent::kAllCleared;
    sink(ev);
  }
}

PrefixTree::Stats PrefixTree::stats() const {
  std::lock_guard<std::mutex> g(st_->mu);
  return {st_->queries, st_->query_tokens, st_->hit_tokens, st_->evictions};
}

// ---------------------------------------------------------------------------- hybrid alias
bool HybridAliasTable::insert(int32_t anchor_page, int32_t slot, const std::vector<int32_t>& pages) {
  if (by_anchor_.count(anchor_page) || by_slot_.count(slot)) return false;
  by_anchor_[anchor_page] = slot;
  by_slot_[slot] = anchor_page;
  pages_[slot] = pages;
  return true;
}

bool HybridAliasTable::remove_by_anchor(int32_t anchor_page) {
  auto it = by_anchor_.find(anchor_page);
  if (it == by_anchor_.end()) return false;
  by_slot_.erase(it->second);
  pages_.erase(it->second);
  by_anchor_.erase(it);
  return true;
}

std::optional<int32_t> HybridAliasTable::slot_for_anchor(int32_t anchor_page) const {
  auto it = by_anchor_.find(anchor_page);
  if (it == by_anchor_.end()) return std::nullopt;
  return it->second;
}

std::optional<int32_t> HybridAliasTable::anchor_for_slot(int32_t slot) const {
  auto it = by_slot_.find(slot);
  if (it == by_slot_.end()) return std::nullopt;
  return it->second;
}

SubPageAllocator::SubPageAllocator(uint32_t slice_tokens, uint32_t page_tokens, uint32_t num_pages)
    : per_page_(std::max<uint32_t>(1, std::min<uint32_t>(32, page_tokens / std::max<uint32_t>(1, slice_tokens)))),
      used_(num_pages, 0) {}

std::optional<std::pair<int32_t, int32_t>> SubPageAllocator::allocate() {
  // Best fit: the most occupied page that still has a free slice, so pages fill up
  // before new ones are opened.
  int best = -1, best_used = -1;
  const uint32_t full = per_page_ == 32 ? 0xffffffffu : ((1u << per_page_) - 1);
  for (size_t p = 0; p < used_.size(); ++p) {
    if (used_[p] == full) continue;
    const int u = __builtin_popcount(used_[p]);
    if (u > best_used) {
      best = int(p);
      best_used = u;
    }
  }
  if (best < 0) return std::nullopt;
  const int slice = __builtin_ctz(~used_[best]);
  used_[best] |= 1u << slice;
  ++active_;
  return std::make_pair(best, slice);
}

void SubPageAllocator::release(int32_t page, int32_t slice) {
  if (page < 0 || size_t(page) >= used_.size()) return;
  if (used_[page] & (1u << slice)) {
    used_[page] &= ~(1u << slice);
    --active_;
  }
}

}  // namespace kv
}  // namespace zs
