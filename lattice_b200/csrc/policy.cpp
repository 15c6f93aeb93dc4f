// Eviction policies (policy.hpp).  Each class cites the reference code whose
// selection rule it restates.
#include "policy.hpp"

#include <algorithm>
#include <utility>

namespace kcmm {
namespace {

// Candidates that have a key, stable-sorted by it (oldest / smallest first),
// truncated to `count`: the shape shared by ref tiering.rs LRU (:79-93), LFU
// (:130-144) and FIFO (:180-194), whose filter_map drops untracked candidates.
template <typename Map>
std::vector<uint32_t> by_key(const Map &m, const std::vector<uint32_t> &cand, size_t count) {
  if (cand.empty() || count == 0) return {};
  std::vector<std::pair<uint32_t, uint64_t>> v;
  for (uint32_t h : cand) {
    auto it = m.find(h);
    if (it != m.end()) v.emplace_back(h, it->second);
  }
  std::stable_sort(v.begin(), v.end(),
                   [](const auto &a, const auto &b) { return a.second < b.second; });
  if (v.size() > count) v.resize(count);
  std::vector<uint32_t> out;
  out.reserve(v.size());
  for (auto &p : v) out.push_back(p.first);
  return out;
}

// ref tiering.rs:56-99: last access time; allocate and access both stamp it.
class Lru final : public EvictionPolicy {
 public:
  void on_allocate(uint32_t b) override { t_[b] = ++tick_; }
  std::vector<uint32_t> select_victims(const std::vector<uint32_t> &c, size_t n) const override {
    return by_key(t_, c, n);
  }
  void on_access(uint32_t b) override { t_[b] = ++tick_; }
  void on_evict(uint32_t b) override { t_.erase(b); }
  const char *name() const override { return "lru"; }

 private:
  std::unordered_map<uint32_t, uint64_t> t_;
  uint64_t tick_ = 0;
};

// ref tiering.rs:103-153: access count, 1 at allocation, +1 per access (an
// access of an untracked block starts it at 1).
class Lfu final : public EvictionPolicy {
 public:
  void on_allocate(uint32_t b) override { c_[b] = 1; }
  std::vector<uint32_t> select_victims(const std::vector<uint32_t> &c, size_t n) const override {
    return by_key(c_, c, n);
  }
  void on_access(uint32_t b) override { c_[b] += 1; }
  void on_evict(uint32_t b) override { c_.erase(b); }
  const char *name() const override { return "lfu"; }

 private:
  std::unordered_map<uint32_t, uint64_t> c_;
};

// ref tiering.rs:157-215: allocation time only; accesses do not reorder.
class Fifo final : public EvictionPolicy {
 public:
  void on_allocate(uint32_t b) override { t_[b] = ++tick_; }
  std::vector<uint32_t> select_victims(const std::vector<uint32_t> &c, size_t n) const override {
    return by_key(t_, c, n);
  }
  void on_access(uint32_t) override {}
  void on_evict(uint32_t b) override { t_.erase(b); }
  const char *name() const override { return "fifo"; }

 private:
  std::unordered_map<uint32_t, uint64_t> t_;
  uint64_t tick_ = 0;
};

// ref tiering.rs:217-446: ARC with lists T1 (seen once) and T2 (seen again),
// most recent at the front, and ghost lists B1 / B2 of entries evicted from
// them (appended at the back, oldest dropped beyond `capacity`).  p is the
// adaptive target size of T1.
class Arc final : public EvictionPolicy {
 public:
  explicit Arc(size_t capacity) : cap_(std::max<size_t>(capacity, 1)) {}

  void on_allocate(uint32_t b) override {
    const bool in_b1 = erase_one(&b1_, b);
    const bool in_b2 = erase_one(&b2_, b);
    if (in_b1) {
      const size_t delta =
          std::max<size_t>(std::max<size_t>(b2_.size(), 1) / std::max<size_t>(b1_.size(), 1), 1);
      p_ = std::min(p_ + delta, cap_);
      t2_.insert(t2_.begin(), b);
    } else if (in_b2) {
      const size_t delta =
          std::max<size_t>(std::max<size_t>(b1_.size(), 1) / std::max<size_t>(b2_.size(), 1), 1);
      p_ = p_ > delta ? p_ - delta : 0;
      t2_.insert(t2_.begin(), b);
    } else {
      t1_.insert(t1_.begin(), b);
    }
    while (t1_.size() + t2_.size() > cap_) replace();
  }

  // Score: position from the LRU end of T1, then |T1| + position from the LRU
  // end of T2, untracked candidates last; stable sort (ref :356-392).
  std::vector<uint32_t> select_victims(const std::vector<uint32_t> &c, size_t n) const override {
    if (c.empty() || n == 0) return {};
    std::vector<std::pair<uint32_t, size_t>> v;
    v.reserve(c.size());
    for (uint32_t h : c) {
      size_t score = t1_.size() + t2_.size() + 1;
      const long p1 = pos_from_tail(t1_, h);
      if (p1 >= 0) {
        score = size_t(p1);
      } else {
        const long p2 = pos_from_tail(t2_, h);
        if (p2 >= 0) score = t1_.size() + size_t(p2);
      }
      v.emplace_back(h, score);
    }
    std::stable_sort(v.begin(), v.end(),
                     [](const auto &a, const auto &b) { return a.second < b.second; });
    if (v.size() > n) v.resize(n);
    std::vector<uint32_t> out;
    for (auto &p : v) out.push_back(p.first);
    return out;
  }

  void on_access(uint32_t b) override {  // ref :394-411
    auto it = std::find(t1_.begin(), t1_.end(), b);
    if (it != t1_.end()) {
      t1_.erase(it);
      t2_.insert(t2_.begin(), b);
      return;
    }
    it = std::find(t2_.begin(), t2_.end(), b);
    if (it != t2_.end()) {
      t2_.erase(it);
      t2_.insert(t2_.begin(), b);
    }
  }

  void on_evict(uint32_t b) override {  // ref :413-441
    auto it = std::find(t1_.begin(), t1_.end(), b);
    if (it != t1_.end()) {
      t1_.erase(it);
      push_ghost(&b1_, b);
      return;
    }
    it = std::find(t2_.begin(), t2_.end(), b);
    if (it != t2_.end()) {
      t2_.erase(it);
      push_ghost(&b2_, b);
    }
  }

  const char *name() const override { return "arc"; }

 private:
  static bool erase_one(std::vector<uint32_t> *v, uint32_t b) {
    auto it = std::find(v->begin(), v->end(), b);
    if (it == v->end()) return false;
    v->erase(it);
    return true;
  }
  static long pos_from_tail(const std::vector<uint32_t> &v, uint32_t h) {
    for (size_t i = v.size(); i-- > 0;) {
      if (v[i] == h) return long(v.size() - 1 - i);
    }
    return -1;
  }
  void push_ghost(std::vector<uint32_t> *g, uint32_t b) {
    if (std::find(g->begin(), g->end(), b) != g->end()) return;
    g->push_back(b);
    while (g->size() > cap_) g->erase(g->begin());
  }
  // ref :268-296: the LRU entry of T1 goes to B1 when T1 is over its target
  // (or T2 is empty), else the LRU entry of T2 goes to B2.
  void replace() {
    if (!t1_.empty() && (t1_.size() > p_ || t2_.empty())) {
      const uint32_t v = t1_.back();
      t1_.pop_back();
      b1_.push_back(v);
      while (b1_.size() > cap_) b1_.erase(b1_.begin());
    } else if (!t2_.empty()) {
      const uint32_t v = t2_.back();
      t2_.pop_back();
      b2_.push_back(v);
      while (b2_.size() > cap_) b2_.erase(b2_.begin());
    }
  }

  std::vector<uint32_t> t1_, t2_, b1_, b2_;
  size_t p_ = 0;
  const size_t cap_;
};

// ref tiering.rs:448-555: LRU over the blocks outside each sequence's first
// `sink` and last `window` positions; a sequence's length is the largest
// registered position + 1.  A block registered in several sequences (shared
// by a fork) keeps its last registration, as the reference's map does.
class SinkWindow final : public EvictionPolicy {
 public:
  SinkWindow(size_t sink, size_t window) : sink_(sink), window_(window) {}
  void register_block(uint32_t b, size_t seq, size_t pos) override { pos_[b] = {seq, pos}; }
  void on_allocate(uint32_t b) override { t_[b] = ++tick_; }
  std::vector<uint32_t> select_victims(const std::vector<uint32_t> &c, size_t n) const override {
    if (c.empty() || n == 0) return {};
    std::map<size_t, size_t> seq_blocks;
    for (const auto &kv : pos_) {
      size_t &m = seq_blocks[kv.second.first];
      m = std::max(m, kv.second.second + 1);
    }
    std::vector<uint32_t> eligible;
    for (uint32_t h : c) {
      auto it = pos_.find(h);
      if (it != pos_.end()) {
        const size_t p = it->second.second;
        if (p < sink_) continue;
        auto sb = seq_blocks.find(it->second.first);
        if (sb != seq_blocks.end()) {
          const size_t start = sb->second > window_ ? sb->second - window_ : 0;
          if (p >= start) continue;
        }
      }
      eligible.push_back(h);
    }
    return by_key(t_, eligible, n);
  }
  void on_access(uint32_t b) override { t_[b] = ++tick_; }
  void on_evict(uint32_t b) override { t_.erase(b); }
  const char *name() const override { return "sink_window"; }

 private:
  std::unordered_map<uint32_t, std::pair<size_t, size_t>> pos_;
  std::unordered_map<uint32_t, uint64_t> t_;
  uint64_t tick_ = 0;
  const size_t sink_, window_;
};

}  // namespace

std::unique_ptr<EvictionPolicy> make_policy(const std::string &name, size_t arc_capacity,
                                            size_t sink_blocks, size_t window_blocks) {
  if (name == "lru") return std::make_unique<Lru>();
  if (name == "lfu") return std::make_unique<Lfu>();
  if (name == "fifo") return std::make_unique<Fifo>();
  if (name == "arc") return std::make_unique<Arc>(arc_capacity);
  if (name == "sink_window") return std::make_unique<SinkWindow>(sink_blocks, window_blocks);
  return nullptr;
}

}  // namespace kcmm
