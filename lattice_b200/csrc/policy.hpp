// Eviction policies of the swap tier: the victim selection of
// ref src/kcmm/tiering.rs:32-540 (trait EvictionPolicy and its LRU, LFU, FIFO,
// ARC and sink-window implementations), keyed by block id instead of the
// physical handle.
//
// The pool drives them as the reference's pool and tiering code do:
//   on_allocate   a block is installed (ref src/kcmm/pool.rs:448)
//   on_access     kcmm_hint / kcmm_protect touch a block (ref src/kcmm/ffi.rs:2334,
//                 2419), and a restored block (ref src/kcmm/tiering.rs:1871)
//   on_evict      a block was swapped out (ref src/kcmm/tiering.rs:1177, 1392)
//   select_victims over the live GPU-resident blocks in id order.
// Each policy object keeps its own per-block state, so a policy switched in at run
// time starts empty, as in ref src/kcmm/tiering.rs:877-895.  Logical ticks stand
// in for the reference's Instant timestamps (same order, never equal).
//
// One difference is deliberate: the reference's sink-window policy only
// protects blocks given to register_block, which no production path calls
// (only its unit tests), so in the reference it acts as LRU.  Here the pool
// registers every table position it creates (register, append, share, fork,
// copy-on-write, and all tables when the policy is switched in), so the first
// `sink` and last `window` blocks of each sequence are protected as documented
// there.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace kcmm {

class EvictionPolicy {
 public:
  virtual ~EvictionPolicy() = default;
  virtual void on_allocate(uint32_t blk) = 0;
  // Up to `count` of `candidates`, in eviction order.
  virtual std::vector<uint32_t> select_victims(const std::vector<uint32_t> &candidates,
                                               size_t count) const = 0;
  virtual void on_access(uint32_t blk) = 0;
  virtual void on_evict(uint32_t blk) = 0;
  virtual const char *name() const = 0;
  // Position of a block in a sequence's table (sink-window only).
  virtual void register_block(uint32_t, size_t, size_t) {}
};

// "lru", "lfu", "fifo", "arc" or "sink_window"; null for an unknown name.
// arc_capacity and (sink, window) size the last two.
std::unique_ptr<EvictionPolicy> make_policy(const std::string &name, size_t arc_capacity,
                                            size_t sink_blocks, size_t window_blocks);

}  // namespace kcmm
