// Internal declarations of the B200 KV-cache manager (not part of the ABI).
//
// Layering (each file cites the reference component it restates):
//   vmm.cpp      physical memory: CUDA VMM (cuMemCreate/cuMemMap) or a host
//                stand-in used by the CPU test-suite       (ref src/cache/cuda_vmm.rs)
//   pool.cpp     lockstep block allocator, block table, sequences, refcounts,
//                swap-tier bookkeeping                     (ref src/kcmm/pool.rs,
//                                                           src/kcmm/superblock.rs,
//                                                           src/kcmm/tiering.rs)
//   ffi.cpp      extern "C" exports of include/kcmm.h      (ref src/kcmm/ffi.rs)
//   kernels/*.cu sm_100a kernels and their launchers       (ref src/cuda/kernels/*.cu)
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "policy.hpp"

namespace kcmm {

// Granularity of one physical allocation (ref src/kcmm/superblock.rs:10).
constexpr size_t kSuperblockBytes = size_t(2) << 20;

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// ---------------------------------------------------------------------------
// Physical memory backends
// ---------------------------------------------------------------------------

class Vmm {
 public:
  virtual ~Vmm() = default;
  // Reserve `bytes` of device VA (2 MiB aligned).  Throws on failure.
  virtual uint64_t reserve(size_t bytes) = 0;
  // Back [va, va+bytes) with a fresh physical allocation, readable and
  // writable from the pool's device.  Throws on failure.
  virtual void create_and_map(uint64_t va, size_t bytes) = 0;
  // Unmap and release everything (called once at destroy).
  virtual void release_all() noexcept = 0;
  // True when the VA is real device memory that kernels may touch.
  virtual bool is_device() const = 0;
  virtual const char *name() const = 0;
};

// CUDA VMM on `device`.  Throws if the driver entry points are missing.
std::unique_ptr<Vmm> make_cuda_vmm(int device);
// Host stand-in: anonymous mmap reservations, no device.  Used only when
// KCMM_VMM_BACKEND=host (CPU tests); every kernel entry point refuses to run
// on such a pool.  KCMM_HOST_VMM_FAIL_AFTER=n makes the (n+1)-th
// create_and_map fail, to exercise the out-of-memory paths.
std::unique_ptr<Vmm> make_host_vmm();
// Encode a 128-byte CUtensorMap for TMA loads of 16-token x 64-dim tiles of
// one kv head from the region at `base` (see vmm.cpp).  False if unsupported.
bool encode_kv_tensor_map(void *out, uint64_t base, uint64_t tokens, int kv_heads, int head_dim);
// 4-D view {64, tokens, head_dim/64, kv_heads} of a layer region whose box
// {64, 16, head_dim/64, 1} is 16 token rows of one head, both head_dim halves:
// it lands in shared memory as [half][16 rows][128 B] (128-byte swizzle).
bool encode_kv_page_tensor_map(void *out, uint64_t base, uint64_t tokens, int kv_heads,
                               int head_dim);

// ---------------------------------------------------------------------------
// Allocator
// ---------------------------------------------------------------------------

struct BlockHandle {
  uint32_t sb = 0;   // superblock index
  uint32_t blk = 0;  // block index inside the superblock
  bool operator==(const BlockHandle &o) const { return sb == o.sb && blk == o.blk; }
};

// Fixed-size block allocator over 2 MiB superblocks.  Free list is LIFO:
// add_superblock pushes blocks 0..n-1, allocation pops from the back, a freed
// block is pushed on the back (ref src/kcmm/superblock.rs:95-121).
class BlockAllocator {
 public:
  explicit BlockAllocator(size_t block_bytes);
  bool try_allocate(BlockHandle *out);
  void add_superblock();
  void free(BlockHandle h) { free_.push_back(h); }
  size_t free_count() const { return free_.size(); }
  size_t superblock_count() const { return sb_count_; }
  size_t total_blocks() const { return sb_count_ * blocks_per_superblock; }
  size_t tail_padding_bytes() const {
    return kSuperblockBytes - blocks_per_superblock * block_bytes;
  }
  const size_t block_bytes;
  const size_t blocks_per_superblock;

 private:
  std::vector<BlockHandle> free_;
  size_t sb_count_ = 0;
};

// ---------------------------------------------------------------------------
// Pool
// ---------------------------------------------------------------------------

enum class Loc : int32_t { Gpu = 0, Cpu = 1, Nvme = 2, Evicting = 3, Restoring = 4 };

struct BlockInfo {
  uint64_t va_offset = 0;      // byte offset inside every layer's K and V region
  BlockHandle handle;
  bool in_use = false;
  Loc loc = Loc::Gpu;
  uint64_t cpu_offset = 0;     // swap slot when loc == Cpu
  uint32_t refcount = 0;       // owners; 1 for an unshared block
  // eviction-policy keys (logical clock, not wall time)
  uint64_t alloc_tick = 0;
  uint64_t access_tick = 0;
  uint64_t access_count = 0;
};

enum class Priority : int32_t { Evictable = 0, Low = 1, Normal = 2, High = 3 };

struct Sequence {
  std::vector<uint32_t> table;
  size_t seq_len = 0;
  bool active = true;
  uint64_t last_access = 0;
  Priority priority = Priority::Normal;
  // Change stamps for device-resident step tables: `version` moves on every
  // table change, `rewrite` only when entries other than the tail change
  // (register, fork, copy-on-write, unregister), so an unchanged `rewrite`
  // means the new entries are all past the old end.
  uint64_t version = 0, rewrite = 0;
};

// What a StepTables object's device arrays hold, as the host last wrote them.
struct StepTableState {
  size_t max_batch = 0;
  std::vector<int64_t> row_seq;  // -1: never written
  std::vector<uint64_t> row_version, row_rewrite;
  std::vector<uint32_t> row_blocks;  // table entries written (the rest are zero)
  std::vector<int32_t> row_len;
  uint64_t log_cursor = 0;  // block-log position the offsets reflect
  size_t offsets_len = 0;   // entries valid in the device offsets array
  bool offsets_init = false;
};

// One sync's changes: 32-bit entries of [tables (max_batch x max_blocks_per_seq) |
// seq_lens (max_batch)] and 64-bit entries of the offsets array.
struct TableUpdates {
  std::vector<uint32_t> idx32;
  std::vector<int32_t> val32;
  std::vector<uint32_t> idx64;
  std::vector<uint64_t> val64;
  size_t offsets_needed = 0;  // entries the offsets array must hold
  bool offsets_full = false;  // every entry was listed (first sync, grown, or log trimmed)
};

struct PoolConfig {
  size_t block_size = 16;
  size_t max_blocks = 16384;
  std::string cpu_cache_path = "/dev/shm/kcmm_swap";
  bool tiering = true;
  std::string eviction_policy = "lru";
  size_t prefetch_window = 4;
  size_t max_batch_blocks = 64;
  int device = 0;
  size_t num_layers = 0, kv_heads = 0, head_dim = 0, max_batch = 0, max_seq_len = 0;
  float low_watermark = 0.2f;
  uint64_t evict_interval_ms = 100;
  size_t sink_blocks = 1, window_blocks = 4;
};

// Operation latencies in microseconds, bucketed at 100, 250, 500, 1000, 2500,
// 5000, 10000 us and above (ref src/kcmm/metrics.rs:29-74).
struct LatencyHistogram {
  uint64_t count = 0, sum_us = 0, min_us = 0, max_us = 0;
  uint64_t buckets[9] = {};
  void record(uint64_t us);
};

// Per-policy counters, keyed by the policy active at the time
// (ref src/kcmm/metrics.rs:14-20, src/kcmm/pool.rs:1263-1292).
struct PolicyStats {
  uint64_t eviction_count = 0, restoration_count = 0, evicted_blocks = 0, restored_blocks = 0;
  double avg_evict_batch_size = 0.0;
};

struct Metrics {
  uint64_t eviction_count = 0, evicted_blocks = 0, eviction_failures = 0;
  uint64_t restoration_count = 0, restored_blocks = 0, restoration_failures = 0;
  uint64_t background_eviction_count = 0;
  LatencyHistogram eviction_latency, restoration_latency;
  std::map<std::string, PolicyStats> policy_stats;
};

// Pinned, device-mapped host memory that backs the swap tier.
struct SwapTier;

class Pool {
 public:
  Pool(const PoolConfig &cfg, std::unique_ptr<Vmm> vmm);
  ~Pool();

  // --- allocation (ref src/kcmm/pool.rs:323-546) ---
  uint32_t alloc_block();
  std::vector<uint32_t> alloc_blocks(size_t n);  // partial success stays installed
  void free_blocks(const uint32_t *ids, size_t n);
  // --- sequences (ref src/kcmm/pool.rs:551-687) ---
  uint32_t register_sequence(std::vector<uint32_t> table);
  void unregister_sequence(size_t seq);
  bool touch(size_t seq);
  bool cool(size_t seq);
  bool set_priority(size_t seq, Priority p);
  void update_seq_len(size_t seq, size_t len);
  size_t seq_len(size_t seq);
  bool append_block(size_t seq, uint32_t blk);
  bool block_table(size_t seq, std::vector<uint32_t> *out);
  size_t active_sequences();
  // --- queries (ref src/kcmm/pool.rs:687-760) ---
  bool block_va_offset(uint32_t blk, uint64_t *out);
  bool sequence_va_offsets(size_t seq, std::vector<uint64_t> *out);
  std::vector<uint64_t> all_offsets_f16();
  std::vector<uint8_t> all_valid();
  bool block_location(uint32_t blk, Loc *out);
  bool block_handle(uint32_t blk, BlockHandle *out);
  uint64_t epoch() const { return epoch_.load(std::memory_order_acquire); }
  // --- statistics (ref src/kcmm/pool.rs:1098-1240) ---
  size_t blocks_in_use();
  size_t total_blocks();
  size_t total_physical_blocks();
  size_t free_physical_blocks();
  size_t superblock_count();
  size_t max_physical_blocks_per_layer() const;
  float physical_idle_ratio();
  bool below_low_watermark(float threshold);
  void collect_metrics(double *ifr, double *pme, double *bu, double *rfi,
                       uint64_t *gpu_blocks, uint64_t *cpu_blocks);
  Metrics metrics();
  // --- refcounts / copy-on-write ---
  void incref(uint32_t blk);
  void decref(uint32_t blk);
  uint32_t refcount(uint32_t blk);
  uint32_t fork_sequence(size_t src);
  std::vector<uint32_t> share_prefix(size_t src, size_t dst, size_t n);
  // Resolve (seq, logical) pairs; every shared block gets a fresh block whose
  // pages are copied on `stream` before the table entry moves.
  std::vector<uint32_t> cow_blocks(const uint32_t *seqs, const uint32_t *logical,
                                   size_t n, void *stream);
  // --- tiering (ref src/kcmm/tiering.rs) ---
  bool tiering_enabled() const { return cfg_.tiering; }
  std::string policy_name();
  void set_policy(const std::string &name);
  void note_access(uint32_t blk);
  size_t evict(size_t count);
  // The victims evict(count) would take now, without moving anything.
  std::vector<uint32_t> preview_victims(size_t count);
  // Background eviction (ref src/kcmm/pool.rs:1308-1405): every
  // evict_interval_ms, when the free-block ratio is below low_watermark, swap
  // out up to min(max_batch_blocks, 16) policy-chosen blocks of inactive
  // (cooled) sequences.  Start is a no-op when running; stop joins the thread.
  void start_background_eviction();
  void stop_background_eviction();
  bool background_eviction_running();
  uint64_t restore_one(uint32_t blk);
  void restore_many(const uint32_t *ids, size_t n);
  void swap_out(const uint32_t *ids, size_t n, void *stream);
  void swap_in(const uint32_t *ids, size_t n, void *stream);
  // --- kernels support ---
  // Device destination offsets (in 2-byte elements) of append rows, computed
  // under the metadata lock exactly like ref src/kcmm/ffi.rs:1138-1186.
  void step_destinations(const uint32_t *seqs, const uint32_t *positions, size_t batch,
                         std::vector<int64_t> *dst_elems);
  void slot_destinations(const int64_t *slots, size_t batch, std::vector<int64_t> *dst_elems);
  // Cached TMA descriptors of a layer's K and V regions for a (kv_heads,
  // head_dim) view; nullptr when the shape has no TMA path.
  const void *tensor_maps(size_t layer, int kv_heads, int head_dim);
  // The V page-box map of the layer (third map above), or null when unavailable.
  const void *v_page_map(size_t layer, int kv_heads, int head_dim);
  // Changes since `st` for the rows seqs[0..batch) of a device step table, and
  // `st` moved to the new state (step_tables.cpp).
  void step_table_updates(const uint32_t *seqs, size_t batch, StepTableState *st,
                          TableUpdates *up);
  void use_device() const;  // make the pool's device current
  void require_device(const char *what) const;
  int32_t *diag_word() const { return diag_; }  // device int32, sticky error bits

  const PoolConfig cfg_;
  const size_t block_size, elem_per_block, block_bytes, step_elems;
  const size_t max_blocks_per_seq, max_blocks_total, num_layers;
  const size_t region_bytes;
  std::vector<uint64_t> va_k, va_v;
  uint64_t *d_layer_bases = nullptr;  // device copy of {va_k[l], va_v[l]} pairs

  std::mutex err_mu;
  std::string last_error;

 private:
  void ensure_capacity_locked();
  uint32_t install_locked(BlockHandle h);
  void release_block_locked(uint32_t blk, std::vector<BlockHandle> *gpu,
                            std::vector<uint64_t> *cpu_slots);
  void finish_release_locked(const std::vector<BlockHandle> &gpu,
                             const std::vector<uint64_t> &cpu_slots,
                             const std::vector<uint32_t> &recycled);
  uint64_t offset_of(BlockHandle h) const {
    return uint64_t(h.sb) * kSuperblockBytes + uint64_t(h.blk) * block_bytes;
  }
  void bump() { epoch_.fetch_add(1, std::memory_order_acq_rel); }
  // Blocks whose offset-table entry (in_use ? va_offset / 2 : 0) changed, in
  // order; entry i has global position block_log_base_ + i.
  void log_block_locked(uint32_t blk);
  void touch_table_locked(Sequence &s, bool rewrite);
  std::vector<uint32_t> select_victims_locked(size_t count);
  void register_positions_locked(size_t seq, size_t from);
  void background_evict_once(float threshold, size_t batch);
  void swap_out_locked(const std::vector<uint32_t> &ids, void *stream, bool background = false);
  void swap_in_locked(const std::vector<uint32_t> &ids, void *stream);
  SwapTier &tier_locked();

  std::unique_ptr<Vmm> vmm_;
  std::mutex tmap_mu_;
  struct TmapEntry {
    size_t layer;
    int kv_heads, head_dim;
    // [0] K and [1] V as {D, Hkv, tokens} with box {64, 1, 16}; [2] V as
    // {64, tokens, D/64, Hkv} with box {64, 16, D/64, 1} (one box = one page of one head)
    alignas(64) unsigned char maps[3][128];
    bool page_ok = false;
  };
  std::vector<std::unique_ptr<TmapEntry>> tmaps_;
  std::mutex mu_;  // guards everything below
  BlockAllocator alloc_;
  std::vector<BlockInfo> blocks_;
  std::vector<uint32_t> recycled_;
  std::vector<size_t> mapped_;  // superblocks backed so far, per region
  std::vector<Sequence> seqs_;
  uint64_t tick_ = 0;
  std::unique_ptr<EvictionPolicy> policy_;
  std::mutex bg_mu_;
  std::condition_variable bg_cv_;
  std::thread bg_thread_;
  bool bg_stop_ = false;
  Metrics metrics_;
  std::unique_ptr<SwapTier> tier_;
  std::atomic<uint64_t> epoch_{0};
  int32_t *diag_ = nullptr;
  std::vector<uint32_t> block_log_;
  uint64_t block_log_base_ = 0;
  uint64_t table_stamp_ = 0;
};

// Best-fit range allocator over the swap buffer, merging on free
// (ref src/kcmm/tiering.rs:552-640).
class CpuSlotAllocator {
 public:
  explicit CpuSlotAllocator(size_t total);
  bool allocate(size_t size, size_t *offset);
  void free(size_t offset, size_t size);
  const std::vector<std::pair<size_t, size_t>> &ranges() const { return free_; }

 private:
  std::vector<std::pair<size_t, size_t>> free_;  // [start, end), sorted
};

}  // namespace kcmm
