// KV-cache pool: lockstep block allocator, block table, sequences, refcounts
// and swap-tier bookkeeping.
//
// Allocation rules restated from the reference (bit-exact block ids and
// offsets are a parity requirement):
//   * one logical allocator stands for the 2*num_layers per-layer K/V pools
//     of ref src/kcmm/pool.rs:228-233; the reference keeps them in lockstep
//     and asserts it (pool.rs:378-400), so a single free list is the same
//     state.  Each new superblock is still backed in every layer region.
//   * capacity: a new superblock is refused once
//     total_physical >= ceil(max_blocks_total / bps) * bps (pool.rs:323-359,
//     1145-1151).
//   * a block id is a recycled index popped LIFO, else the next new index
//     (pool.rs:412-453); va_offset = sb * 2 MiB + blk * block_bytes
//     (pool.rs:406-408).
//   * free releases handles in table order, then appends the recycled ids in
//     table order; any change bumps the block-state epoch (pool.rs:478-546).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "kcmm_internal.hpp"
#include "launch.hpp"

namespace kcmm {

// ---------------------------------------------------------------------------
// BlockAllocator
// ---------------------------------------------------------------------------

BlockAllocator::BlockAllocator(size_t bb)
    : block_bytes(bb), blocks_per_superblock(bb ? kSuperblockBytes / bb : 0) {
  if (bb == 0) throw Error("block_bytes must be positive");
  if (blocks_per_superblock == 0) {
    throw Error("block_bytes (" + std::to_string(bb) + ") too large for a 2 MiB superblock");
  }
}

bool BlockAllocator::try_allocate(BlockHandle *out) {
  if (free_.empty()) return false;
  *out = free_.back();
  free_.pop_back();
  return true;
}

void BlockAllocator::add_superblock() {
  uint32_t sb = uint32_t(sb_count_++);
  free_.reserve(free_.size() + blocks_per_superblock);
  for (size_t i = 0; i < blocks_per_superblock; ++i) free_.push_back({sb, uint32_t(i)});
}

// ---------------------------------------------------------------------------
// CpuSlotAllocator (ref src/kcmm/tiering.rs:552-640)
// ---------------------------------------------------------------------------

CpuSlotAllocator::CpuSlotAllocator(size_t total) {
  if (total > 0) free_.push_back({0, total});
}

bool CpuSlotAllocator::allocate(size_t size, size_t *offset) {
  if (size == 0 || free_.empty()) return false;
  size_t best = SIZE_MAX, best_len = SIZE_MAX;
  for (size_t i = 0; i < free_.size(); ++i) {
    size_t len = free_[i].second - free_[i].first;
    if (len >= size && len < best_len) {  // strict: the first of equal fits wins
      best_len = len;
      best = i;
    }
  }
  if (best == SIZE_MAX) return false;
  *offset = free_[best].first;
  if (best_len == size) {
    free_.erase(free_.begin() + long(best));
  } else {
    free_[best].first += size;
  }
  return true;
}

void CpuSlotAllocator::free(size_t offset, size_t size) {
  if (size == 0) return;
  size_t end = offset + size;
  size_t at = free_.size();
  for (size_t i = 0; i < free_.size(); ++i) {
    if (free_[i].first > offset) {
      at = i;
      break;
    }
  }
  bool prev = at > 0 && free_[at - 1].second == offset;
  bool next = at < free_.size() && free_[at].first == end;
  if (prev && next) {
    free_[at - 1].second = free_[at].second;
    free_.erase(free_.begin() + long(at));
  } else if (prev) {
    free_[at - 1].second = end;
  } else if (next) {
    free_[at].first = offset;
  } else {
    free_.insert(free_.begin() + long(at), {offset, end});
  }
}

// ---------------------------------------------------------------------------
// Swap tier storage
// ---------------------------------------------------------------------------

struct SwapTier {
  uint8_t *host = nullptr;      // host view
  uint8_t *dev_view = nullptr;  // device-mapped view of the same bytes
  size_t bytes = 0;
  bool file_backed = false;
  bool registered = false;
  CpuSlotAllocator slots{0};
  // Copy-engine swap path (created with the tier): device staging buffer, copy
  // stream and the events that order the staging halves.
  dev::SwapStaging staging{};

  ~SwapTier() {
    if (staging.copy_stream) cudaStreamSynchronize(staging.copy_stream);
    for (int h = 0; h < 2; ++h) {
      if (staging.ev_kernel[h]) cudaEventDestroy(staging.ev_kernel[h]);
      if (staging.ev_copy[h]) cudaEventDestroy(staging.ev_copy[h]);
    }
    if (staging.copy_stream) cudaStreamDestroy(staging.copy_stream);
    if (staging.buffer) cudaFree(staging.buffer);
    if (registered) cudaHostUnregister(host);
    if (host) {
      if (file_backed) {
        munmap(host, bytes);
      } else if (registered) {
        // anonymous mapping path
        munmap(host, bytes);
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Pool
// ---------------------------------------------------------------------------

namespace {
size_t checked_block_bytes(const PoolConfig &c) {
  if (c.num_layers == 0 || c.kv_heads == 0 || c.head_dim == 0 || c.max_batch == 0 ||
      c.max_seq_len == 0) {
    throw Error("num_layers, kv_heads, head_dim, max_batch and max_seq_len must be positive");
  }
  if (c.block_size == 0) throw Error("block_size must be positive");
  return c.kv_heads * c.block_size * c.head_dim * 2;
}
}  // namespace

// Bytes of virtual address space per K or V region.  The reference reserves
// align_up(max_blocks_total * block_bytes, 2 MiB) (ref src/kcmm/pool.rs:216-218), but
// its capacity rule (ref src/kcmm/pool.rs:323-340) admits whole superblocks of
// floor(2 MiB / block_bytes) blocks up to ceil(max_blocks_total / blocks_per_superblock)
// of them.  Where block_bytes does not divide 2 MiB (head_dim 192 with one kv head:
// 6144-byte blocks, 341 per superblock) the last admitted superblock lies past that
// reservation and mapping it fails.  The region here holds every admitted superblock;
// block ids, offsets and the capacity error are unchanged.
static size_t region_bytes_for(size_t max_blocks_total, size_t block_bytes) {
  const size_t flat = align_up(max_blocks_total * block_bytes, kSuperblockBytes);
  if (block_bytes == 0 || block_bytes > kSuperblockBytes) return flat;
  const size_t bps = kSuperblockBytes / block_bytes;
  return std::max(flat, (max_blocks_total + bps - 1) / bps * kSuperblockBytes);
}

Pool::Pool(const PoolConfig &cfg, std::unique_ptr<Vmm> vmm)
    : cfg_(cfg),
      block_size(cfg.block_size),
      elem_per_block(cfg.kv_heads * cfg.block_size * cfg.head_dim),
      block_bytes(checked_block_bytes(cfg)),
      step_elems(cfg.kv_heads * cfg.head_dim),
      max_blocks_per_seq((cfg.max_seq_len + cfg.block_size - 1) / cfg.block_size),
      max_blocks_total(cfg.max_batch * ((cfg.max_seq_len + cfg.block_size - 1) / cfg.block_size)),
      num_layers(cfg.num_layers),
      region_bytes(region_bytes_for(max_blocks_total, block_bytes)),
      vmm_(std::move(vmm)),
      alloc_(block_bytes),
      policy_(make_policy(cfg.eviction_policy, cfg.max_blocks, cfg.sink_blocks,
                          cfg.window_blocks)) {
  if (!policy_) policy_ = make_policy("lru", 0, 0, 0);
  // ref src/kcmm/pool.rs:217-225: one K and one V region per layer.
  va_k.resize(num_layers);
  va_v.resize(num_layers);
  for (size_t l = 0; l < num_layers; ++l) {
    va_k[l] = vmm_->reserve(region_bytes);
    va_v[l] = vmm_->reserve(region_bytes);
  }
  if (vmm_->is_device()) {
    use_device();
    std::vector<uint64_t> bases(2 * num_layers);
    for (size_t l = 0; l < num_layers; ++l) {
      bases[2 * l] = va_k[l];
      bases[2 * l + 1] = va_v[l];
    }
    if (cudaMalloc(&d_layer_bases, bases.size() * sizeof(uint64_t)) != cudaSuccess ||
        cudaMemcpy(d_layer_bases, bases.data(), bases.size() * sizeof(uint64_t),
                   cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMalloc(&diag_, sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(diag_, 0, sizeof(int32_t)) != cudaSuccess) {
      throw Error("device allocation of pool metadata failed");
    }
  }
}

Pool::~Pool() {
  stop_background_eviction();
  if (vmm_->is_device()) {
    use_device();
    cudaDeviceSynchronize();
    if (d_layer_bases) cudaFree(d_layer_bases);
    if (diag_) cudaFree(diag_);
  }
  tier_.reset();
  vmm_->release_all();
}

const void *Pool::tensor_maps(size_t layer, int kv_heads, int head_dim) {
  if (!vmm_->is_device() || layer >= num_layers || kv_heads <= 0 || head_dim % 64 != 0) {
    return nullptr;
  }
  std::lock_guard<std::mutex> g(tmap_mu_);
  for (auto &e : tmaps_) {
    if (e->layer == layer && e->kv_heads == kv_heads && e->head_dim == head_dim) return e->maps;
  }
  auto e = std::make_unique<TmapEntry>();
  e->layer = layer;
  e->kv_heads = kv_heads;
  e->head_dim = head_dim;
  const uint64_t tokens = region_bytes / (uint64_t(kv_heads) * head_dim * 2);
  if (!encode_kv_tensor_map(e->maps[0], va_k[layer], tokens, kv_heads, head_dim) ||
      !encode_kv_tensor_map(e->maps[1], va_v[layer], tokens, kv_heads, head_dim)) {
    return nullptr;
  }
  e->page_ok = encode_kv_page_tensor_map(e->maps[2], va_v[layer], tokens, kv_heads, head_dim);
  tmaps_.push_back(std::move(e));
  return tmaps_.back()->maps;
}

const void *Pool::v_page_map(size_t layer, int kv_heads, int head_dim) {
  if (!tensor_maps(layer, kv_heads, head_dim)) return nullptr;
  std::lock_guard<std::mutex> g(tmap_mu_);
  for (auto &e : tmaps_) {
    if (e->layer == layer && e->kv_heads == kv_heads && e->head_dim == head_dim) {
      return e->page_ok ? e->maps[2] : nullptr;
    }
  }
  return nullptr;
}

void Pool::use_device() const {
  if (vmm_->is_device()) cudaSetDevice(cfg_.device);
}

void Pool::require_device(const char *what) const {
  if (!vmm_->is_device()) {
    throw Error(std::string(what) + ": pool has no device memory (host VMM backend)");
  }
}

size_t Pool::max_physical_blocks_per_layer() const {
  size_t bps = alloc_.blocks_per_superblock;
  return bps ? (max_blocks_total + bps - 1) / bps * bps : 0;
}

void Pool::ensure_capacity_locked() {
  if (alloc_.free_count() > 0) return;
  size_t total = alloc_.total_blocks();
  size_t max_phys = max_physical_blocks_per_layer();
  if (total >= max_phys) {
    std::ostringstream os;
    os << "KCMM physical block capacity exhausted: total_physical_blocks=" << total
       << " max_physical_blocks_per_layer=" << max_phys
       << " max_blocks_total=" << max_blocks_total
       << " blocks_per_superblock=" << alloc_.blocks_per_superblock;
    throw Error(os.str());
  }
  // Back the next superblock in every region.  A region already backed by an
  // earlier, partly failed attempt is skipped, so a retry stays consistent.
  size_t sb = alloc_.superblock_count();
  if (mapped_.size() != 2 * num_layers) mapped_.assign(2 * num_layers, 0);
  for (size_t l = 0; l < num_layers; ++l) {
    for (int kv = 0; kv < 2; ++kv) {
      size_t r = 2 * l + size_t(kv);
      if (mapped_[r] > sb) continue;
      uint64_t base = kv ? va_v[l] : va_k[l];
      vmm_->create_and_map(base + sb * kSuperblockBytes, kSuperblockBytes);
      mapped_[r] = sb + 1;
    }
  }
  alloc_.add_superblock();
}

uint32_t Pool::install_locked(BlockHandle h) {
  BlockInfo bi;
  bi.va_offset = offset_of(h);
  bi.handle = h;
  bi.in_use = true;
  bi.loc = Loc::Gpu;
  bi.refcount = 1;
  bi.alloc_tick = bi.access_tick = ++tick_;
  bi.access_count = 1;
  uint32_t idx;
  if (!recycled_.empty()) {
    idx = recycled_.back();
    recycled_.pop_back();
    blocks_[idx] = bi;
  } else {
    idx = uint32_t(blocks_.size());
    blocks_.push_back(bi);
  }
  bump();
  log_block_locked(idx);
  if (cfg_.tiering) policy_->on_allocate(idx);  // ref src/kcmm/pool.rs:446-449
  return idx;
}

void Pool::register_positions_locked(size_t seq, size_t from) {
  const auto &t = seqs_[seq].table;
  for (size_t j = from; j < t.size(); ++j) policy_->register_block(t[j], seq, j);
}

void Pool::log_block_locked(uint32_t blk) {
  constexpr size_t kLogMax = size_t(1) << 20;
  if (block_log_.size() >= kLogMax) {  // readers behind the cut reload the whole array
    const size_t cut = block_log_.size() / 2;
    block_log_.erase(block_log_.begin(), block_log_.begin() + long(cut));
    block_log_base_ += cut;
  }
  block_log_.push_back(blk);
}

void Pool::touch_table_locked(Sequence &s, bool rewrite) {
  s.version = ++table_stamp_;
  if (rewrite) s.rewrite = s.version;
}

uint32_t Pool::alloc_block() {
  std::lock_guard<std::mutex> g(mu_);
  ensure_capacity_locked();
  BlockHandle h;
  if (!alloc_.try_allocate(&h)) throw Error("no free block after ensure_capacity");
  return install_locked(h);
}

std::vector<uint32_t> Pool::alloc_blocks(size_t n) {
  std::vector<uint32_t> out;
  out.reserve(n);
  for (size_t i = 0; i < n; ++i) out.push_back(alloc_block());
  return out;
}

void Pool::release_block_locked(uint32_t blk, std::vector<BlockHandle> *gpu,
                                std::vector<uint64_t> *cpu_slots) {
  BlockInfo &bi = blocks_[blk];
  if (bi.loc == Loc::Gpu || bi.loc == Loc::Cpu || bi.loc == Loc::Nvme) log_block_locked(blk);
  switch (bi.loc) {
    case Loc::Gpu:
      bi.in_use = false;
      gpu->push_back(bi.handle);
      break;
    case Loc::Cpu:
      bi.in_use = false;
      cpu_slots->push_back(bi.cpu_offset);
      break;
    case Loc::Nvme:
      bi.in_use = false;
      break;
    case Loc::Evicting:
    case Loc::Restoring:
      return;  // in flight: physical cleanup skipped (pool.rs:519-525)
  }
  bi.refcount = 0;
}

void Pool::finish_release_locked(const std::vector<BlockHandle> &gpu,
                                 const std::vector<uint64_t> &cpu_slots,
                                 const std::vector<uint32_t> &recycled) {
  for (const BlockHandle &h : gpu) alloc_.free(h);
  if (!cpu_slots.empty() && tier_) {
    size_t slot_bytes = num_layers * 2 * block_bytes;
    for (uint64_t off : cpu_slots) tier_->slots.free(off, slot_bytes);
  }
  if (!recycled.empty()) {
    bump();
    recycled_.insert(recycled_.end(), recycled.begin(), recycled.end());
  }
}

void Pool::free_blocks(const uint32_t *ids, size_t n) {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<BlockHandle> gpu;
  std::vector<uint64_t> cpu;
  std::vector<uint32_t> recycled;
  for (size_t i = 0; i < n; ++i) {
    uint32_t b = ids[i];
    if (b >= blocks_.size() || !blocks_[b].in_use) continue;
    if (blocks_[b].refcount > 1) {  // shared: drop one owner only
      blocks_[b].refcount -= 1;
      continue;
    }
    Loc before = blocks_[b].loc;
    release_block_locked(b, &gpu, &cpu);
    if (before != Loc::Evicting && before != Loc::Restoring) recycled.push_back(b);
  }
  finish_release_locked(gpu, cpu, recycled);
}

uint32_t Pool::register_sequence(std::vector<uint32_t> table) {
  std::lock_guard<std::mutex> g(mu_);
  Sequence s;
  s.table = std::move(table);
  s.last_access = ++tick_;
  touch_table_locked(s, true);
  seqs_.push_back(std::move(s));
  register_positions_locked(seqs_.size() - 1, 0);
  return uint32_t(seqs_.size() - 1);
}

void Pool::unregister_sequence(size_t seq) {
  std::vector<uint32_t> table;
  {
    std::lock_guard<std::mutex> g(mu_);
    if (seq >= seqs_.size()) return;
    table.swap(seqs_[seq].table);
    seqs_[seq].seq_len = 0;
    touch_table_locked(seqs_[seq], true);
  }
  if (!table.empty()) free_blocks(table.data(), table.size());
}

bool Pool::touch(size_t seq) {
  std::lock_guard<std::mutex> g(mu_);
  if (seq >= seqs_.size()) return false;
  seqs_[seq].last_access = ++tick_;
  seqs_[seq].active = true;
  return true;
}

bool Pool::cool(size_t seq) {
  std::lock_guard<std::mutex> g(mu_);
  if (seq >= seqs_.size()) return false;
  seqs_[seq].active = false;
  return true;
}

bool Pool::set_priority(size_t seq, Priority p) {
  std::lock_guard<std::mutex> g(mu_);
  if (seq >= seqs_.size()) return false;
  seqs_[seq].priority = p;
  return true;
}

void Pool::update_seq_len(size_t seq, size_t len) {
  std::lock_guard<std::mutex> g(mu_);
  if (seq < seqs_.size()) seqs_[seq].seq_len = len;
}

size_t Pool::seq_len(size_t seq) {
  std::lock_guard<std::mutex> g(mu_);
  return seq < seqs_.size() ? seqs_[seq].seq_len : 0;
}

bool Pool::append_block(size_t seq, uint32_t blk) {
  std::lock_guard<std::mutex> g(mu_);
  if (seq >= seqs_.size()) return false;
  seqs_[seq].table.push_back(blk);
  touch_table_locked(seqs_[seq], false);
  register_positions_locked(seq, seqs_[seq].table.size() - 1);
  return true;
}

bool Pool::block_table(size_t seq, std::vector<uint32_t> *out) {
  std::lock_guard<std::mutex> g(mu_);
  if (seq >= seqs_.size()) return false;
  *out = seqs_[seq].table;
  return true;
}

size_t Pool::active_sequences() {
  std::lock_guard<std::mutex> g(mu_);
  return seqs_.size();
}

bool Pool::block_va_offset(uint32_t blk, uint64_t *out) {
  std::lock_guard<std::mutex> g(mu_);
  if (blk >= blocks_.size() || !blocks_[blk].in_use) return false;
  *out = blocks_[blk].va_offset;
  return true;
}

bool Pool::sequence_va_offsets(size_t seq, std::vector<uint64_t> *out) {
  std::lock_guard<std::mutex> g(mu_);
  if (seq >= seqs_.size()) return false;
  out->clear();
  for (uint32_t b : seqs_[seq].table) {
    if (b >= blocks_.size() || !blocks_[b].in_use) return false;
    out->push_back(blocks_[b].va_offset);
  }
  return true;
}

std::vector<uint64_t> Pool::all_offsets_f16() {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<uint64_t> v(blocks_.size());
  for (size_t i = 0; i < blocks_.size(); ++i) {
    v[i] = blocks_[i].in_use ? blocks_[i].va_offset / 2 : 0;
  }
  return v;
}

std::vector<uint8_t> Pool::all_valid() {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<uint8_t> v(blocks_.size());
  for (size_t i = 0; i < blocks_.size(); ++i) v[i] = blocks_[i].in_use ? 1 : 0;
  return v;
}

bool Pool::block_location(uint32_t blk, Loc *out) {
  std::lock_guard<std::mutex> g(mu_);
  if (blk >= blocks_.size() || !blocks_[blk].in_use) return false;
  *out = blocks_[blk].loc;
  return true;
}

bool Pool::block_handle(uint32_t blk, BlockHandle *out) {
  std::lock_guard<std::mutex> g(mu_);
  if (blk >= blocks_.size() || !blocks_[blk].in_use) return false;
  *out = blocks_[blk].handle;
  return true;
}

size_t Pool::blocks_in_use() {
  std::lock_guard<std::mutex> g(mu_);
  size_t n = 0;
  for (const auto &b : blocks_) n += b.in_use ? 1 : 0;
  return n;
}

size_t Pool::total_blocks() {
  std::lock_guard<std::mutex> g(mu_);
  return blocks_.size();
}

size_t Pool::total_physical_blocks() {
  std::lock_guard<std::mutex> g(mu_);
  return alloc_.total_blocks();
}

size_t Pool::free_physical_blocks() {
  std::lock_guard<std::mutex> g(mu_);
  return alloc_.free_count();
}

size_t Pool::superblock_count() {
  std::lock_guard<std::mutex> g(mu_);
  return alloc_.superblock_count();
}

float Pool::physical_idle_ratio() {
  // ref src/kcmm/pool.rs:1161-1173
  size_t sbs = superblock_count();
  if (sbs == 0) return 0.0f;
  size_t total = sbs * kSuperblockBytes * num_layers * 2;
  size_t used = blocks_in_use() * block_bytes * num_layers * 2;
  if (used >= total) return 0.0f;
  return float(total - used) / float(total);
}

bool Pool::below_low_watermark(float threshold) {
  // ref src/kcmm/pool.rs:1242-1250
  std::lock_guard<std::mutex> g(mu_);
  size_t total = alloc_.total_blocks();
  if (total == 0) return false;
  float ratio = float(alloc_.free_count()) / float(total);
  return ratio < threshold;
}

void Pool::collect_metrics(double *ifr, double *pme, double *bu, double *rfi,
                           uint64_t *gpu_blocks, uint64_t *cpu_blocks) {
  // UFS metrics, computed in f32 as ref src/kcmm/pool.rs:1179-1236 does.
  std::lock_guard<std::mutex> g(mu_);
  size_t total_physical = alloc_.total_blocks();
  size_t in_use = 0, on_cpu = 0;
  for (const auto &b : blocks_) {
    if (!b.in_use) continue;
    ++in_use;
    if (b.loc == Loc::Cpu) ++on_cpu;
  }
  size_t blocks_used = 0, tokens = 0;
  for (const auto &s : seqs_) {
    blocks_used += s.table.size();
    tokens += s.seq_len;
  }
  size_t sbs = alloc_.superblock_count();
  uint64_t actual_physical = uint64_t(sbs) * kSuperblockBytes * num_layers * 2;
  size_t slots = blocks_used * block_size;
  float f_ifr = slots > 0 ? float(slots > tokens ? slots - tokens : 0) / float(slots) : 0.0f;
  float f_bu = total_physical > 0 ? float(in_use) / float(total_physical) : 0.0f;
  size_t bpt_all = step_elems * num_layers * 2;
  uint64_t ideal = uint64_t(tokens) * bpt_all;
  float f_pme = actual_physical > 0 ? float(ideal) / float(actual_physical) : 1.0f;
  size_t bps = alloc_.blocks_per_superblock;
  size_t active_sbs = (in_use + bps - 1) / bps;
  uint64_t actual_active = uint64_t(active_sbs) * kSuperblockBytes * num_layers * 2;
  float f_rfi = actual_active > 0 ? 1.0f - float(ideal) / float(actual_active) : 0.0f;
  *ifr = double(f_ifr);
  *pme = double(f_pme);
  *bu = double(f_bu);
  *rfi = double(f_rfi);
  *gpu_blocks = in_use - on_cpu;
  *cpu_blocks = on_cpu;
}

Metrics Pool::metrics() {
  std::lock_guard<std::mutex> g(mu_);
  return metrics_;
}

// --- refcounts and copy-on-write -------------------------------------------

void Pool::incref(uint32_t blk) {
  std::lock_guard<std::mutex> g(mu_);
  if (blk >= blocks_.size() || !blocks_[blk].in_use) {
    throw Error("block_idx " + std::to_string(blk) + " is not in use");
  }
  blocks_[blk].refcount += 1;
}

void Pool::decref(uint32_t blk) {
  {
    std::lock_guard<std::mutex> g(mu_);
    if (blk >= blocks_.size() || !blocks_[blk].in_use) {
      throw Error("block_idx " + std::to_string(blk) + " is not in use");
    }
  }
  free_blocks(&blk, 1);
}

uint32_t Pool::refcount(uint32_t blk) {
  std::lock_guard<std::mutex> g(mu_);
  if (blk >= blocks_.size() || !blocks_[blk].in_use) return 0;
  return blocks_[blk].refcount;
}

uint32_t Pool::fork_sequence(size_t src) {
  std::lock_guard<std::mutex> g(mu_);
  if (src >= seqs_.size()) throw Error("seq_idx " + std::to_string(src) + " out of bounds");
  Sequence s = seqs_[src];
  for (uint32_t b : s.table) {
    if (b >= blocks_.size() || !blocks_[b].in_use) {
      throw Error("block_idx " + std::to_string(b) + " is not in use");
    }
  }
  for (uint32_t b : s.table) blocks_[b].refcount += 1;
  s.last_access = ++tick_;
  s.active = true;
  touch_table_locked(s, true);
  seqs_.push_back(std::move(s));
  register_positions_locked(seqs_.size() - 1, 0);
  return uint32_t(seqs_.size() - 1);
}

std::vector<uint32_t> Pool::share_prefix(size_t src, size_t dst, size_t n) {
  std::lock_guard<std::mutex> g(mu_);
  if (src >= seqs_.size() || dst >= seqs_.size()) throw Error("seq_idx out of bounds");
  const auto &t = seqs_[src].table;
  if (n > t.size()) {
    throw Error("num_blocks " + std::to_string(n) + " exceeds source table length " +
                std::to_string(t.size()));
  }
  std::vector<uint32_t> out(t.begin(), t.begin() + long(n));
  for (uint32_t b : out) {
    if (b >= blocks_.size() || !blocks_[b].in_use) {
      throw Error("block_idx " + std::to_string(b) + " is not in use");
    }
  }
  for (uint32_t b : out) blocks_[b].refcount += 1;
  auto &dt = seqs_[dst].table;
  const size_t old_len = dt.size();
  dt.insert(dt.end(), out.begin(), out.end());
  touch_table_locked(seqs_[dst], false);
  register_positions_locked(dst, old_len);
  return out;
}

std::vector<uint32_t> Pool::cow_blocks(const uint32_t *seqs, const uint32_t *logical, size_t n,
                                       void *stream) {
  std::lock_guard<std::mutex> g(mu_);
  // Validate everything before changing state.
  for (size_t i = 0; i < n; ++i) {
    if (seqs[i] >= seqs_.size()) throw Error("seq_idx " + std::to_string(seqs[i]) + " out of bounds");
    const auto &t = seqs_[seqs[i]].table;
    if (logical[i] >= t.size()) {
      throw Error("logical block " + std::to_string(logical[i]) + " >= allocated " +
                  std::to_string(t.size()) + " for seq " + std::to_string(seqs[i]));
    }
    uint32_t b = t[logical[i]];
    if (b >= blocks_.size() || !blocks_[b].in_use || blocks_[b].loc != Loc::Gpu) {
      throw Error("block_idx " + std::to_string(b) + " is not a GPU-resident live block");
    }
  }
  std::vector<uint32_t> out(n);
  std::vector<uint64_t> src_off, dst_off;
  for (size_t i = 0; i < n; ++i) {
    uint32_t &slot = seqs_[seqs[i]].table[logical[i]];
    uint32_t b = slot;
    if (blocks_[b].refcount > 1) {
      ensure_capacity_locked();
      BlockHandle h;
      if (!alloc_.try_allocate(&h)) throw Error("no free block after ensure_capacity");
      uint32_t nb = install_locked(h);
      src_off.push_back(blocks_[b].va_offset);
      dst_off.push_back(blocks_[nb].va_offset);
      blocks_[b].refcount -= 1;
      slot = nb;
      touch_table_locked(seqs_[seqs[i]], true);
      policy_->register_block(nb, seqs[i], logical[i]);
    }
    out[i] = slot;
  }
  if (!src_off.empty()) {
    require_device("kcmm_cow_blocks_on_stream");
    use_device();
    cudaError_t e = dev::copy_blocks(d_layer_bases, int(num_layers), src_off.data(),
                                     dst_off.data(), int(src_off.size()), block_bytes,
                                     static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) throw Error(std::string("block copy launch failed: ") + cudaGetErrorString(e));
  }
  return out;
}

// --- append destinations ---------------------------------------------------

void Pool::step_destinations(const uint32_t *seqs, const uint32_t *positions, size_t batch,
                             std::vector<int64_t> *dst) {
  // ref src/kcmm/ffi.rs:1138-1186
  std::lock_guard<std::mutex> g(mu_);
  dst->resize(batch);
  for (size_t b = 0; b < batch; ++b) {
    size_t s = seqs[b];
    if (s >= seqs_.size()) {
      throw Error("seq_idx " + std::to_string(s) + " out of bounds");
    }
    size_t pos = positions[b];
    size_t lb = pos / block_size, off = pos % block_size;
    const auto &t = seqs_[s].table;
    if (lb >= t.size()) {
      throw Error("logical_block " + std::to_string(lb) + " >= allocated " +
                  std::to_string(t.size()) + " for seq " + std::to_string(s));
    }
    uint32_t blk = t[lb];
    if (blk >= blocks_.size() || !blocks_[blk].in_use || blocks_[blk].loc != Loc::Gpu) {
      throw Error("block_idx " + std::to_string(blk) + " not in use");
    }
    (*dst)[b] = int64_t(blocks_[blk].va_offset / 2 + off * step_elems);
  }
}

void Pool::slot_destinations(const int64_t *slots, size_t batch, std::vector<int64_t> *dst) {
  // ref src/kcmm/ffi.rs:1310-1330
  std::lock_guard<std::mutex> g(mu_);
  dst->resize(batch);
  for (size_t b = 0; b < batch; ++b) {
    int64_t slot = slots[b];
    if (slot < 0) {
      (*dst)[b] = -1;
      continue;
    }
    size_t blk = size_t(slot) / block_size, off = size_t(slot) % block_size;
    if (blk >= blocks_.size() || !blocks_[blk].in_use || blocks_[blk].loc != Loc::Gpu) {
      throw Error("block_idx " + std::to_string(blk) + " from slot " + std::to_string(slot) +
                  " not in use");
    }
    (*dst)[b] = int64_t(blocks_[blk].va_offset / 2 + off * step_elems);
  }
}

// --- tiering ---------------------------------------------------------------

std::string Pool::policy_name() {
  std::lock_guard<std::mutex> g(mu_);
  return policy_->name();
}

void Pool::set_policy(const std::string &name) {
  // ref src/kcmm/tiering.rs:877-895: a fresh policy object; ARC sized by the
  // swap buffer over max_batch_blocks, sink-window protecting 1 + 4 blocks.
  const size_t arc_cap = cfg_.max_blocks * num_layers * 2 * block_bytes /
                         std::max<size_t>(cfg_.max_batch_blocks, 1);
  auto p = make_policy(name, arc_cap, 1, 4);
  if (!p) {
    throw Error("unknown eviction policy '" + name +
                "' (expected lru, lfu, fifo, arc, or sink_window)");
  }
  std::lock_guard<std::mutex> g(mu_);
  policy_ = std::move(p);
  for (size_t s = 0; s < seqs_.size(); ++s) register_positions_locked(s, 0);
}

void Pool::note_access(uint32_t blk) {
  std::lock_guard<std::mutex> g(mu_);
  if (blk < blocks_.size() && blocks_[blk].in_use) {
    blocks_[blk].access_tick = ++tick_;
    blocks_[blk].access_count += 1;
    // the reference reaches the policy through the block's physical handle,
    // which only GPU-resident blocks have (ref src/kcmm/ffi.rs:2330-2336)
    if (blocks_[blk].loc == Loc::Gpu) policy_->on_access(blk);
  }
}

std::vector<uint32_t> Pool::select_victims_locked(size_t count) {
  // Candidates are all live GPU-resident blocks in id order (ffi.rs:1913-1926);
  // the policy orders them (tiering.rs:32-540).
  std::vector<uint32_t> cand;
  for (uint32_t i = 0; i < blocks_.size(); ++i) {
    if (blocks_[i].in_use && blocks_[i].loc == Loc::Gpu) cand.push_back(i);
  }
  return policy_->select_victims(cand, count);
}

std::vector<uint32_t> Pool::preview_victims(size_t count) {
  std::lock_guard<std::mutex> g(mu_);
  return select_victims_locked(count);
}

void Pool::start_background_eviction() {
  if (!cfg_.tiering) throw Error("tiering is disabled");
  require_device("background eviction");
  std::lock_guard<std::mutex> g(bg_mu_);
  if (bg_thread_.joinable()) return;
  bg_stop_ = false;
  bg_thread_ = std::thread([this] {
    use_device();
    const auto interval =
        std::chrono::milliseconds(std::max<uint64_t>(cfg_.evict_interval_ms, 1));
    const float threshold = cfg_.low_watermark;
    const size_t batch = std::min<size_t>(cfg_.max_batch_blocks, 16);
    std::unique_lock<std::mutex> lk(bg_mu_);
    while (!bg_cv_.wait_for(lk, interval, [this] { return bg_stop_; })) {
      lk.unlock();
      try {
        background_evict_once(threshold, batch);
      } catch (const std::exception &) {
        // a failed round (swap tier full, copy error) is counted in the
        // metrics by the swap path; the next round tries again
      }
      lk.lock();
    }
  });
}

void Pool::stop_background_eviction() {
  {
    std::lock_guard<std::mutex> g(bg_mu_);
    if (!bg_thread_.joinable()) return;
    bg_stop_ = true;
  }
  bg_cv_.notify_all();
  bg_thread_.join();
}

bool Pool::background_eviction_running() {
  std::lock_guard<std::mutex> g(bg_mu_);
  return bg_thread_.joinable();
}

void Pool::background_evict_once(float threshold, size_t batch) {
  if (!below_low_watermark(threshold)) return;
  std::lock_guard<std::mutex> g(mu_);
  // candidates: live GPU-resident blocks of inactive sequences, in sequence
  // and table order (ref src/kcmm/pool.rs:1351-1372), each block once
  std::vector<uint32_t> cand;
  std::vector<uint8_t> seen(blocks_.size(), 0);
  for (const Sequence &s : seqs_) {
    if (s.active) continue;
    for (uint32_t b : s.table) {
      if (b < blocks_.size() && !seen[b] && blocks_[b].in_use && blocks_[b].loc == Loc::Gpu) {
        seen[b] = 1;
        cand.push_back(b);
      }
    }
  }
  if (cand.empty()) return;
  std::vector<uint32_t> victims = policy_->select_victims(cand, std::min(batch, cand.size()));
  if (victims.empty()) return;
  SwapTier &t = tier_locked();
  const size_t slot_bytes = num_layers * 2 * block_bytes;
  size_t fits = 0;
  {
    CpuSlotAllocator probe = t.slots;
    size_t off;
    while (fits < victims.size() && probe.allocate(slot_bytes, &off)) ++fits;
  }
  victims.resize(fits);
  if (!victims.empty()) swap_out_locked(victims, nullptr, true);
}

// Swap batches move through the copy engines (device staging buffer +
// cudaMemcpyAsync per run of host slots): 93% of the measured pinned host link
// each way on config 5's 20% swap set, against 87% when the swap kernel stores
// into the mapped host tier directly.  KCMM_SWAP_IMPL=sm selects the latter.
static bool swap_through_copy_engines() {
  static const bool dma = [] {
    const char *v = std::getenv("KCMM_SWAP_IMPL");
    return !(v && std::strcmp(v, "sm") == 0);
  }();
  return dma;
}

SwapTier &Pool::tier_locked() {
  if (tier_) return *tier_;
  require_device("swap tier");
  auto t = std::make_unique<SwapTier>();
  t->bytes = cfg_.max_blocks * num_layers * 2 * block_bytes;  // tiering.rs:738-740
  if (t->bytes == 0) throw Error("swap tier has zero size");
  void *p = MAP_FAILED;
  int fd = -1;
  if (!cfg_.cpu_cache_path.empty()) {
    fd = open(cfg_.cpu_cache_path.c_str(), O_RDWR | O_CREAT, 0600);
    if (fd >= 0 && ftruncate(fd, off_t(t->bytes)) == 0) {
      p = mmap(nullptr, t->bytes, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd, 0);
    }
    if (fd >= 0) close(fd);
  }
  if (p != MAP_FAILED) {
    t->file_backed = true;
  } else {
    p = mmap(nullptr, t->bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (p == MAP_FAILED) throw Error("swap tier: host mapping failed");
  }
  t->host = static_cast<uint8_t *>(p);
  use_device();
  cudaError_t e = cudaHostRegister(t->host, t->bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    munmap(t->host, t->bytes);
    t->host = nullptr;
    throw Error(std::string("swap tier: cudaHostRegister failed: ") + cudaGetErrorString(e));
  }
  t->registered = true;
  void *dv = nullptr;
  e = cudaHostGetDevicePointer(&dv, t->host, 0);
  if (e != cudaSuccess) throw Error(std::string("swap tier: no device view: ") + cudaGetErrorString(e));
  t->dev_view = static_cast<uint8_t *>(dv);
  if (swap_through_copy_engines()) {
    // two halves of 32 MiB, or of one slot if a slot is larger
    dev::SwapStaging &st = t->staging;
    st.bytes = 2 * std::max<size_t>(size_t(32) << 20, num_layers * 2 * block_bytes);
    void *buf = nullptr;
    e = cudaMalloc(&buf, st.bytes);
    if (e == cudaSuccess) st.buffer = static_cast<uint8_t *>(buf);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st.copy_stream, cudaStreamNonBlocking);
    for (int h = 0; h < 2 && e == cudaSuccess; ++h) {
      e = cudaEventCreateWithFlags(&st.ev_kernel[h], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st.ev_copy[h], cudaEventDisableTiming);
    }
    if (e != cudaSuccess)
      throw Error(std::string("swap tier: copy-engine staging: ") + cudaGetErrorString(e));
  }
  t->slots = CpuSlotAllocator(t->bytes);
  tier_ = std::move(t);
  return *tier_;
}

void LatencyHistogram::record(uint64_t us) {
  // ref src/kcmm/metrics.rs:43-64
  count += 1;
  sum_us += us;
  if (count == 1) {
    min_us = max_us = us;
  } else {
    min_us = std::min(min_us, us);
    max_us = std::max(max_us, us);
  }
  static const uint64_t kBounds[8] = {100, 250, 500, 1000, 2500, 5000, 10000, UINT64_MAX};
  for (int i = 0; i < 8; ++i) {
    if (us < kBounds[i]) {
      buckets[i] += 1;
      return;
    }
  }
  buckets[8] += 1;
}

void Pool::swap_out_locked(const std::vector<uint32_t> &ids, void *stream, bool background) {
  if (ids.empty()) return;
  const auto t0 = std::chrono::steady_clock::now();
  SwapTier &t = tier_locked();
  size_t slot_bytes = num_layers * 2 * block_bytes;
  std::vector<uint64_t> va_off, host_off;
  std::vector<uint32_t> taken;
  for (uint32_t b : ids) {
    size_t off;
    if (!t.slots.allocate(slot_bytes, &off)) break;  // swap tier full: stop here
    va_off.push_back(blocks_[b].va_offset);
    host_off.push_back(off);
    taken.push_back(b);
    blocks_[b].loc = Loc::Evicting;
  }
  if (taken.empty()) throw Error("swap tier is full");
  use_device();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e =
      t.staging.buffer
          ? dev::swap_blocks_staged(t.staging, d_layer_bases, int(num_layers), va_off.data(),
                                    host_off.data(), int(taken.size()), block_bytes, t.host, 0, s)
                : dev::swap_blocks(d_layer_bases, int(num_layers), va_off.data(), host_off.data(),
                                   int(taken.size()), block_bytes, t.dev_view, 0, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    for (size_t i = 0; i < taken.size(); ++i) {  // roll back (tiering.rs:960-990)
      blocks_[taken[i]].loc = Loc::Gpu;
      t.slots.free(host_off[i], slot_bytes);
    }
    metrics_.eviction_failures += 1;
    throw Error(std::string("swap-out copy failed: ") + cudaGetErrorString(e));
  }
  for (size_t i = 0; i < taken.size(); ++i) {
    BlockInfo &bi = blocks_[taken[i]];
    alloc_.free(bi.handle);
    bi.loc = Loc::Cpu;
    bi.cpu_offset = host_off[i];
    bump();
    policy_->on_evict(taken[i]);  // ref src/kcmm/tiering.rs:1177
  }
  // ref src/kcmm/pool.rs:1255-1272
  const uint64_t us = uint64_t(std::chrono::duration_cast<std::chrono::microseconds>(
                                   std::chrono::steady_clock::now() - t0)
                                   .count());
  metrics_.eviction_count += 1;
  metrics_.evicted_blocks += taken.size();
  metrics_.eviction_latency.record(us);
  if (background) metrics_.background_eviction_count += 1;
  {
    PolicyStats &ps = metrics_.policy_stats[policy_->name()];
    ps.eviction_count += 1;
    ps.evicted_blocks += taken.size();
    const double n = double(ps.eviction_count);
    ps.avg_evict_batch_size = (ps.avg_evict_batch_size * (n - 1.0) + double(taken.size())) / n;
  }
  if (taken.size() < ids.size()) throw Error("swap tier is full");
}

void Pool::swap_in_locked(const std::vector<uint32_t> &ids, void *stream) {
  if (ids.empty()) return;
  const auto t0 = std::chrono::steady_clock::now();
  SwapTier &t = tier_locked();
  size_t slot_bytes = num_layers * 2 * block_bytes;
  std::vector<uint64_t> va_off, host_off;
  std::vector<BlockHandle> handles;
  for (uint32_t b : ids) {
    ensure_capacity_locked();
    BlockHandle h;
    if (!alloc_.try_allocate(&h)) throw Error("no free block after ensure_capacity");
    handles.push_back(h);
    va_off.push_back(offset_of(h));
    host_off.push_back(blocks_[b].cpu_offset);
    blocks_[b].loc = Loc::Restoring;
  }
  use_device();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e =
      t.staging.buffer
          ? dev::swap_blocks_staged(t.staging, d_layer_bases, int(num_layers), va_off.data(),
                                    host_off.data(), int(ids.size()), block_bytes, t.host, 1, s)
                : dev::swap_blocks(d_layer_bases, int(num_layers), va_off.data(), host_off.data(),
                                   int(ids.size()), block_bytes, t.dev_view, 1, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    for (size_t i = 0; i < ids.size(); ++i) {
      blocks_[ids[i]].loc = Loc::Cpu;
      alloc_.free(handles[i]);
    }
    metrics_.restoration_failures += 1;
    throw Error(std::string("swap-in copy failed: ") + cudaGetErrorString(e));
  }
  for (size_t i = 0; i < ids.size(); ++i) {
    BlockInfo &bi = blocks_[ids[i]];
    t.slots.free(bi.cpu_offset, slot_bytes);
    bi.va_offset = va_off[i];
    bi.handle = handles[i];
    bi.loc = Loc::Gpu;
    bi.access_tick = ++tick_;
    bump();
    log_block_locked(ids[i]);
    policy_->on_access(ids[i]);  // ref src/kcmm/tiering.rs:1871
  }
  // ref src/kcmm/pool.rs:1281-1293
  const uint64_t us = uint64_t(std::chrono::duration_cast<std::chrono::microseconds>(
                                   std::chrono::steady_clock::now() - t0)
                                   .count());
  metrics_.restoration_count += 1;
  metrics_.restored_blocks += ids.size();
  metrics_.restoration_latency.record(us);
  {
    PolicyStats &ps = metrics_.policy_stats[policy_->name()];
    ps.restoration_count += 1;
    ps.restored_blocks += ids.size();
  }
}

size_t Pool::evict(size_t count) {
  std::lock_guard<std::mutex> g(mu_);
  if (!cfg_.tiering || count == 0) return 0;
  std::vector<uint32_t> victims = select_victims_locked(count);
  if (victims.empty()) return 0;
  SwapTier &t = tier_locked();
  size_t slot_bytes = num_layers * 2 * block_bytes;
  size_t fits = 0;
  {
    CpuSlotAllocator probe = t.slots;
    size_t off;
    while (fits < victims.size() && probe.allocate(slot_bytes, &off)) ++fits;
  }
  victims.resize(fits);
  if (victims.empty()) throw Error("swap tier is full");
  swap_out_locked(victims, nullptr);
  return victims.size();
}

void Pool::swap_out(const uint32_t *ids, size_t n, void *stream) {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<uint32_t> v;
  for (size_t i = 0; i < n; ++i) {
    uint32_t b = ids[i];
    if (b >= blocks_.size() || !blocks_[b].in_use) {
      throw Error("block_idx " + std::to_string(b) + " is not in use");
    }
    if (blocks_[b].loc != Loc::Gpu) {
      throw Error("block " + std::to_string(b) + " is not GPU-resident");
    }
    if (std::find(v.begin(), v.end(), b) == v.end()) v.push_back(b);
  }
  swap_out_locked(v, stream);
}

void Pool::swap_in(const uint32_t *ids, size_t n, void *stream) {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<uint32_t> v;
  for (size_t i = 0; i < n; ++i) {
    uint32_t b = ids[i];
    if (b >= blocks_.size() || !blocks_[b].in_use) {
      throw Error("block_idx " + std::to_string(b) + " is not in use");
    }
    if (blocks_[b].loc == Loc::Gpu) continue;  // already resident: skipped
    if (blocks_[b].loc != Loc::Cpu) {
      throw Error("block " + std::to_string(b) + " is in transit; cannot restore");
    }
    if (std::find(v.begin(), v.end(), b) == v.end()) v.push_back(b);
  }
  swap_in_locked(v, stream);
}

uint64_t Pool::restore_one(uint32_t blk) {
  // ref src/kcmm/pool.rs:817-870
  if (!cfg_.tiering) throw Error("tiering is disabled; cannot restore evicted block");
  swap_in(&blk, 1, nullptr);
  std::lock_guard<std::mutex> g(mu_);
  return blocks_[blk].va_offset;
}

void Pool::restore_many(const uint32_t *ids, size_t n) {
  if (!cfg_.tiering) throw Error("tiering is disabled; cannot restore evicted blocks");
  swap_in(ids, n, nullptr);
}

}  // namespace kcmm
