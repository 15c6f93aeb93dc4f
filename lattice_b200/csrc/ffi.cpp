// extern "C" exports of include/kcmm.h.
//
// Argument validation, error strings and return conventions follow
// ref src/kcmm/ffi.rs (cited per function).  Kernels are compiled offline for
// sm_100a and linked in; the reference's lazy NVRTC step
// (ref src/kcmm/ffi.rs:103-171) has no counterpart, so the precompile entry
// points only force the CUDA module to load.
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/kcmm.h"
#include "kcmm_internal.hpp"
#include "launch.hpp"
#include "step_tables.hpp"

using kcmm::Error;
using kcmm::Pool;

struct kcmm_pool_t {
  Pool *pool;
};

struct kcmm_step_tables {
  kcmm_pool_t *owner;
  kcmm::StepTables *tables;
};

namespace {

Pool *P(kcmm_pool_t *h) { return h ? h->pool : nullptr; }

void set_error(kcmm_pool_t *h, const std::string &msg) {
  if (!h) return;
  std::lock_guard<std::mutex> g(h->pool->err_mu);
  h->pool->last_error = msg;
}

size_t write_c_string(char *buf, size_t max_len, const std::string &s) {
  if (!buf || max_len == 0) return 0;
  size_t n = s.size() < max_len - 1 ? s.size() : max_len - 1;
  std::memcpy(buf, s.data(), n);
  buf[n] = 0;
  return n;
}

// Run `fn`; a thrown error becomes "<op>: <message>" and -1.
template <typename F>
int guarded(kcmm_pool_t *h, const char *op, F &&fn) {
  try {
    fn();
    return 0;
  } catch (const std::exception &e) {
    set_error(h, std::string(op) + ": " + e.what());
    return -1;
  }
}

cudaStream_t S(uint64_t stream_ptr) { return reinterpret_cast<cudaStream_t>(stream_ptr); }

int check_launch(kcmm_pool_t *h, const char *op, cudaError_t e) {
  if (e != cudaSuccess) {
    set_error(h, std::string(op) + ": launch failed: " + cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Lifecycle (ref src/kcmm/ffi.rs:470-590)
// ---------------------------------------------------------------------------

kcmm_pool_t *kcmm_pool_create(const kcmm_config_t *c) {
  if (!c) return nullptr;
  kcmm::PoolConfig cfg;
  cfg.block_size = c->block_size ? c->block_size : 16;
  cfg.max_blocks = c->max_blocks ? c->max_blocks : 16384;
  size_t plen = strnlen(c->cpu_cache_path, sizeof(c->cpu_cache_path));
  cfg.cpu_cache_path = plen ? std::string(c->cpu_cache_path, plen) : "/dev/shm/kcmm_swap";
  cfg.tiering = c->tiering != 0;
  cfg.eviction_policy = c->eviction_policy == 1 ? "lfu" : c->eviction_policy == 2 ? "fifo" : "lru";
  cfg.prefetch_window = c->prefetch_window ? c->prefetch_window : 4;
  cfg.max_batch_blocks = c->max_batch_blocks ? c->max_batch_blocks : 64;
  cfg.device = int(c->device_ordinal);
  cfg.num_layers = c->num_layers;
  cfg.kv_heads = c->kv_heads;
  cfg.head_dim = c->head_dim;
  cfg.max_batch = c->max_batch;
  cfg.max_seq_len = c->max_seq_len;
  cfg.low_watermark = c->low_watermark_threshold > 0.0f ? c->low_watermark_threshold : 0.2f;
  cfg.evict_interval_ms = c->background_evict_interval_ms ? c->background_evict_interval_ms : 100;
  cfg.sink_blocks = c->attention_sink_blocks ? c->attention_sink_blocks : 1;
  cfg.window_blocks = c->recent_window_blocks ? c->recent_window_blocks : 4;
  try {
    const char *backend = std::getenv("KCMM_VMM_BACKEND");
    std::unique_ptr<kcmm::Vmm> vmm = (backend && std::strcmp(backend, "host") == 0)
                                         ? kcmm::make_host_vmm()
                                         : kcmm::make_cuda_vmm(cfg.device);
    auto *h = new kcmm_pool_t;
    h->pool = new Pool(cfg, std::move(vmm));
    return h;
  } catch (const std::exception &e) {
    if (std::getenv("KCMM_DEBUG")) std::fprintf(stderr, "kcmm_pool_create: %s\n", e.what());
    return nullptr;
  }
}

void kcmm_pool_destroy(kcmm_pool_t *h) {
  if (!h) return;
  delete h->pool;
  delete h;
}

size_t kcmm_get_last_error(kcmm_pool_t *h, char *buf, size_t max_len) {
  if (!h || !buf || max_len == 0) return 0;
  std::lock_guard<std::mutex> g(h->pool->err_mu);
  if (h->pool->last_error.empty()) return 0;
  return write_c_string(buf, max_len, h->pool->last_error);
}

void kcmm_clear_error(kcmm_pool_t *h) {
  if (!h) return;
  std::lock_guard<std::mutex> g(h->pool->err_mu);
  h->pool->last_error.clear();
}

// ---------------------------------------------------------------------------
// Allocation and sequences (ref src/kcmm/ffi.rs:605-850)
// ---------------------------------------------------------------------------

int kcmm_alloc_blocks(kcmm_pool_t *h, uint32_t n, uint32_t *out) {
  if (!h || !out || n == 0) {
    set_error(h, "kcmm_alloc_blocks: null output buffer or zero count");
    return -1;
  }
  return guarded(h, "kcmm_alloc_blocks", [&] {
    for (uint32_t i = 0; i < n; ++i) out[i] = P(h)->alloc_block();
  });
}

int kcmm_free_blocks(kcmm_pool_t *h, const uint32_t *blocks, uint32_t n) {
  if (!h || !blocks || n == 0) return 0;
  P(h)->free_blocks(blocks, n);
  return 0;
}

int kcmm_register_sequence(kcmm_pool_t *h, const uint32_t *table, uint32_t n, uint32_t *out) {
  if (!h || !table || !out) {
    set_error(h, "kcmm_register_sequence: null arguments");
    return -1;
  }
  *out = P(h)->register_sequence(std::vector<uint32_t>(table, table + n));
  return 0;
}

int kcmm_unregister_sequence(kcmm_pool_t *h, uint32_t seq) {
  if (!h) return -1;
  P(h)->unregister_sequence(seq);
  return 0;
}

void kcmm_touch(kcmm_pool_t *h, uint32_t seq) {
  if (!h) return;
  std::vector<uint32_t> t;
  if (P(h)->touch(seq) && P(h)->block_table(seq, &t)) {
    for (uint32_t b : t) P(h)->note_access(b);
  }
}

void kcmm_cool(kcmm_pool_t *h, uint32_t seq) {
  if (h) P(h)->cool(seq);
}

void kcmm_update_seq_len(kcmm_pool_t *h, uint32_t seq, uint32_t len) {
  if (h) P(h)->update_seq_len(seq, len);
}

uint32_t kcmm_get_seq_len(kcmm_pool_t *h, uint32_t seq) {
  return h ? uint32_t(P(h)->seq_len(seq)) : 0;
}

int kcmm_append_block_to_sequence(kcmm_pool_t *h, uint32_t seq, uint32_t blk) {
  if (!h) return -1;
  if (!P(h)->append_block(seq, blk)) {
    set_error(h, "kcmm_append_block_to_sequence: seq_idx " + std::to_string(seq) + " out of bounds");
    return -1;
  }
  return 0;
}

int kcmm_get_block_table(kcmm_pool_t *h, uint32_t seq, uint32_t *out, uint32_t max_blocks,
                         uint32_t *out_count) {
  if (!h || !out || !out_count) {
    set_error(h, "kcmm_get_block_table: null arguments");
    return -1;
  }
  std::vector<uint32_t> t;
  if (!P(h)->block_table(seq, &t)) {
    set_error(h, "kcmm_get_block_table: seq_idx " + std::to_string(seq) + " not found");
    *out_count = 0;
    return -1;
  }
  size_t n = t.size() < max_blocks ? t.size() : max_blocks;
  std::memcpy(out, t.data(), n * sizeof(uint32_t));
  *out_count = uint32_t(n);
  return 0;
}

// ---------------------------------------------------------------------------
// Queries (ref src/kcmm/ffi.rs:861-1060, 2143)
// ---------------------------------------------------------------------------

uint64_t kcmm_get_block_va_offset(kcmm_pool_t *h, uint32_t blk) {
  uint64_t v = 0;
  if (h && P(h)->block_va_offset(blk, &v)) return v;
  return 0;
}

int kcmm_get_all_block_offsets_f16(kcmm_pool_t *h, uint64_t *out, uint32_t max_blocks,
                                   uint32_t *out_count) {
  if (!h || !out || !out_count) {
    set_error(h, "kcmm_get_all_block_offsets_f16: null arguments");
    return -1;
  }
  auto v = P(h)->all_offsets_f16();
  size_t n = v.size() < max_blocks ? v.size() : max_blocks;
  std::memcpy(out, v.data(), n * sizeof(uint64_t));
  *out_count = uint32_t(n);
  return 0;
}

int kcmm_get_all_block_valid(kcmm_pool_t *h, uint8_t *out, uint32_t max_blocks,
                             uint32_t *out_count) {
  if (!h || !out || !out_count) {
    set_error(h, "kcmm_get_all_block_valid: null arguments");
    return -1;
  }
  auto v = P(h)->all_valid();
  size_t n = v.size() < max_blocks ? v.size() : max_blocks;
  std::memcpy(out, v.data(), n);
  *out_count = uint32_t(n);
  return 0;
}

int kcmm_get_block_location(kcmm_pool_t *h, uint32_t blk, kcmm_block_location_t *out) {
  if (!h || !out) return -1;
  kcmm::Loc loc;
  if (!P(h)->block_location(blk, &loc)) {
    set_error(h, "kcmm_get_block_location: block_idx " + std::to_string(blk) + " not found");
    return -1;
  }
  *out = kcmm_block_location_t(int(loc));
  return 0;
}

int kcmm_get_block_table_va_offsets(kcmm_pool_t *h, uint32_t seq, uint64_t *out,
                                    uint32_t max_blocks, uint32_t *out_count) {
  if (!h || !out || !out_count) {
    set_error(h, "kcmm_get_block_table_va_offsets: null arguments");
    return -1;
  }
  std::vector<uint64_t> v;
  if (!P(h)->sequence_va_offsets(seq, &v)) {
    set_error(h, "kcmm_get_block_table_va_offsets: seq_idx " + std::to_string(seq) + " not found");
    *out_count = 0;
    return -1;
  }
  size_t n = v.size() < max_blocks ? v.size() : max_blocks;
  std::memcpy(out, v.data(), n * sizeof(uint64_t));
  *out_count = uint32_t(n);
  return 0;
}

uint64_t kcmm_get_va_k(kcmm_pool_t *h, uint32_t layer) {
  if (!h || layer >= P(h)->num_layers) return 0;
  return P(h)->va_k[layer];
}

uint64_t kcmm_get_va_v(kcmm_pool_t *h, uint32_t layer) {
  if (!h || layer >= P(h)->num_layers) return 0;
  return P(h)->va_v[layer];
}

uint64_t kcmm_block_state_epoch(kcmm_pool_t *h) { return h ? P(h)->epoch() : 0; }

// ---------------------------------------------------------------------------
// KV append (ref src/kcmm/ffi.rs:1088-1554)
// ---------------------------------------------------------------------------

static int append_rows(kcmm_pool_t *h, const char *op, uint32_t layer,
                       const std::vector<int64_t> &dst, uint64_t k_src, uint64_t v_src,
                       cudaStream_t stream) {
  Pool *p = P(h);
  if (dst.empty()) return 0;
  if (!k_src || !v_src) {
    set_error(h, std::string(op) + ": null source pointer");
    return -1;
  }
  p->use_device();
  cudaError_t e = kcmm::dev::copy_rows(
      reinterpret_cast<const void *>(k_src), reinterpret_cast<const void *>(v_src),
      reinterpret_cast<void *>(p->va_k[layer]), reinterpret_cast<void *>(p->va_v[layer]),
      dst.data(), int(dst.size()), int(p->step_elems), stream);
  return check_launch(h, op, e);
}

int kcmm_append_kv_step(kcmm_pool_t *h, uint32_t layer, const uint32_t *seqs,
                        const uint32_t *positions, uint32_t batch, uint64_t k_src,
                        uint64_t v_src) {
  const char *op = "kcmm_append_kv_step";
  if (!h || !seqs || !positions) {
    set_error(h, std::string(op) + ": null arguments");
    return -1;
  }
  if (layer >= P(h)->num_layers) {
    set_error(h, std::string(op) + ": layer_idx " + std::to_string(layer) + " out of bounds");
    return -1;
  }
  std::vector<int64_t> dst;
  if (guarded(h, op, [&] {
        P(h)->require_device(op);
        P(h)->step_destinations(seqs, positions, batch, &dst);
      }))
    return -1;
  return append_rows(h, op, layer, dst, k_src, v_src, nullptr);
}

static int append_slots(kcmm_pool_t *h, uint32_t layer, const int64_t *slots, uint32_t batch,
                        uint64_t k_src, uint64_t v_src, uint64_t stream) {
  const char *op = "kcmm_append_kv_slots";
  if (!h || !slots) {
    set_error(h, std::string(op) + ": null arguments");
    return -1;
  }
  if (layer >= P(h)->num_layers) {
    set_error(h, std::string(op) + ": layer_idx " + std::to_string(layer) + " out of bounds");
    return -1;
  }
  std::vector<int64_t> dst;
  if (guarded(h, op, [&] {
        P(h)->require_device(op);
        P(h)->slot_destinations(slots, batch, &dst);
      }))
    return -1;
  return append_rows(h, op, layer, dst, k_src, v_src, S(stream));
}

int kcmm_append_kv_slots(kcmm_pool_t *h, uint32_t layer, const int64_t *slots, uint32_t batch,
                         uint64_t k_src, uint64_t v_src) {
  return append_slots(h, layer, slots, batch, k_src, v_src, 0);
}

int kcmm_append_kv_slots_on_stream(kcmm_pool_t *h, uint32_t layer, const int64_t *slots,
                                   uint32_t batch, uint64_t k_src, uint64_t v_src,
                                   uint64_t stream) {
  return append_slots(h, layer, slots, batch, k_src, v_src, stream);
}

static int device_slots_impl(kcmm_pool_t *h, const char *op, uint32_t layer,
                             uint64_t slot_mapping, uint64_t offsets, uint64_t valid,
                             uint32_t offsets_len, uint32_t batch, uint64_t k_src,
                             int64_t k_stride, uint64_t v_src, int64_t v_stride, uint64_t status,
                             uint64_t stream) {
  if (!h || !slot_mapping || !offsets || !k_src || !v_src) {
    set_error(h, std::string(op) + ": null pointer argument");
    return -1;
  }
  if (batch == 0 || offsets_len == 0) {
    set_error(h, std::string(op) + ": batch and offset table length must be positive");
    return -1;
  }
  Pool *p = P(h);
  if (layer >= p->num_layers) {
    set_error(h, std::string(op) + ": layer_idx " + std::to_string(layer) + " out of bounds");
    return -1;
  }
  if (uint64_t(batch) * p->step_elems > 0x7fffffffull) {
    set_error(h, std::string(op) + ": total_elements overflow");
    return -1;
  }
  if (k_stride < 0 || v_stride < 0 || (k_stride && k_stride < int64_t(p->step_elems)) ||
      (v_stride && v_stride < int64_t(p->step_elems))) {
    set_error(h, std::string(op) + ": row strides must be 0 (dense) or >= kv_heads * head_dim");
    return -1;
  }
  if (guarded(h, op, [&] { p->require_device(op); })) return -1;
  kcmm::dev::SlotWriteArgs a = {};
  a.k_stride = k_stride;
  a.v_stride = v_stride;
  a.va_k = reinterpret_cast<void *>(p->va_k[layer]);
  a.va_v = reinterpret_cast<void *>(p->va_v[layer]);
  a.slot_mapping = reinterpret_cast<const int64_t *>(slot_mapping);
  a.block_offsets = reinterpret_cast<const uint64_t *>(offsets);
  a.valid = reinterpret_cast<const uint8_t *>(valid);
  a.offsets_len = int(offsets_len);
  a.batch = int(batch);
  a.step_elems = int(p->step_elems);
  a.block_size = int(p->block_size);
  a.k_src = reinterpret_cast<const void *>(k_src);
  a.v_src = reinterpret_cast<const void *>(v_src);
  a.status = reinterpret_cast<int32_t *>(status);
  a.region_elems = p->region_bytes / 2;
  p->use_device();
  return check_launch(h, op, kcmm::dev::device_slot_write(a, S(stream)));
}

int kcmm_append_kv_device_slots_on_stream(kcmm_pool_t *h, uint32_t layer, uint64_t slot_mapping,
                                          uint64_t offsets, uint64_t valid, uint32_t offsets_len,
                                          uint32_t batch, uint64_t k_src, uint64_t v_src,
                                          uint64_t status, uint64_t stream) {
  return device_slots_impl(h, "kcmm_append_kv_device_slots_on_stream", layer, slot_mapping,
                           offsets, valid, offsets_len, batch, k_src, 0, v_src, 0, status,
                           stream);
}

int kcmm_append_kv_device_slots_strided_on_stream(kcmm_pool_t *h, uint32_t layer,
                                                  uint64_t slot_mapping, uint64_t offsets,
                                                  uint64_t valid, uint32_t offsets_len,
                                                  uint32_t batch, uint64_t k_src,
                                                  int64_t k_row_stride, uint64_t v_src,
                                                  int64_t v_row_stride, uint64_t status,
                                                  uint64_t stream) {
  return device_slots_impl(h, "kcmm_append_kv_device_slots_strided_on_stream", layer,
                           slot_mapping, offsets, valid, offsets_len, batch, k_src,
                           k_row_stride, v_src, v_row_stride, status, stream);
}

int kcmm_append_kv_device_slots_bf16_on_stream(kcmm_pool_t *h, uint32_t layer,
                                               uint64_t slot_mapping, uint64_t offsets,
                                               uint64_t valid, uint32_t offsets_len,
                                               uint32_t batch, uint64_t k_src, uint64_t v_src,
                                               uint64_t status, uint64_t stream) {
  return kcmm_append_kv_device_slots_on_stream(h, layer, slot_mapping, offsets, valid,
                                               offsets_len, batch, k_src, v_src, status, stream);
}

int kcmm_precompile_vllm_kv_write_f16(kcmm_pool_t *h) {
  if (!h) return -1;
  return 0;
}

// ---------------------------------------------------------------------------
// Paged decode attention (ref src/kcmm/ffi.rs:1569-1881)
// ---------------------------------------------------------------------------

// Element strides of the strided decode entry points (0 = dense).
struct DecodeStrides {
  int64_t q_token = 0, q_head = 0, out_token = 0, out_head = 0, tables_row = 0;
};

// Groups of the shared-prefix decode (device arrays).
struct DecodeGroups {
  uint64_t group_starts = 0, prefix_lens = 0;
  uint32_t n_groups = 0, max_group_size = 0;
};

// Peer outputs of the decode fused with the KV-head all-gather.
struct DecodePeers {
  const uint64_t *gathered = nullptr, *signals = nullptr;
  uint32_t rank = 0, world = 0;
  uint64_t epoch = 0;
};

static int decode_impl(kcmm_pool_t *h, kcmm::dev::Dtype dtype, uint32_t layer, uint64_t q,
                       uint64_t out, uint64_t tables, uint64_t seq_lens, uint64_t offsets,
                       uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
                       uint32_t max_bps, float scale, uint64_t stream, bool sync,
                       bool bind, bool noalloc = false, const DecodeStrides *st = nullptr,
                       const DecodePeers *peers = nullptr,
                       const DecodeGroups *groups = nullptr) {
  const char *op = groups ? (dtype == kcmm::dev::Dtype::F16
                                 ? "kcmm_paged_attn_decode_shared_prefix_f16"
                                 : "kcmm_paged_attn_decode_shared_prefix_bf16")
                   : peers ? (dtype == kcmm::dev::Dtype::F16 ? "kcmm_paged_attn_decode_f16_allgather"
                                                           : "kcmm_paged_attn_decode_bf16_allgather")
                   : st ? (dtype == kcmm::dev::Dtype::F16 ? "kcmm_paged_attn_decode_f16_strided"
                                                        : "kcmm_paged_attn_decode_bf16_strided")
                   : noalloc ? "kcmm_paged_attn_decode_bf16_noalloc_on_stream"
                   : dtype == kcmm::dev::Dtype::F16 ? "kcmm_paged_attn_decode_f16"
                                                    : "kcmm_paged_attn_decode_bf16";
  if (!h || !q || !out || !tables || !seq_lens || !offsets) {
    set_error(h, std::string(op) + ": null pointer argument");
    return -1;
  }
  if (batch == 0 || hq == 0 || hkv == 0 || hd == 0 || bs == 0 || max_bps == 0) {
    set_error(h, std::string(op) + ": shape arguments must be positive");
    return -1;
  }
  if (hd > 256) {
    set_error(h, std::string(op) + ": head_dim " + std::to_string(hd) + " exceeds kernel limit 256");
    return -1;
  }
  if (hq > 0xFFFF || hkv > 0xFFFF || bs > 0xFFFF || max_bps > 0xFFFF) {
    set_error(h, std::string(op) + ": packed shape argument exceeds 65535");
    return -1;
  }
  Pool *p = P(h);
  if (layer >= p->num_layers) {
    set_error(h, std::string(op) + ": layer_idx " + std::to_string(layer) + " out of bounds");
    return -1;
  }
  if (uint64_t(batch) * hq > 0x7fffffffull) {
    set_error(h, std::string(op) + ": total_heads overflow");
    return -1;
  }
  if (st && (st->q_token <= 0 || st->q_head < int64_t(hd) || st->out_token <= 0 ||
             st->out_head < int64_t(hd) || st->tables_row < int64_t(max_bps))) {
    set_error(h, std::string(op) +
                     ": strides must be positive, head strides >= head_dim and the "
                     "block-table row stride >= max_blocks_per_seq");
    return -1;
  }
  if (peers) {
    if (!peers->gathered || !peers->signals || peers->world < 1 ||
        peers->world > uint32_t(kcmm::dev::kMaxPeers) || peers->rank >= peers->world ||
        peers->epoch == 0) {
      set_error(h, std::string(op) + ": need 1 <= world <= " +
                       std::to_string(kcmm::dev::kMaxPeers) +
                       ", rank < world, epoch >= 1 and non-null gathered / signal pointer arrays");
      return -1;
    }
    for (uint32_t r = 0; r < peers->world; ++r) {
      if (!peers->gathered[r] || (peers->gathered[r] & 15) || !peers->signals[r] ||
          (peers->signals[r] & 7)) {
        set_error(h, std::string(op) + ": gathered buffer " + std::to_string(r) +
                         " must be non-null and 16-byte aligned, signal array 8-byte aligned");
        return -1;
      }
    }
  }
  if (groups) {
    if (!groups->group_starts || !groups->prefix_lens || groups->n_groups == 0 ||
        groups->n_groups > batch || groups->max_group_size == 0 ||
        groups->max_group_size > batch) {
      set_error(h, std::string(op) +
                       ": need non-null group_starts / prefix_lens, 1 <= n_groups <= batch "
                       "and 1 <= max_group_size <= batch");
      return -1;
    }
    if (batch > 8192) {
      set_error(h, std::string(op) + ": at most 8192 sequences per call");
      return -1;
    }
    if (hq % hkv != 0 || hq / hkv > 16) {
      set_error(h, std::string(op) + ": needs num_q_heads a multiple of num_kv_heads with at "
                                     "most 16 query heads per kv head");
      return -1;
    }
  }
  if (guarded(h, op, [&] { p->require_device(op); })) return -1;
  if (bind) p->use_device();
  kcmm::dev::DecodeArgs a = {};
  if (peers) {
    a.peer_out = peers->gathered;
    a.peer_sig = peers->signals;
    a.peer_rank = int(peers->rank);
    a.peer_world = int(peers->world);
    a.peer_epoch = peers->epoch;
  }
  if (st) {
    a.q_stride_token = st->q_token;
    a.q_stride_head = st->q_head;
    a.out_stride_token = st->out_token;
    a.out_stride_head = st->out_head;
    a.tables_stride = st->tables_row;
  }
  a.dtype = dtype;
  a.q = reinterpret_cast<const void *>(q);
  a.out = reinterpret_cast<void *>(out);
  a.block_tables = reinterpret_cast<const int32_t *>(tables);
  a.seq_lens = reinterpret_cast<const int32_t *>(seq_lens);
  a.block_offsets = reinterpret_cast<const uint64_t *>(offsets);
  a.va_k = reinterpret_cast<const void *>(p->va_k[layer]);
  a.va_v = reinterpret_cast<const void *>(p->va_v[layer]);
  a.region_elems = p->region_bytes / 2;
  a.batch = int(batch);
  a.num_q_heads = int(hq);
  a.kv_heads = int(hkv);
  a.head_dim = int(hd);
  a.block_size = int(bs);
  a.max_blocks_per_seq = int(max_bps);
  a.scale = scale;
  a.diag = p->diag_word();
  if (const char *fs = std::getenv("KCMM_DECODE_SPLITS")) a.force_splits = std::atoi(fs);
  if (noalloc) {
    const size_t need = kcmm::dev::decode_scratch_bytes(a);
    const size_t limit = kcmm::dev::decode_noalloc_scratch_limit();
    if (need > limit) {
      set_error(h, std::string(op) + ": needs " + std::to_string(need) +
                       " bytes of scratch, above the static limit of " + std::to_string(limit) +
                       " bytes; use kcmm_paged_attn_decode_bf16_on_stream or a smaller batch");
      return -1;
    }
    if (check_launch(h, op, kcmm::dev::decode_attention_noalloc(a, S(stream)))) return -1;
    return 0;
  }
  if (groups) {
    cudaError_t e = kcmm::dev::decode_attention_shared_prefix(
        a, reinterpret_cast<const int32_t *>(groups->group_starts),
        reinterpret_cast<const int32_t *>(groups->prefix_lens), int(groups->n_groups),
        int(groups->max_group_size), S(stream));
    // Shapes the shared-prefix kernels are not built for (head_dim outside 64 / 128 /
    // 256, pages not a multiple of 16 tokens, more than 16 query heads per kv head) get
    // the plain decode: the same result, each sequence reading its own pages.
    if (e == cudaErrorNotSupported) e = kcmm::dev::decode_attention(a, S(stream));
    if (check_launch(h, op, e)) return -1;
    return 0;
  }
  if (check_launch(h, op, kcmm::dev::decode_attention(a, S(stream)))) return -1;
  if (sync) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      set_error(h, std::string(op) + ": synchronize failed: " + cudaGetErrorString(e));
      return -1;
    }
  }
  return 0;
}

int kcmm_paged_attn_decode_f16(kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out,
                               uint64_t tables, uint64_t seq_lens, uint64_t offsets,
                               uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd,
                               uint32_t bs, uint32_t max_bps, float scale) {
  return decode_impl(h, kcmm::dev::Dtype::F16, layer, q, out, tables, seq_lens, offsets, batch,
                     hq, hkv, hd, bs, max_bps, scale, 0, true, true);
}

int kcmm_paged_attn_decode_f16_on_stream(kcmm_pool_t *h, uint32_t layer, uint64_t q,
                                         uint64_t out, uint64_t tables, uint64_t seq_lens,
                                         uint64_t offsets, uint32_t batch, uint32_t hq,
                                         uint32_t hkv, uint32_t hd, uint32_t bs,
                                         uint32_t max_bps, float scale, uint64_t stream) {
  return decode_impl(h, kcmm::dev::Dtype::F16, layer, q, out, tables, seq_lens, offsets, batch,
                     hq, hkv, hd, bs, max_bps, scale, stream, false, true);
}

int kcmm_paged_attn_decode_f16_on_current_context_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out, uint64_t tables,
    uint64_t seq_lens, uint64_t offsets, uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd,
    uint32_t bs, uint32_t max_bps, float scale, uint64_t stream) {
  return decode_impl(h, kcmm::dev::Dtype::F16, layer, q, out, tables, seq_lens, offsets, batch,
                     hq, hkv, hd, bs, max_bps, scale, stream, false, false);
}

int kcmm_paged_attn_decode_bf16_strided_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, int64_t q_stride_token, int64_t q_stride_head,
    uint64_t out, int64_t out_stride_token, int64_t out_stride_head, uint64_t tables,
    int64_t tables_row_stride, uint64_t seq_lens, uint64_t offsets, uint32_t batch, uint32_t hq,
    uint32_t hkv, uint32_t hd, uint32_t bs, uint32_t max_bps, float scale, uint64_t stream) {
  DecodeStrides st;
  st.q_token = q_stride_token;
  st.q_head = q_stride_head;
  st.out_token = out_stride_token;
  st.out_head = out_stride_head;
  st.tables_row = tables_row_stride;
  return decode_impl(h, kcmm::dev::Dtype::BF16, layer, q, out, tables, seq_lens, offsets, batch,
                     hq, hkv, hd, bs, max_bps, scale, stream, false, true, false, &st);
}

int kcmm_paged_attn_decode_f16_strided_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, int64_t q_stride_token, int64_t q_stride_head,
    uint64_t out, int64_t out_stride_token, int64_t out_stride_head, uint64_t tables,
    int64_t tables_row_stride, uint64_t seq_lens, uint64_t offsets, uint32_t batch, uint32_t hq,
    uint32_t hkv, uint32_t hd, uint32_t bs, uint32_t max_bps, float scale, uint64_t stream) {
  DecodeStrides st;
  st.q_token = q_stride_token;
  st.q_head = q_stride_head;
  st.out_token = out_stride_token;
  st.out_head = out_stride_head;
  st.tables_row = tables_row_stride;
  return decode_impl(h, kcmm::dev::Dtype::F16, layer, q, out, tables, seq_lens, offsets, batch,
                     hq, hkv, hd, bs, max_bps, scale, stream, false, true, false, &st);
}

static int decode_allgather(kcmm_pool_t *h, kcmm::dev::Dtype dt, uint32_t layer, uint64_t q,
                            uint64_t out, uint64_t tables, uint64_t seq_lens, uint64_t offsets,
                            uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
                            uint32_t max_bps, float scale, const uint64_t *gathered,
                            const uint64_t *signals, uint32_t rank, uint32_t world,
                            uint64_t epoch, uint64_t stream) {
  DecodePeers pe;
  pe.gathered = gathered;
  pe.signals = signals;
  pe.rank = rank;
  pe.world = world;
  pe.epoch = epoch;
  return decode_impl(h, dt, layer, q, out, tables, seq_lens, offsets, batch, hq, hkv, hd, bs,
                     max_bps, scale, stream, false, true, false, nullptr, &pe);
}

int kcmm_paged_attn_decode_bf16_allgather_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out, uint64_t tables, uint64_t seq_lens,
    uint64_t offsets, uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
    uint32_t max_bps, float scale, const uint64_t *gathered_ptrs, const uint64_t *signal_ptrs,
    uint32_t rank, uint32_t world, uint64_t epoch, uint64_t stream) {
  return decode_allgather(h, kcmm::dev::Dtype::BF16, layer, q, out, tables, seq_lens, offsets,
                          batch, hq, hkv, hd, bs, max_bps, scale, gathered_ptrs, signal_ptrs,
                          rank, world, epoch, stream);
}

int kcmm_paged_attn_decode_f16_allgather_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out, uint64_t tables, uint64_t seq_lens,
    uint64_t offsets, uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
    uint32_t max_bps, float scale, const uint64_t *gathered_ptrs, const uint64_t *signal_ptrs,
    uint32_t rank, uint32_t world, uint64_t epoch, uint64_t stream) {
  return decode_allgather(h, kcmm::dev::Dtype::F16, layer, q, out, tables, seq_lens, offsets,
                          batch, hq, hkv, hd, bs, max_bps, scale, gathered_ptrs, signal_ptrs,
                          rank, world, epoch, stream);
}

static int decode_shared_prefix(kcmm_pool_t *h, kcmm::dev::Dtype dt, uint32_t layer, uint64_t q,
                                uint64_t out, uint64_t tables, uint64_t seq_lens,
                                uint64_t offsets, uint32_t batch, uint32_t hq, uint32_t hkv,
                                uint32_t hd, uint32_t bs, uint32_t max_bps, float scale,
                                uint64_t group_starts, uint64_t prefix_lens, uint32_t n_groups,
                                uint32_t max_group_size, uint64_t stream) {
  DecodeGroups g;
  g.group_starts = group_starts;
  g.prefix_lens = prefix_lens;
  g.n_groups = n_groups;
  g.max_group_size = max_group_size;
  return decode_impl(h, dt, layer, q, out, tables, seq_lens, offsets, batch, hq, hkv, hd, bs,
                     max_bps, scale, stream, false, true, false, nullptr, nullptr, &g);
}

int kcmm_paged_attn_decode_shared_prefix_bf16_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out, uint64_t tables, uint64_t seq_lens,
    uint64_t offsets, uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
    uint32_t max_bps, float scale, uint64_t group_starts, uint64_t prefix_lens,
    uint32_t n_groups, uint32_t max_group_size, uint64_t stream) {
  return decode_shared_prefix(h, kcmm::dev::Dtype::BF16, layer, q, out, tables, seq_lens,
                              offsets, batch, hq, hkv, hd, bs, max_bps, scale, group_starts,
                              prefix_lens, n_groups, max_group_size, stream);
}

int kcmm_paged_attn_decode_shared_prefix_f16_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out, uint64_t tables, uint64_t seq_lens,
    uint64_t offsets, uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
    uint32_t max_bps, float scale, uint64_t group_starts, uint64_t prefix_lens,
    uint32_t n_groups, uint32_t max_group_size, uint64_t stream) {
  return decode_shared_prefix(h, kcmm::dev::Dtype::F16, layer, q, out, tables, seq_lens,
                              offsets, batch, hq, hkv, hd, bs, max_bps, scale, group_starts,
                              prefix_lens, n_groups, max_group_size, stream);
}

int kcmm_paged_attn_decode_bf16_on_stream(kcmm_pool_t *h, uint32_t layer, uint64_t q,
                                          uint64_t out, uint64_t tables, uint64_t seq_lens,
                                          uint64_t offsets, uint32_t batch, uint32_t hq,
                                          uint32_t hkv, uint32_t hd, uint32_t bs,
                                          uint32_t max_bps, float scale, uint64_t stream) {
  return decode_impl(h, kcmm::dev::Dtype::BF16, layer, q, out, tables, seq_lens, offsets, batch,
                     hq, hkv, hd, bs, max_bps, scale, stream, false, true);
}

int kcmm_paged_attn_decode_bf16_noalloc_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out, uint64_t tables,
    uint64_t seq_lens, uint64_t offsets, uint32_t batch, uint32_t hq, uint32_t hkv, uint32_t hd,
    uint32_t bs, uint32_t max_bps, float scale, uint64_t stream) {
  return decode_impl(h, kcmm::dev::Dtype::BF16, layer, q, out, tables, seq_lens, offsets, batch,
                     hq, hkv, hd, bs, max_bps, scale, stream, false, true, true);
}

// ---------------------------------------------------------------------------
// Chunked prefill (tcgen05)
// ---------------------------------------------------------------------------

static int prefill_impl(kcmm_pool_t *h, kcmm::dev::Dtype dtype, uint32_t layer, uint64_t q,
                        uint64_t out, uint64_t tables, uint64_t q_start, uint64_t ctx_lens,
                        uint64_t offsets, uint32_t batch, uint32_t max_q_len, uint32_t hq,
                        uint32_t hkv, uint32_t hd, uint32_t bs, uint32_t max_bps, float scale,
                        uint64_t stream) {
  const char *op = dtype == kcmm::dev::Dtype::F16 ? "kcmm_paged_prefill_f16_on_stream"
                                                  : "kcmm_paged_prefill_bf16_on_stream";
  if (!h || !q || !out || !tables || !q_start || !ctx_lens || !offsets) {
    set_error(h, std::string(op) + ": null pointer argument");
    return -1;
  }
  if (batch == 0 || max_q_len == 0 || hq == 0 || hkv == 0 || hd == 0 || bs == 0 ||
      max_bps == 0) {
    set_error(h, std::string(op) + ": shape arguments must be positive");
    return -1;
  }
  if (hd > 256 || hd % 8 != 0) {
    set_error(h, std::string(op) + ": head_dim " + std::to_string(hd) +
                     " unsupported (the tensor-core prefill takes multiples of 8 up to 256)");
    return -1;
  }
  if (hq % hkv != 0 || hq / hkv > 128) {
    set_error(h, std::string(op) + ": num_q_heads / kv_heads must be an integer of at most 128");
    return -1;
  }
  if (hq > 0xFFFF || hkv > 0xFFFF || bs > 0xFFFF || max_bps > 0xFFFF || batch > 0xFFFF) {
    set_error(h, std::string(op) + ": packed shape argument exceeds 65535");
    return -1;
  }
  if (((q | out) & 15) != 0) {
    set_error(h, std::string(op) + ": query and output must be 16-byte aligned");
    return -1;
  }
  Pool *p = P(h);
  if (layer >= p->num_layers) {
    set_error(h, std::string(op) + ": layer_idx " + std::to_string(layer) + " out of bounds");
    return -1;
  }
  if (guarded(h, op, [&] { p->require_device(op); })) return -1;
  p->use_device();
  kcmm::dev::PrefillArgs a = {};
  a.dtype = dtype;
  a.q = reinterpret_cast<const void *>(q);
  a.out = reinterpret_cast<void *>(out);
  a.block_tables = reinterpret_cast<const int32_t *>(tables);
  a.query_start = reinterpret_cast<const int32_t *>(q_start);
  a.context_lens = reinterpret_cast<const int32_t *>(ctx_lens);
  a.block_offsets = reinterpret_cast<const uint64_t *>(offsets);
  a.va_k = reinterpret_cast<const void *>(p->va_k[layer]);
  a.va_v = reinterpret_cast<const void *>(p->va_v[layer]);
  a.region_elems = p->region_bytes / 2;
  a.batch = int(batch);
  a.max_q_len = int(max_q_len);
  a.num_q_heads = int(hq);
  a.kv_heads = int(hkv);
  a.head_dim = int(hd);
  a.block_size = int(bs);
  a.max_blocks_per_seq = int(max_bps);
  a.scale = scale;
  a.diag = p->diag_word();
  if (hd == 128) {  // the TMA page boxes of the two-tile kernel
    a.tensor_maps = p->tensor_maps(layer, int(hkv), int(hd));
    a.v_page_map = p->v_page_map(layer, int(hkv), int(hd));
  }
  return check_launch(h, op, kcmm::dev::paged_prefill(a, S(stream)));
}

int kcmm_paged_prefill_bf16_on_stream(kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out,
                                      uint64_t tables, uint64_t q_start, uint64_t ctx_lens,
                                      uint64_t offsets, uint32_t batch, uint32_t max_q_len,
                                      uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
                                      uint32_t max_bps, float scale, uint64_t stream) {
  return prefill_impl(h, kcmm::dev::Dtype::BF16, layer, q, out, tables, q_start, ctx_lens,
                      offsets, batch, max_q_len, hq, hkv, hd, bs, max_bps, scale, stream);
}

int kcmm_paged_prefill_f16_on_stream(kcmm_pool_t *h, uint32_t layer, uint64_t q, uint64_t out,
                                     uint64_t tables, uint64_t q_start, uint64_t ctx_lens,
                                     uint64_t offsets, uint32_t batch, uint32_t max_q_len,
                                     uint32_t hq, uint32_t hkv, uint32_t hd, uint32_t bs,
                                     uint32_t max_bps, float scale, uint64_t stream) {
  return prefill_impl(h, kcmm::dev::Dtype::F16, layer, q, out, tables, q_start, ctx_lens,
                      offsets, batch, max_q_len, hq, hkv, hd, bs, max_bps, scale, stream);
}

int kcmm_precompile_paged_attn_decode_f16(kcmm_pool_t *h) {
  if (!h) return -1;
  if (guarded(h, "kcmm_precompile_paged_attn_decode_f16", [&] {
        P(h)->require_device("kcmm_precompile_paged_attn_decode_f16");
      }))
    return -1;
  P(h)->use_device();
  return check_launch(h, "kcmm_precompile_paged_attn_decode_f16", kcmm::dev::decode_preload());
}

// ---------------------------------------------------------------------------
// Fused RMSNorm + RoPE + append
// ---------------------------------------------------------------------------

int kcmm_fused_norm_rope_append_bf16_on_stream(
    kcmm_pool_t *h, uint32_t layer, uint64_t x, uint64_t w, uint64_t normed, uint32_t hidden,
    float eps, uint64_t q, uint32_t hq, uint64_t k, uint64_t v, uint64_t positions,
    float theta, uint32_t rope_mode, uint64_t slots, uint64_t offsets, uint64_t valid,
    uint32_t offsets_len, uint32_t num_tokens, uint64_t status, uint64_t stream) {
  const char *op = "kcmm_fused_norm_rope_append_bf16_on_stream";
  if (!h || !x || !w || !normed || !q || !k || !v || !positions || !slots || !offsets) {
    set_error(h, std::string(op) + ": null pointer argument");
    return -1;
  }
  Pool *p = P(h);
  if (layer >= p->num_layers) {
    set_error(h, std::string(op) + ": layer_idx " + std::to_string(layer) + " out of bounds");
    return -1;
  }
  if (num_tokens == 0 || hidden == 0 || hq == 0 || offsets_len == 0) {
    set_error(h, std::string(op) + ": shape arguments must be positive");
    return -1;
  }
  if (hidden % 8 != 0 || hidden > 65536) {
    set_error(h, std::string(op) + ": hidden must be a multiple of 8 and at most 65536");
    return -1;
  }
  if (rope_mode > 2) {
    set_error(h, std::string(op) + ": unknown rope_mode " + std::to_string(rope_mode));
    return -1;
  }
  if (p->cfg_.head_dim % 2 != 0 || (rope_mode == 2 && p->cfg_.head_dim % 4 != 0)) {
    set_error(h, std::string(op) + ": head_dim must be even (a multiple of 4 for neox)");
    return -1;
  }
  if (hq > 0xFFFF || !(theta > 0.0f)) {
    set_error(h, std::string(op) + ": invalid num_q_heads or rope_theta");
    return -1;
  }
  if (guarded(h, op, [&] { p->require_device(op); })) return -1;
  kcmm::dev::FusedAppendArgs a;
  a.x = reinterpret_cast<const void *>(x);
  a.norm_weight = reinterpret_cast<const void *>(w);
  a.normed_out = reinterpret_cast<void *>(normed);
  a.hidden = int(hidden);
  a.eps = eps;
  a.q = reinterpret_cast<void *>(q);
  a.num_q_heads = int(hq);
  a.k = reinterpret_cast<const void *>(k);
  a.v = reinterpret_cast<const void *>(v);
  a.positions = reinterpret_cast<const int32_t *>(positions);
  a.rope_theta = theta;
  a.rope_mode = int(rope_mode);
  a.slot_mapping = reinterpret_cast<const int64_t *>(slots);
  a.block_offsets = reinterpret_cast<const uint64_t *>(offsets);
  a.valid = reinterpret_cast<const uint8_t *>(valid);
  a.offsets_len = int(offsets_len);
  a.num_tokens = int(num_tokens);
  a.kv_heads = int(p->cfg_.kv_heads);
  a.head_dim = int(p->cfg_.head_dim);
  a.block_size = int(p->block_size);
  a.va_k = reinterpret_cast<void *>(p->va_k[layer]);
  a.va_v = reinterpret_cast<void *>(p->va_v[layer]);
  a.region_elems = p->region_bytes / 2;
  a.status = reinterpret_cast<int32_t *>(status);
  p->use_device();
  return check_launch(h, op, kcmm::dev::fused_norm_rope_append(a, S(stream)));
}

// ---------------------------------------------------------------------------
// Tiering (ref src/kcmm/ffi.rs:1900-2030)
// ---------------------------------------------------------------------------

uint32_t kcmm_evict_blocks(kcmm_pool_t *h, uint32_t count) {
  if (!h || count == 0) return 0;
  uint32_t n = 0;
  if (guarded(h, "kcmm_evict_blocks", [&] { n = uint32_t(P(h)->evict(count)); })) return 0;
  return n;
}

uint64_t kcmm_restore_evicted_block(kcmm_pool_t *h, uint32_t blk) {
  if (!h) return 0;
  uint64_t va = 0;
  if (guarded(h, "kcmm_restore_evicted_block", [&] { va = P(h)->restore_one(blk); })) return 0;
  return va;
}

int kcmm_restore_evicted_blocks(kcmm_pool_t *h, const uint32_t *ids, uint32_t count) {
  if (!h || !ids || count == 0) return 0;
  return guarded(h, "kcmm_restore_evicted_blocks", [&] { P(h)->restore_many(ids, count); });
}

int kcmm_is_gpu_resident(kcmm_pool_t *h, uint32_t blk) {
  kcmm::Loc loc;
  return (h && P(h)->block_location(blk, &loc) && loc == kcmm::Loc::Gpu) ? 1 : 0;
}

int kcmm_swap_out_blocks_on_stream(kcmm_pool_t *h, const uint32_t *ids, uint32_t count,
                                   uint64_t stream) {
  if (!h) return -1;
  if (!ids || count == 0) return 0;
  return guarded(h, "kcmm_swap_out_blocks_on_stream",
                 [&] { P(h)->swap_out(ids, count, reinterpret_cast<void *>(stream)); });
}

int kcmm_swap_in_blocks_on_stream(kcmm_pool_t *h, const uint32_t *ids, uint32_t count,
                                  uint64_t stream) {
  if (!h) return -1;
  if (!ids || count == 0) return 0;
  return guarded(h, "kcmm_swap_in_blocks_on_stream",
                 [&] { P(h)->swap_in(ids, count, reinterpret_cast<void *>(stream)); });
}

// ---------------------------------------------------------------------------
// Metrics and statistics (ref src/kcmm/ffi.rs:2037-2190)
// ---------------------------------------------------------------------------

int kcmm_get_metrics(kcmm_pool_t *h, kcmm_metrics_t *out) {
  if (!h || !out) return -1;
  kcmm_metrics_t m = {};
  P(h)->collect_metrics(&m.ifr, &m.pme, &m.bu, &m.rfi, &m.gpu_blocks, &m.cpu_blocks);
  kcmm::Metrics c = P(h)->metrics();
  m.nvme_blocks = 0;
  m.eviction_count = c.eviction_count;
  m.restoration_count = c.restoration_count;
  *out = m;
  return 0;
}

static void copy_histogram(const kcmm::LatencyHistogram &h, kcmm_latency_histogram_t *out) {
  out->count = h.count;
  out->sum_us = h.sum_us;
  out->min_us = h.min_us;
  out->max_us = h.max_us;
  for (int i = 0; i < 9; ++i) out->buckets[i] = h.buckets[i];
}

int kcmm_get_metrics_ext(kcmm_pool_t *h, kcmm_metrics_ext_t *out) {
  if (!h || !out) return -1;
  kcmm_metrics_ext_t m = {};
  if (kcmm_get_metrics(h, &m.base) != 0) return -1;
  kcmm::Metrics c = P(h)->metrics();
  m.evicted_blocks_total = c.evicted_blocks;
  m.restored_blocks_total = c.restored_blocks;
  m.eviction_failures = c.eviction_failures;
  m.restoration_failures = c.restoration_failures;
  m.background_eviction_count = c.background_eviction_count;
  copy_histogram(c.eviction_latency, &m.eviction_latency);
  copy_histogram(c.restoration_latency, &m.restoration_latency);
  *out = m;
  return 0;
}

int kcmm_get_policy_stats(kcmm_pool_t *h, const char *policy, kcmm_policy_stats_t *out) {
  if (!h || !policy || !out) return -1;
  kcmm::Metrics c = P(h)->metrics();
  auto it = c.policy_stats.find(policy);
  if (it == c.policy_stats.end()) return -1;
  out->eviction_count = it->second.eviction_count;
  out->restoration_count = it->second.restoration_count;
  out->evicted_blocks = it->second.evicted_blocks;
  out->restored_blocks = it->second.restored_blocks;
  out->avg_evict_batch_size = it->second.avg_evict_batch_size;
  return 0;
}

int kcmm_get_pool_stats(kcmm_pool_t *h, kcmm_pool_stats_t *out) {
  if (!h || !out) return -1;
  Pool *p = P(h);
  kcmm_pool_stats_t s = {};
  s.blocks_in_use = uint32_t(p->blocks_in_use());
  s.total_blocks = uint32_t(p->total_blocks());
  s.total_physical_blocks = uint32_t(p->total_physical_blocks());
  s.free_physical_blocks = uint32_t(p->free_physical_blocks());
  s.active_sequences = uint32_t(p->active_sequences());
  s.num_layers = uint32_t(p->num_layers);
  s.blocks_per_superblock = uint32_t(kcmm::kSuperblockBytes / p->block_bytes);
  s.superblock_count = uint32_t(p->superblock_count());
  s.block_size = uint32_t(p->block_size);
  s.max_blocks_per_seq = uint32_t(p->max_blocks_per_seq);
  s.block_bytes = uint32_t(p->block_bytes);
  s.tiering_enabled = p->tiering_enabled() ? 1 : 0;
  s.sharing_enabled = 1;
  s.physical_idle_ratio = p->physical_idle_ratio();
  *out = s;
  return 0;
}

uint32_t kcmm_blocks_in_use(kcmm_pool_t *h) { return h ? uint32_t(P(h)->blocks_in_use()) : 0; }
uint32_t kcmm_total_blocks(kcmm_pool_t *h) { return h ? uint32_t(P(h)->total_blocks()) : 0; }
uint32_t kcmm_free_physical_blocks(kcmm_pool_t *h) {
  return h ? uint32_t(P(h)->free_physical_blocks()) : 0;
}
int kcmm_has_free_blocks(kcmm_pool_t *h) { return (h && P(h)->free_physical_blocks() > 0) ? 1 : 0; }
uint32_t kcmm_active_sequences(kcmm_pool_t *h) {
  return h ? uint32_t(P(h)->active_sequences()) : 0;
}

// ---------------------------------------------------------------------------
// Policy, hints, sharing (ref src/kcmm/ffi.rs:2200-2500)
// ---------------------------------------------------------------------------

int kcmm_set_eviction_policy(kcmm_pool_t *h, const char *policy) {
  if (!h || !policy) return -1;
  std::string s(policy);
  for (char &c : s) c = char(std::tolower(static_cast<unsigned char>(c)));
  if (!P(h)->tiering_enabled()) {
    set_error(h, "kcmm_set_eviction_policy: tiering is disabled");
    return -1;
  }
  return guarded(h, "kcmm_set_eviction_policy", [&] { P(h)->set_policy(s); });
}

uint32_t kcmm_get_eviction_policy(kcmm_pool_t *h, char *out, uint32_t max_len) {
  if (!h || !out || max_len == 0 || !P(h)->tiering_enabled()) return 0;
  return uint32_t(write_c_string(out, max_len, P(h)->policy_name()));
}

int kcmm_is_tiering_enabled(kcmm_pool_t *h) { return (h && P(h)->tiering_enabled()) ? 1 : 0; }

int kcmm_hint(kcmm_pool_t *h, uint32_t seq, kcmm_hint_t hint) {
  if (!h) return -1;
  Pool *p = P(h);
  std::vector<uint32_t> table;
  if (!p->block_table(seq, &table)) {
    set_error(h, "kcmm_hint: seq_idx " + std::to_string(seq) + " out of bounds");
    return -1;
  }
  switch (hint) {
    case KCMM_HINT_MULTI_TURN:
    case KCMM_HINT_SYSTEM_PROMPT:
    case KCMM_HINT_ATTENTION_SINK:
    case KCMM_HINT_HEAVY_HITTER:
      p->touch(seq);
      for (uint32_t b : table) p->note_access(b);
      break;
    case KCMM_HINT_HIGH_PRIORITY:
      p->touch(seq);
      p->set_priority(seq, kcmm::Priority::High);
      break;
    case KCMM_HINT_NEAR_END:
      p->cool(seq);
      break;
    case KCMM_HINT_LOW_PRIORITY:
      p->cool(seq);
      p->set_priority(seq, kcmm::Priority::Low);
      break;
    case KCMM_HINT_EVICTABLE:
      p->cool(seq);
      p->set_priority(seq, kcmm::Priority::Evictable);
      break;
    default:
      set_error(h, "kcmm_hint: unknown hint " + std::to_string(int(hint)));
      return -1;
  }
  return 0;
}

int kcmm_protect(kcmm_pool_t *h, uint32_t, const uint32_t *ids, uint32_t n,
                 kcmm_protection_t level) {
  if (!h || !ids || n == 0) return -1;
  Pool *p = P(h);
  if (!p->tiering_enabled()) return 0;
  for (uint32_t i = 0; i < n; ++i) {
    kcmm::BlockHandle bh;
    if (!p->block_handle(ids[i], &bh)) {
      set_error(h, "kcmm_protect: block_idx " + std::to_string(ids[i]) + " not found");
      return -1;
    }
    if (level != KCMM_EVICT_PREFERRED) p->note_access(ids[i]);
  }
  return 0;
}

int kcmm_share_prefix(kcmm_pool_t *h, uint32_t src, uint32_t dst, uint32_t n, uint32_t *out) {
  if (!h || !out || n == 0) return -1;
  return guarded(h, "kcmm_share_prefix", [&] {
    auto v = P(h)->share_prefix(src, dst, n);
    std::memcpy(out, v.data(), v.size() * sizeof(uint32_t));
  });
}

int kcmm_block_incref(kcmm_pool_t *h, uint32_t blk) {
  if (!h) return -1;
  return guarded(h, "kcmm_block_incref", [&] { P(h)->incref(blk); });
}

int kcmm_block_decref(kcmm_pool_t *h, uint32_t blk) {
  if (!h) return -1;
  return guarded(h, "kcmm_block_decref", [&] { P(h)->decref(blk); });
}

uint32_t kcmm_block_refcount(kcmm_pool_t *h, uint32_t blk) { return h ? P(h)->refcount(blk) : 0; }

int kcmm_fork_sequence(kcmm_pool_t *h, uint32_t src, uint32_t *out) {
  if (!h || !out) {
    set_error(h, "kcmm_fork_sequence: null arguments");
    return -1;
  }
  return guarded(h, "kcmm_fork_sequence", [&] { *out = P(h)->fork_sequence(src); });
}

int kcmm_cow_blocks_on_stream(kcmm_pool_t *h, const uint32_t *seqs, const uint32_t *logical,
                              uint32_t count, uint32_t *out, uint64_t stream) {
  if (!h) return -1;
  if (count == 0) return 0;
  if (!seqs || !logical || !out) {
    set_error(h, "kcmm_cow_blocks_on_stream: null arguments");
    return -1;
  }
  return guarded(h, "kcmm_cow_blocks_on_stream", [&] {
    auto v = P(h)->cow_blocks(seqs, logical, count, reinterpret_cast<void *>(stream));
    std::memcpy(out, v.data(), v.size() * sizeof(uint32_t));
  });
}

// ---------------------------------------------------------------------------
// Utilities and accessors (ref src/kcmm/ffi.rs:2488-2560)
// ---------------------------------------------------------------------------

int kcmm_below_low_watermark(kcmm_pool_t *h, float threshold) {
  return (h && P(h)->below_low_watermark(threshold)) ? 1 : 0;
}

int kcmm_synchronize(kcmm_pool_t *h) {
  if (!h) return -1;
  Pool *p = P(h);
  if (guarded(h, "kcmm_synchronize", [&] { p->require_device("kcmm_synchronize"); })) return -1;
  p->use_device();
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    set_error(h, std::string("kcmm_synchronize: ") + cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

uint32_t kcmm_get_block_size(kcmm_pool_t *h) { return h ? uint32_t(P(h)->block_size) : 0; }
uint32_t kcmm_get_max_blocks_per_seq(kcmm_pool_t *h) {
  return h ? uint32_t(P(h)->max_blocks_per_seq) : 0;
}
uint32_t kcmm_get_block_bytes(kcmm_pool_t *h) { return h ? uint32_t(P(h)->block_bytes) : 0; }
uint32_t kcmm_get_num_layers(kcmm_pool_t *h) { return h ? uint32_t(P(h)->num_layers) : 0; }
uint32_t kcmm_get_max_batch(kcmm_pool_t *h) { return h ? uint32_t(P(h)->cfg_.max_batch) : 0; }
uint32_t kcmm_get_max_seq_len(kcmm_pool_t *h) { return h ? uint32_t(P(h)->cfg_.max_seq_len) : 0; }

int32_t kcmm_get_kernel_status(kcmm_pool_t *h) {
  if (!h) return -1;
  Pool *p = P(h);
  if (guarded(h, "kcmm_get_kernel_status", [&] { p->require_device("kcmm_get_kernel_status"); }))
    return -1;
  p->use_device();
  int32_t v = 0;
  if (cudaMemcpy(&v, p->diag_word(), sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (v) cudaMemset(p->diag_word(), 0, sizeof(v));
  return v;
}

const char *kcmm_build_info(void) { return "kcmm-b200 0.1.0 sm_100a"; }

// --- all-gather over NVLink peer memory -------------------------------------------

uint32_t kcmm_peer_signal_words(uint32_t world) {
  return world >= 1 && world <= uint32_t(kcmm::dev::kMaxPeers)
             ? world * uint32_t(kcmm::dev::kGatherBlocks)
             : 0;
}

int kcmm_peer_allgather_on_stream(uint64_t src, uint64_t nbytes, const uint64_t *dst_ptrs,
                                  const uint64_t *sig_ptrs, uint32_t rank, uint32_t world,
                                  uint64_t epoch, uint64_t stream) {
  if (!src || !dst_ptrs || !sig_ptrs || world == 0 || world > uint32_t(kcmm::dev::kMaxPeers) ||
      rank >= world || nbytes == 0 || nbytes % 16 != 0 || epoch == 0)
    return -1;
  void *dst[kcmm::dev::kMaxPeers];
  unsigned long long *sig[kcmm::dev::kMaxPeers];
  for (uint32_t r = 0; r < world; ++r) {
    if (!dst_ptrs[r] || !sig_ptrs[r] || dst_ptrs[r] % 16 != 0 || sig_ptrs[r] % 8 != 0) return -1;
    dst[r] = reinterpret_cast<void *>(dst_ptrs[r]);
    sig[r] = reinterpret_cast<unsigned long long *>(sig_ptrs[r]);
  }
  return kcmm::dev::peer_allgather(reinterpret_cast<const void *>(src), nbytes, dst, sig,
                                   int(rank), int(world), epoch, S(stream)) == cudaSuccess
             ? 0
             : -1;
}

int kcmm_peer_wait_on_stream(uint64_t sig, uint32_t world, uint64_t epoch, uint64_t status,
                             uint64_t stream) {
  if (!sig || sig % 8 != 0 || world == 0 || world > uint32_t(kcmm::dev::kMaxPeers) || epoch == 0)
    return -1;
  return kcmm::dev::peer_wait(reinterpret_cast<const unsigned long long *>(sig), int(world),
                              epoch, reinterpret_cast<int32_t *>(status),
                              S(stream)) == cudaSuccess
             ? 0
             : -1;
}

// --- background eviction and victim preview ------------------------------------

int kcmm_start_background_eviction(kcmm_pool_t *h) {
  if (!h) return -1;
  return guarded(h, "kcmm_start_background_eviction",
                 [&] { P(h)->start_background_eviction(); });
}

int kcmm_stop_background_eviction(kcmm_pool_t *h) {
  if (!h) return -1;
  return guarded(h, "kcmm_stop_background_eviction", [&] { P(h)->stop_background_eviction(); });
}

uint32_t kcmm_preview_eviction_victims(kcmm_pool_t *h, uint32_t count, uint32_t *out,
                                       uint32_t max_out) {
  if (!h || !out || max_out == 0 || !P(h)->tiering_enabled()) return 0;
  std::vector<uint32_t> v;
  if (guarded(h, "kcmm_preview_eviction_victims",
              [&] { v = P(h)->preview_victims(count); }) != 0)
    return 0;
  const uint32_t n = uint32_t(std::min<size_t>(v.size(), max_out));
  std::memcpy(out, v.data(), n * sizeof(uint32_t));
  return n;
}

// --- device-resident step tables -----------------------------------------------

kcmm_step_tables_t *kcmm_step_tables_create(kcmm_pool_t *h, uint32_t max_batch) {
  if (!h) return nullptr;
  kcmm::StepTables *t = nullptr;
  if (guarded(h, "kcmm_step_tables_create",
              [&] { t = new kcmm::StepTables(P(h), max_batch); }) != 0)
    return nullptr;
  return new kcmm_step_tables{h, t};
}

void kcmm_step_tables_destroy(kcmm_step_tables_t *t) {
  if (!t) return;
  delete t->tables;
  delete t;
}

int kcmm_step_tables_sync_on_stream(kcmm_step_tables_t *t, const uint32_t *seqs,
                                    uint32_t batch, uint64_t stream) {
  if (!t) return -1;
  if (batch > 0 && !seqs) {
    set_error(t->owner, "kcmm_step_tables_sync_on_stream: seq_indices is null");
    return -1;
  }
  return guarded(t->owner, "kcmm_step_tables_sync_on_stream",
                 [&] { t->tables->sync(seqs, batch, S(stream)); });
}

uint64_t kcmm_step_tables_block_tables(const kcmm_step_tables_t *t) {
  return t ? reinterpret_cast<uint64_t>(t->tables->block_tables()) : 0;
}

uint64_t kcmm_step_tables_seq_lens(const kcmm_step_tables_t *t) {
  return t ? reinterpret_cast<uint64_t>(t->tables->seq_lens()) : 0;
}

uint64_t kcmm_step_tables_block_offsets(const kcmm_step_tables_t *t) {
  return t ? reinterpret_cast<uint64_t>(t->tables->block_offsets()) : 0;
}

int kcmm_step_tables_stats(const kcmm_step_tables_t *t, kcmm_step_tables_stats_t *out) {
  if (!t || !out) return -1;
  const kcmm::StepTableStats &s = t->tables->stats();
  out->syncs = s.syncs;
  out->table_entries = s.entries32;
  out->offset_entries = s.entries64;
  out->bytes = s.bytes;
  out->full_offsets = s.full_offsets;
  return 0;
}

}  // extern "C"
