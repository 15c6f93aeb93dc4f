// Device-resident step tables: the block tables, sequence lengths and block
// offsets a decode step reads, kept on the device between steps and brought up
// to date by the entries that changed.
//
// The reference rebuilds all three on the host every step and copies the
// tables and lengths to the device once per layer
// (src/model/llama_transformer.rs:277-303 and :338-339; the offsets through
// get_all_block_offsets_f16, src/kcmm/pool.rs:724-735).  Here a sync compares
// the pool with what the device holds:
//   * a row whose sequence changed, or whose table was rewritten (fork, copy-on-
//     write, unregister), is written whole, with zeros past the table as in the
//     reference's build; a row that only grew gets its new tail entries;
//   * a length is written when it differs;
//   * offsets entries are written for the blocks the pool logged since the last
//     sync (install, release, swap-in), or all of them on the first sync, after
//     the array grew, or when the log was trimmed past this reader.
// The changes travel as one packed list (one host-to-device copy from pinned
// memory) and one scatter kernel applies them, both on the caller's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "kcmm_internal.hpp"
#include "launch.hpp"
#include "step_tables.hpp"

namespace kcmm {

void Pool::step_table_updates(const uint32_t *seqs, size_t batch, StepTableState *st,
                              TableUpdates *up) {
  std::lock_guard<std::mutex> g(mu_);
  up->idx32.clear();
  up->val32.clear();
  up->idx64.clear();
  up->val64.clear();
  const size_t mbps = max_blocks_per_seq;
  const size_t len_base = st->max_batch * mbps;
  for (size_t b = 0; b < batch; ++b) {
    if (seqs[b] >= seqs_.size()) {
      throw Error("seq_idx " + std::to_string(seqs[b]) + " out of bounds");
    }
  }
  for (size_t b = 0; b < batch; ++b) {
    const Sequence &q = seqs_[seqs[b]];
    const uint32_t n = uint32_t(std::min(q.table.size(), mbps));
    const bool same = st->row_seq[b] == int64_t(seqs[b]);
    uint32_t from = 0;
    if (same && st->row_rewrite[b] == q.rewrite) {
      from = st->row_version[b] == q.version ? n : std::min(st->row_blocks[b], n);
    }
    for (uint32_t j = from; j < n; ++j) {
      up->idx32.push_back(uint32_t(b * mbps + j));
      up->val32.push_back(int32_t(q.table[j]));
    }
    for (uint32_t j = std::max(n, from); j < st->row_blocks[b]; ++j) {  // zeros past the table
      up->idx32.push_back(uint32_t(b * mbps + j));
      up->val32.push_back(0);
    }
    st->row_seq[b] = int64_t(seqs[b]);
    st->row_version[b] = q.version;
    st->row_rewrite[b] = q.rewrite;
    st->row_blocks[b] = n;
    const int32_t len = int32_t(q.seq_len);
    if (st->row_len[b] != len || !same) {
      up->idx32.push_back(uint32_t(len_base + b));
      up->val32.push_back(len);
      st->row_len[b] = len;
    }
  }
  const size_t total = blocks_.size();
  up->offsets_needed = total;
  const uint64_t log_end = block_log_base_ + block_log_.size();
  up->offsets_full = !st->offsets_init || st->log_cursor < block_log_base_;
  auto entry = [&](size_t i) { return blocks_[i].in_use ? blocks_[i].va_offset / 2 : 0; };
  if (up->offsets_full) {
    for (size_t i = 0; i < total; ++i) {
      up->idx64.push_back(uint32_t(i));
      up->val64.push_back(entry(i));
    }
  } else {
    for (uint64_t k = st->log_cursor; k < log_end; ++k) {
      const uint32_t blk = block_log_[size_t(k - block_log_base_)];
      up->idx64.push_back(blk);
      up->val64.push_back(entry(blk));
    }
  }
  st->log_cursor = log_end;
  st->offsets_len = total;
  st->offsets_init = true;
}

StepTables::StepTables(Pool *pool, size_t max_batch) : pool_(pool) {
  if (max_batch == 0 || max_batch > 65535) throw Error("max_batch must be in [1, 65535]");
  pool_->require_device("kcmm_step_tables_create");
  pool_->use_device();
  st_.max_batch = max_batch;
  st_.row_seq.assign(max_batch, -1);
  st_.row_version.assign(max_batch, 0);
  st_.row_rewrite.assign(max_batch, 0);
  st_.row_blocks.assign(max_batch, 0);
  st_.row_len.assign(max_batch, 0);
  i32_len_ = max_batch * pool_->max_blocks_per_seq + max_batch;
  if (cudaMalloc(&d_i32_, i32_len_ * sizeof(int32_t)) != cudaSuccess ||
      cudaMemset(d_i32_, 0, i32_len_ * sizeof(int32_t)) != cudaSuccess) {
    cudaGetLastError();
    release();
    throw Error("step tables: device allocation failed");
  }
  for (auto &e : done_) {
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      release();
      throw Error("step tables: event creation failed");
    }
  }
}

StepTables::~StepTables() { release(); }

void StepTables::release() {
  pool_->use_device();
  cudaDeviceSynchronize();  // nothing in flight reads what is freed below
  if (d_i32_) cudaFree(d_i32_);
  if (d_off_) cudaFree(d_off_);
  for (int i = 0; i < 2; ++i) {
    if (d_stage_[i]) cudaFree(d_stage_[i]);
    if (h_stage_[i]) cudaFreeHost(h_stage_[i]);
    if (done_[i]) cudaEventDestroy(done_[i]);
    d_stage_[i] = nullptr;
    h_stage_[i] = nullptr;
    done_[i] = nullptr;
  }
  d_i32_ = nullptr;
  d_off_ = nullptr;
}

void StepTables::sync(const uint32_t *seqs, size_t batch, cudaStream_t stream) {
  if (batch > st_.max_batch) {
    throw Error("batch " + std::to_string(batch) + " exceeds the tables' max_batch " +
                std::to_string(st_.max_batch));
  }
  pool_->use_device();
  StepTableState next = st_;
  pool_->step_table_updates(seqs, batch, &next, &up_);
  // the offsets array grows in stream order; a grown array is written whole
  if (up_.offsets_needed > off_cap_) {
    size_t cap = std::max<size_t>(up_.offsets_needed + up_.offsets_needed / 2, 1024);
    uint64_t *fresh = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&fresh), cap * 8, stream);
    if (e != cudaSuccess) throw Error(std::string("step tables: ") + cudaGetErrorString(e));
    if (d_off_) cudaFreeAsync(d_off_, stream);
    d_off_ = fresh;
    off_cap_ = cap;
    if (!up_.offsets_full) {
      next.offsets_init = false;  // list every entry instead of the logged ones
      StepTableState again = st_;
      again.offsets_init = false;
      pool_->step_table_updates(seqs, batch, &again, &up_);
      next = again;
    }
  }
  const size_t n32 = up_.idx32.size(), n64 = up_.idx64.size();
  stats_.syncs += 1;
  if (n32 == 0 && n64 == 0) {
    st_ = next;
    return;
  }
  // [idx32 n32][val32 n32][idx64 n64][pad to 8][val64 n64]
  size_t off64 = (n32 * 8 + n64 * 4 + 7) / 8 * 8;
  const size_t bytes = off64 + n64 * 8;
  const int slot = int(stats_.syncs & 1);
  if (cudaEventSynchronize(done_[slot]) != cudaSuccess) {  // host buffer free again
    cudaGetLastError();
  }
  if (bytes > stage_cap_[slot]) {
    const size_t cap = std::max<size_t>(bytes + bytes / 2, 4096);
    if (h_stage_[slot]) cudaFreeHost(h_stage_[slot]);
    if (d_stage_[slot]) cudaFreeAsync(d_stage_[slot], stream);
    h_stage_[slot] = nullptr;
    d_stage_[slot] = nullptr;
    stage_cap_[slot] = 0;
    if (cudaMallocHost(&h_stage_[slot], cap) != cudaSuccess ||
        cudaMallocAsync(&d_stage_[slot], cap, stream) != cudaSuccess) {
      cudaGetLastError();
      throw Error("step tables: staging allocation failed");
    }
    stage_cap_[slot] = cap;
  }
  unsigned char *h = static_cast<unsigned char *>(h_stage_[slot]);
  std::memcpy(h, up_.idx32.data(), n32 * 4);
  std::memcpy(h + n32 * 4, up_.val32.data(), n32 * 4);
  std::memcpy(h + n32 * 8, up_.idx64.data(), n64 * 4);
  std::memcpy(h + off64, up_.val64.data(), n64 * 8);
  cudaError_t e = cudaMemcpyAsync(d_stage_[slot], h, bytes, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaEventRecord(done_[slot], stream);
  if (e == cudaSuccess)
    e = dev::apply_table_updates(d_stage_[slot], int(n32), int(n64), off64, d_i32_, d_off_,
                                 stream);
  if (e != cudaSuccess) throw Error(std::string("step tables: ") + cudaGetErrorString(e));
  st_ = next;
  stats_.entries32 += n32;
  stats_.entries64 += n64;
  stats_.bytes += bytes;
  if (up_.offsets_full) stats_.full_offsets += 1;
}

}  // namespace kcmm
