// Device-resident step tables (step_tables.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "kcmm_internal.hpp"

namespace kcmm {

struct StepTableStats {
  uint64_t syncs = 0, entries32 = 0, entries64 = 0, bytes = 0, full_offsets = 0;
};

class StepTables {
 public:
  StepTables(Pool *pool, size_t max_batch);
  ~StepTables();
  StepTables(const StepTables &) = delete;
  StepTables &operator=(const StepTables &) = delete;

  // Bring rows [0, batch) up to date for sequences seqs[0..batch), and the
  // offsets array for every block of the pool.  Syncs of one object must be
  // ordered on the device (one stream, or events between streams).
  void sync(const uint32_t *seqs, size_t batch, cudaStream_t stream);

  Pool *pool() const { return pool_; }
  int32_t *block_tables() const { return d_i32_; }
  int32_t *seq_lens() const { return d_i32_ + st_.max_batch * pool_->max_blocks_per_seq; }
  uint64_t *block_offsets() const { return d_off_; }
  size_t max_batch() const { return st_.max_batch; }
  const StepTableStats &stats() const { return stats_; }

 private:
  void release();
  Pool *pool_;
  StepTableState st_;
  TableUpdates up_;
  StepTableStats stats_;
  int32_t *d_i32_ = nullptr;  // [max_batch x max_blocks_per_seq tables | max_batch lens]
  size_t i32_len_ = 0;
  uint64_t *d_off_ = nullptr;
  size_t off_cap_ = 0;
  void *h_stage_[2] = {nullptr, nullptr};
  void *d_stage_[2] = {nullptr, nullptr};
  size_t stage_cap_[2] = {0, 0};
  cudaEvent_t done_[2] = {nullptr, nullptr};
};

}  // namespace kcmm
