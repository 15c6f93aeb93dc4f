/*
 * TEST INFRASTRUCTURE -- the reference's own CUDA kernels, compiled as host
 * C++ from their sources (which stay under the reference tree; nothing is
 * copied), with a small executor for grid/block indices and __syncthreads.
 * Built by oracle/Makefile into oracle/_ref/libref_kernels.so; used by the
 * tests to pin the oracle, and by bench.py as the reference arm (the
 * reference's path timed on the host cores).
 *
 * Kernels included (paths in the reference project):
 *   src/cuda/kernels/kcmm_vllm_paged_attn.cu  kcmm_vllm_paged_attn_decode_f16
 *   src/cuda/kernels/paged_attn_decode.cu     paged_attn_decode_f16 (engine; D <= 64)
 *   src/cuda/kernels/kcmm_vllm_kv_write.cu    kcmm_vllm_kv_write_slots_f16
 *   src/cuda/kernels/rms_norm.cu              rms_norm_f16
 *   src/cuda/kernels/rope.cu                  rope_f16
 *   src/cuda/kernels/kv_gather.cu             gather_kv_layer / scatter_kv_layer
 * With KCMM_SHIM_BF16 the same attention source is built over bfloat16 storage
 * (exported as ref_paged_attn_bf16) for the bf16 CPU baseline, and with
 * KCMM_SHIM_F32 over fp32 storage (ref_paged_attn_f32) for the fp32 CPU toy.
 * Those two builds carry only the attention kernel; the executor's globals
 * come from the default build.
 */
#include <ucontext.h>

#include <algorithm>
#include <atomic>
#include <functional>
#include <thread>
#include <vector>

#include "cuda_fp16.h"

#if defined(KCMM_SHIM_BF16) || defined(KCMM_SHIM_F32)
#define KCMM_SHIM_ALT 1
#endif

#ifndef KCMM_SHIM_ALT
thread_local kcmm_shim_dim3 blockIdx, threadIdx, blockDim, gridDim;
#endif

namespace {

// ---- executor --------------------------------------------------------------

struct FiberSched {
  ucontext_t main_ctx;
  std::vector<ucontext_t> ctx;
  std::vector<std::vector<char>> stacks;
  std::vector<char> done;
  unsigned current = 0;
  const std::function<void()> *body = nullptr;
};
thread_local FiberSched *g_sched = nullptr;

void fiber_entry() {
  FiberSched *s = g_sched;
  (*s->body)();
  s->done[s->current] = 1;
  swapcontext(&s->ctx[s->current], &s->main_ctx);
}

// Run one CTA of `threads` threads with barrier support.
void run_cta_fibers(unsigned threads, const std::function<void()> &body) {
  static thread_local FiberSched sched;
  FiberSched &s = sched;
  g_sched = &s;
  s.body = &body;
  if (s.ctx.size() < threads) {
    s.ctx.resize(threads);
    s.stacks.resize(threads);
  }
  s.done.assign(threads, 0);
  for (unsigned t = 0; t < threads; ++t) {
    s.stacks[t].resize(256 * 1024);
    getcontext(&s.ctx[t]);
    s.ctx[t].uc_stack.ss_sp = s.stacks[t].data();
    s.ctx[t].uc_stack.ss_size = s.stacks[t].size();
    s.ctx[t].uc_link = &s.main_ctx;
    makecontext(&s.ctx[t], fiber_entry, 0);
  }
  bool pending = true;
  while (pending) {
    pending = false;
    for (unsigned t = 0; t < threads; ++t) {
      if (s.done[t]) continue;
      s.current = t;
      threadIdx.x = t;
      swapcontext(&s.main_ctx, &s.ctx[t]);
      if (!s.done[t]) pending = true;
    }
  }
  g_sched = nullptr;
}

// Launch grid x block; CTAs spread over `workers` OS threads.
void launch(unsigned grid, unsigned block, int workers, bool barriers,
            const std::function<void()> &body) {
  std::atomic<unsigned> next{0};
  auto worker = [&] {
    blockDim.x = block;
    gridDim.x = grid;
    for (;;) {
      unsigned b = next.fetch_add(1);
      if (b >= grid) break;
      blockIdx.x = b;
      if (barriers) {
        run_cta_fibers(block, body);
      } else {
        for (unsigned t = 0; t < block; ++t) {
          threadIdx.x = t;
          body();
        }
      }
    }
  };
  workers = std::max(1, workers);
  if (workers == 1) {
    worker();
    return;
  }
  std::vector<std::thread> pool;
  for (int i = 0; i < workers; ++i) pool.emplace_back(worker);
  for (auto &t : pool) t.join();
}

}  // namespace

#ifndef KCMM_SHIM_ALT
void __syncthreads() {
  FiberSched *s = g_sched;
  if (!s) return;
  swapcontext(&s->ctx[s->current], &s->main_ctx);
  threadIdx.x = s->current;
}
#endif

// ---- the reference kernels -------------------------------------------------

#ifdef KCMM_SHIM_BF16
#define kcmm_vllm_paged_attn_decode_f16 ref_body_attn_bf16
#include "kcmm_vllm_paged_attn.cu"
#undef kcmm_vllm_paged_attn_decode_f16
#elif defined(KCMM_SHIM_F32)
#define kcmm_vllm_paged_attn_decode_f16 ref_body_attn_f32
#include "kcmm_vllm_paged_attn.cu"
#undef kcmm_vllm_paged_attn_decode_f16
#else
#include "kcmm_vllm_paged_attn.cu"
#include "paged_attn_decode.cu"
#include "kcmm_vllm_kv_write.cu"
// dynamic shared memory of rms_norm_f16 (`extern __shared__ float shared[]`):
// one buffer per OS thread, i.e. per CTA being executed
thread_local float shared[4096];
#include "rms_norm.cu"
#include "rope.cu"
#include "kv_gather.cu"
#endif

using u64 = unsigned long long;

extern "C" {

#ifdef KCMM_SHIM_BF16
void ref_paged_attn_bf16(const uint16_t *q, const uint16_t *va_k, const uint16_t *va_v,
                         const int32_t *tables, const int32_t *seq_lens, const uint64_t *offsets,
                         uint16_t *out, int batch, int hq, int hkv, int d, int bs, int max_bps,
                         float scale, int workers) {
  const int total = batch * hq;
  const int packed_heads = (hkv << 16) | hq;
  const int packed_blocks = (max_bps << 16) | bs;
  launch((total + 127) / 128, 128, workers, false, [&] {
    ref_body_attn_bf16(u64(q), u64(va_k), u64(va_v), u64(tables), u64(seq_lens), u64(offsets),
                       u64(out), total, packed_heads, d, packed_blocks, scale);
  });
}
#elif defined(KCMM_SHIM_F32)
// block_offsets_f16 is read as an element index into the float regions
void ref_paged_attn_f32(const float *q, const float *va_k, const float *va_v,
                        const int32_t *tables, const int32_t *seq_lens, const uint64_t *offsets,
                        float *out, int batch, int hq, int hkv, int d, int bs, int max_bps,
                        float scale, int workers) {
  const int total = batch * hq;
  const int packed_heads = (hkv << 16) | hq;
  const int packed_blocks = (max_bps << 16) | bs;
  launch((total + 127) / 128, 128, workers, false, [&] {
    ref_body_attn_f32(u64(q), u64(va_k), u64(va_v), u64(tables), u64(seq_lens), u64(offsets),
                      u64(out), total, packed_heads, d, packed_blocks, scale);
  });
}
#else
// launch shape of ref src/kcmm/ffi.rs:1812-1818 (128 threads, 1 per (b, q head))
void ref_paged_attn_f16(const uint16_t *q, const uint16_t *va_k, const uint16_t *va_v,
                        const int32_t *tables, const int32_t *seq_lens, const uint64_t *offsets,
                        uint16_t *out, int batch, int hq, int hkv, int d, int bs, int max_bps,
                        float scale, int workers) {
  const int total = batch * hq;
  const int packed_heads = (hkv << 16) | hq;
  const int packed_blocks = (max_bps << 16) | bs;
  launch((total + 127) / 128, 128, workers, false, [&] {
    kcmm_vllm_paged_attn_decode_f16(u64(q), u64(va_k), u64(va_v), u64(tables), u64(seq_lens),
                                    u64(offsets), u64(out), total, packed_heads, d,
                                    packed_blocks, scale);
  });
}

// engine kernel (ref src/cuda/kernels/mod.rs:183-211); head_dim <= 64 only
void ref_paged_attn_engine_f16(const uint16_t *q, const uint16_t *va_k, const uint16_t *va_v,
                               const int32_t *tables, const int32_t *seq_lens,
                               const uint64_t *offsets, uint16_t *out, int batch, int hq,
                               int hkv, int d, int bs, int max_bps, int workers) {
  const int total = batch * hq;
  const int packed = (max_bps << 16) | bs;
  launch((total + 127) / 128, 128, workers, false, [&] {
    paged_attn_decode_f16(reinterpret_cast<const __half *>(q),
                          reinterpret_cast<const __half *>(va_k),
                          reinterpret_cast<const __half *>(va_v), tables, seq_lens,
                          reinterpret_cast<const unsigned long long *>(offsets),
                          reinterpret_cast<__half *>(out), total, hq, hkv, d, packed);
  });
}

// launch shape of ref src/kcmm/ffi.rs:1502-1508 (one thread per element)
void ref_kv_write_slots_f16(uint16_t *va_k, uint16_t *va_v, const int64_t *slots,
                            const uint64_t *offsets, const uint8_t *valid, const uint16_t *k_src,
                            const uint16_t *v_src, int32_t *status, int batch, int step, int bs,
                            int offsets_len) {
  const int total = batch * step;
  launch((total + 255) / 256, 256, 1, false, [&] {
    kcmm_vllm_kv_write_slots_f16(u64(va_k), u64(va_v), u64(slots), u64(offsets), u64(valid),
                                 u64(k_src), u64(v_src), u64(status), total, step, bs,
                                 offsets_len);
  });
}

// launch shape of ref src/cuda/kernels/mod.rs:76-91 (256 threads, 1 KiB smem)
void ref_rms_norm_f16(const uint16_t *x, const uint16_t *w, uint16_t *y, int rows, int cols,
                      float eps, int workers) {
  launch(rows, 256, workers, true, [&] {
    rms_norm_f16(reinterpret_cast<const __half *>(x), reinterpret_cast<const __half *>(w),
                 reinterpret_cast<__half *>(y), rows, cols, eps);
  });
}

// ref src/cuda/kernels/mod.rs:93-111: one position for the whole launch
void ref_rope_f16(uint16_t *q, uint16_t *k, int batch, int hq, int hkv, int half_dim, int pos) {
  const int n = std::max(batch * hq * half_dim, batch * hkv * half_dim);
  launch((n + 1023) / 1024, 1024, 1, false, [&] {
    rope_f16(reinterpret_cast<__half *>(q), reinterpret_cast<__half *>(k), batch, hq, hkv,
             half_dim, pos);
  });
}

void ref_gather_kv(const uint64_t *src_ptrs, uint16_t *dst, int half_count, int num_blocks) {
  const int n = half_count * num_blocks;
  launch((n + 255) / 256, 256, 1, false, [&] {
    gather_kv_layer(reinterpret_cast<const unsigned long long *>(src_ptrs),
                    reinterpret_cast<__half *>(dst), half_count, num_blocks);
  });
}

void ref_scatter_kv(const uint16_t *src, const uint64_t *dst_ptrs, int half_count,
                    int num_blocks) {
  const int n = half_count * num_blocks;
  launch((n + 255) / 256, 256, 1, false, [&] {
    scatter_kv_layer(reinterpret_cast<const __half *>(src),
                     reinterpret_cast<const unsigned long long *>(dst_ptrs), half_count,
                     num_blocks);
  });
}
#endif

}  // extern "C"
