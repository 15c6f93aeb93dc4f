/*
 * TEST INFRASTRUCTURE -- host stand-ins for the few CUDA built-ins that the
 * reference's kernel sources use, so that those sources compile unchanged
 * as host C++ (oracle/ref_host.cpp).  Only oracle/_ref is built with it.
 *
 *   __half            16-bit storage; IEEE binary16 by default, bfloat16
 *                     when KCMM_SHIM_BF16 is defined (bf16 timing builds),
 *                     and a plain float when KCMM_SHIM_F32 is defined (the
 *                     fp32 CPU toy: the kernels index elements through
 *                     `__half *`, so the same source then runs on fp32 data).
 *   blockIdx/...      per-OS-thread launch coordinates set by the executor.
 *   __syncthreads     a barrier implemented with ucontext fibers.
 */
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

struct kcmm_shim_dim3 {
  unsigned x = 0, y = 0, z = 0;
};
extern thread_local kcmm_shim_dim3 blockIdx, threadIdx, blockDim, gridDim;

#define __global__
#define __device__
#define __forceinline__ inline
#define __shared__ thread_local

#ifdef KCMM_SHIM_F32
struct __half {
  float v;
};
static inline float __half2float(__half h) { return h.v; }
static inline __half __float2half(float f) { return __half{f}; }
#elif defined(KCMM_SHIM_BF16)
struct __half {
  uint16_t bits;
};
static inline float __half2float(__half h) {
  uint32_t u = uint32_t(h.bits) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
static inline __half __float2half(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return __half{uint16_t(u >> 16)};
}
#else
struct __half {
  uint16_t bits;
};
static inline float __half2float(__half h) {
  _Float16 v;
  std::memcpy(&v, &h.bits, 2);
  return float(v);
}
static inline __half __float2half(float f) {
  _Float16 v = _Float16(f);
  __half h;
  std::memcpy(&h.bits, &v, 2);
  return h;
}
#endif

static inline float rsqrtf(float x) { return 1.0f / std::sqrt(x); }

// Single-threaded per CTA (fibers of one CTA run on one OS thread), so a
// plain read-modify-write is atomic here.
static inline int atomicCAS(int *addr, int compare, int val) {
  int old = *addr;
  if (old == compare) *addr = val;
  return old;
}

void __syncthreads();
