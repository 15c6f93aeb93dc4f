// KV append kernels for sm_100a: host-addressed row copies, the
// device-slot write (vLLM reshape_and_cache) and the fused
// RMSNorm + RoPE + append.
//
// All three move 16-bit words without converting them (bf16 and f16 share
// the kernels) and use 16-byte accesses whenever source, destination and row
// length allow it; a row that does not qualify falls back to 2-byte accesses
// instead of faulting.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <cmath>

#include "../launch.hpp"
#include "pdl.cuh"
#include "ptx.cuh"

namespace kcmm {
namespace dev {
namespace {

constexpr int kRowsPerLaunch = 480;  // keeps the parameter block under 4 KB

struct RowCopyParams {
  const uint16_t *k_src;
  const uint16_t *v_src;
  uint16_t *va_k;
  uint16_t *va_v;
  int rows;
  int row_elems;
  int row_base;  // index of the first row of this launch in k_src/v_src
  int64_t dst[kRowsPerLaunch];
};

// One CTA per row; restates the per-row cuMemcpyDtoDAsync pair of
// ref src/kcmm/ffi.rs:1168-1186 as one launch.
__global__ void copy_rows_kernel(const RowCopyParams p) {
  const int r = blockIdx.x;
  const int64_t dst = p.dst[r];
  if (dst < 0) return;
  const int64_t src = int64_t(p.row_base + r) * p.row_elems;
  const uint16_t *ks = p.k_src + src;
  const uint16_t *vs = p.v_src + src;
  uint16_t *kd = p.va_k + dst;
  uint16_t *vd = p.va_v + dst;
  const bool vec = ((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs) |
                     reinterpret_cast<uintptr_t>(kd) | reinterpret_cast<uintptr_t>(vd)) &
                    15) == 0 &&
                   (p.row_elems & 7) == 0;
  if (vec) {
    for (int c = threadIdx.x; c < p.row_elems / 8; c += blockDim.x) {
      reinterpret_cast<uint4 *>(kd)[c] = reinterpret_cast<const uint4 *>(ks)[c];
      reinterpret_cast<uint4 *>(vd)[c] = reinterpret_cast<const uint4 *>(vs)[c];
    }
  } else {
    for (int c = threadIdx.x; c < p.row_elems; c += blockDim.x) {
      kd[c] = ks[c];
      vd[c] = vs[c];
    }
  }
}

// Device-slot write: one CTA per token row.  Status semantics follow
// ref src/cuda/kernels/kcmm_vllm_kv_write.cu:37-56 (first error wins):
// 1 = block id outside the offsets table, 2 = block marked free, and, as an
// addition, 3 = offset outside the layer region (the reference would fault).
__global__ void slot_write_kernel(const SlotWriteArgs a) {
  const int row = blockIdx.x;
  __shared__ int64_t s_dst;
  if (threadIdx.x == 0) {
    int64_t dst = -1;
    const int64_t slot = a.slot_mapping[row];
    if (slot >= 0) {
      const int64_t blk = slot / a.block_size;
      // both lookups in flight together when the block id is in range
      const bool in_range = blk < a.offsets_len;
      const uint8_t live = in_range && a.valid ? a.valid[blk] : uint8_t(1);
      const uint64_t off = in_range ? a.block_offsets[blk] : 0;
      if (!in_range) {
        if (a.status) atomicCAS(a.status, 0, 1);
      } else if (live == 0) {
        if (a.status) atomicCAS(a.status, 0, 2);
      } else {
        const int64_t d = int64_t(off) + (slot % a.block_size) * a.step_elems;
        if (uint64_t(d) + uint64_t(a.step_elems) > a.region_elems) {
          if (a.status) atomicCAS(a.status, 0, 3);
        } else {
          dst = d;
        }
      }
    }
    s_dst = dst;
  }
  __syncthreads();
  const int64_t dst = s_dst;
  if (dst < 0) return;
  const uint16_t *ks = static_cast<const uint16_t *>(a.k_src) +
                       int64_t(row) * (a.k_stride ? a.k_stride : a.step_elems);
  const uint16_t *vs = static_cast<const uint16_t *>(a.v_src) +
                       int64_t(row) * (a.v_stride ? a.v_stride : a.step_elems);
  uint16_t *kd = static_cast<uint16_t *>(a.va_k) + dst;
  uint16_t *vd = static_cast<uint16_t *>(a.va_v) + dst;
  const bool vec = ((reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs) |
                     reinterpret_cast<uintptr_t>(kd) | reinterpret_cast<uintptr_t>(vd)) &
                    15) == 0 &&
                   (a.step_elems & 7) == 0;
  if (vec) {
    for (int c = threadIdx.x; c < a.step_elems / 8; c += blockDim.x) {
      reinterpret_cast<uint4 *>(kd)[c] = reinterpret_cast<const uint4 *>(ks)[c];
      reinterpret_cast<uint4 *>(vd)[c] = reinterpret_cast<const uint4 *>(vs)[c];
    }
  } else {
    for (int c = threadIdx.x; c < a.step_elems; c += blockDim.x) {
      kd[c] = ks[c];
      vd[c] = vs[c];
    }
  }
}

// ---------------------------------------------------------------------------
// Fused RMSNorm + RoPE + KV append (bf16), one CTA per token.
// ---------------------------------------------------------------------------

constexpr int kFusedThreads = 256;

__device__ __forceinline__ float bf(uint16_t v) {
  return __uint_as_float(uint32_t(v) << 16);
}
__device__ __forceinline__ uint16_t to_bf(float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t *>(&h);
}

struct Vec8 {
  uint16_t e[8];
};
__device__ __forceinline__ Vec8 load8(const uint16_t *p, bool vec) {
  Vec8 v;
  if (vec) {
    *reinterpret_cast<uint4 *>(v.e) = *reinterpret_cast<const uint4 *>(p);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v.e[i] = p[i];
  }
  return v;
}
__device__ __forceinline__ void store8(uint16_t *p, const Vec8 &v, bool vec) {
  if (vec) {
    *reinterpret_cast<uint4 *>(p) = *reinterpret_cast<const uint4 *>(v.e);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = v.e[i];
  }
}

// Rotate `heads` rows of head_dim elements at src into dst (dst may equal src).
// cs/sn hold cos/sin per pair frequency (head_dim/2 entries).
__device__ __forceinline__ void rope_rows(const uint16_t *src, uint16_t *dst, int heads, int D,
                                          int mode, const float *cs, const float *sn,
                                          bool vec) {
  const int half = D / 2;
  if (mode != 2) {
    // interleaved pairs (2i, 2i+1) of each head
    const int chunks = heads * D / 8;
    if ((D & 7) == 0) {
      for (int c = threadIdx.x; c < chunks; c += kFusedThreads) {
        const int e0 = c * 8, d0 = e0 % D;
        Vec8 v = load8(src + e0, vec);
        Vec8 o;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = d0 / 2 + j;
          const float x0 = bf(v.e[2 * j]), x1 = bf(v.e[2 * j + 1]);
          o.e[2 * j] = to_bf(x0 * cs[i] - x1 * sn[i]);
          o.e[2 * j + 1] = to_bf(x0 * sn[i] + x1 * cs[i]);
        }
        store8(dst + e0, o, vec);
      }
    } else {
      for (int pi = threadIdx.x; pi < heads * half; pi += kFusedThreads) {
        const int h = pi / half, i = pi % half;
        const int e = h * D + 2 * i;
        const float x0 = bf(src[e]), x1 = bf(src[e + 1]);
        dst[e] = to_bf(x0 * cs[i] - x1 * sn[i]);
        dst[e + 1] = to_bf(x0 * sn[i] + x1 * cs[i]);
      }
    }
  } else {
    // half-split pairs (i, i + D/2)
    if ((half & 7) == 0) {
      const int per_head = half / 8;
      for (int c = threadIdx.x; c < heads * per_head; c += kFusedThreads) {
        const int h = c / per_head, i0 = (c % per_head) * 8;
        const uint16_t *s = src + h * D;
        uint16_t *d = dst + h * D;
        Vec8 a = load8(s + i0, vec), b = load8(s + i0 + half, vec);
        Vec8 oa, ob;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + j;
          const float x0 = bf(a.e[j]), x1 = bf(b.e[j]);
          oa.e[j] = to_bf(x0 * cs[i] - x1 * sn[i]);
          ob.e[j] = to_bf(x0 * sn[i] + x1 * cs[i]);
        }
        store8(d + i0, oa, vec);
        store8(d + i0 + half, ob, vec);
      }
    } else {
      for (int pi = threadIdx.x; pi < heads * half; pi += kFusedThreads) {
        const int h = pi / half, i = pi % half;
        const int e = h * D + i;
        const float x0 = bf(src[e]), x1 = bf(src[e + half]);
        dst[e] = to_bf(x0 * cs[i] - x1 * sn[i]);
        dst[e + half] = to_bf(x0 * sn[i] + x1 * cs[i]);
      }
    }
  }
}

__global__ void __launch_bounds__(kFusedThreads) fused_kernel(const FusedAppendArgs a) {
  extern __shared__ float fsm[];  // cs[D/2], sn[D/2]
  __shared__ float red[kFusedThreads / 32];
  __shared__ int64_t s_dst;
  ptx::grid_dependency_wait();  // a programmatic dependent: see pdl.cuh
  ptx::launch_dependents();
  const int t = blockIdx.x;
  const int D = a.head_dim, half = D / 2;
  float *cs = fsm;
  float *sn = fsm + half;

  // Slot resolution (thread 0) -- same rules as the device-slot write.
  if (threadIdx.x == 0) {
    int64_t dst = -1;
    const int64_t slot = a.slot_mapping[t];
    const int step = a.kv_heads * D;
    if (slot >= 0) {
      const int64_t blk = slot / a.block_size;
      if (blk >= a.offsets_len) {
        if (a.status) atomicCAS(a.status, 0, 1);
      } else if (a.valid && a.valid[blk] == 0) {
        if (a.status) atomicCAS(a.status, 0, 2);
      } else {
        const int64_t d = int64_t(a.block_offsets[blk]) + (slot % a.block_size) * step;
        if (uint64_t(d) + uint64_t(step) > a.region_elems) {
          if (a.status) atomicCAS(a.status, 0, 3);
        } else {
          dst = d;
        }
      }
    }
    s_dst = dst;
  }

  // Rotary table for this token's position (ref src/cuda/kernels/rope.cu:18,
  // with the base as a parameter): theta_i = 1 / base^e_i.
  const float pos = float(a.positions[t]);
  for (int i = threadIdx.x; i < half; i += kFusedThreads) {
    const float e = a.rope_mode == 0 ? float(2 * (i / 2)) / float(D) : float(2 * i) / float(D);
    const float theta = 1.0f / powf(a.rope_theta, e);
    float s, c;
    sincosf(pos * theta, &s, &c);
    cs[i] = c;
    sn[i] = s;
  }

  // RMSNorm (ref src/cuda/kernels/rms_norm.cu:14-35): out = ((x * inv_rms) * w)
  const int H = a.hidden;
  const uint16_t *x = static_cast<const uint16_t *>(a.x) + int64_t(t) * H;
  const uint16_t *w = static_cast<const uint16_t *>(a.norm_weight);
  uint16_t *y = static_cast<uint16_t *>(a.normed_out) + int64_t(t) * H;
  const bool xvec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                      reinterpret_cast<uintptr_t>(y)) &
                     15) == 0;
  float ss = 0.f;
  for (int c = threadIdx.x; c < H / 8; c += kFusedThreads) {
    Vec8 v = load8(x + c * 8, xvec);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = bf(v.e[j]);
      ss += f * f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kFusedThreads / 32; ++i) total += red[i];
  const float inv_rms = 1.0f / sqrtf(total / float(H) + a.eps);
  for (int c = threadIdx.x; c < H / 8; c += kFusedThreads) {
    Vec8 v = load8(x + c * 8, xvec), wv = load8(w + c * 8, xvec), o;
#pragma unroll
    for (int j = 0; j < 8; ++j) o.e[j] = to_bf((bf(v.e[j]) * inv_rms) * bf(wv.e[j]));
    store8(y + c * 8, o, xvec);
  }

  // RoPE on q (in place) and k (straight into the page), V copied.
  const int step = a.kv_heads * D;
  uint16_t *q = static_cast<uint16_t *>(a.q) + int64_t(t) * a.num_q_heads * D;
  const bool qvec = (reinterpret_cast<uintptr_t>(q) & 15) == 0;
  rope_rows(q, q, a.num_q_heads, D, a.rope_mode, cs, sn, qvec);
  const int64_t dst = s_dst;
  if (dst >= 0) {
    const uint16_t *k = static_cast<const uint16_t *>(a.k) + int64_t(t) * step;
    const uint16_t *v = static_cast<const uint16_t *>(a.v) + int64_t(t) * step;
    uint16_t *kd = static_cast<uint16_t *>(a.va_k) + dst;
    uint16_t *vd = static_cast<uint16_t *>(a.va_v) + dst;
    const bool kvec = ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(kd)) & 15) == 0;
    rope_rows(k, kd, a.kv_heads, D, a.rope_mode, cs, sn, kvec);
    const bool vvec = ((reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(vd)) & 15) == 0 &&
                      (step & 7) == 0;
    if (vvec) {
      for (int c = threadIdx.x; c < step / 8; c += kFusedThreads) {
        reinterpret_cast<uint4 *>(vd)[c] = reinterpret_cast<const uint4 *>(v)[c];
      }
    } else {
      for (int c = threadIdx.x; c < step; c += kFusedThreads) vd[c] = v[c];
    }
  }
}

// ---------------------------------------------------------------------------
// Rotation of one 16-byte chunk with a cos/sin table.
// ---------------------------------------------------------------------------

// Rotate the 8-element chunk `in` of a head row starting at element d0.
// Interleaved modes rotate pairs (2i, 2i+1) inside the chunk; for neox the chunk
// holds the low halves of pairs (i, i + D/2) and `partner` the high halves.
__device__ __forceinline__ void rot_chunk(uint4 &lo, uint4 *partner, int pair0, const float *cs,
                                          const float *sn, bool neox) {
  uint16_t *e = reinterpret_cast<uint16_t *>(&lo);
  if (!neox) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float c = cs[pair0 + j], s = sn[pair0 + j];
      const float x0 = bf(e[2 * j]), x1 = bf(e[2 * j + 1]);
      e[2 * j] = to_bf(x0 * c - x1 * s);
      e[2 * j + 1] = to_bf(x0 * s + x1 * c);
    }
  } else {
    uint16_t *f = reinterpret_cast<uint16_t *>(partner);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float c = cs[pair0 + j], s = sn[pair0 + j];
      const float x0 = bf(e[j]), x1 = bf(f[j]);
      e[j] = to_bf(x0 * c - x1 * s);
      f[j] = to_bf(x0 * s + x1 * c);
    }
  }
}

// ---------------------------------------------------------------------------
// Fused RMSNorm + RoPE + KV append, split form (the default for aligned rows):
// three CTAs per token, one per independent part of the op.
//   blockIdx.y == 0  rotary of the k heads into the page, V row copied
//   blockIdx.y == 1  rotary of the q heads, in place
//   blockIdx.y == 2  RMSNorm of the hidden row (x, w -> normed)
// Only the K/V CTA waits for the two dependent lookups of the slot (slot
// mapping, then the offsets / valid tables); its CTAs come first in the grid,
// so those lookups are issued before the bulk of the loads.  The norm and q
// CTAs store as soon as their own loads land.  Against one CTA per token that
// does all three parts, this cut 32 layers of config 3 (one CUDA graph) from
// 169 to 137 us on B200.
// Rotary factors: theta_i comes from the launcher (the reference formula
// 1/powf(base, e_i) in fp32, ref src/cuda/kernels/rope.cu:18).  The first
// head_dim/2 threads of a rotary CTA form angle = pos * theta_i in fp32 like the
// reference, reduce it exactly to [-pi, pi] in double precision and put
// __cosf/__sinf of it (absolute error below 2^-21 on that interval) in a shared
// table.  Every thread evaluating the factors of its own pairs instead was
// slower in the 32-layer graph (167 us).
// Requirements (checked by the launcher): 16-byte aligned rows, head_dim % 16 ==
// 0, head_dim <= 256, and hidden, num_q_heads * head_dim and kv_heads * head_dim
// at most C * 8 * kSplitThreads for the chunk budget C (8-element chunks per
// thread) the launcher picks: 4 when they fit 4096, else 8.
// ---------------------------------------------------------------------------

constexpr int kSplitThreads = 128;

// Slot resolution with the device-slot write's status rules; -1 = write nothing.
__device__ __forceinline__ int64_t resolve_slot(const FusedAppendArgs &a, int64_t slot,
                                                int step) {
  if (slot < 0) return -1;
  const int64_t blk = slot / a.block_size;
  if (blk >= a.offsets_len) {
    if (a.status) atomicCAS(a.status, 0, 1);
    return -1;
  }
  // both lookups in flight together (one round trip, not two)
  const uint8_t live = a.valid ? a.valid[blk] : uint8_t(1);
  const uint64_t off = a.block_offsets[blk];
  if (live == 0) {
    if (a.status) atomicCAS(a.status, 0, 2);
    return -1;
  }
  const int64_t d = int64_t(off) + (slot % a.block_size) * step;
  if (uint64_t(d) + uint64_t(step) > a.region_elems) {
    if (a.status) atomicCAS(a.status, 0, 3);
    return -1;
  }
  return d;
}

// cos / sin of the fp32 angle pos * theta: the angle minus the nearest multiple
// of 2 pi, formed in double precision (|angle| <= 2^24 keeps it exact to well
// below the fp32 ulp of the result), then the hardware approximations.
__device__ __forceinline__ void rotary(float pos, float theta, float &c, float &s) {
  const float ang = pos * theta;
  constexpr double kTwoPi = 6.283185307179586476925286766559;
  constexpr double kInvTwoPi = 0.15915494309189533576888376337251;
  const double k = rint(double(ang) * kInvTwoPi);
  const float r = float(fma(-k, kTwoPi, double(ang)));
  s = __sinf(r);
  c = __cosf(r);
}

template <int C>
__global__ void __launch_bounds__(kSplitThreads) fused_split_kernel(const FusedAppendArgs a) {
  __shared__ float red[kSplitThreads / 32];
  __shared__ int64_t s_dst;
  __shared__ float tcs[128], tsn[128];  // cos / sin per pair index
  ptx::grid_dependency_wait();  // a programmatic dependent: see pdl.cuh
  ptx::launch_dependents();
  const int t = blockIdx.x, tid = threadIdx.x;
  const int role = blockIdx.y;
  const int D = a.head_dim, half = D / 2, cph = D / 8;
  const bool neox = a.rope_mode == 2;
  if (role == 0) {
    const int step = a.kv_heads * D, nk = step / 8;
    int64_t slot = -1;
    if (tid == 0) slot = a.slot_mapping[t];
    const float pos = float(a.positions[t]);
    const uint4 *k = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.k) + int64_t(t) * step);
    const uint4 *v = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.v) + int64_t(t) * step);
    uint4 kr[C], kh[C], vr[C];
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = tid + i * kSplitThreads;
      if (c < nk) {
        kr[i] = k[c];
        vr[i] = v[c];
        if (neox && (c % cph) * 8 < half) kh[i] = k[c + half / 8];
      }
    }
    if (tid == 0) s_dst = resolve_slot(a, slot, step);
    for (int i = tid; i < half; i += kSplitThreads) rotary(pos, a.inv_freq[i], tcs[i], tsn[i]);
    __syncthreads();  // the table and s_dst
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = tid + i * kSplitThreads;
      const int d0 = (c % cph) * 8;
      if (c < nk && (!neox || d0 < half)) rot_chunk(kr[i], &kh[i], neox ? d0 : d0 / 2, tcs, tsn, neox);
    }
    const int64_t dst = s_dst;
    if (dst < 0) return;
    uint4 *kd = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.va_k) + dst);
    uint4 *vd = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.va_v) + dst);
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = tid + i * kSplitThreads;
      if (c < nk) {
        vd[c] = vr[i];
        const int d0 = (c % cph) * 8;
        if (!neox) {
          kd[c] = kr[i];
        } else if (d0 < half) {
          kd[c] = kr[i];
          kd[c + half / 8] = kh[i];
        }
      }
    }
    return;
  }
  if (role == 1) {
    const float pos = float(a.positions[t]);
    const int nq = a.num_q_heads * D / 8;
    uint4 *q = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.q) + int64_t(t) * a.num_q_heads * D);
    uint4 qr[C];
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = tid + i * kSplitThreads;
      if (c < nq) qr[i] = q[c];
    }
    for (int i = tid; i < half; i += kSplitThreads) rotary(pos, a.inv_freq[i], tcs[i], tsn[i]);
    __syncthreads();
    // A thread stores only the chunks it rotates (neox: a low-half chunk and its
    // high partner, which no other thread writes), so the in-place update needs
    // no second barrier.
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = tid + i * kSplitThreads;
      if (c < nq) {
        const int d0 = (c % cph) * 8;
        if (!neox) {
          rot_chunk(qr[i], nullptr, d0 / 2, tcs, tsn, false);
          q[c] = qr[i];
        } else if (d0 < half) {
          uint4 hi = q[c + half / 8];
          rot_chunk(qr[i], &hi, d0, tcs, tsn, true);
          q[c] = qr[i];
          q[c + half / 8] = hi;
        }
      }
    }
    return;
  }
  // RMSNorm (ref src/cuda/kernels/rms_norm.cu:14-35): bf16((x * inv_rms) * w)
  const int H = a.hidden, nx = H / 8;
  const uint4 *x = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.x) + int64_t(t) * H);
  const uint4 *w = reinterpret_cast<const uint4 *>(a.norm_weight);
  uint4 xr[C], wr[C];
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = tid + i * kSplitThreads;
    if (c < nx) {
      xr[i] = x[c];
      wr[i] = w[c];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < C; ++i) {
    if (tid + i * kSplitThreads < nx) {
      const uint16_t *e = reinterpret_cast<const uint16_t *>(&xr[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float f = bf(e[j]);
        ss += f * f;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kSplitThreads / 32; ++i) total += red[i];
  const float inv_rms = 1.0f / sqrtf(total / float(H) + a.eps);
  uint4 *y = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.normed_out) + int64_t(t) * H);
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = tid + i * kSplitThreads;
    if (c < nx) {
      const uint16_t *xe = reinterpret_cast<const uint16_t *>(&xr[i]);
      const uint16_t *we = reinterpret_cast<const uint16_t *>(&wr[i]);
      uint4 out;
      uint16_t *oe = reinterpret_cast<uint16_t *>(&out);
#pragma unroll
      for (int j = 0; j < 8; ++j) oe[j] = to_bf((bf(xe[j]) * inv_rms) * bf(we[j]));
      y[c] = out;
    }
  }
}

}  // namespace

cudaError_t copy_rows(const void *k_src, const void *v_src, void *va_k, void *va_v,
                      const int64_t *dst_elems_host, int rows, int row_elems,
                      cudaStream_t stream) {
  for (int base = 0; base < rows; base += kRowsPerLaunch) {
    RowCopyParams p;
    p.k_src = static_cast<const uint16_t *>(k_src);
    p.v_src = static_cast<const uint16_t *>(v_src);
    p.va_k = static_cast<uint16_t *>(va_k);
    p.va_v = static_cast<uint16_t *>(va_v);
    p.rows = std::min(kRowsPerLaunch, rows - base);
    p.row_elems = row_elems;
    p.row_base = base;
    for (int r = 0; r < p.rows; ++r) p.dst[r] = dst_elems_host[base + r];
    const int threads = std::min(256, std::max(32, (row_elems / 8 + 31) / 32 * 32));
    copy_rows_kernel<<<p.rows, threads, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t device_slot_write(const SlotWriteArgs &a, cudaStream_t stream) {
  const int threads = std::min(256, std::max(32, (a.step_elems / 8 + 31) / 32 * 32));
  slot_write_kernel<<<a.batch, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t fused_norm_rope_append(const FusedAppendArgs &args, cudaStream_t stream) {
  FusedAppendArgs a = args;
  // theta_i = 1 / base^e_i in fp32, the reference formula (ref src/cuda/kernels/rope.cu:18
  // with the base as a parameter); e_i = 2 floor(i/2) / D (reference mode) or 2i / D
  for (int i = 0; i < a.head_dim / 2 && i < 128; ++i) {
    const float e = a.rope_mode == 0 ? float(2 * (i / 2)) / float(a.head_dim)
                                     : float(2 * i) / float(a.head_dim);
    a.inv_freq[i] = 1.0f / powf(a.rope_theta, e);
  }
  const uintptr_t align = reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.norm_weight) |
                          reinterpret_cast<uintptr_t>(a.normed_out) | reinterpret_cast<uintptr_t>(a.q) |
                          reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
                          reinterpret_cast<uintptr_t>(a.va_k) | reinterpret_cast<uintptr_t>(a.va_v);
  const int step = a.kv_heads * a.head_dim;
  const int widest = std::max(a.hidden, std::max(a.num_q_heads * a.head_dim, step));
  const bool split = (align & 15) == 0 && a.head_dim % 16 == 0 && a.head_dim <= 256 &&
                     a.hidden % 8 == 0 && widest <= 8 * 8 * kSplitThreads &&
                     !(std::getenv("KCMM_FUSED_IMPL") &&
                       std::strcmp(std::getenv("KCMM_FUSED_IMPL"), "table") == 0);
  if (split) {
    const dim3 grid(a.num_tokens, 3);
    if (widest <= 4 * 8 * kSplitThreads)
      return launch_pdl(fused_split_kernel<4>, grid, dim3(kSplitThreads), 0, stream, a);
    return launch_pdl(fused_split_kernel<8>, grid, dim3(kSplitThreads), 0, stream, a);
  }
  const size_t smem = size_t(a.head_dim) * sizeof(float);
  return launch_pdl(fused_kernel, dim3(a.num_tokens), dim3(kFusedThreads), smem, stream, a);
}

}  // namespace dev
}  // namespace kcmm
