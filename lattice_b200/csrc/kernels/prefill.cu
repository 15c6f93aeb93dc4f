// Chunked prefill attention over paged KV on the sm_100a tensor cores (tcgen05).
//
// A chunk of q_len new tokens of sequence b sits at absolute positions
// [ctx_len - q_len, ctx_len); its K/V rows are already in the pages.  Query
// token t attends causally to keys [0, ctx_len - q_len + t].  The reference
// has no prefill kernel (its prefill is a token-by-token decode loop,
// ref src/model/transformer.rs:50-65); the arithmetic is the decode kernel's
// softmax(scale * q.k) v (ref src/cuda/kernels/kcmm_vllm_paged_attn.cu:40-101)
// with a causal limit per query row.
//
// CTA = 128 query rows x one kv head: TT = 128 / G tokens x the G query heads
// of the GQA group (row r = token r / G, head r % G), so every K/V tile feeds
// all heads of the group.  4 warps; thread r owns row r (TMEM lane r).
//   per KV tile of 128 tokens (pages gathered by cp.async into 128-byte-swizzled
//   shared memory, double buffered):
//     S  = Q K^T      tcgen05.mma M128 N128 K16 x 8, fp32 in TMEM columns [0,128)
//     softmax         tcgen05.ld S row -> causal mask, online max/sum in the
//                     log2 domain, P -> swizzled shared memory as two 16-bit
//                     tiles, P_hi = round(P) and P_lo = round(P - P_hi)
//     O += P_hi V + P_lo V   tcgen05.mma M128 N128 K16 x 16 (V as an MN-major
//                     operand), fp32 in TMEM columns [128,256)
//   The P.V operands must share V's 16-bit type; a single rounded P leaves a
//   relative error of 2^-9 per weight, which rows over a few keys with
//   cancelling values do not average out.  The hi/lo pair carries P to ~2^-17.
//   The running max is only raised when a tile's max exceeds it by more than
//   2^8 (the rescale of O in TMEM is skipped otherwise); P stays <= 2^8.
// Every mbarrier wait is bounded; a wait that runs out sets the pool's
// diagnostic bit, the CTA drains its copies, frees its TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "../launch.hpp"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace kcmm {
namespace dev {
namespace {

constexpr int kRows = 128;   // query rows per CTA (MMA M)
constexpr int kKvTile = 128;  // keys per tile (MMA N of S, K of P.V)
constexpr int kHd = 128;      // head_dim
constexpr uint32_t kTile = 128 * 128 * 2;  // one 128 x 128 16-bit tile: 32 KB
constexpr uint32_t kHalf = 128 * 128;      // one 64-column half (128 rows x 128 B)
constexpr uint32_t kOffQ = 0;                    // the Q tile opens every kernel's layout
constexpr uint64_t kLimitNs = 1000000000ull;     // an MMA that has not finished in 1 s

struct PrefillParams {
  const uint16_t *q;
  uint16_t *out;
  const int32_t *tables;
  const int32_t *q_start;   // [batch + 1]
  const int32_t *ctx_lens;  // [batch]
  const uint64_t *offsets;  // 2-byte units
  const uint16_t *va_k;
  const uint16_t *va_v;
  uint64_t region_elems;
  int hq, hkv, G, bs, max_bps, tt;  // G: query heads per kv head padded to a power of two
  int gr;                            // the real query heads per kv head (rows j >= gr idle)
  int d;  // head_dim (the single-role kernel; the others are built for 128)
  float scale_log2;
  uint32_t idesc_qk, idesc_pv;
  int32_t *diag;
};

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  // byte offset of 16-byte chunk `chunk` (0..15) of a 256-byte row inside a
  // [2 halves][128 rows][128 B] tile with the 128-byte swizzle
  return uint32_t((chunk >> 3) * kHalf + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// The same for the V tiles of the warp-specialised kernel, stored box-major:
// [8 boxes of 16 keys][2 halves][16 rows][128 B], the layout one 4-D page box lands in.
__device__ __forceinline__ uint32_t swz_v(int row, int chunk) {
  return uint32_t((row >> 4) * 4096 + (chunk >> 3) * 2048 + (row & 15) * 128 +
                  (((chunk & 7) ^ (row & 7)) << 4));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// Online-softmax step for one row over one key tile, in place: s[c] becomes
// P = exp2(s * scale_log2 - m) with keys past `qpos` masked out (when the tile
// reaches past the CTA's first row).  The running max m is only raised when the
// tile's max exceeds it by more than 8 (log2 units).  Returns the row sum of P;
// alpha = exp2(m_old - m_new) rescales the earlier sum and O.
template <int N>
__device__ __forceinline__ float masked_max(float (&s)[N], int k0, int qpos, bool need_mask) {
  if (need_mask) {
#pragma unroll
    for (int c = 0; c < N; ++c) s[c] = k0 + c > qpos ? -INFINITY : s[c];
  }
  // four independent chains of three-input max
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int c = 0; c < N; c += 8) {
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = ptx::max3(m[i], s[c + 2 * i], s[c + 2 * i + 1]);
  }
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// Given the tile's row max mx (already in log2 units), update the running max and
// turn s into P in place; returns the sum of this thread's P values.
template <int N>
__device__ __forceinline__ float exp_given_max(float (&s)[N], float mx, float scale_log2,
                                               bool has_prev, float &m_run, float &alpha,
                                               bool &rescale) {
  float m_new = m_run;
  if (mx > m_run + 8.f) m_new = mx;  // first tile: m_run = -inf
  alpha = ptx::fast_exp2(m_run - m_new);  // 0 on the first tile, else <= 1
  rescale = has_prev && m_new != m_run;
  m_run = m_new;
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < N; ++c) {
    s[c] = ptx::fast_exp2(fmaf(s[c], scale_log2, -m_new));
    sum[c & 3] += s[c];
  }
  return (sum[0] + sum[1]) + (sum[2] + sum[3]);
}

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162 *>(&v));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<__half2 *>(&v));
}

// P row -> the P_hi and P_lo tiles (128-byte swizzle, keys along the row).
template <typename T>
__device__ __forceinline__ void store_p(const float (&s)[128], uint32_t pa, uint32_t pl, int row) {
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    uint32_t w[4], r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = s[c * 8 + 2 * e], bb = s[c * 8 + 2 * e + 1];
      w[e] = pack2<T>(a, bb);
      const float2 hv = unpack2<T>(w[e]);
      r[e] = pack2<T>(a - hv.x, bb - hv.y);
    }
    const uint32_t so = swz(row, c);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(pa + so), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3])
                 : "memory");
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(pl + so), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
  }
}

// P values of N keys of one row -> TMEM as 16-bit pairs (element 2c in the low half of
// column c): P_hi at column t_hi, P_lo = round(P - P_hi) at column t_lo.
template <typename T, int N>
__device__ __forceinline__ void store_p_tmem(const float (&s)[N], uint32_t t_hi, uint32_t t_lo) {
#pragma unroll
  for (int part = 0; part < N / 64; ++part) {
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = pack2<T>(s[64 * part + 2 * i], s[64 * part + 2 * i + 1]);
    tc::st32u(t_hi + 32 * part, w);
  }
#pragma unroll
  for (int part = 0; part < N / 64; ++part) {
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float a = s[64 * part + 2 * i], b = s[64 * part + 2 * i + 1];
      const float2 hv = unpack2<T>(pack2<T>(a, b));
      w[i] = pack2<T>(a - hv.x, b - hv.y);
    }
    tc::st32u(t_lo + 32 * part, w);
  }
  tc::wait_st();
}

// The 128 P values of one row -> TMEM as 16-bit pairs, 16 columns per store so that
// few packed words are live at once: P_hi at columns t_hi .. t_hi + 63, P_lo =
// round(P - P_hi) at t_lo .. t_lo + 63.
template <typename T>
__device__ __forceinline__ void store_p_row128(const float (&s)[128], uint32_t t_hi,
                                               uint32_t t_lo) {
#pragma unroll
  for (int part = 0; part < 4; ++part) {
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = pack2<T>(s[32 * part + 2 * i], s[32 * part + 2 * i + 1]);
    tc::st16u(t_hi + 16 * part, w);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = s[32 * part + 2 * i], b = s[32 * part + 2 * i + 1];
      const float2 hv = unpack2<T>(pack2<T>(a, b));
      w[i] = pack2<T>(a - hv.x, b - hv.y);
    }
    tc::st16u(t_lo + 16 * part, w);
  }
  tc::wait_st();
}

// The P_hi half of store_p_row128 alone.
template <typename T>
__device__ __forceinline__ void store_p_hi128(const float (&s)[128], uint32_t t_hi) {
#pragma unroll
  for (int part = 0; part < 4; ++part) {
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = pack2<T>(s[32 * part + 2 * i], s[32 * part + 2 * i + 1]);
    tc::st16u(t_hi + 16 * part, w);
  }
}
// One row of O (128 fp32 columns in TMEM) to global memory as it is.
__device__ __forceinline__ void store_o_row_f32(uint32_t t_row, float *dst) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float o[32];
    tc::ld32(t_row + c * 32, o);
    tc::wait_ld();
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4 *>(dst + c * 32 + q * 4) =
          make_float4(o[q * 4], o[q * 4 + 1], o[q * 4 + 2], o[q * 4 + 3]);
  }
}

// Store N columns of one row of O (fp32 in TMEM) / l to global memory.
template <typename T, int N = 128>
__device__ __forceinline__ void store_o_row(uint32_t t_row, float inv, uint16_t *dst, bool ok) {
#pragma unroll
  for (int c = 0; c < N / 32; ++c) {
    float o[32];
    tc::ld32(t_row + c * 32, o);
    tc::wait_ld();
    if (ok) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 v;
        v.x = pack2<T>(o[q * 8 + 0] * inv, o[q * 8 + 1] * inv);
        v.y = pack2<T>(o[q * 8 + 2] * inv, o[q * 8 + 3] * inv);
        v.z = pack2<T>(o[q * 8 + 4] * inv, o[q * 8 + 5] * inv);
        v.w = pack2<T>(o[q * 8 + 6] * inv, o[q * 8 + 7] * inv);
        *reinterpret_cast<uint4 *>(dst + c * 32 + q * 8) = v;
      }
    }
  }
}

// N columns of an O row *= f (all lanes of the warp execute this; f = 1 for rows that
// keep their max).
template <int N = 128>
__device__ __forceinline__ void scale_o_row(uint32_t t_row, float f) {
#pragma unroll
  for (int c = 0; c < N / 32; ++c) {
    float o[32];
    tc::ld32(t_row + c * 32, o);
    tc::wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e) o[e] *= f;
    tc::st32(t_row + c * 32, o);
  }
  tc::wait_st();
}

// Shared memory and TMEM of the single-role kernel for head_dim padded to DP (64, 128,
// 192 or 256) and KT keys per tile (128, or 64 where DP > 128 so that the tiles fit):
// Q [DP/64][128 rows][128 B], K and V [2 stages][DP/64][KT rows][128 B], P_hi and P_lo
// [KT/64][128 rows][128 B], all with the 128-byte swizzle, then a ring of key rows
// [3 tiles][KT] and the two halves' row values [2][128] (tile max, final sum).  TMEM
// (512 columns): S of tiles j even / odd in columns [0, KT) / [KT, 2 KT), O in
// [256, 256 + DP).
template <int DP, int KT>
struct OneRole {
  static constexpr uint32_t kQ = 128u * DP * 2;   // Q tile bytes
  static constexpr uint32_t kKV = uint32_t(KT) * DP * 2;  // one K or V stage
  static constexpr uint32_t kP = 128u * KT * 2;   // one P tile
  static constexpr uint32_t kKvBlk = uint32_t(KT) * 128;  // a 64-column block of K or V
  static constexpr uint32_t kOffK = kQ;
  static constexpr uint32_t kOffV = kOffK + 2 * kKV;
  static constexpr uint32_t kOffP = kOffV + 2 * kKV;
  static constexpr uint32_t kOffRow = kOffP + 2 * kP;        // [3 tiles][KT] key rows
  static constexpr uint32_t kOffX = kOffRow + 3 * KT * 4;    // [2 halves][128 rows] f32
  static constexpr uint32_t kOffBar = kOffX + 2 * 128 * 4;   // 2 mbarriers, TMEM slot, fail
  static constexpr size_t kSmem = kOffBar + 64 + 1024;
  static constexpr uint32_t kCols = 512;
  static_assert(kSmem <= 232448, "shared memory of one CTA");
};

constexpr uint32_t kNoRow = 0xFFFFFFFFu;  // a key past the range or with a bad address
constexpr int kOneRoleThreads = 256;      // two threads per query row
// keys per tile of the single-role kernel for head_dim padded to dp
constexpr int one_role_kt(int dp) { return dp <= 64 ? 128 : 64; }

// byte offset of 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled tile whose
// 64-column blocks are `blk` bytes apart
__device__ __forceinline__ uint32_t swz_blk(int row, int chunk, uint32_t blk) {
  return uint32_t((chunk >> 3) * blk + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// The single-role kernel: every thread loads with cp.async, thread 0 issues the MMAs,
// threads r and r + 128 (warps w and w + 4 reach the same TMEM lanes) run the softmax
// of row r over the first and second half of each key tile and own the first and
// second half of O's columns; they combine the tile's row max through shared memory at
// the barrier that follows the S read, and their row sums at the end.  It serves head
// dims other than 128 (p.d <= DP,
// a multiple of 8; the columns past p.d are zero in Q and V and are not stored), and
// head_dim 128 where the block size is not a multiple of 16.
// Pipeline, per key tile j (K and V stages j & 1, S buffer j & 1):
//   wait S(j) -> read S(j) -> K(j+1) landed: issue S(j+1) -> copy K(j+2) into the
//   stage S(j) has freed -> softmax(j) in registers -> wait P.V(j-1) -> rescale O,
//   store P(j) -> copy V(j+1) into the stage P.V(j-1) has freed -> V(j) landed:
//   issue P.V(j).
// So the tensor pipe computes S(j+1) and P.V(j-1) while the threads run softmax(j),
// and every copy is issued one tile ahead.  Each thread commits one cp.async group per
// K tile and one per V tile, in the order K(j+2), V(j+1) within tile j (after K(0),
// K(1), V(0) up front), empty where the tile does not exist, so "K(j+1) landed" is
// wait_group 1 and "V(j) landed" is wait_group 2.  The copies read each key's row
// address from a shared ring of 3 tiles (element offset / 8, or kNoRow): thread n
// resolves key n of tile j+3 during tile j (block table, then offsets table, the two
// loads issued around the softmax) into the slot of tile j, whose last copy (V(j)) was
// issued in tile j-1, so no copy waits on a table lookup.
template <typename T, int DP, int KT>
__global__ void __launch_bounds__(kOneRoleThreads, 1) prefill_kernel(const PrefillParams p) {
  using L = OneRole<DP, KT>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;  // 1024-aligned base (swizzle atoms)
  unsigned char *smem = smem_raw + (sb - raw);
  volatile int &s_fail = *reinterpret_cast<volatile int *>(smem + L::kOffBar + 20);
  uint32_t *rows = reinterpret_cast<uint32_t *>(smem + L::kOffRow);  // [3][KT]
  float *xch = reinterpret_cast<float *>(smem + L::kOffX);            // [2][128]
  constexpr int NT = kOneRoleThreads, KH = KT / 2, OH = DP / 2;

  const int tid = threadIdx.x, warp = tid >> 5, half = tid >> 7;
  // query tiles last-first: the longest causal items start first
  const int qt = int(gridDim.x) - 1 - int(blockIdx.x), h = blockIdx.y, b = blockIdx.z;
  const int q0 = p.q_start[b];
  const int qlen = p.q_start[b + 1] - q0;
  const int ctx = p.ctx_lens[b];
  if (qt * p.tt >= qlen) return;  // no rows for this CTA
  if (ctx < qlen || ctx > p.max_bps * p.bs) {
    if (tid == 0) atomicOr(p.diag, int32_t(kDiagBadLaunch));
    return;
  }
  const int D = p.d, DC = p.d / 8;  // head_dim, its 16-byte chunks
  const int base_pos = ctx - qlen;
  const int ti_hi = min((qt + 1) * p.tt, qlen);
  const int kv_hi = base_pos + ti_hi;  // keys [0, kv_hi) reach some row of this CTA
  const int nt = (kv_hi + KT - 1) / KT;

  const int row = tid & 127;
  const int ti = qt * p.tt + row / p.G;
  const bool row_ok = ti < qlen && row % p.G < p.gr;
  const int qpos = row_ok ? base_pos + ti : kv_hi - 1;

  const uint32_t bar_s = sb + L::kOffBar, bar_o = sb + L::kOffBar + 8,
                 slot = sb + L::kOffBar + 16;
  if (warp == 0) {
    tc::tmem_alloc(slot, L::kCols);
    tc::tmem_relinquish();
    tc::fence_before_sync();
  }
  if (tid == 0) {
    ptx::mbar_init(bar_s, 1);
    ptx::mbar_init(bar_o, 1);
    ptx::fence_mbarrier_init();
    s_fail = 0;
  }

  // --- Q tile: row r = (token, head) pair, zero rows past the chunk and columns past D --
  {
#pragma unroll 4
    for (int it = 0; it < 128 * DP / 8 / NT; ++it) {
      const int idx = it * NT + tid, r = idx / (DP / 8), c = idx % (DP / 8);
      const int t_r = qt * p.tt + r / p.G, h_r = h * p.gr + r % p.G;
      const bool ok = t_r < qlen && r % p.G < p.gr && c < DC;
      const uint16_t *src = ok ? p.q + (size_t(q0 + t_r) * p.hq + h_r) * D + c * 8 : p.q;
      ptx::cp_async16(sb + swz_blk(r, c, kHalf), src, ok ? 16u : 0u);
    }
    ptx::cp_async_commit();
  }

  const size_t tok_stride = size_t(p.hkv) * D;
  const int32_t *table = p.tables + size_t(b) * p.max_bps;
  bool bad = false;
  // Key n of tile t: its block id (first load), then its row (second load) into the
  // ring slot t % 3.  Threads n >= KT take no key.
  auto key_block = [&](int t) -> int {
    const int kv = t * KT + tid;
    return tid < KT && t < nt && kv < kv_hi ? table[kv / p.bs] : -1;
  };
  auto key_row = [&](int t, int blk) {
    if (tid >= KT) return;
    uint32_t r = kNoRow;
    if (blk >= 0) {
      const int kv = t * KT + tid;
      const uint64_t off = p.offsets[blk];
      const uint64_t elem = off + uint64_t(kv % p.bs) * tok_stride + uint64_t(h) * D;
      if ((off & 7) == 0 && elem + uint64_t(D) <= p.region_elems && (elem >> 3) < kNoRow) {
        r = uint32_t(elem >> 3);
      } else {
        bad = true;
      }
    }
    rows[(t % 3) * KT + tid] = r;
  };
  // One K or V tile of keys [j * KT, j * KT + KT) into stage st from the ring, then a
  // commit (an empty group for a tile past the last).
  auto load_tile = [&](int j, int st, bool is_v) {
    if (j < nt) {
      const uint32_t dst = sb + (is_v ? L::kOffV : L::kOffK) + st * L::kKV;
      const uint16_t *base = is_v ? p.va_v : p.va_k;
      const uint32_t *rj = rows + (j % 3) * KT;
#pragma unroll 4
      for (int it = 0; it < KT * DP / 8 / NT; ++it) {
        const int idx = it * NT + tid, n = idx / (DP / 8), c = idx % (DP / 8);
        const uint32_t r = rj[n];
        const bool ok = r != kNoRow && c < DC;
        ptx::cp_async16(dst + swz_blk(n, c, L::kKvBlk),
                        ok ? base + (uint64_t(r) << 3) + c * 8 : base, ok ? 16u : 0u);
      }
    }
    ptx::cp_async_commit();
  };

  {  // rows of tiles 0, 1 and 2
    const int b0 = key_block(0), b1 = key_block(1), b2 = key_block(2);
    key_row(0, b0);
    key_row(1, b1);
    key_row(2, b2);
  }
  __syncthreads();
  load_tile(0, 0, false);
  load_tile(1, 1, false);
  load_tile(0, 0, true);
  ptx::cp_async_wait<2>();  // Q and K(0)
  ptx::fence_proxy_async_smem();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + L::kOffBar + 16);
  const uint32_t lane_base = uint32_t(warp * 32) << 16;
  const uint32_t tO = tmem + 256;
  // S(j) = Q K(j)^T into S buffer j & 1 (thread 0)
  auto issue_s = [&](int j) {
    const uint32_t ka = sb + L::kOffK + (j & 1) * L::kKV, tS = tmem + (j & 1) * KT;
#pragma unroll
    for (int k = 0; k < DP / 16; ++k) {
      const uint32_t in_row = uint32_t(k & 3) * 32;
      tc::mma_ss(tS, tc::sw128_desc(sb + (k >> 2) * kHalf + in_row, 16, 1024),
                 tc::sw128_desc(ka + (k >> 2) * L::kKvBlk + in_row, 16, 1024), p.idesc_qk,
                 k > 0);
    }
    tc::commit(bar_s);
  };
  if (tid == 0) {
    tc::fence_after_sync();
    issue_s(0);
  }

  float m_run = -INFINITY, l_run = 0.f;
  bool failed = false;
  const uint32_t pa = sb + L::kOffP, pl = pa + L::kP;
  for (int j = 0; j < nt; ++j) {
    if (!ptx::mbar_wait_bounded(bar_s, uint32_t(j & 1), kLimitNs)) s_fail = 1;
    tc::fence_after_sync();
    float s[KH];
#pragma unroll
    for (int c = 0; c < KH / 32; ++c)
      tc::ld32(tmem + (j & 1) * KT + half * KH + lane_base + c * 32, s + c * 32);
    tc::wait_ld();
    const float mx_half = masked_max<KH>(s, j * KT + half * KH, qpos,
                                         j * KT + KT - 1 > base_pos + qt * p.tt) *
                          p.scale_log2;
    xch[half * 128 + row] = mx_half;  // read by the other half after the barrier
    // S(j) is read by every thread and K(j + 1) has landed: S(j + 1) may start
    ptx::cp_async_wait<1>();
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (s_fail) {
      failed = true;
      break;
    }
    if (tid == 0 && j + 1 < nt) {
      tc::fence_after_sync();
      issue_s(j + 1);
    }
    load_tile(j + 2, j & 1, false);  // the K stage S(j) has finished with
    const int blk3 = key_block(j + 3);  // in flight during the softmax

    float alpha;
    bool rescale;
    const float mx = fmaxf(mx_half, xch[(half ^ 1) * 128 + row]);  // the row's tile max
    const float sum = exp_given_max<KH>(s, mx, p.scale_log2, j > 0, m_run, alpha, rescale);
    l_run = l_run * alpha + sum;  // this half's share of the row sum

    if (j > 0) {  // P.V(j - 1) done: P, O and V stage (j + 1) & 1 are free
      if (!ptx::mbar_wait_bounded(bar_o, uint32_t((j - 1) & 1), kLimitNs)) s_fail = 1;
      tc::fence_after_sync();
    }
    if (__any_sync(0xffffffffu, rescale))
      scale_o_row<OH>(tO + half * OH + lane_base, rescale ? alpha : 1.f);
#pragma unroll
    for (int c = 0; c < KH / 8; ++c) {  // P half row -> P_hi, P_lo (keys along the row)
      uint32_t w[4], r[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = s[c * 8 + 2 * e], bb = s[c * 8 + 2 * e + 1];
        w[e] = pack2<T>(a, bb);
        const float2 hv = unpack2<T>(w[e]);
        r[e] = pack2<T>(a - hv.x, bb - hv.y);
      }
      const uint32_t so = swz_blk(row, half * (KH / 8) + c, kHalf);
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(pa + so), "r"(w[0]),
                   "r"(w[1]), "r"(w[2]), "r"(w[3])
                   : "memory");
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(pl + so), "r"(r[0]),
                   "r"(r[1]), "r"(r[2]), "r"(r[3])
                   : "memory");
    }
    load_tile(j + 1, (j + 1) & 1, true);  // the V stage P.V(j - 1) has finished with
    key_row(j + 3, blk3);  // slot (j + 3) % 3: tile j's, whose copies are all issued
    ptx::cp_async_wait<2>();  // V(j)
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (s_fail) {
      failed = true;
      break;
    }
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t va = sb + L::kOffV + (j & 1) * L::kKV;
#pragma unroll
      for (int k = 0; k < KT / 16; ++k) {
        const uint32_t ao = uint32_t((k >> 2) * kHalf + (k & 3) * 32);
        // V: rows = keys (K), 64-element blocks of head_dim (N) kKvBlk apart
        const uint64_t vd = tc::sw128_desc(va + uint32_t(k) * 2048, L::kKvBlk, 1024);
        tc::mma_ss(tO, tc::sw128_desc(pa + ao, 16, 1024), vd, p.idesc_pv,
                   (j > 0 || k > 0) ? 1u : 0u);
        tc::mma_ss(tO, tc::sw128_desc(pl + ao, 16, 1024), vd, p.idesc_pv, 1u);
      }
      tc::commit(bar_o);
    }
  }

  if (!failed) {
    if (!ptx::mbar_wait_bounded(bar_o, uint32_t((nt - 1) & 1), kLimitNs)) s_fail = 1;
    tc::fence_after_sync();
  }
  xch[half * 128 + row] = l_run;
  __syncthreads();
  failed = failed || s_fail;
  if (!failed) {
    const float l = l_run + xch[(half ^ 1) * 128 + row];
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint16_t *dst = p.out + (size_t(q0 + ti) * p.hq + h * p.gr + row % p.G) * D + half * OH;
    {  // this half's columns of O, 8 per store, those below D
#pragma unroll
      for (int c = 0; c < OH / 32; ++c) {
        float o[32];
        tc::ld32(tO + half * OH + lane_base + c * 32, o);
        tc::wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (row_ok && half * OH + c * 32 + q * 8 < D) {
            uint4 v;
            v.x = pack2<T>(o[q * 8 + 0] * inv, o[q * 8 + 1] * inv);
            v.y = pack2<T>(o[q * 8 + 2] * inv, o[q * 8 + 3] * inv);
            v.z = pack2<T>(o[q * 8 + 4] * inv, o[q * 8 + 5] * inv);
            v.w = pack2<T>(o[q * 8 + 6] * inv, o[q * 8 + 7] * inv);
            *reinterpret_cast<uint4 *>(dst + c * 32 + q * 8) = v;
          }
        }
      }
    }
  } else {
    ptx::cp_async_wait<0>();
    if (tid == 0) atomicOr(p.diag, int32_t(kDiagWaitTimeout));
  }
  if (bad) atomicOr(p.diag, int32_t(kDiagBadOffset));
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, L::kCols);
  }
}

// --- warp-specialised kernel: producer warps, MMA issuer, softmax warps -------------------
//
// warps 0-7  softmax: warp w owns rows 32*(w%4) .. +31 (its TMEM lane quarter) and key /
//            head_dim columns [64*(w/4), +64): two warps share each row and trade their
//            partial row max through shared memory.  S_j from TMEM -> P_hi/P_lo written
//            back over S_j's own TMEM columns (16-bit pairs: P_hi in the first 64
//            columns, P_lo in the last 64), O rescale in TMEM, epilogue
// warp 8     K producer: Q, then K tiles into a 3-stage ring
// warp 10    V producer: V tiles into a 2-stage ring
// TMA variant: 16-token page boxes by TMA.  K boxes ({64, 1, 16}: one head_dim half,
//            2 KB) 0-3 from warp 8 and 4-7 from warp 11; V boxes ({64, 16, 2, 1}: both
//            halves of a page, 4 KB, landing box-major) from warps 10 and 12.  TMA
//            issue costs ~90 cycles a box, so V boxes halve V's cost.  V tiles that
//            reach past the context are gathered with zero-filling cp.async instead.
// Gather variant (layouts the tensor map cannot address): warps 8 and 10 copy whole
//            tiles with 16-byte cp.async from all lanes.
// warp 9     MMA issuer (lane 0) and TMEM owner: QK runs two tiles ahead of P.V, so
//            softmax of one tile overlaps the tensor work of its neighbours.  P.V takes
//            P from TMEM (A operand) and V from shared memory.
// TMEM columns: S/P buffers [0,128), [128,256), [256,384) and O [384,512).  QK of tile
// j+2 is issued before P.V of tile j, into the buffer of tile j-1; tensor-core
// operations of the CTA execute in issue order, so it runs after P.V of tile j-1 has
// read P_(j-1) from those columns.



constexpr uint32_t kWsTmemCols = 512;
constexpr int kKStages = 3;                              // K ring depth
constexpr int kVStages = 2;                              // V ring depth
constexpr uint32_t kWsOffK = kOffQ + kTile;
constexpr uint32_t kWsOffV = kWsOffK + kKStages * kTile;
constexpr uint32_t kWsOffBar = kWsOffV + kVStages * kTile;  // no P tiles in shared memory
constexpr uint32_t kWsOffXch = kWsOffBar + 256;          // row-max exchange [2 parity][2 half][128]
constexpr size_t kWsSmem = kWsOffXch + 2 * 2 * 128 * 4 + 1024;  // + alignment slack
// Kernel parameters with the layer's tensor maps for the TMA variant: K as {D, Hkv,
// tokens} with box {64, 1, 16}, V as {64, tokens, 2, Hkv} with box {64, 16, 2, 1} (a
// whole 16-token page of one head per box); row_shift = log2(Hkv * D).
struct alignas(64) WsParams {
  CUtensorMap tmk;
  CUtensorMap tmv;
  PrefillParams p;
  uint32_t row_shift;
  // Pair kernel work split (1-D grid): items (qt fastest, then kv head, then sequence)
  // below n_whole run whole; each later item runs as nsplit CTAs over consecutive KV
  // ranges that write partial rows to part_o, merged by prefill_merge_kernel.
  int nqt, n_whole, nsplit;
  float *part_o;  // [split items][nsplit][256 rows][128]; then m and l: [..][256] each
};
template <bool TMA>
constexpr int ws_threads() { return TMA ? 13 * 32 : 11 * 32; }
constexpr int kSBufs = 3;  // S/P buffers in TMEM: QK of tile j+2 issues before P.V of tile j
// kSFull/kPFull: one per S buffer; kODone: one per tile parity; kPair: one per row quarter.
// Each waiter's barrier can complete at most once past the phase it waits on, so the
// parity waits are unambiguous.
// kOFinal: single use, committed after the last P.V (the epilogue's wait cannot use
// kODone: softmax may finish its last tile while P.V of tile nt-3, on the same
// barrier, is still running, and a parity wait would then pass one phase early).
enum WsBar { kQFull = 0, kKFull = 1, kKEmpty = 4, kVFull = 7, kVEmpty = 10, kSFull = 13,
             kPFull = 16, kODone = 19, kPair = 21, kOFinal = 25, kSlot = 26 };

// Page lookups for the 16-token boxes of successive KV tiles, four tiles ahead.  The
// producer warp's lanes form 4 groups of 8 (lane = 8 * group + box); group g serves
// tiles g, g+4, g+8, ...  After its tile j is issued the group loads the block ids of
// tile j+4, and two tiles later their offsets, so each dependent global load has two
// tiles of time to return.
// With 8-token pages a box spans two pages: each lane also follows the block holding
// the box's rows 8-15 (blk2 / off2) and hands out its base as e1; otherwise e1 is the
// row 8 of the same page.  TWO = false (the TMA kernels, 16-token pages only) compiles
// the second page out.
template <bool TWO>
struct BoxLookup {
  const int32_t *table;
  const uint64_t *offsets;
  int bs, kv_hi, nt, bx, grp, j, j0;
  int tile;        // tile this lane's group is gathering
  int blk, blk2;   // its block ids (-1: past the keys in use); blk2 for 8-token pages
  uint64_t off, off2;  // their block offsets (valid once loaded)
  __device__ int blk_of(int t) const {
    const int key = t * kKvTile + bx * 16;
    return (t < nt && key < kv_hi) ? table[key / bs] : -1;
  }
  __device__ int blk2_of(int t) const {
    const int key = t * kKvTile + bx * 16 + 8;
    return (TWO && bs == 8 && t < nt && key < kv_hi) ? table[key / bs] : -1;
  }
  // Tiles j0, j0 + 1, ... below nt_ (the end of the CTA's range).
  __device__ BoxLookup(const int32_t *tb, const uint64_t *of, int bs_, int kv_hi_, int nt_,
                       int lane, int j0_ = 0)
      : table(tb), offsets(of), bs(bs_), kv_hi(kv_hi_), nt(nt_), bx(lane & 7), grp(lane >> 3),
        j(j0_), j0(j0_), tile(j0_ + (lane >> 3)) {
    blk = blk_of(tile);
    blk2 = TWO ? blk2_of(tile) : -1;
    off = blk >= 0 ? offsets[blk] : 0;
    off2 = TWO && blk2 >= 0 ? offsets[blk2] : 0;
  }
  // Element offset (2-byte units) of the first token row of this lane's box (lane & 7)
  // in the next tile, from the group that holds it; false when the box lies past the
  // keys in use, or its block offset is misaligned or its 16 rows leave the region.
  // All 32 lanes must call this together.
  __device__ bool next(uint32_t row_stride, uint64_t region_elems, int64_t *e0, int64_t *e1,
                       bool *bad) {
    const int g = (j - j0) & 3;
    int64_t zz = 0, zz2 = 0;
    bool live = false;
    if (grp == g && blk >= 0) {
      zz = int64_t(off + uint64_t((j * kKvTile + bx * 16) % bs) * row_stride);
      if (TWO && bs == 8) {  // rows 0-7 in this page, rows 8-15 (if in use) in blk2's
        zz2 = int64_t(off2);
        live = (off & 7) == 0 && uint64_t(zz) + 8ull * row_stride <= region_elems &&
               (blk2 < 0 || ((off2 & 7) == 0 && off2 + 8ull * row_stride <= region_elems));
      } else {
        zz2 = zz + 8 * int64_t(row_stride);
        live = (off & 7) == 0 && uint64_t(zz) + 16ull * row_stride <= region_elems;
      }
      if (!live) *bad = true;
    }
    const int src = (g << 3) | bx;
    zz = __shfl_sync(0xffffffffu, zz, src);
    if constexpr (TWO) {
      zz2 = __shfl_sync(0xffffffffu, zz2, src);
    } else {
      zz2 = zz + 8 * int64_t(row_stride);
    }
    live = __shfl_sync(0xffffffffu, int(live), src) != 0;
    if (grp == g) {  // start gathering tile j + 4
      tile = j + 4;
      blk = blk_of(tile);
      if constexpr (TWO) blk2 = blk2_of(tile);
    }
    if (j - j0 >= 2 && grp == ((j - j0 + 2) & 3)) {  // tile j + 2
      off = blk >= 0 ? offsets[blk] : 0;
      if constexpr (TWO) off2 = blk2 >= 0 ? offsets[blk2] : 0;
    }
    ++j;
    *e0 = zz;
    *e1 = zz2;
    return live;
  }
};

// Bounded wait that also gives up as soon as another role has failed.
__device__ __forceinline__ bool ws_wait(uint32_t bar, uint32_t parity, volatile int *fail) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((n & 63) == 0) {
      if (*fail) return false;
      if (ptx::globaltimer_ns() - t0 > kLimitNs) {
        *fail = 1;
        return false;
      }
    }
  }
}

// One warp copies a 128-key tile of one kv head into the swizzled [2 halves][128
// rows][128 B] layout with 16-byte cp.async: each half-warp moves one 256-byte token
// row per step.  Box b (keys 16b .. 16b+15) has its rows 0-7 from element e0 and rows
// 8-15 from element e1 of lane b (TWO; otherwise all 16 rows from e0); keys past
// kv_hi and boxes that are not live are zero-filled.
template <bool BOXV = false, int B0 = 0, int NB = 8, bool TWO = false>
__device__ __forceinline__ void gather_tile(const uint16_t *va, uint32_t dst, int64_t e0,
                                            int64_t e1, bool live, int j, int kv_hi,
                                            uint32_t row_stride, int h, int lane) {
  const int hw = lane >> 4, c = lane & 15;
#pragma unroll
  for (int b = B0; b < B0 + NB; ++b) {
    const int64_t eb = __shfl_sync(0xffffffffu, e0, b);
    const int64_t eb1 = TWO ? __shfl_sync(0xffffffffu, e1, b) : 0;
    const bool lb = __shfl_sync(0xffffffffu, int(live), b) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 2 * i + hw, row = b * 16 + r;
      const bool ok = lb && j * kKvTile + row < kv_hi;
      const int64_t er = !TWO || i < 4 ? eb + int64_t(r) * row_stride
                                       : eb1 + int64_t(r - 8) * row_stride;
      const uint16_t *src = va + er + h * kHd + c * 8;
      ptx::cp_async16(dst + (BOXV ? swz_v(row, c) : swz(row, c)), ok ? src : va, ok ? 16u : 0u);
    }
  }
}

template <typename T, bool TMA>
__global__ void __launch_bounds__(ws_threads<TMA>(), 1)
    prefill_ws_kernel(const __grid_constant__ WsParams P) {
  const PrefillParams &p = P.p;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  unsigned char *smem = smem_raw + (sb - raw);
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = p.q_start[b];
  const int qlen = p.q_start[b + 1] - q0;
  const int ctx = p.ctx_lens[b];
  if (qt * p.tt >= qlen) return;
  if (ctx < qlen || ctx > p.max_bps * p.bs) {
    if (tid == 0) atomicOr(p.diag, int32_t(kDiagBadLaunch));
    return;
  }
  const int base_pos = ctx - qlen;
  const int ti_hi = min((qt + 1) * p.tt, qlen);
  const int kv_hi = base_pos + ti_hi;
  const int nt = (kv_hi + kKvTile - 1) / kKvTile;
  auto bar = [&](int i) { return sb + kWsOffBar + uint32_t(i) * 8; };

  if (tid == 0) {
    ptx::mbar_init(bar(kQFull), 32);
    for (int i = 0; i < kVStages; ++i) {
      // V: 32 arrivals per producer warp (cp.async noinc, or one expect_tx + 31 plain)
      ptx::mbar_init(bar(kVFull + i), TMA ? 64 : 32);
      ptx::mbar_init(bar(kVEmpty + i), 1);
    }
    for (int i = 0; i < 2; ++i) ptx::mbar_init(bar(kODone + i), 1);
    ptx::mbar_init(bar(kOFinal), 1);
    for (int i = 0; i < kSBufs; ++i) {
      ptx::mbar_init(bar(kSFull + i), 1);
      ptx::mbar_init(bar(kPFull + i), 256);
    }
    for (int i = 0; i < kKStages; ++i) {
      // K: one expect_tx per TMA producer warp, or 32 cp.async arrivals
      ptx::mbar_init(bar(kKFull + i), TMA ? 2 : 32);
      ptx::mbar_init(bar(kKEmpty + i), 1);
    }
    for (int i = 0; i < 4; ++i) ptx::mbar_init(bar(kPair + i), 64);
    ptx::fence_mbarrier_init();
    s_fail = 0;
  }
  if (warp == 9) {
    tc::tmem_alloc(bar(kSlot), kWsTmemCols);
    tc::tmem_relinquish();
    tc::fence_before_sync();
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + kWsOffBar + kSlot * 8);
  volatile int *fail = &s_fail;
  const int32_t *table = p.tables + size_t(b) * p.max_bps;
  const uint32_t row_stride = uint32_t(p.hkv) * kHd;  // elements per token row
  // Roles: warps 0-7 softmax, 8 K producer part 0 (+Q), 9 MMA, 10 V producer part 0;
  // with TMA, 11 = K part 1 and 12 = V part 1 (a part = boxes 4*part .. 4*part+3 of a
  // tile).
  const bool k_prod = warp == 8 || (TMA && warp == 11);
  const bool v_prod = warp == 10 || (TMA && warp == 12);

  if (k_prod) {
    // ---------------- K producer (warp 8 also loads Q) ----------------
    if (warp == 8) {
      for (int it = 0; it < 64; ++it) {
        const int idx = it * 32 + lane, r = idx >> 4, c = idx & 15;
        const int t_r = qt * p.tt + r / p.G, h_r = h * p.gr + r % p.G;
        const bool ok = t_r < qlen && r % p.G < p.gr;
        const uint16_t *src = ok ? p.q + (size_t(q0 + t_r) * p.hq + h_r) * kHd + c * 8 : p.q;
        ptx::cp_async16(sb + kOffQ + swz(r, c), src, ok ? 16u : 0u);
      }
      ptx::cp_async_mbar_arrive(bar(kQFull));
    }
    const int part = warp == 8 ? 0 : 1;
    if (TMA && lane == 0) ptx::prefetch_tensormap(&P.tmk);
    bool bad = false;
    BoxLookup<!TMA> lk(table, p.offsets, p.bs, kv_hi, nt, lane);
    for (int j = 0; j < nt; ++j) {
      const int st = j % kKStages;
      int64_t e0 = 0, e1 = 0;
      bool live = lk.next(row_stride, p.region_elems, &e0, &e1, &bad);
      // QK of tile j - kKStages must have finished reading this stage
      if (j >= kKStages &&
          !ws_wait(bar(kKEmpty + st), uint32_t((j / kKStages - 1) & 1), fail))
        break;
      const uint32_t dst = sb + kWsOffK + st * kTile;
      if constexpr (TMA) {
        if (live && (e0 & (row_stride - 1)) != 0) {  // not a whole token row: no TMA box
          live = false;
          bad = true;
        }
        const bool mine = ((lane & 7) >> 2) == part;
        const uint32_t lm = __ballot_sync(0xffffffffu, live && mine && lane < 8);
        if (lane == 0) ptx::mbar_arrive_expect_tx(bar(kKFull + st), uint32_t(__popc(lm)) * 4096u);
        __syncwarp();
        if (lane < 16 && live && mine) {  // lanes 8..15: second head_dim half of the boxes
          const int bx = lane & 7, half = lane >> 3;
          ptx::tma_load_3d(dst + half * kHalf + bx * 2048, &P.tmk, half * 64, h,
                           int(e0 >> P.row_shift), bar(kKFull + st));
        }
      } else {
        gather_tile<false, 0, 8, !TMA>(p.va_k, dst, e0, e1, live, j, kv_hi, row_stride, h, lane);
        ptx::cp_async_mbar_arrive(bar(kKFull + st));
      }
    }
    ptx::cp_async_wait<0>();
    if (bad) atomicOr(p.diag, int32_t(kDiagBadOffset));
  } else if (v_prod) {
    // ---------------- V producer ----------------
    const int part = warp == 10 ? 0 : 1;
    if (TMA && lane == 0) ptx::prefetch_tensormap(&P.tmv);
    bool bad = false;
    BoxLookup<!TMA> lk(table, p.offsets, p.bs, kv_hi, nt, lane);
    for (int j = 0; j < nt; ++j) {
      const int st = j % kVStages;
      int64_t e0 = 0, e1 = 0;
      bool live = lk.next(row_stride, p.region_elems, &e0, &e1, &bad);
      // P.V of tile j - kVStages must have finished reading this stage
      if (j >= kVStages &&
          !ws_wait(bar(kVEmpty + st), uint32_t((j / kVStages - 1) & 1), fail))
        break;
      const uint32_t dst = sb + kWsOffV + st * kTile;
      if constexpr (TMA) {
        const bool aligned = (e0 & (row_stride - 1)) == 0;
        const bool mine = ((lane & 7) >> 2) == part;
        const uint32_t lm = __ballot_sync(0xffffffffu, live && aligned && mine && lane < 8);
        // whole tile inside the context and all 4 boxes loadable: TMA, else zero-filling copies
        if (j * kKvTile + kKvTile <= kv_hi && __popc(lm) == 4) {
          if (lane == 0) {
            ptx::mbar_arrive_expect_tx(bar(kVFull + st), 4u * 4096u);
          } else {
            ptx::mbar_arrive(bar(kVFull + st));
          }
          __syncwarp();
          if (lane < 8 && mine) {  // one box = 16 token rows x both head_dim halves
            ptx::tma_load_4d(dst + lane * 4096, &P.tmv, 0, int(e0 >> P.row_shift), 0, h,
                             bar(kVFull + st));
          }
        } else {
          if (part == 0) {
            gather_tile<true, 0, 4, !TMA>(p.va_v, dst, e0, e1, live, j, kv_hi, row_stride, h, lane);
          } else {
            gather_tile<true, 4, 4, !TMA>(p.va_v, dst, e0, e1, live, j, kv_hi, row_stride, h, lane);
          }
          ptx::cp_async_mbar_arrive(bar(kVFull + st));
        }
      } else {
        gather_tile<true, 0, 8, !TMA>(p.va_v, dst, e0, e1, live, j, kv_hi, row_stride, h, lane);
        ptx::cp_async_mbar_arrive(bar(kVFull + st));
      }
    }
    ptx::cp_async_wait<0>();
    if (bad) atomicOr(p.diag, int32_t(kDiagBadOffset));
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    const uint32_t qa = sb + kOffQ;
    const uint32_t tO = tmem + kSBufs * 128;
    auto issue_qk = [&](int j) {
      const uint32_t ka = sb + kWsOffK + (j % kKStages) * kTile, tS = tmem + (j % kSBufs) * 128;
      if (lane == 0) {
        tc::fence_after_sync();
        ptx::fence_proxy_async_smem();  // cp.async-written K (and Q) -> tensor-core reads
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t o = uint32_t((k >> 2) * kHalf + (k & 3) * 32);
          tc::mma_ss(tS, tc::sw128_desc(qa + o, 16, 1024), tc::sw128_desc(ka + o, 16, 1024),
                     p.idesc_qk, k > 0);
        }
        tc::commit(bar(kSFull + j % kSBufs));
        tc::commit(bar(kKEmpty + j % kKStages));
      }
      __syncwarp();
    };
    bool ok = ws_wait(bar(kQFull), 0, fail) && ws_wait(bar(kKFull), 0, fail);
    if (ok) issue_qk(0);
    if (ok && nt > 1) {
      ok = ws_wait(bar(kKFull + 1), 0, fail);
      if (ok) issue_qk(1);
    }
    for (int j = 0; ok && j < nt; ++j) {
      // QK of tile j+2 goes into the buffer of tile j-1, whose P.V was issued last
      // iteration (tensor-core operations run in issue order)
      if (j + 2 < nt) {
        if (!ws_wait(bar(kKFull + (j + 2) % kKStages), uint32_t(((j + 2) / kKStages) & 1), fail))
          break;
        issue_qk(j + 2);
      }
      if (!ws_wait(bar(kPFull + j % kSBufs), uint32_t((j / kSBufs) & 1), fail)) break;
      if (!ws_wait(bar(kVFull + j % kVStages), uint32_t((j / kVStages) & 1), fail)) break;
      if (lane == 0) {
        tc::fence_after_sync();
        ptx::fence_proxy_async_smem();  // cp.async-written V -> tensor-core reads
        const uint32_t va = sb + kWsOffV + (j % kVStages) * kTile;
        const uint32_t tp = tmem + (j % kSBufs) * 128;  // P_hi columns [0,64), P_lo [64,128)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // V box k: 16 keys (K) x head_dim (N), the two halves 2048 B apart
          const uint64_t vd = tc::sw128_desc(va + uint32_t(k) * 4096, 2048, 1024);
          tc::mma_ts(tO, tp + k * 8, vd, p.idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
          tc::mma_ts(tO, tp + 64 + k * 8, vd, p.idesc_pv, 1u);
        }
        tc::commit(bar(kODone + (j & 1)));
        tc::commit(bar(kVEmpty + j % kVStages));
        if (j == nt - 1) tc::commit(bar(kOFinal));
      }
      __syncwarp();
    }
  } else if (warp < 8) {
    // ---------------- softmax warps ----------------
    const int q4 = warp & 3, hf = warp >> 2;
    const int row = q4 * 32 + lane;
    const int ti = qt * p.tt + row / p.G;
    const bool row_ok = ti < qlen;
    const int qpos = row_ok ? base_pos + ti : kv_hi - 1;
    const uint32_t lane_base = uint32_t(q4 * 32) << 16;
    const uint32_t tO = tmem + kSBufs * 128 + lane_base + hf * 64;
    float *xch = reinterpret_cast<float *>(smem + kWsOffXch);
    const uint32_t pbar = bar(kPair + q4);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (!ws_wait(bar(kSFull + j % kSBufs), uint32_t((j / kSBufs) & 1), fail)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float s[64];
      const uint32_t tS = tmem + (j % kSBufs) * 128 + lane_base;
      tc::ld32(tS + hf * 64, s);
      tc::ld32(tS + hf * 64 + 32, s + 32);
      tc::wait_ld();
      const bool need_mask = j * kKvTile + kKvTile - 1 > base_pos + qt * p.tt;
      float mx = masked_max<64>(s, j * kKvTile + hf * 64, qpos, need_mask) * p.scale_log2;
      // trade the partial row max with the warp holding the other 64 keys of the rows;
      // this also orders both warps' reads of S_j before either writes P_j over it
      xch[((j & 1) * 2 + hf) * 128 + row] = mx;
      tc::fence_before_sync();
      ptx::mbar_arrive(pbar);
      if (!ws_wait(pbar, uint32_t(j & 1), fail)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      mx = fmaxf(mx, xch[((j & 1) * 2 + (hf ^ 1)) * 128 + row]);
      float alpha;
      bool rescale;
      const float sum = exp_given_max<64>(s, mx, p.scale_log2, j > 0, m_run, alpha, rescale);
      l_run = l_run * alpha + sum;
      store_p_tmem<T, 64>(s, tS + hf * 32, tS + 64 + hf * 32);
      if (__any_sync(0xffffffffu, rescale)) {
        // O *= alpha once P.V of tile j-1 is done (P.V of tile j waits for this
        // tile's P, so it cannot have run)
        if (!ws_wait(bar(kODone + ((j - 1) & 1)), uint32_t(((j - 1) >> 1) & 1), fail)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        scale_o_row<64>(tO, rescale ? alpha : 1.f);
      }
      tc::fence_before_sync();
      ptx::mbar_arrive(bar(kPFull + j % kSBufs));
    }
    // row sum = both halves' partial sums (same running max in both warps)
    if (ok) {
      xch[((nt & 1) * 2 + hf) * 128 + row] = l_run;
      ptx::mbar_arrive(pbar);
      if (ws_wait(pbar, uint32_t(nt & 1), fail)) {
        l_run += xch[((nt & 1) * 2 + (hf ^ 1)) * 128 + row];
      } else {
        ok = false;
      }
    }
    // every P.V done
    if (ok && ws_wait(bar(kOFinal), 0, fail)) {
      tc::fence_after_sync();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint16_t *dst = p.out + (size_t(q0 + ti) * p.hq + h * p.gr + row % p.G) * kHd + hf * 64;
      store_o_row<T, 64>(tO, inv, dst, row_ok && row % p.G < p.gr);  // idle rows: no store
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (s_fail && tid == 0) atomicOr(p.diag, int32_t(kDiagWaitTimeout));
  if (warp == 9) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kWsTmemCols);
  }
}

// --- two query tiles per CTA: the pair kernel (the default) ------------------------------
//
// A CTA owns 256 query rows of one kv head: tile 0 = rows 0-127, tile 1 = rows 128-255
// (row = token * G + head, as above), so every K/V tile that crosses from L2 feeds both
// tiles' MMAs: half the TMA boxes per FLOP of prefill_ws_kernel.
// warps 0-3  softmax of tile 0, warps 4-7 softmax of tile 1: one thread per row, all
//            128 keys of a KV tile (warp w reads its TMEM lane quarter w % 4)
// warp 8     Q (both tiles), then K boxes 0-3 of every KV tile (all 8 without TMA)
// warp 9     MMA issuer and TMEM owner
// warp 10    V (all 8 page boxes of a tile)
// warp 11    K boxes 4-7 (TMA variant; idle otherwise)
// TMEM: S/P of tile 0 [0,128), S/P of tile 1 [128,256), O of tile 0 [256,384), O of
// tile 1 [384,512).  Per KV tile j the issue order is
//   P.V(0, j), QK(0, j+1), P.V(1, j), QK(1, j+1)
// so the tensor pipe works on one tile while the other tile's softmax runs.  QK(x, j+1)
// overwrites S/P of tile x after P.V(x, j) read it (tensor-core operations of a CTA
// execute in issue order), and its completion also covers P.V(x, j), so the softmax
// may rescale O(x) as soon as S(x, j+1) is ready.
// P_lo: a single rounding of P to 16 bits leaves a relative error of up to 2^-9 per
// weight.  Over a row with many comparable weights the errors average out; over few
// dominant weights (short rows, peaked rows, cancelling values) they do not.  Each
// softmax thread bounds its row's tile: with s2 = sum(P^2) over the tile and L the
// running sum including it, sqrt(s2) <= L / 64 keeps the tile's rounding error
// (standard deviation) within about 2^-9 / sqrt(3) / 64 of the largest |v|.  s2 is
// bounded by max(P) * sum(P), both known without a pass over the values.  A warp with a
// row above the bound marks the tile and stores its rows' P_lo; the other warps store
// zeros in the P_lo columns, so a marked tile's P_lo MMAs see P_lo where it is needed
// and nothing elsewhere, and an unmarked tile runs no P_lo MMAs.  On a long context
// only the first few KV tiles of every row are marked.
constexpr int kPrThreads = 12 * 32;
constexpr int kPrKStages = 3;
constexpr int kPrVStages = 2;
constexpr uint32_t kPrOffQ = 0;  // two Q tiles
constexpr uint32_t kPrOffK = 2 * kTile;
constexpr uint32_t kPrOffV = kPrOffK + kPrKStages * kTile;
constexpr uint32_t kPrOffBar = kPrOffV + kPrVStages * kTile;
constexpr size_t kPrSmem = kPrOffBar + 256 + 1024;  // barriers and flags + alignment slack
constexpr float kLoTau2 = 1.0f / 4096.0f;            // (1/64)^2
// Register split of the pair kernel: the launch gives every thread kPrLaunchRegs
// (__launch_bounds__(384, 1)); the softmax warpgroups then take kPrSoftmaxRegs and the
// producer / MMA warpgroup keeps kPrOtherRegs.  setmaxnreg.inc waits until the
// warpgroup's registers are free in the CTA's pool, so the split must not exceed the
// pool: 256 * 208 + 128 * 80 = 63,488 <= 384 * 168 = 64,512.  The launcher checks the
// compiled kernel's register count against it before every launch.
constexpr int kPrLaunchRegs = 168;
constexpr int kPrSoftmaxRegs = 208;
constexpr int kPrOtherRegs = 80;
static_assert(256 * kPrSoftmaxRegs + 128 * kPrOtherRegs <= kPrThreads * kPrLaunchRegs,
              "register split exceeds the launch pool");
enum PrBar { kPrQFull = 0, kPrKFull = 1, kPrKEmpty = 4, kPrVFull = 7, kPrVEmpty = 9,
             kPrSFull = 11, kPrPFull = 13, kPrOFinal = 15, kPrSlot = 17, kPrLoFlags = 18 };

template <typename T, bool TMA>
__global__ void __launch_bounds__(kPrThreads, 1)
    prefill_pair_kernel(const __grid_constant__ WsParams P) {
  const PrefillParams &p = P.p;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  unsigned char *smem = smem_raw + (sb - raw);
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Work item of this CTA, and for the split tail its part.
  const int lin = int(blockIdx.x);
  const bool split = lin >= P.n_whole;
  const int item = split ? P.n_whole + (lin - P.n_whole) / P.nsplit : lin;
  const int part = split ? (lin - P.n_whole) % P.nsplit : 0;
  // Query tiles run last-first: under the causal mask the last tile of a chunk attends
  // the most keys, so the longest items start first and the short ones fill the tail.
  const int qt = P.nqt - 1 - item % P.nqt, h = (item / P.nqt) % p.hkv,
            b = item / (P.nqt * p.hkv);
  const int tt = 2 * p.tt;  // tokens per CTA (p.tt per tile)
  const int q0 = p.q_start[b];
  const int qlen = p.q_start[b + 1] - q0;
  const int ctx = p.ctx_lens[b];
  if (qt * tt >= qlen) return;
  if (ctx < qlen || ctx > p.max_bps * p.bs) {
    if (tid == 0) atomicOr(p.diag, int32_t(kDiagBadLaunch));
    return;
  }
  const int base_pos = ctx - qlen;
  const int ti_hi = min((qt + 1) * tt, qlen);
  const int kv_hi = base_pos + ti_hi;
  const int nt = (kv_hi + kKvTile - 1) / kKvTile;
  // KV tiles [j_lo, j_hi) of this CTA.  Every part of a split item but the last ends at
  // or below the CTA's first query row, so its rows see no causal mask, and the last
  // part (which holds the diagonal) gives every row at least one key.
  int j_lo = 0, j_hi = nt;
  float *part_o = nullptr, *part_m = nullptr, *part_l = nullptr;
  if (split) {
    const int cap = (base_pos + qt * tt) / kKvTile;
    auto bound = [&](int k) { return k >= P.nsplit ? nt : min(k * nt / P.nsplit, cap); };
    j_lo = bound(part);
    j_hi = bound(part + 1);
    const size_t slot = size_t(item - P.n_whole) * P.nsplit + part;
    const size_t n_slots = size_t(gridDim.x - P.n_whole);
    part_o = P.part_o + slot * 256 * kHd;
    part_m = P.part_o + n_slots * 256 * kHd + slot * 256;
    part_l = part_m + n_slots * 256;
    if (j_hi == j_lo) {  // nothing below the first row: the part carries no weight
      for (int r = tid; r < 256; r += kPrThreads) part_l[r] = 0.f;
      return;
    }
  }
  const int n_loc = j_hi - j_lo;  // this CTA's tiles; loop counters below run over them
  auto bar = [&](int i) { return sb + kPrOffBar + uint32_t(i) * 8; };
  volatile int *lo_flag = reinterpret_cast<volatile int *>(smem + kPrOffBar + kPrLoFlags * 8);

  if (tid == 0) {
    ptx::mbar_init(bar(kPrQFull), 32);
    for (int i = 0; i < kPrKStages; ++i) {
      ptx::mbar_init(bar(kPrKFull + i), TMA ? 2 : 32);
      ptx::mbar_init(bar(kPrKEmpty + i), 1);
    }
    for (int i = 0; i < kPrVStages; ++i) {
      ptx::mbar_init(bar(kPrVFull + i), 32);
      ptx::mbar_init(bar(kPrVEmpty + i), 1);
    }
    for (int x = 0; x < 2; ++x) {
      ptx::mbar_init(bar(kPrSFull + x), 1);
      ptx::mbar_init(bar(kPrPFull + x), 128);
      ptx::mbar_init(bar(kPrOFinal + x), 1);
    }
    for (int i = 0; i < 8; ++i) lo_flag[i] = -1;  // [tile][j % 4] = j when tile j needs P_lo
    ptx::fence_mbarrier_init();
    s_fail = 0;
  }
  if (warp == 9) {
    tc::tmem_alloc(bar(kPrSlot), kWsTmemCols);
    tc::tmem_relinquish();
    tc::fence_before_sync();
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + kPrOffBar + kPrSlot * 8);
  volatile int *fail = &s_fail;
  const int32_t *table = p.tables + size_t(b) * p.max_bps;
  const uint32_t row_stride = uint32_t(p.hkv) * kHd;  // elements per token row
  if (warp >= 8) {
  // producer / MMA warpgroup: gives registers back to the softmax warpgroups
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPrOtherRegs));
  if (warp == 8 || (TMA && warp == 11)) {
    // ---------------- K producers (warp 8 loads Q first) ----------------
    if (warp == 8) {
      for (int it = 0; it < 128; ++it) {
        const int idx = it * 32 + lane, r = idx >> 4, c = idx & 15;  // r: CTA row 0..255
        const int t_r = qt * tt + r / p.G, h_r = h * p.gr + r % p.G;
        const bool ok = t_r < qlen && r % p.G < p.gr;
        const uint16_t *src = ok ? p.q + (size_t(q0 + t_r) * p.hq + h_r) * kHd + c * 8 : p.q;
        ptx::cp_async16(sb + kPrOffQ + uint32_t(r >> 7) * kTile + swz(r & 127, c), src,
                        ok ? 16u : 0u);
      }
      ptx::cp_async_mbar_arrive(bar(kPrQFull));
    }
    const int part = warp == 8 ? 0 : 1;
    if (TMA && lane == 0) ptx::prefetch_tensormap(&P.tmk);
    bool bad = false;
    BoxLookup<!TMA> lk(table, p.offsets, p.bs, kv_hi, j_hi, lane, j_lo);
    for (int jj = 0; jj < n_loc; ++jj) {
      const int j = j_lo + jj, st = jj % kPrKStages;
      int64_t e0 = 0, e1 = 0;
      bool live = lk.next(row_stride, p.region_elems, &e0, &e1, &bad);
      // both tiles' QK of tile jj - kPrKStages must have finished reading this stage
      if (jj >= kPrKStages &&
          !ws_wait(bar(kPrKEmpty + st), uint32_t((jj / kPrKStages - 1) & 1), fail))
        break;
      const uint32_t dst = sb + kPrOffK + st * kTile;
      if constexpr (TMA) {
        if (live && (e0 & (row_stride - 1)) != 0) {  // not a whole token row: no TMA box
          live = false;
          bad = true;
        }
        const bool mine = ((lane & 7) >> 2) == part;
        const uint32_t lm = __ballot_sync(0xffffffffu, live && mine && lane < 8);
        if (lane == 0) ptx::mbar_arrive_expect_tx(bar(kPrKFull + st), uint32_t(__popc(lm)) * 4096u);
        __syncwarp();
        if (lane < 16 && live && mine) {  // lanes 8..15: second head_dim half of the boxes
          const int bx = lane & 7, half = lane >> 3;
          ptx::tma_load_3d(dst + half * kHalf + bx * 2048, &P.tmk, half * 64, h,
                           int(e0 >> P.row_shift), bar(kPrKFull + st));
        }
      } else {
        gather_tile<false, 0, 8, !TMA>(p.va_k, dst, e0, e1, live, j, kv_hi, row_stride, h, lane);
        ptx::cp_async_mbar_arrive(bar(kPrKFull + st));
      }
    }
    ptx::cp_async_wait<0>();
    if (bad) atomicOr(p.diag, int32_t(kDiagBadOffset));
  } else if (warp == 10) {
    // ---------------- V producer ----------------
    if (TMA && lane == 0) ptx::prefetch_tensormap(&P.tmv);
    bool bad = false;
    BoxLookup<!TMA> lk(table, p.offsets, p.bs, kv_hi, j_hi, lane, j_lo);
    for (int jj = 0; jj < n_loc; ++jj) {
      const int j = j_lo + jj, st = jj % kPrVStages;
      int64_t e0 = 0, e1 = 0;
      bool live = lk.next(row_stride, p.region_elems, &e0, &e1, &bad);
      // both tiles' P.V of tile jj - kPrVStages must have finished reading this stage
      if (jj >= kPrVStages &&
          !ws_wait(bar(kPrVEmpty + st), uint32_t((jj / kPrVStages - 1) & 1), fail))
        break;
      const uint32_t dst = sb + kPrOffV + st * kTile;
      bool boxes = false;
      if constexpr (TMA) {
        const bool aligned = (e0 & (row_stride - 1)) == 0;
        const uint32_t lm = __ballot_sync(0xffffffffu, live && aligned && lane < 8);
        // whole tile inside the context and all 8 boxes loadable: TMA, else zero-filling copies
        boxes = j * kKvTile + kKvTile <= kv_hi && __popc(lm) == 8;
      }
      if (boxes) {
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(bar(kPrVFull + st), 8u * 4096u);
        } else {
          ptx::mbar_arrive(bar(kPrVFull + st));
        }
        __syncwarp();
        if (lane < 8) {  // one box = 16 token rows x both head_dim halves
          ptx::tma_load_4d(dst + lane * 4096, &P.tmv, 0, int(e0 >> P.row_shift), 0, h,
                           bar(kPrVFull + st));
        }
      } else {
        gather_tile<true, 0, 8, !TMA>(p.va_v, dst, e0, e1, live, j, kv_hi, row_stride, h, lane);
        ptx::cp_async_mbar_arrive(bar(kPrVFull + st));
      }
    }
    ptx::cp_async_wait<0>();
    if (bad) atomicOr(p.diag, int32_t(kDiagBadOffset));
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    auto issue_qk = [&](int x, int j) {
      const uint32_t qa = sb + kPrOffQ + uint32_t(x) * kTile;
      const uint32_t ka = sb + kPrOffK + (j % kPrKStages) * kTile;
      const uint32_t tS = tmem + uint32_t(x) * 128;
      if (lane == 0) {
        tc::fence_after_sync();
        ptx::fence_proxy_async_smem();  // cp.async-written K (and Q) -> tensor-core reads
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t o = uint32_t((k >> 2) * kHalf + (k & 3) * 32);
          tc::mma_ss(tS, tc::sw128_desc(qa + o, 16, 1024), tc::sw128_desc(ka + o, 16, 1024),
                     p.idesc_qk, k > 0);
        }
        tc::commit(bar(kPrSFull + x));
      }
      __syncwarp();
    };
    auto issue_pv = [&](int x, int j) {
      if (lane == 0) {
        tc::fence_after_sync();
        ptx::fence_proxy_async_smem();  // cp.async-written V -> tensor-core reads
        const uint32_t va = sb + kPrOffV + (j % kPrVStages) * kTile;
        const uint32_t tp = tmem + uint32_t(x) * 128;  // P_hi columns [0,64), P_lo [64,128)
        const uint32_t tO = tmem + 256 + uint32_t(x) * 128;
        const bool lo = lo_flag[x * 4 + (j & 3)] == j;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // V box k: 16 keys (K) x head_dim (N), the two halves 2048 B apart
          const uint64_t vd = tc::sw128_desc(va + uint32_t(k) * 4096, 2048, 1024);
          tc::mma_ts(tO, tp + k * 8, vd, p.idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        if (lo) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint64_t vd = tc::sw128_desc(va + uint32_t(k) * 4096, 2048, 1024);
            tc::mma_ts(tO, tp + 64 + k * 8, vd, p.idesc_pv, 1u);
          }
        }
        if (j == n_loc - 1) tc::commit(bar(kPrOFinal + x));
      }
      __syncwarp();
    };
    bool ok = ws_wait(bar(kPrQFull), 0, fail) && ws_wait(bar(kPrKFull), 0, fail);
    if (ok) {
      issue_qk(0, 0);
      issue_qk(1, 0);
      if (lane == 0) tc::commit(bar(kPrKEmpty));
      __syncwarp();
    }
    for (int j = 0; ok && j < n_loc; ++j) {  // j: this CTA's tile index (from j_lo)
      const uint32_t ph = uint32_t(j & 1);
      if (!ws_wait(bar(kPrPFull), ph, fail)) break;
      if (!ws_wait(bar(kPrVFull + j % kPrVStages), uint32_t((j / kPrVStages) & 1), fail)) break;
      issue_pv(0, j);
      const bool more = j + 1 < n_loc;
      if (more) {
        if (!ws_wait(bar(kPrKFull + (j + 1) % kPrKStages), uint32_t(((j + 1) / kPrKStages) & 1),
                     fail))
          break;
        issue_qk(0, j + 1);
      }
      if (!ws_wait(bar(kPrPFull + 1), ph, fail)) break;
      issue_pv(1, j);
      if (lane == 0) tc::commit(bar(kPrVEmpty + j % kPrVStages));
      __syncwarp();
      if (more) {
        issue_qk(1, j + 1);
        if (lane == 0) tc::commit(bar(kPrKEmpty + (j + 1) % kPrKStages));
        __syncwarp();
      }
    }
  }
  } else {
    // ---------------- softmax warps ----------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPrSoftmaxRegs));
    const int x = warp >> 2, q4 = warp & 3;
    const int row = q4 * 32 + lane;           // TMEM lane = row of tile x
    const int crow = x * 128 + row;           // row of the CTA
    const int ti = qt * tt + crow / p.G;
    const bool row_ok = ti < qlen;
    const int qpos = row_ok ? base_pos + ti : kv_hi - 1;
    const uint32_t lane_base = uint32_t(q4 * 32) << 16;
    const uint32_t tS = tmem + uint32_t(x) * 128 + lane_base;
    const uint32_t tO = tmem + 256 + uint32_t(x) * 128 + lane_base;
    const int first_pos = base_pos + qt * tt + x * p.tt;  // position of the tile's first row
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_loc; ++j) {  // j: this CTA's tile index, key tile j_lo + j
      if (!ws_wait(bar(kPrSFull + x), uint32_t(j & 1), fail)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::ld32(tS + 32 * c, s + 32 * c);
      tc::wait_ld();
      const int k0 = (j_lo + j) * kKvTile;
      const bool need_mask = k0 + kKvTile - 1 > first_pos;
      const float mx = masked_max<128>(s, k0, qpos, need_mask) * p.scale_log2;
      float alpha;
      bool rescale;
      const float sum = exp_given_max<128>(s, mx, p.scale_log2, j > 0, m_run, alpha, rescale);
      l_run = l_run * alpha + sum;
      // sum(P^2) <= max(P) * sum(P), with max(P) = 2^(mx - m_run) from the tile's max
      const float pmax = ptx::fast_exp2(mx - m_run);
      // A warp whose rows need P_lo marks the tile and stores it; the others store
      // zeros there, which is what skipping P_lo gives their rows if another warp's
      // rows make the tile run its P_lo MMAs.
      // The bound is loose on flat rows (max(P) is several times the mean), so a warp
      // that fails it evaluates sum(P^2) itself before marking the tile.
      bool mark = __any_sync(0xffffffffu, pmax * sum > kLoTau2 * l_run * l_run);
      if (mark) {
        float q2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 128; ++c) q2[c & 3] = fmaf(s[c], s[c], q2[c & 3]);
        const float s2 = (q2[0] + q2[1]) + (q2[2] + q2[3]);
        mark = __any_sync(0xffffffffu, s2 > kLoTau2 * l_run * l_run);
      }
      if (mark) {
        if (lane == 0) lo_flag[x * 4 + (j & 3)] = j;
        store_p_row128<T>(s, tS, tS + 64);
      } else {
        store_p_hi128<T>(s, tS);
        const uint32_t z[16] = {};
#pragma unroll
        for (int part = 0; part < 4; ++part) tc::st16u(tS + 64 + 16 * part, z);
        tc::wait_st();
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // O(x) *= alpha: P.V(x, j-1) completed before S(x, j) (same issuer, in order)
        scale_o_row<128>(tO, rescale ? alpha : 1.f);
      }
      tc::fence_before_sync();
      ptx::mbar_arrive(bar(kPrPFull + x));
    }
    if (ok && ws_wait(bar(kPrOFinal + x), 0, fail)) {
      tc::fence_after_sync();
      if (split) {  // unnormalised O with the row's running max and sum, for the merge
        store_o_row_f32(tO, part_o + size_t(crow) * kHd);
        part_m[crow] = m_run;
        part_l[crow] = l_run;
      } else {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        uint16_t *dst = p.out + (size_t(q0 + ti) * p.hq + h * p.gr + crow % p.G) * kHd;
        store_o_row<T, 128>(tO, inv, dst, row_ok && crow % p.G < p.gr);  // idle rows: no store
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (s_fail && tid == 0) atomicOr(p.diag, int32_t(kDiagWaitTimeout));
  if (warp == 9) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kWsTmemCols);
  }
}

// Merge of the split tail: one warp per CTA row of a split item, 4 head-dim columns a
// lane.  Each part holds its rows' unnormalised O, running max m (log2 units) and sum l;
// a part with l = 0 saw no key and carries no weight (its O is not read).
//   out = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p,  M = max over parts with l_p > 0
template <typename T>
__global__ void __launch_bounds__(256) prefill_merge_kernel(const __grid_constant__ WsParams P) {
  const PrefillParams &p = P.p;
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
  const int n_items = int((gridDim.x * 8) / 256);
  const int r = int(blockIdx.x) * 8 + warp;  // row over all split items
  const int si = r / 256, crow = r % 256;
  const int item = P.n_whole + si;
  const int qt = P.nqt - 1 - item % P.nqt, h = (item / P.nqt) % p.hkv,
            b = item / (P.nqt * p.hkv);  // the pair kernel's item order
  const int q0 = p.q_start[b];
  const int qlen = p.q_start[b + 1] - q0;
  const int ti = qt * 2 * p.tt + crow / p.G;
  if (ti >= qlen || crow % p.G >= p.gr) return;
  const size_t n_slots = size_t(n_items) * P.nsplit;
  const float *om = P.part_o + n_slots * 256 * kHd;
  const float *ol = om + n_slots * 256;
  float M = -INFINITY;
  for (int k = 0; k < P.nsplit; ++k) {
    const size_t slot = size_t(si) * P.nsplit + k;
    if (ol[slot * 256 + crow] > 0.f) M = fmaxf(M, om[slot * 256 + crow]);
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float L = 0.f;
  for (int k = 0; k < P.nsplit; ++k) {
    const size_t slot = size_t(si) * P.nsplit + k;
    const float l = ol[slot * 256 + crow];
    if (!(l > 0.f)) continue;
    const float w = exp2f(om[slot * 256 + crow] - M);
    const float4 o =
        *reinterpret_cast<const float4 *>(P.part_o + (slot * 256 + crow) * kHd + lane * 4);
    acc.x += w * o.x;
    acc.y += w * o.y;
    acc.z += w * o.z;
    acc.w += w * o.w;
    L += w * l;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint2 v;
  v.x = pack2<T>(acc.x * inv, acc.y * inv);
  v.y = pack2<T>(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2 *>(p.out + (size_t(q0 + ti) * p.hq + h * p.gr + crow % p.G) * kHd +
                             lane * 4) = v;
}

}  // namespace

static int prefill_sm_count() {
  static int counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

namespace {

using OneRoleFn = void (*)(const PrefillParams);

// The single-role kernel for head_dim d: padded to the next multiple of 64, with
// 64-key tiles above 128 so that Q, two K/V stages and P fit in shared memory.
template <typename T>
bool pick_one_role(int d, OneRoleFn *fn, size_t *smem) {
  if (d <= 0 || d > 256 || d % 8 != 0) return false;
  if (d <= 64) {
    *fn = prefill_kernel<T, 64, one_role_kt(64)>;
    *smem = OneRole<64, one_role_kt(64)>::kSmem;
  } else if (d <= 128) {
    *fn = prefill_kernel<T, 128, one_role_kt(128)>;
    *smem = OneRole<128, one_role_kt(128)>::kSmem;
  } else if (d <= 192) {
    *fn = prefill_kernel<T, 192, one_role_kt(192)>;
    *smem = OneRole<192, one_role_kt(192)>::kSmem;
  } else {
    *fn = prefill_kernel<T, 256, one_role_kt(256)>;
    *smem = OneRole<256, one_role_kt(256)>::kSmem;
  }
  return true;
}

}  // namespace

cudaError_t paged_prefill(const PrefillArgs &a, cudaStream_t stream) {
  if (a.head_dim <= 0 || a.head_dim > 256 || a.head_dim % 8 != 0 || a.kv_heads <= 0 ||
      a.num_q_heads % a.kv_heads != 0)
    return cudaErrorInvalidValue;
  const int G = a.num_q_heads / a.kv_heads;
  if (G < 1 || G > kRows) return cudaErrorInvalidValue;
  // A CTA's rows are (token, head) pairs, token = row / Gp: a group that does not divide
  // the 128 rows is padded to the next power of two, its extra rows idle (zero queries,
  // never stored), e.g. 7 query heads per kv head run as 8.
  int Gp = 1;
  while (Gp < G) Gp *= 2;
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.out)) & 15)
    return cudaErrorInvalidValue;
  if (a.batch <= 0 || a.max_q_len <= 0) return cudaSuccess;
  PrefillParams p;
  p.q = static_cast<const uint16_t *>(a.q);
  p.out = static_cast<uint16_t *>(a.out);
  p.tables = a.block_tables;
  p.q_start = a.query_start;
  p.ctx_lens = a.context_lens;
  p.offsets = a.block_offsets;
  p.va_k = static_cast<const uint16_t *>(a.va_k);
  p.va_v = static_cast<const uint16_t *>(a.va_v);
  p.region_elems = a.region_elems;
  p.hq = a.num_q_heads;
  p.hkv = a.kv_heads;
  p.G = Gp;
  p.gr = G;
  p.bs = a.block_size;
  p.max_bps = a.max_blocks_per_seq;
  p.tt = kRows / Gp;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  const bool bf16 = a.dtype == Dtype::BF16;
  p.idesc_qk = tc::idesc_f16(bf16, 128, 128, false, false);
  p.idesc_pv = tc::idesc_f16(bf16, 128, 128, false, true);
  p.diag = a.diag;
  p.d = a.head_dim;
  dim3 grid((a.max_q_len + p.tt - 1) / p.tt, a.kv_heads, a.batch);
  // the single-role kernel: S = 128 x KT, O = 128 x DP
  auto one_role = [&]() -> cudaError_t {
    OneRoleFn fn;
    size_t smem;
    const bool ok = bf16 ? pick_one_role<__nv_bfloat16>(a.head_dim, &fn, &smem)
                         : pick_one_role<__half>(a.head_dim, &fn, &smem);
    if (!ok) return cudaErrorInvalidValue;
    const int dp = (a.head_dim + 63) / 64 * 64, kt = one_role_kt(dp);
    PrefillParams q = p;
    q.idesc_qk = tc::idesc_f16(bf16, 128, kt, false, false);
    q.idesc_pv = tc::idesc_f16(bf16, 128, dp, false, true);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    fn<<<grid, kOneRoleThreads, smem, stream>>>(q);
    return cudaGetLastError();
  };
  if (a.head_dim != kHd) return one_role();
  // The warp-specialised kernels gather 16-token boxes: block_size a multiple of 16, or 8
  // (a box over two pages).  Otherwise (or with KCMM_PREFILL_IMPL=cpasync) the
  // single-role kernel runs.
  const char *impl = std::getenv("KCMM_PREFILL_IMPL");
  const bool single = impl && std::strcmp(impl, "cpasync") == 0;
  const bool gather = impl && std::strcmp(impl, "gather") == 0;
  if ((a.block_size % 16 == 0 || a.block_size == 8) && !single) {
    // TMA boxes address 16 whole token rows of the {D, Hkv, tokens} view: pages of a
    // multiple of 16 tokens, and Hkv * D a power of two dividing the 2 MiB superblock
    // (1 Mi elements).  8-token pages take the copy-gather producers (two pages a box).
    const uint32_t rs = uint32_t(a.kv_heads) * kHd;
    const bool tma = !gather && a.block_size % 16 == 0 && a.tensor_maps && a.v_page_map &&
                     (rs & (rs - 1)) == 0 && (1u << 20) % rs == 0;
    WsParams wp;
    std::memset(static_cast<void *>(&wp), 0, sizeof(wp));
    wp.p = p;
    wp.row_shift = uint32_t(__builtin_ctz(rs));
    if (tma) {
      std::memcpy(&wp.tmk, a.tensor_maps, sizeof(CUtensorMap));
      std::memcpy(&wp.tmv, a.v_page_map, sizeof(CUtensorMap));
    }
    const bool ws = impl && std::strcmp(impl, "ws") == 0;
    auto pfn = tma ? (bf16 ? prefill_pair_kernel<__nv_bfloat16, true>
                           : prefill_pair_kernel<__half, true>)
                   : (bf16 ? prefill_pair_kernel<__nv_bfloat16, false>
                           : prefill_pair_kernel<__half, false>);
    // the pair kernel's register split needs the launch register count it was built
    // for (a smaller pool would leave setmaxnreg.inc waiting): otherwise the one-tile kernel
    cudaFuncAttributes fa;
    const bool regs_ok = cudaFuncGetAttributes(&fa, pfn) == cudaSuccess &&
                         fa.numRegs * kPrThreads >= 256 * kPrSoftmaxRegs + 128 * kPrOtherRegs;
    if (!ws && regs_ok) {  // two query tiles per CTA (prefill_pair_kernel)
      auto fn = pfn;
      cudaError_t e =
          cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPrSmem));
      if (e != cudaSuccess) return e;
      // One CTA per SM: the items past the last whole wave run split over their KV range
      // into up to 4 parts, so the tail fills the SMs instead of leaving them half idle.
      const int nqt = (a.max_q_len + 2 * p.tt - 1) / (2 * p.tt);
      const int items = nqt * a.kv_heads * a.batch;
      const int sms = prefill_sm_count();
      const int rem = items % sms;
      const char *sp = std::getenv("KCMM_PREFILL_SPLIT");
      int nsplit = 1;
      if (rem > 0 && !(sp && std::strcmp(sp, "0") == 0)) nsplit = std::min(4, sms / rem);
      float *part = nullptr;
      if (nsplit > 1) {
        const size_t bytes = size_t(rem) * nsplit * 256 * (kHd + 2) * sizeof(float);
        part = static_cast<float *>(stream_scratch(stream, bytes));
        if (!part) nsplit = 1;  // no per-stream buffer (e.g. under graph capture)
      }
      wp.nqt = nqt;
      wp.nsplit = nsplit;
      wp.n_whole = nsplit > 1 ? items - rem : items;
      wp.part_o = part;
      const int ctas = wp.n_whole + (items - wp.n_whole) * nsplit;
      fn<<<ctas, kPrThreads, kPrSmem, stream>>>(wp);
      e = cudaGetLastError();
      if (e != cudaSuccess || nsplit == 1) return e;
      auto mfn = bf16 ? prefill_merge_kernel<__nv_bfloat16> : prefill_merge_kernel<__half>;
      mfn<<<(items - wp.n_whole) * 256 / 8, 256, 0, stream>>>(wp);
      return cudaGetLastError();
    }
    auto fn = tma ? (bf16 ? prefill_ws_kernel<__nv_bfloat16, true> : prefill_ws_kernel<__half, true>)
                  : (bf16 ? prefill_ws_kernel<__nv_bfloat16, false> : prefill_ws_kernel<__half, false>);
    cudaError_t e =
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kWsSmem));
    if (e != cudaSuccess) return e;
    fn<<<grid, tma ? ws_threads<true>() : ws_threads<false>(), kWsSmem, stream>>>(wp);
    return cudaGetLastError();
  }
  return one_role();
}

}  // namespace dev
}  // namespace kcmm
