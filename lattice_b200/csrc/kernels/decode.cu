// Paged decode attention for sm_100a.
//
// Computes, for every sequence b and query head h (ref
// src/cuda/kernels/kcmm_vllm_paged_attn.cu:40-101 is the scalar original):
//   out[b,h,:] = sum_t softmax_t(scale * q[b,h,:] . k_t) v_t,  t < seq_lens[b]
// with k_t / v_t at va_{k,v} + offsets[table[b][t/bs]] + (t%bs)*Hkv*D + kvh*D
// and kvh = h*Hkv/Hq.  seq_lens[b] <= 0 leaves out[b] untouched.
//
// B200 design (the path is HBM-bound: ~4 FLOP per byte):
//   * work item = (sequence, kv head, <=16 query heads of its group, split of
//     the context).  All query heads of a GQA group share one CTA, so each KV
//     page is read from HBM once per group.
//   * the context is cut into 16-token units.  The 32 lanes of a warp issue the
//     unit's K and V rows as 16-byte cp.async copies into a padded shared-memory
//     tile (rows past the context zero-filled); each lane arrives on the stage's
//     mbarrier when its copies land.  Each warp runs its own NS-deep ring, so
//     ~W*NS units (W*NS*8.7 KB at D=128) are in flight per CTA.  One
//     cp.async.bulk per row instead (lane r copies row r, lane 0 arms the
//     mbarrier with the unit's bytes) ran 33% slower on the Llama-3-8B decode
//     shape on B200 (151.8 against 114.2 us per call): 256-byte bulk copies
//     cost the TMA engine more per byte than the LSU path.
//   * QK^T and PV run on the tensor pipe (m16n8k16, fp32 accumulate) from
//     ldmatrix'd tiles: this keeps the issue slots per byte far below the HBM
//     rate; softmax is online, in the log2 domain, with warp shuffles.
//   * warps of a CTA merge in shared memory; splits of a sequence merge in a
//     second pass through their log-sum-exp.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include "../launch.hpp"
#include "pdl.cuh"
#include "ptx.cuh"

namespace kcmm {
namespace dev {
namespace {

constexpr int kUnit = 16;            // tokens per pipeline unit
constexpr int kWarps = 4;            // warps per decode CTA
constexpr int kStages = 3;           // depth of each warp's unit ring
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // a KV unit that has not landed in 1 s
                                                  // is reported, never waited on forever

struct DecodeParams {
  const void *q;
  void *out;
  const int32_t *tables;
  const int32_t *seq_lens;
  const uint64_t *offsets;
  const void *va_k;
  const void *va_v;
  uint64_t region_elems;
  int batch, hq, hkv, bs, max_bps;
  float scale_log2;
  int units_per_split, num_splits, n_head_tiles;
  float *part_o;
  float *part_lse;
  int32_t *diag;
  // Element strides: q and out rows are q + b*q_sb + h*q_sh (head_dim contiguous),
  // block-table rows tables + b*bt_stride.  Dense: (hq*D, D), (hq*D, D), max_bps.
  int64_t q_sb, q_sh, o_sb, o_sh;
  int64_t bt_stride;
};

__device__ __forceinline__ int ceil_div_dev(int a, int b) { return (a + b - 1) / b; }

__device__ __forceinline__ void head_range(int kvh, int ht, int hq, int hkv, int *lo, int *hi) {
  // query heads h with h*hkv/hq == kvh form [ceil(kvh*hq/hkv), ceil((kvh+1)*hq/hkv))
  int g_lo = int((int64_t(kvh) * hq + hkv - 1) / hkv);
  int g_hi = int((int64_t(kvh + 1) * hq + hkv - 1) / hkv);
  *lo = g_lo + ht * 16;
  *hi = min(g_hi, *lo + 16);
}

// Shared-prefix (cascade) decode: sequences in batch order form groups
// [group_starts[g], group_starts[g+1]) whose first prefix_lens[g] tokens are the
// same pages (beams of one request, or requests on one system prompt).  The
// prefix is attended once per group with all members' query rows stacked in the
// CTA's 16 rows (members_per_tile = 16 / G members per tile, tiles_per_group
// tiles), each member's own tokens by a second kind of CTA, and the two sets of
// partials merge through their log-sum-exp.
struct CascadeParams {
  const int32_t *group_starts;  // [n_groups + 1]
  const int32_t *prefix_lens;   // [n_groups], tokens
  int n_groups, max_group_size, members_per_tile, tiles_per_group;
  int fit;          // CTAs per prefix tile that one wave of the GPU holds (>= 1)
  int max_a;        // prefix slots of a row: at most this many prefix splits
  // Written by shared_prefix_prep_kernel (scratch):
  int32_t *seq_slots;  // [batch]: partial slots of sequence b (prefix + own splits)
  int32_t *count;      // [1]: work entries
  int32_t *cursor;     // [1]: next (entry, kv head) item of the persistent CTAs, zeroed by prep
  int4 *work;          // [2 per entry] the work entries, prefix work first
};

// A member whose own tokens past the shared prefix take at most this many 16-token
// units attends them inside its group's last prefix piece (rows of the other members
// masked) instead of in a work entry of its own: for beams a few tokens past their
// common prefix, a separate entry would cost a CTA's whole start-up for one unit.
constexpr int kFoldUnits = 4;
// Bit of the prep kernel's per-sequence group word: the member's own units are folded.
constexpr int kFoldFlag = 1 << 30;

// One work entry (two int4): what a CTA of the shared-prefix decode attends.
//   a = {mode (1 prefix, 2 own tokens), table row b, first unit, end unit}
//   c = {first member (mode 1), member mask | fold mask << 16 (mode 1), partial slot,
//        tokens}
// Mode 1 rows are (member m of the mask, query head); mode 2 rows are sequence
// b's heads.  `tokens` bounds the keys (the shared units, or the context).  A
// mode-1 entry also attends the own units of the members in its fold mask, each
// through the member's own table row with the other members' rows masked.

// One CTA resolves the groups and writes the work list, so the attention CTAs
// start from one entry, as the plain decode starts from its sequence.  A
// sequence shares its group's prefix when the group is well formed (0 <= start <
// end <= batch, and its start maps back to it), the sequence lies in the group's
// range and is among its first max_group_size members.  Starts are meant to
// ascend; where they do not, the search below still gives every sequence at most
// one group.  A group's units are its prefix length capped by every sharing
// member's context, in whole 16-token units; they are split into
// max(fit, units / (32 * 4)) pieces (at most max_a), each sequence's own
// units into pieces of DecodeParams.units_per_split.
__global__ void shared_prefix_prep_kernel(const DecodeParams p, const CascadeParams c) {
  ptx::grid_dependency_wait();
  ptx::launch_dependents();
  extern __shared__ int32_t prep_smem[];
  int32_t *gs = prep_smem;                      // [n_groups + 1]
  int32_t *sg = prep_smem + c.n_groups + 1;     // [batch]: group shared, or -1
  int32_t *gu = sg + p.batch;                   // [n_groups]: units shared
  int32_t *gn = gu + c.n_groups;                // [n_groups]: prefix splits
  int32_t *sl = gn + c.n_groups;                // [batch]: seq_lens, capped
  int32_t *gp = sl + p.batch;                   // [n_groups]: prefix_lens
  __shared__ int n_work;
  const int cap = p.max_bps * p.bs;
  // every global input in one pass: the rest of the kernel works from shared memory
  for (int i = threadIdx.x; i <= c.n_groups; i += blockDim.x) gs[i] = c.group_starts[i];
  for (int i = threadIdx.x; i < c.n_groups; i += blockDim.x) gp[i] = c.prefix_lens[i];
  for (int i = threadIdx.x; i < p.batch; i += blockDim.x) sl[i] = min(p.seq_lens[i], cap);
  if (threadIdx.x == 0) n_work = 0;
  __syncthreads();
  auto group_of = [&](int b) {  // the last group whose start is <= b
    int lo = 0, hi = c.n_groups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (gs[mid] <= b) {
        lo = mid;
      } else {
        hi = mid - 1;
      }
    }
    return lo;
  };
  auto well_formed = [&](int g) {
    const int s0 = gs[g], s1 = gs[g + 1];
    return s0 >= 0 && s1 <= p.batch && s0 < s1 && group_of(s0) == g;
  };
  for (int b = threadIdx.x; b < p.batch; b += blockDim.x) {
    const int g = group_of(b);
    const bool in = well_formed(g) && b >= gs[g] && b < gs[g + 1] && b - gs[g] < c.max_group_size;
    sg[b] = in ? g : -1;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < c.n_groups; g += blockDim.x) {
    int pl = 0;
    if (well_formed(g)) {
      pl = gp[g];
      const int s_end = min(gs[g + 1], gs[g] + c.max_group_size);
      for (int m = gs[g]; m < s_end; ++m) {
        if (sg[m] == g) pl = min(pl, sl[m]);
      }
    }
    const int pu = max(pl, 0) / kUnit;
    const int want = pu > 0 ? min(c.max_a, min(pu, max(c.fit, ceil_div_dev(pu, 32 * 4)))) : 0;
    const int ups = want > 0 ? ceil_div_dev(pu, want) : 1;  // <= 32 units per warp
    const int ns = want > 0 ? ceil_div_dev(pu, ups) : 0;    // every piece non-empty
    gu[g] = pu;
    gn[g] = ns;
    if (ns == 0) continue;
    for (int t = 0; t < c.tiles_per_group; ++t) {
      int mask = 0, fold = 0;
      // the last piece is the smallest; members with few own units join it while the
      // piece stays within 32 units per warp
      int room = 32 * kWarps - (pu - (ns - 1) * ups);
      for (int m = 0; m < c.members_per_tile; ++m) {
        const int bm = gs[g] + t * c.members_per_tile + m;
        if (bm < p.batch && sg[bm] == g) {
          mask |= 1 << m;
          const int own = ceil_div_dev(sl[bm], kUnit) - pu;
          if (own > 0 && own <= kFoldUnits && own <= room) {
            room -= own;
            fold |= 1 << m;
            sg[bm] = g | kFoldFlag;
          }
        }
      }
      if (!mask) continue;
      const int at = atomicAdd(&n_work, ns);
      for (int k = 0; k < ns; ++k) {
        c.work[2 * (at + k)] = make_int4(1, gs[g], k * ups, min(k * ups + ups, pu));
        c.work[2 * (at + k) + 1] = make_int4(gs[g] + t * c.members_per_tile,
                                             mask | (k == ns - 1 ? fold << 16 : 0), k,
                                             pu * kUnit);
      }
    }
  }
  __syncthreads();  // prefix work first: the long items start first
  for (int b = threadIdx.x; b < p.batch; b += blockDim.x) {
    const int len = sl[b];
    const bool folded = sg[b] >= 0 && (sg[b] & kFoldFlag);
    const int g = sg[b] >= 0 ? sg[b] & ~kFoldFlag : -1;
    const int pu = g >= 0 ? gu[g] : 0;
    const int na = g >= 0 ? gn[g] : 0;
    const int n_units = len > 0 ? ceil_div_dev(len, kUnit) : 0;
    const int nb = n_units > pu && !folded ? ceil_div_dev(n_units - pu, p.units_per_split) : 0;
    c.seq_slots[b] = len > 0 ? na + nb : 0;
    if (nb == 0) continue;
    const int at = atomicAdd(&n_work, nb);
    for (int k = 0; k < nb; ++k) {
      const int u0 = pu + k * p.units_per_split;
      c.work[2 * (at + k)] = make_int4(2, b, u0, min(u0 + p.units_per_split, n_units));
      c.work[2 * (at + k) + 1] = make_int4(0, 0, na + k, len);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *c.count = n_work;
    *c.cursor = 0;
  }
}

template <typename T, int D, int W, int NS>
struct Cfg {
  static constexpr int RS = D + 8;                  // padded row (elements)
  static constexpr int STAGE = 2 * kUnit * RS;      // K tile + V tile (elements)
  static constexpr int Q_ELEMS = 16 * RS;
  static constexpr size_t SMEM =
      size_t(Q_ELEMS + W * NS * STAGE) * sizeof(T) + size_t(W * NS) * 8 + 16;
  static constexpr int KS = D / 16;  // k-steps of QK^T, also 16-wide d slabs of PV
  static constexpr int ND = D / 8;   // 8-wide output tiles
};

// Shared memory holds the CTA to 2 per SM (108.9 KB each at D = 128).  The
// launch bound says so, which lets ptxas schedule the main loop with up to 255
// registers.  Without it ptxas may aim at 3 CTAs per SM (at most 168 registers)
// after unrelated edits to the kernel, and the loop then runs about 10% slower on
// the Llama-3-8B decode shape (measured: 129.8 us against 117.3 us per call).
//
// MODE 0: the plain decode, item = blockIdx.z = sequence.
// MODE 1: a prefix entry of the shared-prefix decode (ea / ec, written by
//         shared_prefix_prep_kernel): rows are (member, query head) pairs of the
//         entry's member mask, keys the group's shared units read through its
//         first member's block table; a partial into the entry's slot.
// MODE 2: an own-tokens entry: one sequence's units past its shared prefix; a
//         partial into the entry's slot, after the prefix ones.
//
// rb counts the units that already went through this warp's ring (the persistent
// shared-prefix CTAs run many entries on barriers initialised once): unit k of this
// call uses stage (rb + k) % NS at phase parity ((rb + k) / NS) & 1.  MODE 0 passes 0
// and initialises its barriers here.  Returns false when a wait ran out (the CTA
// has reported it and must stop).
// TWO (MODE 0 only): 8-token pages, a unit's rows 8-15 read from the next page.
template <typename T, int D, int W, int NS, int MODE, bool TWO = false>
__device__ __forceinline__ bool decode_body(const DecodeParams &p, const int item,
                                            const int split, int &rb, const int4 ea = int4{},
                                            const int4 ec = int4{}, const int kvh_in = 0) {
  using C = Cfg<T, D, W, NS>;
  using MMA = ptx::Mma<T>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T *qs = reinterpret_cast<T *>(smem_raw);
  T *stages = qs + C::Q_ELEMS;
  uint64_t *bars = reinterpret_cast<uint64_t *>(stages + W * NS * C::STAGE);
  __shared__ int s_fail;
  // Launched as a programmatic dependent of the previous kernel on the stream:
  // nothing is read before that kernel has completed.  The merge launch that
  // follows may be scheduled once every CTA of this grid has started.
  ptx::grid_dependency_wait();
  ptx::launch_dependents();

  const int kvh = MODE == 0 ? int(blockIdx.y) / p.n_head_tiles : kvh_in;
  const int ht = MODE == 0 ? int(blockIdx.y) % p.n_head_tiles : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  int b, seq_len, u_begin, u_end, n_splits_b, G, lo, hi;
  int NR = 0, slot0 = 0, mbase = 0;  // MODE 1/2 only
  unsigned members = 0;              // MODE 1: bit m = member m of the tile is a row source
  unsigned fold = 0;                 // MODE 1: bit m = member m's own units are in this entry
  int n_total;                       // units of this CTA (MODE 1: prefix, then folded own)
  if constexpr (MODE == 0) {
    b = item;
    seq_len = p.seq_lens[b];
    if (seq_len <= 0) return true;
    seq_len = min(seq_len, p.max_bps * p.bs);
    const int n_units = ceil_div_dev(seq_len, kUnit);
    u_begin = split * p.units_per_split;
    if (u_begin >= n_units) return true;
    u_end = min(u_begin + p.units_per_split, n_units);
    head_range(kvh, ht, p.hq, p.hkv, &lo, &hi);
    G = hi - lo;
    if (G <= 0) return true;
    n_splits_b = ceil_div_dev(n_units, p.units_per_split);
    n_total = u_end - u_begin;
  } else {
    // the work entry of the shared-prefix decode
    b = ea.y;
    u_begin = ea.z;
    u_end = ea.w;
    slot0 = ec.z;
    seq_len = ec.w;
    head_range(kvh, 0, p.hq, p.hkv, &lo, &hi);
    G = hi - lo;
    if (G <= 0 || u_begin >= u_end) return true;
    n_total = u_end - u_begin;
    if constexpr (MODE == 1) {
      mbase = ec.x;
      members = unsigned(ec.y) & 0xffffu;
      fold = unsigned(ec.y) >> 16;
      NR = (32 - __clz(int(members))) * G;  // up to the last member in the mask
      const int pu = seq_len / kUnit, cap = p.max_bps * p.bs;
      for (unsigned f = fold; f; f &= f - 1) {
        const int len = min(p.seq_lens[mbase + __ffs(int(f)) - 1], cap);
        n_total += ceil_div_dev(len, kUnit) - pu;
      }
    } else {
      NR = G;
    }
    n_splits_b = 2;  // partials only
  }

  // ---- stage Q (rows >= G are zero) and init barriers --------------------
  const T *qg = static_cast<const T *>(p.q) + int64_t(b) * p.q_sb + int64_t(lo) * p.q_sh;
  for (int i = threadIdx.x; i < 16 * (D / 8); i += W * 32) {
    int r = i / (D / 8), c = (i % (D / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    bool row_live;
    const T *src;
    if constexpr (MODE == 1) {  // row r = (member r / G, head lo + r % G)
      const int m = r / G;
      row_live = r < NR && ((members >> m) & 1u);
      src = static_cast<const T *>(p.q) + int64_t(mbase + m) * p.q_sb +
            int64_t(lo + r - m * G) * p.q_sh + c;
    } else {
      row_live = r < G;
      src = qg + int64_t(r) * p.q_sh + c;
    }
    if (row_live) {
      if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        v = *reinterpret_cast<const uint4 *>(src);
      } else {
        T tmp[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) tmp[e] = src[e];
        v = *reinterpret_cast<uint4 *>(tmp);
      }
    }
    *reinterpret_cast<uint4 *>(qs + r * C::RS + c) = v;
  }
  if (threadIdx.x == 0) s_fail = 0;
  uint64_t *my_bars = bars + warp * NS;
  if constexpr (MODE == 0) {
    if (lane == 0) {
      for (int s = 0; s < NS; ++s) ptx::mbar_init(ptx::smem_u32(my_bars + s), 32);
    }
  }
  ptx::fence_proxy_async_smem();
  __syncthreads();

  // ---- Q fragments (A operand, rows = heads) ------------------------------
  uint32_t qa[C::KS][4];
  {
    const int mi = lane >> 3, r = lane & 7;
    const int row = (mi & 1) * 8 + r;
#pragma unroll
    for (int ks = 0; ks < C::KS; ++ks) {
      int col = ks * 16 + (mi >> 1) * 8;
      ptx::ldsm_x4(ptx::smem_u32(qs + row * C::RS + col), qa[ks][0], qa[ks][1], qa[ks][2],
                   qa[ks][3]);
    }
  }

  // ---- per-warp unit list and page addresses -----------------------------
  const int n_w = (n_total - warp + W - 1) / W;  // units owned by this warp (<= 32)
  const int64_t row_stride = int64_t(p.hkv) * D;  // elements between tokens
  int64_t my_elem = 0;
  // 8-token pages: a unit's rows 8-15 lie in the next page, based here
  constexpr bool two_pages = TWO;
  static_assert(!TWO || MODE == 0, "two-page units are a plain-decode layout");
  int64_t my_elem2 = 0;
  int my_ok = 0;
  int my_meta = 0;  // MODE 1: valid tokens | (folded member + 1) << 8 (0: a shared unit)
  if (lane < n_w) {
    int u = u_begin + warp + lane * W;
    int tb = b;  // table row
    if constexpr (MODE == 1) {
      const int i = warp + lane * W;
      if (i < u_end - u_begin) {
        my_meta = kUnit;
      } else {  // the (i - prefix)-th own unit of the folded members, in member order
        const int pu = seq_len / kUnit, cap = p.max_bps * p.bs;
        int j = i - (u_end - u_begin);
        for (unsigned f = fold; f; f &= f - 1) {
          const int m = __ffs(int(f)) - 1;
          const int len = min(p.seq_lens[mbase + m], cap);
          const int own = ceil_div_dev(len, kUnit) - pu;
          if (j < own) {
            u = pu + j;
            tb = mbase + m;
            my_meta = min(kUnit, len - u * kUnit) | ((m + 1) << 8);
            break;
          }
          j -= own;
        }
      }
    }
    int tok0 = u * kUnit;
    int page = tok0 / p.bs;
    int blk = p.tables[int64_t(tb) * p.bt_stride + page];
    if constexpr (MODE == 1) {  // the caller's promise: every member holds the same block
      for (int m = 0; m < 16; ++m) {
        if ((my_meta >> 8) == 0 && ((members >> m) & 1u) &&
            p.tables[int64_t(mbase + m) * p.bt_stride + page] != blk)
          atomicOr(p.diag, int32_t(kDiagBadLaunch));
      }
    }
    // second page of the unit (8-token pages), read only when the unit reaches it
    const int blk2 = two_pages && tok0 + 8 < seq_len
                         ? p.tables[int64_t(tb) * p.bt_stride + page + 1] : blk;
    const int rows_a = two_pages ? 8 : kUnit;  // rows of the unit in the first page
    if (blk >= 0 && blk2 >= 0) {
      const uint64_t off = p.offsets[blk], off2 = p.offsets[blk2];
      const int64_t e = int64_t(off) + int64_t(tok0 % p.bs) * row_stride + int64_t(kvh) * D;
      const int64_t e2 = int64_t(off2) + int64_t(kvh) * D;
      const bool aligned = ((off | off2) & 7) == 0;
      const bool inside = uint64_t(e + (rows_a - 1) * row_stride + D) <= p.region_elems &&
                          (!two_pages || uint64_t(e2 + 7 * row_stride + D) <= p.region_elems);
      my_ok = aligned && inside;
      my_elem = e;
      my_elem2 = two_pages ? e2 : e;
    }
    if (!my_ok) atomicOr(p.diag, int32_t(kDiagBadOffset));
  }

  const T *vak = static_cast<const T *>(p.va_k);
  const T *vav = static_cast<const T *>(p.va_v);
  T *wst = stages + warp * NS * C::STAGE;

  // One unit = 16 K rows + 16 V rows of D elements, moved as 16-byte cp.async
  // chunks spread over the 32 lanes (rows past the context are zero-filled);
  // each lane then arrives on the stage's mbarrier once its copies land.
  auto issue = [&](int k) {
    const int st = (rb + k) % NS;
    const uint32_t bar = ptx::smem_u32(my_bars + st);
    const int64_t elem = __shfl_sync(0xffffffffu, my_elem, k);
    const int64_t elem2 = two_pages ? __shfl_sync(0xffffffffu, my_elem2, k) : elem;
    const int ok = __shfl_sync(0xffffffffu, my_ok, k);
    int nvalid;
    if constexpr (MODE == 1) {
      nvalid = ok ? (__shfl_sync(0xffffffffu, my_meta, k) & 0xff) : 0;
    } else {
      const int u = u_begin + warp + k * W;
      nvalid = ok ? min(kUnit, seq_len - u * kUnit) : 0;
    }
    const uint32_t ks_tile = ptx::smem_u32(wst + st * C::STAGE);
    const uint32_t vs_tile = ks_tile + kUnit * C::RS * sizeof(T);
    constexpr int CPR = D / 8;  // 16-byte chunks per row
#pragma unroll
    for (int j = lane; j < kUnit * CPR; j += 32) {
      const int r = j / CPR, c = j % CPR;
      const int64_t off = (two_pages && r >= 8 ? elem2 + int64_t(r - 8) * row_stride
                                               : elem + int64_t(r) * row_stride) + c * 8;
      const uint32_t n = r < nvalid ? 16u : 0u;
      const uint32_t so = uint32_t((r * C::RS + c * 8) * sizeof(T));
      ptx::cp_async16(ks_tile + so, vak + (n ? off : 0), n);
      ptx::cp_async16(vs_tile + so, vav + (n ? off : 0), n);
    }
    ptx::cp_async_mbar_arrive(bar);
  };

  // ---- main loop -----------------------------------------------------------
  float o[C::ND][4];
#pragma unroll
  for (int i = 0; i < C::ND; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int g = lane >> 2, t = lane & 3;
  bool failed = false;

  for (int k = 0; k < NS && k < n_w; ++k) issue(k);

  for (int k = 0; k < n_w; ++k) {
    const int st = (rb + k) % NS;
    const uint32_t bar = ptx::smem_u32(my_bars + st);
    const bool landed =
        ptx::mbar_wait_bounded(bar, uint32_t(((rb + k) / NS) & 1), kWaitLimitNs);
    if (!__all_sync(0xffffffffu, landed)) {  // warp-uniform exit
      failed = true;
      break;
    }
    __syncwarp();
    const int ok = __shfl_sync(0xffffffffu, my_ok, k);
    int nvalid;
    bool live0 = true, live1 = true;  // MODE 1 own unit: only its member's rows attend it
    if constexpr (MODE == 1) {
      const int meta = __shfl_sync(0xffffffffu, my_meta, k);
      nvalid = meta & 0xff;
      const int mm = (meta >> 8) - 1;
      if (mm >= 0) {
        live0 = (lane >> 2) / G == mm;
        live1 = ((lane >> 2) + 8) / G == mm;
      }
    } else {
      const int u = u_begin + warp + k * W;
      nvalid = min(kUnit, seq_len - u * kUnit);
    }
    const T *ks_tile = wst + st * C::STAGE;
    const T *vs_tile = ks_tile + kUnit * C::RS;
    if (ok) {
      // S = Q K^T : 16 heads x 16 tokens in two n-tiles
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      {
        const int mi = lane >> 3, r = lane & 7;
        const int tok = (mi >> 1) * 8 + r;
#pragma unroll
        for (int ks = 0; ks < C::KS; ++ks) {
          uint32_t b0, b1, b2, b3;
          ptx::ldsm_x4(ptx::smem_u32(ks_tile + tok * C::RS + ks * 16 + (mi & 1) * 8), b0, b1, b2,
                       b3);
          MMA::run(s[0], qa[ks], b0, b1);
          MMA::run(s[1], qa[ks], b2, b3);
        }
      }
      // online softmax (log2 domain)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int tok = nt * 8 + 2 * t + (j & 1);
          float v = tok < nvalid && (j < 2 ? live0 : live1) ? s[nt][j] * p.scale_log2 : -INFINITY;
          s[nt][j] = v;
        }
        mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      float e0 = mn0, e1 = mn1;  // exponent base
      if constexpr (MODE == 1) {
        // a row that has seen only masked keys keeps a zero sum and a max of -inf
        if (e0 == -INFINITY) e0 = 0.f;
        if (e1 == -INFINITY) e1 = 0.f;
      }
      const float a0 = ptx::fast_exp2(m0 - e0), a1 = ptx::fast_exp2(m1 - e1);
      m0 = mn0;
      m1 = mn1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = ptx::fast_exp2(s[nt][0] - e0);
        s[nt][1] = ptx::fast_exp2(s[nt][1] - e0);
        s[nt][2] = ptx::fast_exp2(s[nt][2] - e1);
        s[nt][3] = ptx::fast_exp2(s[nt][3] - e1);
        ps0 += s[nt][0] + s[nt][1];
        ps1 += s[nt][2] + s[nt][3];
      }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
#pragma unroll
      for (int i = 0; i < C::ND; ++i) {
        o[i][0] *= a0;
        o[i][1] *= a0;
        o[i][2] *= a1;
        o[i][3] *= a1;
      }
      uint32_t pa[4], pl[4];  // P = hi + lo (16-bit each)
      MMA::split(s[0][0], s[0][1], pa[0], pl[0]);
      MMA::split(s[0][2], s[0][3], pa[1], pl[1]);
      MMA::split(s[1][0], s[1][1], pa[2], pl[2]);
      MMA::split(s[1][2], s[1][3], pa[3], pl[3]);
      // O += P V
      {
        const int mi = lane >> 3, r = lane & 7;
        const int tok = (mi & 1) * 8 + r;
#pragma unroll
        for (int j = 0; j < C::KS; ++j) {
          uint32_t b0, b1, b2, b3;
          ptx::ldsm_x4_t(ptx::smem_u32(vs_tile + tok * C::RS + j * 16 + (mi >> 1) * 8), b0, b1,
                         b2, b3);
          MMA::run(o[2 * j], pa, b0, b1);
          MMA::run(o[2 * j], pl, b0, b1);
          MMA::run(o[2 * j + 1], pa, b2, b3);
          MMA::run(o[2 * j + 1], pl, b2, b3);
        }
      }
    }
    __syncwarp();
    if (k + NS < n_w) issue(k + NS);
  }
  rb += n_w;

  if (failed) {
    // Let copies still in flight land before the CTA's shared memory is
    // released (bounded as well), then report.
    for (int k = 0; k < NS && k < n_w; ++k) {
      ptx::mbar_wait_bounded(ptx::smem_u32(my_bars + k), 0, 1000000ull);
      ptx::mbar_wait_bounded(ptx::smem_u32(my_bars + k), 1, 1000000ull);
    }
    if (lane == 0) {
      atomicOr(p.diag, int32_t(kDiagWaitTimeout));
      s_fail = 1;
    }
  }

  // ---- merge the warps of this CTA ----------------------------------------
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  __syncthreads();
  if (s_fail) return false;
  float *cO = reinterpret_cast<float *>(stages);  // [W][16][D]
  float *cm = cO + W * 16 * D;                     // [W][16]
  float *cl = cm + W * 16;                         // [W][16]
  {
    float *wo = cO + warp * 16 * D;
#pragma unroll
    for (int i = 0; i < C::ND; ++i) {
      int d = i * 8 + 2 * t;
      const int nr = MODE == 0 ? G : NR;
      if (g < nr) *reinterpret_cast<float2 *>(wo + g * D + d) = make_float2(o[i][0], o[i][1]);
      if (g + 8 < nr) *reinterpret_cast<float2 *>(wo + (g + 8) * D + d) = make_float2(o[i][2], o[i][3]);
    }
    if (t == 0) {
      cm[warp * 16 + g] = m0;
      cl[warp * 16 + g] = l0;
      cm[warp * 16 + g + 8] = m1;
      cl[warp * 16 + g + 8] = l1;
    }
  }
  __syncthreads();
  const int64_t head0 = int64_t(b) * p.hq + lo;
  for (int i = threadIdx.x; i < (MODE == 0 ? G : NR) * (D / 2); i += W * 32) {
    const int h = i / (D / 2), d = (i % (D / 2)) * 2;
    if constexpr (MODE == 1) {
      if (!((members >> (h / G)) & 1u)) continue;
    }
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, cm[w * 16 + h]);
    float L = 0.f, x0 = 0.f, x1 = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      float mw = cm[w * 16 + h];
      if (mw == -INFINITY) continue;  // warp saw no unit
      float sc = ptx::fast_exp2(mw - M);
      L += cl[w * 16 + h] * sc;
      x0 += cO[(w * 16 + h) * D + d] * sc;
      x1 += cO[(w * 16 + h) * D + d + 1] * sc;
    }
    const float inv = 1.f / L;
    if (n_splits_b == 1) {
      T *dst = static_cast<T *>(p.out) + int64_t(b) * p.o_sb + int64_t(lo + h) * p.o_sh + d;
      dst[0] = ptx::from_f32<T>(x0 * inv);
      dst[1] = ptx::from_f32<T>(x1 * inv);
    } else {
      int64_t row;
      if constexpr (MODE == 1) {
        const int m = h / G;
        row = (int64_t(mbase + m) * p.hq + lo + (h - m * G)) * p.num_splits + slot0;
      } else if constexpr (MODE == 2) {
        row = (head0 + h) * p.num_splits + slot0;
      } else {
        row = (head0 + h) * p.num_splits + split;
      }
      *reinterpret_cast<float2 *>(p.part_o + row * D + d) = make_float2(x0 * inv, x1 * inv);
      if (d == 0) p.part_lse[row] = M + log2f(L);
    }
  }
  return true;
}

template <typename T, int D, int W, int NS, bool TWO = false>
__global__ void __launch_bounds__(W * 32, 2) decode_kernel(const DecodeParams p) {
  int rb = 0;
  decode_body<T, D, W, NS, 0, TWO>(p, blockIdx.z, blockIdx.x, rb);
}

// Shared-prefix decode: persistent CTAs (at most 2 per SM) take items
// entry * Hkv + kv head of the prep kernel's work list through an atomic cursor,
// with the kv head fastest, so items start in list order (prefix work first: the
// long items start together in the first wave) and no CTA is launched for work
// the arguments could have asked for but did not.  Each warp's unit ring and
// its mbarriers run on across the items.
template <typename T, int D, int W, int NS>
__global__ void __launch_bounds__(W * 32, 2)
    decode_shared_prefix_kernel(const DecodeParams p, const CascadeParams cp) {
  using C = Cfg<T, D, W, NS>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ int s_item;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<T *>(smem_raw) + C::Q_ELEMS +
                                                W * NS * C::STAGE);
  if (lane == 0) {
    for (int s = 0; s < NS; ++s) ptx::mbar_init(ptx::smem_u32(bars + warp * NS + s), 32);
  }
  ptx::grid_dependency_wait();  // the work list is the prep kernel's output
  const int n = *cp.count * p.hkv;
  int rb = 0;
  for (;;) {
    __syncthreads();  // the previous item's reads of shared memory are done
    if (threadIdx.x == 0) s_item = atomicAdd(cp.cursor, 1);
    __syncthreads();
    const int item = s_item;
    if (item >= n) break;
    const int entry = item / p.hkv, kvh = item % p.hkv;
    const int4 ea = cp.work[2 * entry], ec = cp.work[2 * entry + 1];
    const bool ok = ea.x == 1 ? decode_body<T, D, W, NS, 1>(p, 0, 0, rb, ea, ec, kvh)
                              : decode_body<T, D, W, NS, 2>(p, 0, 0, rb, ea, ec, kvh);
    if (!ok) break;
  }
  ptx::launch_dependents();
}

// Second pass: combine the splits of each (sequence, head) through their
// log-sum-exp, one warp per row, 4-dimension slices per lane.  Sequences that fit
// one split were written by the first pass.
template <typename T>
__global__ void merge_kernel(const DecodeParams p, int D, int rows) {
  ptx::grid_dependency_wait();
  ptx::launch_dependents();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // b * hq + h
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int b = row / p.hq;
  int seq_len = p.seq_lens[b];
  if (seq_len <= 0) return;
  seq_len = min(seq_len, p.max_bps * p.bs);
  const int n_units = ceil_div_dev(seq_len, kUnit);
  const int ns = ceil_div_dev(n_units, p.units_per_split);
  if (ns <= 1) return;
  const float *lse = p.part_lse + int64_t(row) * p.num_splits;
  float M = -INFINITY;
  for (int s = lane; s < ns; s += 32) M = fmaxf(M, lse[s]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float wsum = 0.f;
  for (int s = lane; s < ns; s += 32) wsum += ptx::fast_exp2(lse[s] - M);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  const float inv = 1.f / wsum;
  const float *po = p.part_o + int64_t(row) * p.num_splits * D;
  T *dst = static_cast<T *>(p.out) + int64_t(b) * p.o_sb + int64_t(row % p.hq) * p.o_sh;
  for (int d = lane * 4; d < D; d += 128) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int s = 0; s < ns; ++s) {
      const float w = ptx::fast_exp2(lse[s] - M);
      const float4 v = *reinterpret_cast<const float4 *>(po + int64_t(s) * D + d);
      acc.x += v.x * w;
      acc.y += v.y * w;
      acc.z += v.z * w;
      acc.w += v.w * w;
    }
    dst[d] = ptx::from_f32<T>(acc.x * inv);
    dst[d + 1] = ptx::from_f32<T>(acc.y * inv);
    dst[d + 2] = ptx::from_f32<T>(acc.z * inv);
    dst[d + 3] = ptx::from_f32<T>(acc.w * inv);
  }
}

// Merge of the shared-prefix decode: every row's slots are its group's prefix
// splits followed by its own suffix splits, all of them partials.
template <typename T>
__global__ void merge_shared_prefix_kernel(const DecodeParams p, const CascadeParams cp, int D,
                                           int rows) {
  ptx::grid_dependency_wait();
  ptx::launch_dependents();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // b * hq + h
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int b = row / p.hq;
  const int ns = cp.seq_slots[b];  // 0 for an empty sequence: left untouched
  if (ns <= 0) return;
  const float *lse = p.part_lse + int64_t(row) * p.num_splits;
  float M = -INFINITY;
  for (int s = lane; s < ns; s += 32) M = fmaxf(M, lse[s]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float wsum = 0.f;
  for (int s = lane; s < ns; s += 32) wsum += ptx::fast_exp2(lse[s] - M);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  const float inv = 1.f / wsum;
  const float *po = p.part_o + int64_t(row) * p.num_splits * D;
  T *dst = static_cast<T *>(p.out) + int64_t(b) * p.o_sb + int64_t(row % p.hq) * p.o_sh;
  for (int d = lane * 4; d < D; d += 128) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int s = 0; s < ns; ++s) {
      const float w = ptx::fast_exp2(lse[s] - M);
      const float4 v = *reinterpret_cast<const float4 *>(po + int64_t(s) * D + d);
      acc.x += v.x * w;
      acc.y += v.y * w;
      acc.z += v.z * w;
      acc.w += v.w * w;
    }
    dst[d] = ptx::from_f32<T>(acc.x * inv);
    dst[d + 1] = ptx::from_f32<T>(acc.y * inv);
    dst[d + 2] = ptx::from_f32<T>(acc.z * inv);
    dst[d + 3] = ptx::from_f32<T>(acc.w * inv);
  }
}

// Peer outputs of merge_gather_kernel: rank r's gathered buffer holds
// [2][world][batch][hq][D] 16-bit values; epoch e writes this rank's rows to slot
// `rank` of half e & 1 of every buffer (kernels/peer.cu says why two halves), then
// this CTA's flag in every rank's signal array is raised to epoch.
struct PeerOut {
  uint16_t *dst[kMaxPeers];
  unsigned long long *sig[kMaxPeers];
  int rank, world;
  unsigned long long epoch;
};

// merge_kernel fused with the all-gather of the KV-head split: kGatherBlocks
// CTAs of 32 warps walk all rows, one warp per row (the per-CTA flags fix the
// CTA count, so the parallelism comes from wide CTAs; with 4-warp CTAs the
// 70B head-split merge was latency-bound at 45 us).  A row that needed merging is merged as in merge_kernel
// and written to the local output and to every rank's buffer; a row that the
// first pass finished (one split) is copied from the local output to the
// buffers.  The stores to other GPUs are plain stores over NVLink; the CTA's
// flags follow a system-scope fence (kernels/peer.cu has the waiting side).
constexpr int kMergeGatherThreads = 1024;

template <typename T>
__global__ void __launch_bounds__(kMergeGatherThreads) merge_gather_kernel(const DecodeParams p, int D, int rows, const PeerOut g) {
  ptx::grid_dependency_wait();
  ptx::launch_dependents();
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const int64_t slice = int64_t(p.batch) * p.hq * D;
  for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < rows; row += gridDim.x * wpb) {
    const int b = row / p.hq;
    int seq_len = p.seq_lens[b];
    if (seq_len <= 0) continue;  // left untouched, here and in the peers' buffers
    seq_len = min(seq_len, p.max_bps * p.bs);
    const int n_units = ceil_div_dev(seq_len, kUnit);
    const int ns = ceil_div_dev(n_units, p.units_per_split);
    T *local = static_cast<T *>(p.out) + int64_t(b) * p.o_sb + int64_t(row % p.hq) * p.o_sh;
    const int64_t goff = (int64_t(g.epoch & 1ull) * g.world + g.rank) * slice + int64_t(row) * D;
    if (ns <= 1) {
      for (int d = lane * 4; d < D; d += 128) {
        const uint16_t *src = reinterpret_cast<const uint16_t *>(local) + d;
        const uint2 v = make_uint2(uint32_t(src[0]) | (uint32_t(src[1]) << 16),
                                   uint32_t(src[2]) | (uint32_t(src[3]) << 16));
        for (int r = 0; r < g.world; ++r) *reinterpret_cast<uint2 *>(g.dst[r] + goff + d) = v;
      }
      continue;
    }
    const float *lse = p.part_lse + int64_t(row) * p.num_splits;
    float M = -INFINITY;
    for (int s = lane; s < ns; s += 32) M = fmaxf(M, lse[s]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float wsum = 0.f;
    for (int s = lane; s < ns; s += 32) wsum += ptx::fast_exp2(lse[s] - M);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
    const float inv = 1.f / wsum;
    const float *po = p.part_o + int64_t(row) * p.num_splits * D;
    for (int d = lane * 4; d < D; d += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int s = 0; s < ns; ++s) {
        const float w = ptx::fast_exp2(lse[s] - M);
        const float4 v = *reinterpret_cast<const float4 *>(po + int64_t(s) * D + d);
        acc.x += v.x * w;
        acc.y += v.y * w;
        acc.z += v.z * w;
        acc.w += v.w * w;
      }
      T o[4] = {ptx::from_f32<T>(acc.x * inv), ptx::from_f32<T>(acc.y * inv),
                ptx::from_f32<T>(acc.z * inv), ptx::from_f32<T>(acc.w * inv)};
#pragma unroll
      for (int k = 0; k < 4; ++k) local[d + k] = o[k];
      const uint16_t *u = reinterpret_cast<const uint16_t *>(o);
      const uint2 v = make_uint2(uint32_t(u[0]) | (uint32_t(u[1]) << 16),
                                 uint32_t(u[2]) | (uint32_t(u[3]) << 16));
      for (int r = 0; r < g.world; ++r) *reinterpret_cast<uint2 *>(g.dst[r] + goff + d) = v;
    }
  }
  // The CTA barrier orders every thread's stores (peers' memory included) before
  // the flag threads' system-scope fence and release store, which carry them to
  // the other GPUs (cumulativity: the pattern of a cooperative grid barrier).
  __syncthreads();
  if (int(threadIdx.x) < g.world) {
    __threadfence_system();
    unsigned long long *f = g.sig[threadIdx.x] + g.rank * kGatherBlocks + blockIdx.x;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(g.epoch) : "memory");
  }
}

// Fallback for shapes outside the tensor-core path (head_dim not a multiple
// of 16, block_size not a multiple of 16): one warp per (sequence, head),
// plain loads, same math.
template <typename T>
__global__ void decode_generic_kernel(const DecodeParams p, int D) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= p.batch * p.hq) return;
  const int b = warp_global / p.hq, h = warp_global % p.hq;
  const int kvh = int(int64_t(h) * p.hkv / p.hq);
  int seq_len = p.seq_lens[b];
  if (seq_len <= 0) return;
  seq_len = min(seq_len, p.max_bps * p.bs);
  const T *q = static_cast<const T *>(p.q) + int64_t(b) * p.q_sb + int64_t(h) * p.q_sh;
  float qv[8], acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int d = lane + 32 * i;
    qv[i] = d < D ? ptx::to_f32(q[d]) : 0.f;
    acc[i] = 0.f;
  }
  const T *vak = static_cast<const T *>(p.va_k);
  const T *vav = static_cast<const T *>(p.va_v);
  float m = -INFINITY, l = 0.f;
  for (int tok = 0; tok < seq_len; ++tok) {
    int blk = p.tables[int64_t(b) * p.bt_stride + tok / p.bs];
    int64_t e = blk < 0 ? -1
                        : int64_t(p.offsets[blk]) + int64_t(tok % p.bs) * p.hkv * D +
                              int64_t(kvh) * D;
    if (e < 0 || uint64_t(e + D) > p.region_elems) {
      if (lane == 0) atomicOr(p.diag, int32_t(kDiagBadOffset));
      continue;
    }
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int d = lane + 32 * i;
      if (d < D) part += qv[i] * ptx::to_f32(vak[e + d]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    float s = part * p.scale_log2;
    float mn = fmaxf(m, s);
    float a = ptx::fast_exp2(m - mn), pr = ptx::fast_exp2(s - mn);
    m = mn;
    l = l * a + pr;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int d = lane + 32 * i;
      if (d < D) acc[i] = acc[i] * a + pr * ptx::to_f32(vav[e + d]);
    }
  }
  if (l == 0.f) return;
  T *out = static_cast<T *>(p.out) + int64_t(b) * p.o_sb + int64_t(h) * p.o_sh;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int d = lane + 32 * i;
    if (d < D) out[d] = ptx::from_f32<T>(acc[i] / l);
  }
}


// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

using KernelFn = void (*)(const DecodeParams);

template <typename T, int D>
KernelFn fast_kernel(bool two_pages) {
  return two_pages ? decode_kernel<T, D, kWarps, kStages, true>
                   : decode_kernel<T, D, kWarps, kStages, false>;
}

// two_pages: 8-token pages (each 16-token unit spans two of them)
template <typename T>
bool pick_fast(int D, KernelFn *fn, size_t *smem, bool two_pages = false) {
  switch (D) {
#define KCMM_CASE(DD)                                 \
  case DD:                                            \
    *fn = fast_kernel<T, DD>(two_pages);              \
    *smem = Cfg<T, DD, kWarps, kStages>::SMEM;        \
    return true;
    KCMM_CASE(32)
    KCMM_CASE(64)
    KCMM_CASE(80)
    KCMM_CASE(96)
    KCMM_CASE(112)
    KCMM_CASE(128)
    KCMM_CASE(160)
    KCMM_CASE(192)
    KCMM_CASE(256)
#undef KCMM_CASE
    default:
      return false;
  }
}

struct Occupancy {
  std::mutex mu;
  int sm_count = 0;
};
Occupancy &occ() {
  static Occupancy o;
  return o;
}

int sm_count() {
  Occupancy &o = occ();
  std::lock_guard<std::mutex> g(o.mu);
  if (o.sm_count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&o.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (o.sm_count <= 0) o.sm_count = 148;
  }
  return o.sm_count;
}

struct Plan {
  bool fast = false;
  KernelFn fn = nullptr;
  size_t smem = 0;
  int n_head_tiles = 1, units_per_split = 1, num_splits = 1;
  size_t scratch_bytes = 0;
};

Plan make_plan(const DecodeArgs &a) {
  Plan pl;
  const int D = a.head_dim;
  // 16-token units within a page, or across two 8-token pages
  bool shape_ok = D % 16 == 0 && (a.block_size % kUnit == 0 || a.block_size == 8);
  if (shape_ok) {
    const bool two = a.block_size == 8;
    pl.fast = a.dtype == Dtype::BF16 ? pick_fast<__nv_bfloat16>(D, &pl.fn, &pl.smem, two)
                                     : pick_fast<__half>(D, &pl.fn, &pl.smem, two);
  }
  if (!pl.fast) return pl;
  const int g_max = (a.num_q_heads + a.kv_heads - 1) / a.kv_heads;
  pl.n_head_tiles = (g_max + 15) / 16;
  const int max_units =
      int((int64_t(a.max_blocks_per_seq) * a.block_size + kUnit - 1) / kUnit);
  const int64_t items = int64_t(a.batch) * a.kv_heads * pl.n_head_tiles;
  // Aim at ~6 waves of 2 resident CTAs per SM over the worst-case context (on
  // the Llama-3-8B decode shape: 4 splits, 113.6 us, against 117.4 us at 8 waves
  // and 119.4 us at 6 splits); at least 16 units per split so each warp's ring
  // fills, at most 32 units per warp.
  const int64_t target = int64_t(sm_count()) * 2 * 6;
  int64_t want_splits = std::max<int64_t>(1, (target + items - 1) / items);
  int ups = int((max_units + want_splits - 1) / want_splits);
  // At most 16 splits: every CTA pays a start-up of a few microseconds before its
  // first unit lands, so few long items want few large CTAs.  Measured on the
  // Llama-3-70B head-split shards (8 sequences of 32k tokens): 1 kv head 70.6 us
  // with 128 splits against 35.5 us with 16; 4 kv heads 124.4 us against 100.1 us.
  ups = std::max(ups, (max_units + 15) / 16);
  ups = std::max(ups, 16);
  ups = std::min(ups, 32 * kWarps);
  if (a.force_splits > 0) ups = std::max(1, std::min((max_units + a.force_splits - 1) / a.force_splits, 32 * kWarps));
  pl.units_per_split = ups;
  pl.num_splits = (max_units + ups - 1) / ups;
  if (pl.num_splits > 1) {
    size_t rows = size_t(a.batch) * a.num_q_heads * pl.num_splits;
    pl.scratch_bytes = rows * size_t(D) * 4 + rows * 4;
  }
  return pl;
}

cudaMemPool_t scratch_pool(int dev) {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  std::lock_guard<std::mutex> g(mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    if (cudaMemPoolCreate(&pools[dev], &props) != cudaSuccess) return nullptr;
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
  }
  return pools[dev];
}

cudaError_t scratch_acquire(const DecodeArgs &a, size_t bytes, cudaStream_t stream, void **out,
                            bool *owned) {
  *owned = false;
  if (a.scratch) {
    if (a.scratch_bytes < bytes) return cudaErrorInvalidValue;
    *out = a.scratch;
    return cudaSuccess;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  cudaMemPool_t mp = scratch_pool(dev);
  if (!mp) return cudaErrorMemoryAllocation;
  cudaError_t e = cudaMallocFromPoolAsync(out, bytes, mp, stream);
  if (e == cudaSuccess) *owned = true;
  return e;
}

}  // namespace

size_t decode_scratch_bytes(const DecodeArgs &a) { return make_plan(a).scratch_bytes; }

// Split scratch kept per (device, stream) between calls, so a call makes no
// stream-ordered allocation between its kernels and the next call's launch can
// overlap the previous merge (programmatic dependent launch).  Calls on one
// stream run in order, and each kernel waits for the previous one before it
// touches memory, so they can share one buffer; a larger call replaces it in
// stream order.  Streams are keyed by cudaStreamGetId (never reused in a
// process).  Returns null while the stream is being captured (a graph may be
// replayed on any stream) or once kMaxCachedStreams streams hold a buffer: the
// caller then allocates for the call alone.
constexpr size_t kMaxCachedStreams = 16;

void *stream_scratch(cudaStream_t stream, size_t bytes) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cs != cudaStreamCaptureStatusNone) return nullptr;
  unsigned long long id = 0;
  int dev = 0;
  if (cudaStreamGetId(stream, &id) != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  struct Entry {
    void *ptr = nullptr;
    size_t bytes = 0;
  };
  static std::mutex mu;
  static std::map<std::pair<int, unsigned long long>, Entry> cache;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find({dev, id});
  if (it == cache.end()) {
    if (cache.size() >= kMaxCachedStreams) return nullptr;
    it = cache.emplace(std::make_pair(dev, id), Entry{}).first;
  }
  Entry &en = it->second;
  if (en.bytes >= bytes) return en.ptr;
  cudaMemPool_t mp = scratch_pool(dev);
  if (!mp) return nullptr;
  void *fresh = nullptr;
  const size_t want = std::max(bytes, en.bytes + en.bytes / 2);
  if (cudaMallocFromPoolAsync(&fresh, want, mp, stream) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (en.ptr) cudaFreeAsync(en.ptr, stream);
  en.ptr = fresh;
  en.bytes = want;
  return fresh;
}

cudaError_t decode_attention(const DecodeArgs &a, cudaStream_t stream) {
  DecodeParams p = {};
  p.q = a.q;
  p.out = a.out;
  p.tables = a.block_tables;
  p.seq_lens = a.seq_lens;
  p.offsets = a.block_offsets;
  p.va_k = a.va_k;
  p.va_v = a.va_v;
  p.region_elems = a.region_elems;
  p.batch = a.batch;
  p.hq = a.num_q_heads;
  p.hkv = a.kv_heads;
  p.bs = a.block_size;
  p.max_bps = a.max_blocks_per_seq;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.diag = a.diag;
  const int64_t dense_row = int64_t(a.num_q_heads) * a.head_dim;
  p.q_sb = a.q_stride_token ? a.q_stride_token : dense_row;
  p.q_sh = a.q_stride_head ? a.q_stride_head : a.head_dim;
  p.o_sb = a.out_stride_token ? a.out_stride_token : dense_row;
  p.o_sh = a.out_stride_head ? a.out_stride_head : a.head_dim;
  p.bt_stride = a.tables_stride ? a.tables_stride : a.max_blocks_per_seq;

  Plan pl = make_plan(a);
  if (!pl.fast && a.peer_world > 0) return cudaErrorNotSupported;  // tensor-core path only
  if (!pl.fast) {
    const int threads = 256;
    const int64_t warps = int64_t(a.batch) * a.num_q_heads;
    const int blocks = int((warps * 32 + threads - 1) / threads);
    if (a.dtype == Dtype::BF16) {
      decode_generic_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(p, a.head_dim);
    } else {
      decode_generic_kernel<__half><<<blocks, threads, 0, stream>>>(p, a.head_dim);
    }
    return cudaGetLastError();
  }
  p.units_per_split = pl.units_per_split;
  p.num_splits = pl.num_splits;
  p.n_head_tiles = pl.n_head_tiles;

  void *scratch = nullptr;
  bool owned = false;
  if (pl.scratch_bytes) {
    if (a.scratch) {
      if (a.scratch_bytes < pl.scratch_bytes) return cudaErrorInvalidValue;
      scratch = a.scratch;
    } else if ((scratch = stream_scratch(stream, pl.scratch_bytes)) != nullptr) {
      // kept for the stream
    } else {
      int dev = 0;
      cudaGetDevice(&dev);
      cudaMemPool_t mp = scratch_pool(dev);
      if (!mp) return cudaErrorMemoryAllocation;
      cudaError_t e = cudaMallocFromPoolAsync(&scratch, pl.scratch_bytes, mp, stream);
      if (e != cudaSuccess) return e;
      owned = true;
    }
    size_t rows = size_t(a.batch) * a.num_q_heads * pl.num_splits;
    p.part_o = static_cast<float *>(scratch);
    p.part_lse = p.part_o + rows * size_t(a.head_dim);
  }

  cudaError_t e = cudaFuncSetAttribute(pl.fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(pl.smem));
  if (e != cudaSuccess) return e;
  dim3 grid(pl.num_splits, a.kv_heads * pl.n_head_tiles, a.batch);
  e = launch_pdl(pl.fn, grid, dim3(kWarps * 32), pl.smem, stream, p);
  if (e == cudaSuccess && a.peer_world > 0) {
    // merge fused with the all-gather: always launched (it also forwards the
    // rows the first pass finished)
    PeerOut g = {};
    for (int r = 0; r < a.peer_world; ++r) {
      g.dst[r] = reinterpret_cast<uint16_t *>(a.peer_out[r]);
      g.sig[r] = reinterpret_cast<unsigned long long *>(a.peer_sig[r]);
    }
    g.rank = a.peer_rank;
    g.world = a.peer_world;
    g.epoch = a.peer_epoch;
    const int rows = a.batch * a.num_q_heads;
    if (a.dtype == Dtype::BF16) {
      e = launch_pdl(merge_gather_kernel<__nv_bfloat16>, dim3(kGatherBlocks),
                     dim3(kMergeGatherThreads), 0, stream, p, a.head_dim, rows, g);
    } else {
      e = launch_pdl(merge_gather_kernel<__half>, dim3(kGatherBlocks),
                     dim3(kMergeGatherThreads), 0, stream, p, a.head_dim, rows, g);
    }
  } else if (e == cudaSuccess && pl.num_splits > 1) {
    const int rows = a.batch * a.num_q_heads;
    const dim3 mgrid((rows + 3) / 4);
    if (a.dtype == Dtype::BF16) {
      e = launch_pdl(merge_kernel<__nv_bfloat16>, mgrid, dim3(128), 0, stream, p, a.head_dim, rows);
    } else {
      e = launch_pdl(merge_kernel<__half>, mgrid, dim3(128), 0, stream, p, a.head_dim, rows);
    }
  }
  if (owned) {
    cudaError_t f = cudaFreeAsync(scratch, stream);
    if (e == cudaSuccess) e = f;
  }
  return e;
}

namespace {

using SharedPrefixFn = void (*)(const DecodeParams, const CascadeParams);

template <typename T>
bool pick_shared_prefix(int D, SharedPrefixFn *fn, size_t *smem) {
  switch (D) {
#define KCMM_CASE(DD)                                                  \
  case DD:                                                             \
    *fn = decode_shared_prefix_kernel<T, DD, kWarps, kStages>;         \
    *smem = Cfg<T, DD, kWarps, kStages>::SMEM;                         \
    return true;
    KCMM_CASE(64)
    KCMM_CASE(128)
    KCMM_CASE(256)
#undef KCMM_CASE
    default:
      return false;
  }
}

// Units per split for `items` work items over at most max_units units, aiming
// at `waves` waves of 2 CTAs per SM (16..32*W units, at most 16 splits).  The
// plain decode's rule is 6 waves, which balances contexts of unequal length;
// the prefix items of a group are few and equally long, and there CTAs of 4
// units per warp spend most of their time starting up and draining their ring
// (measured on the beam-search shape: 63 us at 8 splits of 16 units).
int units_per_split_for(int64_t items, int max_units, int waves) {
  const int64_t target = int64_t(sm_count()) * 2 * waves;
  const int64_t want = std::max<int64_t>(1, (target + items - 1) / std::max<int64_t>(items, 1));
  int ups = int((max_units + want - 1) / want);
  ups = std::max(ups, (max_units + 15) / 16);
  ups = std::max(ups, 16);
  return std::min(ups, 32 * kWarps);
}

struct SharedPrefixPlan {
  SharedPrefixFn fn = nullptr;
  size_t smem = 0, scratch_bytes = 0, resolved_off = 0;
  int mt = 0, tiles = 0, fit = 1, max_a = 0, b_ups = 0, b_splits = 0;
  int64_t max_work = 0;
};

// Groups resolved in one CTA's shared memory: group_starts, two words per
// sequence and three per group (at most 192 KB).
constexpr int kSharedPrefixMaxBatch = 8192;

SharedPrefixPlan make_shared_prefix_plan(const DecodeArgs &a, int n_groups, int max_group) {
  SharedPrefixPlan pl;
  const int G = (a.num_q_heads + a.kv_heads - 1) / a.kv_heads;
  if (a.head_dim % 16 != 0 || a.block_size % kUnit != 0 || G > 16 ||
      a.num_q_heads % a.kv_heads != 0)
    return pl;
  const bool ok = a.dtype == Dtype::BF16
                      ? pick_shared_prefix<__nv_bfloat16>(a.head_dim, &pl.fn, &pl.smem)
                      : pick_shared_prefix<__half>(a.head_dim, &pl.fn, &pl.smem);
  if (!ok) {
    pl.fn = nullptr;
    return pl;
  }
  const int max_units =
      int((int64_t(a.max_blocks_per_seq) * a.block_size + kUnit - 1) / kUnit);
  pl.mt = 16 / G;
  pl.tiles = (max_group + pl.mt - 1) / pl.mt;
  // Prefix tiles are few and equally long: split each into as many pieces as
  // one wave of 2 CTAs per SM holds for all of them (at least one; at most 32
  // units per warp), so every piece starts at once and none waits for a slot.
  const int64_t prefix_ctas = int64_t(n_groups) * pl.tiles * a.kv_heads;
  pl.fit = int(std::max<int64_t>(1, std::min<int64_t>(16, int64_t(sm_count()) * 2 / prefix_ctas)));
  pl.max_a = std::max(pl.fit, (max_units + 32 * kWarps - 1) / (32 * kWarps));
  pl.b_ups = units_per_split_for(int64_t(a.batch) * a.kv_heads, max_units, 6);
  pl.b_splits = (max_units + pl.b_ups - 1) / pl.b_ups;
  const size_t rows = size_t(a.batch) * a.num_q_heads * size_t(pl.max_a + pl.b_splits);
  pl.resolved_off = (rows * size_t(a.head_dim) * 4 + rows * 4 + 15) & ~size_t(15);
  pl.max_work = int64_t(n_groups) * pl.tiles * pl.max_a + int64_t(a.batch) * pl.b_splits;
  // seq_slots, the count and the cursor, then the 32-byte work entries (16-byte aligned)
  pl.scratch_bytes = pl.resolved_off + ((size_t(a.batch) + 2) * 4 + 15) / 16 * 16 +
                     size_t(pl.max_work) * 32;
  return pl;
}

}  // namespace

cudaError_t decode_attention_shared_prefix(const DecodeArgs &a, const int32_t *group_starts,
                                           const int32_t *prefix_lens, int n_groups,
                                           int max_group, cudaStream_t stream) {
  const SharedPrefixPlan pl = make_shared_prefix_plan(a, n_groups, max_group);
  if (!pl.fn) return cudaErrorNotSupported;
  // batches the prep kernel cannot resolve in one CTA's shared memory: not supported
  // (the caller falls back to the plain decode)
  if (a.batch > kSharedPrefixMaxBatch || pl.max_work * a.kv_heads > 0x7fffffff)
    return cudaErrorNotSupported;
  DecodeParams p = {};
  p.q = a.q;
  p.out = a.out;
  p.tables = a.block_tables;
  p.seq_lens = a.seq_lens;
  p.offsets = a.block_offsets;
  p.va_k = a.va_k;
  p.va_v = a.va_v;
  p.region_elems = a.region_elems;
  p.batch = a.batch;
  p.hq = a.num_q_heads;
  p.hkv = a.kv_heads;
  p.bs = a.block_size;
  p.max_bps = a.max_blocks_per_seq;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.diag = a.diag;
  p.q_sb = int64_t(a.num_q_heads) * a.head_dim;
  p.q_sh = a.head_dim;
  p.o_sb = p.q_sb;
  p.o_sh = a.head_dim;
  p.bt_stride = a.max_blocks_per_seq;
  p.units_per_split = pl.b_ups;
  p.num_splits = pl.max_a + pl.b_splits;  // slot stride of a row
  p.n_head_tiles = 1;
  CascadeParams cp = {};
  cp.group_starts = group_starts;
  cp.prefix_lens = prefix_lens;
  cp.n_groups = n_groups;
  cp.max_group_size = max_group;
  cp.members_per_tile = pl.mt;
  cp.tiles_per_group = pl.tiles;
  cp.fit = pl.fit;
  cp.max_a = pl.max_a;

  void *scratch = nullptr;
  bool owned = false;
  cudaError_t e = cudaSuccess;
  if (a.scratch) {
    if (a.scratch_bytes < pl.scratch_bytes) return cudaErrorInvalidValue;
    scratch = a.scratch;
  } else if ((scratch = stream_scratch(stream, pl.scratch_bytes)) == nullptr) {
    e = scratch_acquire(a, pl.scratch_bytes, stream, &scratch, &owned);
    if (e != cudaSuccess) return e;
  }
  const size_t rows = size_t(a.batch) * a.num_q_heads * size_t(p.num_splits);
  p.part_o = static_cast<float *>(scratch);
  p.part_lse = p.part_o + rows * size_t(a.head_dim);
  char *res = static_cast<char *>(scratch) + pl.resolved_off;
  cp.seq_slots = reinterpret_cast<int32_t *>(res);
  cp.count = cp.seq_slots + a.batch;
  cp.cursor = cp.count + 1;
  cp.work = reinterpret_cast<int4 *>(res + ((size_t(a.batch) + 2) * 4 + 15) / 16 * 16);

  const size_t prep_smem = (size_t(n_groups) * 4 + 1 + size_t(a.batch) * 2) * 4;
  e = cudaFuncSetAttribute(shared_prefix_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(prep_smem));
  if (e == cudaSuccess)
    e = launch_pdl(shared_prefix_prep_kernel, dim3(1), dim3(1024), prep_smem, stream, p, cp);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(pl.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(pl.smem));
  if (e == cudaSuccess) {
    dim3 grid(unsigned(std::min<int64_t>(pl.max_work * a.kv_heads, int64_t(sm_count()) * 2)));
    e = launch_pdl(pl.fn, grid, dim3(kWarps * 32), pl.smem, stream, p, cp);
  }
  if (e == cudaSuccess) {
    const int nrows = a.batch * a.num_q_heads;
    const dim3 mgrid((nrows + 3) / 4);
    if (a.dtype == Dtype::BF16) {
      e = launch_pdl(merge_shared_prefix_kernel<__nv_bfloat16>, mgrid, dim3(128), 0, stream, p,
                     cp, a.head_dim, nrows);
    } else {
      e = launch_pdl(merge_shared_prefix_kernel<__half>, mgrid, dim3(128), 0, stream, p, cp,
                     a.head_dim, nrows);
    }
  }
  if (owned) {
    cudaError_t f = cudaFreeAsync(scratch, stream);
    if (e == cudaSuccess) e = f;
  }
  return e;
}

cudaError_t decode_preload() {
  cudaFuncAttributes attr;
  for (int D : {64, 128}) {
    KernelFn fn;
    size_t smem;
    pick_fast<__nv_bfloat16>(D, &fn, &smem);
    cudaError_t e = cudaFuncGetAttributes(&attr, fn);
    if (e != cudaSuccess) return e;
    pick_fast<__half>(D, &fn, &smem);
    e = cudaFuncGetAttributes(&attr, fn);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace dev
}  // namespace kcmm
