// Persistent "stream-K" paged decode attention for sm_100a (included by decode.cu).
//
// Work decomposition.  Every (sequence b, kv head, tile of <=16 query heads)
// is a *segment* of ceil(L_b/16) 16-token *units*.  The segments of all
// sequences, laid end to end, form one flat unit space of U units; CTA c of a
// one-wave persistent grid of P CTAs takes the contiguous slice
// [c*U/P, (c+1)*U/P).  Every CTA therefore streams the same number of KV bytes
// (+-1 unit) whatever the mix of context lengths, with no atomics and no work
// queue.  A slice may start or end inside a segment: the CTA then emits a
// partial result (o, lse) for that *piece*, and a second pass merges the
// pieces of a segment by log-sum-exp; segments that lie inside one slice are
// written to `out` directly.
//
// Inside a CTA the warps are specialised.  One producer warp walks the slice
// in order and streams every unit's K and V rows into a deep shared-memory
// ring (R stages, ~20 at head_dim 128, i.e. ~170 KB in flight per SM) with
// one-row `cp.async.bulk` copies (TMA engine; the [bs][Hkv][D] page layout
// needs no tensor map), a full/empty mbarrier pair per stage, and page
// addresses looked up 32 units at a time, one batch ahead.  C consumer warps
// take the units round-robin and run QK^T and PV on the tensor pipe
// (m16n8k16, fp32 accumulate) with an online softmax in the log2 domain.  Q
// tiles arrive by bulk copy into S slots, one per in-flight piece.  When a
// consumer leaves a piece it deposits (o, m, l) into the piece's merge slot;
// the last consumer to arrive merges the C deposits, frees the slot and starts
// the Q load of the piece S places ahead.  Every wait is bounded in wall time.

namespace kcmm {
namespace dev {
namespace sk {

struct alignas(64) Params {
  CUtensorMap tmk;  // K region of the layer: {D, Hkv, tokens}, box {64, 1, 16}, 128B swizzle
  CUtensorMap tmv;  // V region, same view
  uint64_t region_tokens;
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
  int n_head_tiles;  // ceil(group / 16)
  int g_max;         // rows of a head tile (<= 16)
  float *part_o;     // [(segments + P) * g_max * D]
  float *part_lse;   // [(segments + P) * g_max]
  int64_t *cum_out;  // [B+1] unit prefix, written by CTA 0 for the merge pass
  int32_t *segcum_out;  // [B+1] segment prefix
  int32_t *diag;
};

constexpr int kUnitTok = 16;
constexpr uint64_t kLimitNs = 1000000000ull;

struct Layout {
  size_t rings, qslots, merge_o, merge_ml, bars, info, cum, segcum, lens, total;
};

__host__ __device__ inline size_t al16(size_t x) { return (x + 15) & ~size_t(15); }

// Shared-memory plan of a CTA with C consumer warps, S piece slots and an
// R-stage ring (identical on host and device).
template <int D, int C, int S>
__host__ __device__ inline Layout layout(int batch, int g_max, int R) {
  constexpr int RS = D + 8;
  Layout L;
  size_t o = 0;
  L.rings = o;  // 1024-aligned at run time; stage = K + V tiles of 16 x D, 128B-swizzled
  o = al16(o + size_t(R) * 2 * kUnitTok * D * 2);
  L.qslots = o;
  o = al16(o + size_t(S) * 16 * RS * 2);
  L.merge_o = o;
  o = al16(o + size_t(S) * C * g_max * D * 4);
  L.merge_ml = o;
  o = al16(o + size_t(S) * C * g_max * 2 * 4);
  L.bars = o;
  o = al16(o + size_t(2 * R + S) * 8);
  L.info = o;
  o = al16(o + size_t(R + 2 * S) * 4);
  L.cum = o;
  o = al16(o + size_t(batch + 1) * 8);
  L.segcum = o;
  o = al16(o + size_t(batch + 1) * 4);
  L.lens = o;
  o = al16(o + size_t(batch) * 4);
  L.total = o + 1024;  // slack for aligning the base to 1024 bytes
  return L;
}

// Largest c in [0, P) with floor(c*U/P) <= u.
__device__ __forceinline__ int cta_of(int64_t u, int64_t U, int P) {
  int c = int((u * P) / U);
  if (c >= P) c = P - 1;
  while (c + 1 < P && ((int64_t(c) + 1) * U) / P <= u) ++c;
  while (c > 0 && (int64_t(c) * U) / P > u) --c;
  return c;
}

struct Loc {
  int b, segl, unit, nunits;
  int64_t seg_start;  // first unit of the segment in the flat space
  int sc;             // compact segment index
};

__device__ __forceinline__ Loc locate(int64_t u, const int64_t *cum, const int32_t *segcum,
                                      int B, int segs_per_seq) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (cum[mid] <= u) lo = mid; else hi = mid - 1;
  }
  Loc r;
  r.b = lo;
  r.nunits = int(cum[lo + 1] - cum[lo]) / segs_per_seq;  // one sequence: fits 32 bits
  const int rem = int(u - cum[lo]);
  r.segl = rem / r.nunits;
  r.unit = rem - r.segl * r.nunits;
  r.seg_start = cum[lo] + int64_t(r.segl) * r.nunits;
  r.sc = segcum[lo] + r.segl;
  return r;
}

// Sequence holding compact segment sc.
__device__ __forceinline__ int seq_of_segment(int sc, const int32_t *segcum, int B) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (segcum[mid] <= sc) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void heads_of(int segl, int nht, int hq, int hkv, int *lo, int *G) {
  const int kvh = segl / nht, ht = segl % nht;
  const int g_lo = int((int64_t(kvh) * hq + hkv - 1) / hkv);
  const int g_hi = int((int64_t(kvh + 1) * hq + hkv - 1) / hkv);
  *lo = g_lo + ht * 16;
  *G = max(0, min(g_hi, *lo + 16) - *lo);
}

template <typename T, int D, int C, int NP, int S>
__global__ void __launch_bounds__((C + NP) * 32)
    sk_decode_kernel(const __grid_constant__ Params p, int R) {
  using MMA = ptx::Mma<T>;
  constexpr int RS = D + 8;
  constexpr int HALVES = D / 64;                 // 64-dim half-tiles per K or V tile
  constexpr int TILE_B = HALVES * kUnitTok * 128;  // bytes of one K (or V) tile
  constexpr int KS = D / 16, ND = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout Lo = layout<D, C, S>(p.batch, p.g_max, R);
  unsigned char *ring = smem + Lo.rings;
  T *qslots = reinterpret_cast<T *>(smem + Lo.qslots);
  float *merge_o = reinterpret_cast<float *>(smem + Lo.merge_o);
  float *merge_ml = reinterpret_cast<float *>(smem + Lo.merge_ml);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Lo.bars);
  uint64_t *empty = full + R;
  uint64_t *qbars = empty + R;
  int *info = reinterpret_cast<int *>(smem + Lo.info);
  int *slot_cnt = info + R;
  int *slot_gen = slot_cnt + S;
  int64_t *cum = reinterpret_cast<int64_t *>(smem + Lo.cum);
  int32_t *segcum = reinterpret_cast<int32_t *>(smem + Lo.segcum);
  int32_t *lens = reinterpret_cast<int32_t *>(smem + Lo.lens);
  __shared__ int s_fail;

  const int c = blockIdx.x, P = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int B = p.batch;
  const int nht = p.n_head_tiles;
  const int segs_per_seq = p.hkv * nht;
  const int max_len = p.max_bps * p.bs;
  const int g_max = p.g_max;

  // ---- prefix sums over sequences (warp 0) ---------------------------------
  if (warp == 0) {
    const int per = (B + 31) / 32, b0 = lane * per;
    int64_t su = 0;
    int ss = 0;
    for (int i = 0; i < per; ++i) {
      const int b = b0 + i;
      if (b < B) {
        int L = p.seq_lens[b];
        L = L > 0 ? min(L, max_len) : 0;
        lens[b] = L;
        const int nu = (L + kUnitTok - 1) / kUnitTok;
        su += int64_t(nu) * segs_per_seq;
        ss += nu > 0 ? segs_per_seq : 0;
      }
    }
    int64_t iu = su;
    int is = ss;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t vu = __shfl_up_sync(0xffffffffu, iu, o);
      const int vs = __shfl_up_sync(0xffffffffu, is, o);
      if (lane >= o) {
        iu += vu;
        is += vs;
      }
    }
    int64_t ru = iu - su;
    int rs = is - ss;
    for (int i = 0; i < per; ++i) {
      const int b = b0 + i;
      if (b < B) {
        cum[b] = ru;
        segcum[b] = rs;
        const int nu = (lens[b] + kUnitTok - 1) / kUnitTok;
        ru += int64_t(nu) * segs_per_seq;
        rs += nu > 0 ? segs_per_seq : 0;
      }
    }
    if (lane == 31) {
      cum[B] = iu;
      segcum[B] = is;
    }
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < R; ++s) {
      ptx::mbar_init(ptx::smem_u32(full + s), 1);
      ptx::mbar_init(ptx::smem_u32(empty + s), 1);
    }
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(ptx::smem_u32(qbars + s), 1);
      slot_cnt[s] = 0;
      slot_gen[s] = 0;
    }
    s_fail = 0;
  }
  ptx::fence_proxy_async_smem();
  __syncthreads();

  const int64_t U = cum[B];
  if (c == 0) {
    for (int b = threadIdx.x; b <= B; b += (C + NP) * 32) {
      p.cum_out[b] = cum[b];
      p.segcum_out[b] = segcum[b];
    }
  }
  const int64_t lo = (int64_t(c) * U) / P, hi = (int64_t(c) + 1) * U / P;
  if (lo >= hi) return;
  const int n = int(hi - lo);  // units of this slice
  const Loc first = locate(lo, cum, segcum, B, segs_per_seq);
  const Loc last = locate(hi - 1, cum, segcum, B, segs_per_seq);
  const int sc0 = first.sc;
  const int n_pieces = last.sc - sc0 + 1;
  const int64_t row_stride = int64_t(p.hkv) * D;
  const T *qg = static_cast<const T *>(p.q);

  // Q tile of piece k -> slot k % S, issued by one whole warp.
  auto issue_q = [&](int k) {
    const int sc = sc0 + k;
    const int b = seq_of_segment(sc, segcum, B);
    int hlo, G;
    heads_of(sc - segcum[b], nht, p.hq, p.hkv, &hlo, &G);
    const int slot = k % S;
    const uint32_t bar = ptx::smem_u32(qbars + slot);
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive_expect_tx(bar, uint32_t(G * D * sizeof(T)));
    __syncwarp();
    if (lane < G) {
      ptx::bulk_g2s(ptx::smem_u32(qslots + slot * 16 * RS + lane * RS),
                    qg + (int64_t(b) * p.hq + hlo + lane) * D, uint32_t(D * sizeof(T)), bar);
    }
  };

  if (warp >= C) {
    // ======================= producer warps ===============================
    // NP producer warps share the ring: producer pw issues the quads of units
    // q*4 .. q*4+3 with q % NP == pw (a warp issues its TMA loads one after
    // another, so several warps are needed to keep the ring full).
    const int pw = warp - C;
    if (pw == 0) {
      for (int k = 0; k < S && k < n_pieces; ++k) issue_q(k);
    }
    if (lane == 0) {
      ptx::prefetch_tensormap(&p.tmk);
      ptx::prefetch_tensormap(&p.tmv);
    }
    constexpr int kQuad = 4;
    // lane l of batch t stands for unit 4 * (pw + NP * (8t + l/4)) + l%4
    auto unit_of = [&](int batch, int l) { return kQuad * (pw + NP * (8 * batch + (l >> 2))) + (l & 3); };
    // Page lookups run as a 3-stage register pipeline over these batches: at
    // the start of batch t the table entries of batch t+2 and the offsets of
    // batch t+1 are requested, and the coordinates of batch t are finished
    // from values that arrived one batch earlier -- no instruction waits on a
    // fresh load.
    int a_blk = -1, a_inf = 0, a_tok = 0;  // stage A: block id + unit facts of batch t+2
    uint64_t b_off = 0;                    // stage B: page offset of batch t+1
    int b_blk = -1, b_inf = 0, b_tok = 0;
    int64_t c_z = 0;                       // stage C: TMA token coordinate of batch t
    int c_inf = 0;                         // (kvh << 6) | (nvalid << 1) | ok
    auto stage_a = [&](int batch) {
      const int i = unit_of(batch, lane);
      a_blk = -1;
      a_inf = 0;
      a_tok = 0;
      if (i < n) {
        const Loc l = locate(lo + i, cum, segcum, B, segs_per_seq);
        const int tok0 = l.unit * kUnitTok;
        const int nvalid = min(kUnitTok, lens[l.b] - tok0);
        a_blk = p.tables[int64_t(l.b) * p.max_bps + tok0 / p.bs];
        a_inf = ((l.segl / nht) << 6) | (nvalid << 1) | 1;
        a_tok = tok0 % p.bs;
      }
    };
    auto stage_b = [&]() {
      b_blk = a_blk;
      b_inf = a_inf;
      b_tok = a_tok;
      b_off = (b_inf & 1) && b_blk >= 0 ? p.offsets[b_blk] : 0;
    };
    auto stage_c = [&]() {
      int ok = 0;
      int64_t z = 0;
      if (b_inf & 1) {
        if (b_blk >= 0) {
          z = int64_t(b_off / uint64_t(row_stride)) + b_tok;
          const int nvalid = (b_inf >> 1) & 31;
          ok = b_off % uint64_t(row_stride) == 0 && uint64_t(z + nvalid) <= p.region_tokens;
        }
        if (!ok) atomicOr(p.diag, int32_t(kDiagBadOffset));
      }
      c_z = z;
      c_inf = (b_inf & ~1) | ok;
    };
    stage_a(0);
    stage_b();
    stage_c();
    stage_a(1);
    stage_b();
    stage_a(2);
    const int grp = lane >> 3, gl = lane & 7;
    const unsigned gmask = 0xffu << (grp * 8);
    bool stop = false;
    for (int qi = 0; !stop; ++qi) {  // qi-th quad of this producer
      const int i0 = kQuad * (pw + NP * qi);
      if (i0 >= n) break;
      if ((qi & 7) == 0 && qi > 0) {  // rotate: B -> C, A -> B, new A
        stage_c();
        stage_b();
        stage_a((qi >> 3) + 2);
      }
      const int i = i0 + grp;
      const int src = ((qi & 7) << 2) | grp;
      const int64_t z = __shfl_sync(0xffffffffu, c_z, src);
      const int inf = __shfl_sync(0xffffffffu, c_inf, src);
      const bool live = i < n;
      const int ok = live && (inf & 1), kvh = inf >> 6;
      const int st = i % R;
      bool freed = true;
      if (live && i >= R) {  // wait until the consumer of unit i-R released the stage
        freed = ptx::mbar_wait_bounded(ptx::smem_u32(empty + st),
                                       uint32_t(((i / R) - 1) & 1), kLimitNs);
      }
      if (!__all_sync(0xffffffffu, freed)) {
        if (lane == 0) {
          atomicOr(p.diag, int32_t(kDiagWaitTimeout));
          s_fail = 1;
        }
        stop = true;
        break;
      }
      const uint32_t bar = ptx::smem_u32(full + st);
      if (live && gl == 0) {
        info[st] = ok;
        ptx::mbar_arrive_expect_tx(bar, ok ? uint32_t(2 * TILE_B) : 0u);
      }
      __syncwarp(gmask);
      if (ok && gl < 2 * HALVES) {  // one lane per 16 x 64 half-tile
        const int h = gl % HALVES;
        const bool v = gl >= HALVES;
        const uint32_t dst = ptx::smem_u32(ring + size_t(st) * 2 * TILE_B) + (v ? TILE_B : 0) +
                             h * kUnitTok * 128;
        ptx::tma_load_3d(dst, v ? static_cast<const void *>(&p.tmv) : &p.tmk, h * 64, kvh,
                         int(z), bar);
      }
      __syncwarp();
    }
    // drain: the last loads this warp issued must land before it leaves (the
    // consumers normally wait for them too; this covers a consumer that gave up)
    for (int qi = 0;; ++qi) {
      const int i0 = kQuad * (pw + NP * qi);
      if (i0 >= n) break;
      if (lane < kQuad && i0 + lane < n && i0 + lane >= n - R) {
        const int i = i0 + lane;
        ptx::mbar_wait_bounded(ptx::smem_u32(full + (i % R)), uint32_t((i / R) & 1), 2000000ull);
      }
    }
    return;
  }

  // ======================== consumer warps ================================
  const int g = lane >> 2, t = lane & 3;
  float o[ND][4];
  float m0, m1, l0, l1;
  auto reset = [&]() {
#pragma unroll
    for (int i = 0; i < ND; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  };
  reset();

  auto merge_piece = [&](int k) {
    const int slot = k % S;
    const int sc = sc0 + k;
    const int b = seq_of_segment(sc, segcum, B);
    const int segl = sc - segcum[b];
    int hlo, G;
    heads_of(segl, nht, p.hq, p.hkv, &hlo, &G);
    const int nunits = int((cum[b + 1] - cum[b]) / segs_per_seq);
    const int64_t s_start = cum[b] + int64_t(segl) * nunits, s_end = s_start + nunits;
    const bool whole = s_start >= lo && s_end <= hi;
    // pieces of segment sc live at rows sc + c (c = CTA), which never collide:
    // the CTAs holding pieces of segment sc+1 start at or after those of sc
    const int64_t gidx = int64_t(sc) + c;
    const float *mo = merge_o + size_t(slot) * C * g_max * D;
    const float *mml = merge_ml + size_t(slot) * C * g_max * 2;
    for (int idx = lane; idx < G * (D / 2); idx += 32) {
      const int h = idx / (D / 2), d = (idx % (D / 2)) * 2;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < C; ++w) M = fmaxf(M, mml[(w * g_max + h) * 2]);
      float Ls = 0.f, x0 = 0.f, x1 = 0.f;
#pragma unroll
      for (int w = 0; w < C; ++w) {
        const float mw = mml[(w * g_max + h) * 2];
        if (mw == -INFINITY) continue;
        const float sc_w = ptx::fast_exp2(mw - M);
        Ls += mml[(w * g_max + h) * 2 + 1] * sc_w;
        const float2 v = *reinterpret_cast<const float2 *>(mo + (size_t(w) * g_max + h) * D + d);
        x0 += v.x * sc_w;
        x1 += v.y * sc_w;
      }
      const float inv = 1.f / Ls;
      if (whole) {
        T *dst = static_cast<T *>(p.out) + (int64_t(b) * p.hq + hlo + h) * D + d;
        dst[0] = ptx::from_f32<T>(x0 * inv);
        dst[1] = ptx::from_f32<T>(x1 * inv);
      } else {
        *reinterpret_cast<float2 *>(p.part_o + (gidx * g_max + h) * D + d) =
            make_float2(x0 * inv, x1 * inv);
        if (d == 0) p.part_lse[gidx * g_max + h] = M + log2f(Ls);
      }
    }
  };

  auto finalize = [&](int k) {
    const int slot = k % S, gen = k / S;
    if (lane == 0) {  // wait until the slot's previous piece has been merged
      volatile int *vg = slot_gen + slot;
      if (*vg != gen) {
        const uint64_t t0 = ptx::globaltimer_ns();
        while (*vg != gen) {
          if (ptx::globaltimer_ns() - t0 > kLimitNs) {
            atomicOr(p.diag, int32_t(kDiagWaitTimeout));
            s_fail = 1;
            break;
          }
        }
      }
      __threadfence_block();
    }
    __syncwarp();
    float lq0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
    lq0 += __shfl_xor_sync(0xffffffffu, lq0, 2);
    float lq1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
    lq1 += __shfl_xor_sync(0xffffffffu, lq1, 2);
    float *mo = merge_o + (size_t(slot) * C + warp) * g_max * D;
    float *mml = merge_ml + (size_t(slot) * C + warp) * g_max * 2;
#pragma unroll
    for (int i = 0; i < ND; ++i) {
      const int d = i * 8 + 2 * t;
      if (g < g_max) *reinterpret_cast<float2 *>(mo + g * D + d) = make_float2(o[i][0], o[i][1]);
      if (g + 8 < g_max)
        *reinterpret_cast<float2 *>(mo + (g + 8) * D + d) = make_float2(o[i][2], o[i][3]);
    }
    if (t == 0) {
      if (g < g_max) {
        mml[g * 2] = m0;
        mml[g * 2 + 1] = lq0;
      }
      if (g + 8 < g_max) {
        mml[(g + 8) * 2] = m1;
        mml[(g + 8) * 2 + 1] = lq1;
      }
    }
    __threadfence_block();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(slot_cnt + slot, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == C - 1) {
      __threadfence_block();
      merge_piece(k);
      __syncwarp();
      if (lane == 0) {
        slot_cnt[slot] = 0;
        __threadfence_block();
        *reinterpret_cast<volatile int *>(slot_gen + slot) = gen + 1;
      }
      __syncwarp();
      if (k + S < n_pieces) issue_q(k + S);
    }
  };

  uint32_t qa[KS][4];
  int cur = 0;
  bool have_q = false;
  bool failed = false;
  // segment cursor: advanced incrementally (units only move forward)
  int cb = 0, csegl = 0, cnu = 1, csc = 0;
  int64_t cstart = 0, cend = 0;
  if (warp < n) {
    const Loc l0 = locate(lo + warp, cum, segcum, B, segs_per_seq);
    cb = l0.b;
    csegl = l0.segl;
    cnu = l0.nunits;
    csc = l0.sc;
    cstart = l0.seg_start;
    cend = cstart + cnu;
  }
  for (int i = warp; i < n; i += C) {
    const int64_t u = lo + i;
    while (u >= cend) {  // next segment (sequences without units hold none)
      if (++csegl == segs_per_seq) {
        csegl = 0;
        do {
          ++cb;
        } while (cum[cb + 1] == cum[cb]);
        cnu = int(cum[cb + 1] - cum[cb]) / segs_per_seq;
      }
      ++csc;
      cstart = cend;
      cend = cstart + cnu;
    }
    const int unit = int(u - cstart);
    const int k = csc - sc0;
    const int nvalid = min(kUnitTok, lens[cb] - unit * kUnitTok);
    while (cur < k) {
      finalize(cur);
      ++cur;
      reset();
      have_q = false;
    }
    if (!have_q) {
      const bool q_in = ptx::mbar_wait_bounded(ptx::smem_u32(qbars + cur % S),
                                               uint32_t((cur / S) & 1), kLimitNs);
      if (!__all_sync(0xffffffffu, q_in)) {
        failed = true;
        break;
      }
      const T *qt = qslots + (cur % S) * 16 * RS;
      const int mi2 = lane >> 3, r = lane & 7;
      const int row = (mi2 & 1) * 8 + r;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        ptx::ldsm_x4(ptx::smem_u32(qt + row * RS + ks * 16 + (mi2 >> 1) * 8), qa[ks][0],
                     qa[ks][1], qa[ks][2], qa[ks][3]);
      }
      have_q = true;
    }
    const int st = i % R;
    const bool landed =
        ptx::mbar_wait_bounded(ptx::smem_u32(full + st), uint32_t((i / R) & 1), kLimitNs);
    if (!__all_sync(0xffffffffu, landed)) {
      failed = true;
      break;
    }
    const uint32_t kt = ptx::smem_u32(ring + size_t(st) * 2 * TILE_B);
    const uint32_t vt = kt + TILE_B;
    // byte address of 16-byte chunk (token, dim d0..d0+7) in a swizzled tile
    auto sw = [](uint32_t tile, int tok, int d0) -> uint32_t {
      return tile + (d0 >> 6) * (kUnitTok * 128) + tok * 128 +
             ((((d0 & 63) >> 3) ^ (tok & 7)) << 4);
    };
    if (info[st] && nvalid < kUnitTok) {
      // rows past the context hold whatever the page holds: zero V there so
      // that P = 0 meets 0, not a stale NaN
      for (int idx = lane; idx < (kUnitTok - nvalid) * (D / 8); idx += 32) {
        const int tok = nvalid + idx / (D / 8), d0 = (idx % (D / 8)) * 8;
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(sw(vt, tok, d0)), "r"(0)
                     : "memory");
      }
      ptx::fence_proxy_async_smem();  // before the stage is refilled by TMA
      __syncwarp();
    }
    if (info[st]) {
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      {
        const int mi2 = lane >> 3, r = lane & 7;
        const int tok = (mi2 >> 1) * 8 + r;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t b0, b1, b2, b3;
          ptx::ldsm_x4(sw(kt, tok, ks * 16 + (mi2 & 1) * 8), b0, b1, b2, b3);
          MMA::run(s[0], qa[ks], b0, b1);
          MMA::run(s[1], qa[ks], b2, b3);
        }
      }
      if (nvalid == kUnitTok) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int j = 0; j < 4; ++j) s[nt][j] *= p.scale_log2;
      } else {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int tok = nt * 8 + 2 * t + (j & 1);
            s[nt][j] = tok < nvalid ? s[nt][j] * p.scale_log2 : -INFINITY;
          }
      }
      float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
      float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float a0 = ptx::fast_exp2(m0 - mn0), a1 = ptx::fast_exp2(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = ptx::fast_exp2(s[nt][0] - mn0);
        s[nt][1] = ptx::fast_exp2(s[nt][1] - mn0);
        s[nt][2] = ptx::fast_exp2(s[nt][2] - mn1);
        s[nt][3] = ptx::fast_exp2(s[nt][3] - mn1);
        ps0 += s[nt][0] + s[nt][1];
        ps1 += s[nt][2] + s[nt][3];
      }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
      if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
        for (int d = 0; d < ND; ++d) {
          o[d][0] *= a0;
          o[d][1] *= a0;
          o[d][2] *= a1;
          o[d][3] *= a1;
        }
      }
      uint32_t pa[4], pl[4];  // P = hi + lo (16-bit each)
      MMA::split(s[0][0], s[0][1], pa[0], pl[0]);
      MMA::split(s[0][2], s[0][3], pa[1], pl[1]);
      MMA::split(s[1][0], s[1][1], pa[2], pl[2]);
      MMA::split(s[1][2], s[1][3], pa[3], pl[3]);
      {
        const int mi2 = lane >> 3, r = lane & 7;
        const int tok = (mi2 & 1) * 8 + r;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          uint32_t b0, b1, b2, b3;
          ptx::ldsm_x4_t(sw(vt, tok, j * 16 + (mi2 >> 1) * 8), b0, b1, b2, b3);
          MMA::run(o[2 * j], pa, b0, b1);
          MMA::run(o[2 * j], pl, b0, b1);
          MMA::run(o[2 * j + 1], pa, b2, b3);
          MMA::run(o[2 * j + 1], pl, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(empty + st));  // release the stage
  }
  if (failed) {
    if (lane == 0) {
      atomicOr(p.diag, int32_t(kDiagWaitTimeout));
      s_fail = 1;
    }
    return;
  }
  // deposit every remaining piece (a consumer with no unit in a piece deposits
  // an empty partial so that the merge count completes)
  while (cur < n_pieces) {
    if (s_fail) break;
    finalize(cur);
    ++cur;
    reset();
  }
}

// ---------------------------------------------------------------------------
// Stream-K decode with per-warp cp.async rings (the default path).
//
// Same flat-unit slicing, pieces and merge slots as above, but every warp is
// its own producer: warp w takes units w, w+W, ... of the slice and keeps NS
// of them in flight in a private ring, each unit moved as 16-byte cp.async
// (LDGSTS) chunks by all 32 lanes -- issue cost is spread over every lane of
// every warp, which keeps far more bytes in flight per SM than a single
// issuing thread can.  Each lane's copies arrive on the stage's mbarrier
// (cp.async.mbarrier.arrive.noinc, 32 arrivals per phase).  Tiles are stored
// unpadded with the 16-byte chunk c of row r at chunk c ^ (r & 7), so the
// ldmatrix reads of 8 consecutive rows hit 8 distinct bank groups.
// ---------------------------------------------------------------------------

template <int D, int W, int S>
__host__ __device__ inline Layout layout_ld(int batch, int g_max, int NS) {
  Layout L;
  size_t o = 0;
  L.rings = o;  // W * NS stages of K + V tiles (16 x D each)
  o = al16(o + size_t(W) * NS * 2 * kUnitTok * D * 2);
  L.qslots = o;
  o = al16(o + size_t(S) * 16 * (D + 8) * 2);
  L.merge_o = o;
  o = al16(o + size_t(S) * W * g_max * D * 4);
  L.merge_ml = o;
  o = al16(o + size_t(S) * W * g_max * 2 * 4);
  L.bars = o;
  o = al16(o + size_t(W * NS + S) * 8);
  L.info = o;
  o = al16(o + size_t(2 * S) * 4);
  L.cum = o;
  o = al16(o + size_t(batch + 1) * 8);
  L.segcum = o;
  o = al16(o + size_t(batch + 1) * 4);
  L.lens = o;
  o = al16(o + size_t(batch) * 4);
  L.total = o;
  return L;
}

template <typename T, int D, int W, int S>
__global__ void __launch_bounds__(W * 32) sk_ld_kernel(const Params p, int NS) {
  using MMA = ptx::Mma<T>;
  constexpr int RS = D + 8;  // padded Q slot rows
  constexpr int TILE_B = kUnitTok * D * 2;
  constexpr int CPR = D / 8;  // 16-byte chunks per row
  constexpr int KS = D / 16, ND = D / 8;
  extern __shared__ __align__(128) unsigned char smem[];
  const Layout Lo = layout_ld<D, W, S>(p.batch, p.g_max, NS);
  unsigned char *rings = smem + Lo.rings;
  T *qslots = reinterpret_cast<T *>(smem + Lo.qslots);
  float *merge_o = reinterpret_cast<float *>(smem + Lo.merge_o);
  float *merge_ml = reinterpret_cast<float *>(smem + Lo.merge_ml);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Lo.bars);
  uint64_t *qbars = bars + W * NS;
  int *slot_cnt = reinterpret_cast<int *>(smem + Lo.info);
  int *slot_gen = slot_cnt + S;
  int64_t *cum = reinterpret_cast<int64_t *>(smem + Lo.cum);
  int32_t *segcum = reinterpret_cast<int32_t *>(smem + Lo.segcum);
  int32_t *lens = reinterpret_cast<int32_t *>(smem + Lo.lens);
  __shared__ int s_fail;

  const int c = blockIdx.x, P = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int B = p.batch;
  const int nht = p.n_head_tiles;
  const int segs_per_seq = p.hkv * nht;
  const int max_len = p.max_bps * p.bs;
  const int g_max = p.g_max;

  // ---- prefix sums over sequences (warp 0) ---------------------------------
  if (warp == 0) {
    const int per = (B + 31) / 32, b0 = lane * per;
    int64_t su = 0;
    int ss = 0;
    for (int i = 0; i < per; ++i) {
      const int b = b0 + i;
      if (b < B) {
        int L = p.seq_lens[b];
        L = L > 0 ? min(L, max_len) : 0;
        lens[b] = L;
        const int nu = (L + kUnitTok - 1) / kUnitTok;
        su += int64_t(nu) * segs_per_seq;
        ss += nu > 0 ? segs_per_seq : 0;
      }
    }
    int64_t iu = su;
    int is = ss;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t vu = __shfl_up_sync(0xffffffffu, iu, o);
      const int vs = __shfl_up_sync(0xffffffffu, is, o);
      if (lane >= o) {
        iu += vu;
        is += vs;
      }
    }
    int64_t ru = iu - su;
    int rs = is - ss;
    for (int i = 0; i < per; ++i) {
      const int b = b0 + i;
      if (b < B) {
        cum[b] = ru;
        segcum[b] = rs;
        const int nu = (lens[b] + kUnitTok - 1) / kUnitTok;
        ru += int64_t(nu) * segs_per_seq;
        rs += nu > 0 ? segs_per_seq : 0;
      }
    }
    if (lane == 31) {
      cum[B] = iu;
      segcum[B] = is;
    }
  }
  if (lane == 0) {
    for (int st = 0; st < NS; ++st) ptx::mbar_init(ptx::smem_u32(bars + warp * NS + st), 32);
  }
  if (threadIdx.x == 0) {
    for (int st = 0; st < S; ++st) {
      ptx::mbar_init(ptx::smem_u32(qbars + st), 1);
      slot_cnt[st] = 0;
      slot_gen[st] = 0;
    }
    s_fail = 0;
  }
  ptx::fence_proxy_async_smem();
  __syncthreads();

  const int64_t U = cum[B];
  if (c == 0) {
    for (int b = threadIdx.x; b <= B; b += W * 32) {
      p.cum_out[b] = cum[b];
      p.segcum_out[b] = segcum[b];
    }
  }
  const int64_t lo = (int64_t(c) * U) / P, hi = (int64_t(c) + 1) * U / P;
  if (lo >= hi) return;
  const int n = int(hi - lo);
  const Loc first = locate(lo, cum, segcum, B, segs_per_seq);
  const Loc last = locate(hi - 1, cum, segcum, B, segs_per_seq);
  const int sc0 = first.sc;
  const int n_pieces = last.sc - sc0 + 1;
  const int64_t row_stride = int64_t(p.hkv) * D;
  const T *qg = static_cast<const T *>(p.q);

  auto issue_q = [&](int k) {  // Q tile of piece k -> slot k % S (whole warp)
    const int sc = sc0 + k;
    const int b = seq_of_segment(sc, segcum, B);
    int hlo, G;
    heads_of(sc - segcum[b], nht, p.hq, p.hkv, &hlo, &G);
    const int slot = k % S;
    const uint32_t bar = ptx::smem_u32(qbars + slot);
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive_expect_tx(bar, uint32_t(G * D * sizeof(T)));
    __syncwarp();
    if (lane < G) {
      ptx::bulk_g2s(ptx::smem_u32(qslots + slot * 16 * RS + lane * RS),
                    qg + (int64_t(b) * p.hq + hlo + lane) * D, uint32_t(D * sizeof(T)), bar);
    }
  };
  if (warp == 0) {
    for (int k = 0; k < S && k < n_pieces; ++k) issue_q(k);
  }

  // ---- this warp's unit stream: positions j -> unit i = warp + j*W ----------
  const int n_w = n > warp ? (n - warp + W - 1) / W : 0;
  // page lookups: 3-stage register pipeline over batches of 32 positions
  int a_blk = -1, a_inf = 0, a_tok = 0;
  uint64_t b_off = 0;
  int b_blk = -1, b_inf = 0, b_tok = 0;
  int64_t c_e = 0;  // element offset of the unit's first row for its kv head
  int c_inf = 0;    // (nvalid << 1) | ok
  auto stage_a = [&](int batch) {
    const int j = batch * 32 + lane;
    a_blk = -1;
    a_inf = 0;
    a_tok = 0;
    if (j < n_w) {
      const Loc l = locate(lo + warp + int64_t(j) * W, cum, segcum, B, segs_per_seq);
      const int tok0 = l.unit * kUnitTok;
      const int nvalid = min(kUnitTok, lens[l.b] - tok0);
      a_blk = p.tables[int64_t(l.b) * p.max_bps + tok0 / p.bs];
      a_inf = ((l.segl / nht) << 6) | (nvalid << 1) | 1;
      a_tok = tok0 % p.bs;
    }
  };
  auto stage_b = [&]() {
    b_blk = a_blk;
    b_inf = a_inf;
    b_tok = a_tok;
    b_off = (b_inf & 1) && b_blk >= 0 ? p.offsets[b_blk] : 0;
  };
  auto stage_c = [&]() {
    int ok = 0;
    int64_t e = 0;
    if (b_inf & 1) {
      if (b_blk >= 0) {
        e = int64_t(b_off) + int64_t(b_tok) * row_stride + int64_t(b_inf >> 6) * D;
        ok = (b_off & 7) == 0 && uint64_t(e + (kUnitTok - 1) * row_stride + D) <= p.region_elems;
      }
      if (!ok) atomicOr(p.diag, int32_t(kDiagBadOffset));
    }
    c_e = e;
    c_inf = (((b_inf >> 1) & 31) << 1) | ok;
  };
  stage_a(0);
  stage_b();
  stage_c();
  stage_a(1);
  stage_b();
  stage_a(2);

  const T *vak = static_cast<const T *>(p.va_k);
  const T *vav = static_cast<const T *>(p.va_v);
  unsigned char *wring = rings + size_t(warp) * NS * 2 * TILE_B;
  uint64_t *wbars = bars + warp * NS;

  // Issue position j into stage j % NS.  Must be called by the whole warp with
  // j's batch current in stage C.  Chunk q = lane + 32m of a tile is row
  // q / CPR, 16-byte column q % CPR (32-bit offsets from the unit's first row).
  constexpr int M = kUnitTok * CPR / 32;
  const int rs32 = int(row_stride);
  auto issue = [&](int j) {
    const int64_t e = __shfl_sync(0xffffffffu, c_e, j & 31);
    const int inf = __shfl_sync(0xffffffffu, c_inf, j & 31);
    const int nvalid = (inf & 1) ? (inf >> 1) : 0;
    const int st = j % NS;
    const uint32_t kt = ptx::smem_u32(wring + size_t(st) * 2 * TILE_B);
    const uint32_t vt = kt + TILE_B;
    const T *kb = vak + e, *vb = vav + e;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int q = lane + 32 * m, r = q / CPR, ch = q % CPR;
      const int pc = ch < (CPR & ~7) ? (ch ^ (r & 7)) : ch;  // swizzle full 8-chunk groups only
      const uint32_t so = uint32_t(r * (D * 2) + (pc << 4));
      const bool live = r < nvalid;
      const int go = live ? r * rs32 + ch * 8 : 0;
      const uint32_t nb = live ? 16u : 0u;
      ptx::cp_async16(kt + so, kb + go, nb);
      ptx::cp_async16(vt + so, vb + go, nb);
    }
    ptx::cp_async_mbar_arrive(ptx::smem_u32(wbars + st));
    return inf;
  };

  // ---- accumulators, pieces -------------------------------------------------
  const int g = lane >> 2, t = lane & 3;
  float o[ND][4];
  float m0, m1, l0, l1;
  auto reset = [&]() {
#pragma unroll
    for (int i = 0; i < ND; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  };
  reset();

  auto merge_piece = [&](int k) {
    const int slot = k % S;
    const int sc = sc0 + k;
    const int b = seq_of_segment(sc, segcum, B);
    const int segl = sc - segcum[b];
    int hlo, G;
    heads_of(segl, nht, p.hq, p.hkv, &hlo, &G);
    const int nunits = int(cum[b + 1] - cum[b]) / segs_per_seq;
    const int64_t s_start = cum[b] + int64_t(segl) * nunits, s_end = s_start + nunits;
    const bool whole = s_start >= lo && s_end <= hi;
    const int64_t gidx = int64_t(sc) + c;  // rows sc + c never collide (see merge pass)
    const float *mo = merge_o + size_t(slot) * W * g_max * D;
    const float *mml = merge_ml + size_t(slot) * W * g_max * 2;
    for (int idx = lane; idx < G * (D / 2); idx += 32) {
      const int h = idx / (D / 2), d = (idx % (D / 2)) * 2;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < W; ++w) M = fmaxf(M, mml[(w * g_max + h) * 2]);
      float Ls = 0.f, x0 = 0.f, x1 = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float mw = mml[(w * g_max + h) * 2];
        if (mw == -INFINITY) continue;
        const float sc_w = ptx::fast_exp2(mw - M);
        Ls += mml[(w * g_max + h) * 2 + 1] * sc_w;
        const float2 v = *reinterpret_cast<const float2 *>(mo + (size_t(w) * g_max + h) * D + d);
        x0 += v.x * sc_w;
        x1 += v.y * sc_w;
      }
      const float inv = 1.f / Ls;
      if (whole) {
        T *dst = static_cast<T *>(p.out) + (int64_t(b) * p.hq + hlo + h) * D + d;
        dst[0] = ptx::from_f32<T>(x0 * inv);
        dst[1] = ptx::from_f32<T>(x1 * inv);
      } else {
        *reinterpret_cast<float2 *>(p.part_o + (gidx * g_max + h) * D + d) =
            make_float2(x0 * inv, x1 * inv);
        if (d == 0) p.part_lse[gidx * g_max + h] = M + log2f(Ls);
      }
    }
  };

  auto finalize = [&](int k) {
    const int slot = k % S, gen = k / S;
    if (lane == 0) {
      volatile int *vg = slot_gen + slot;
      if (*vg != gen) {
        const uint64_t t0 = ptx::globaltimer_ns();
        while (*vg != gen) {
          if (ptx::globaltimer_ns() - t0 > kLimitNs) {
            atomicOr(p.diag, int32_t(kDiagWaitTimeout));
            s_fail = 1;
            break;
          }
        }
      }
      __threadfence_block();
    }
    __syncwarp();
    float lq0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
    lq0 += __shfl_xor_sync(0xffffffffu, lq0, 2);
    float lq1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
    lq1 += __shfl_xor_sync(0xffffffffu, lq1, 2);
    float *mo = merge_o + (size_t(slot) * W + warp) * g_max * D;
    float *mml = merge_ml + (size_t(slot) * W + warp) * g_max * 2;
#pragma unroll
    for (int i = 0; i < ND; ++i) {
      const int d = i * 8 + 2 * t;
      if (g < g_max) *reinterpret_cast<float2 *>(mo + g * D + d) = make_float2(o[i][0], o[i][1]);
      if (g + 8 < g_max)
        *reinterpret_cast<float2 *>(mo + (g + 8) * D + d) = make_float2(o[i][2], o[i][3]);
    }
    if (t == 0) {
      if (g < g_max) {
        mml[g * 2] = m0;
        mml[g * 2 + 1] = lq0;
      }
      if (g + 8 < g_max) {
        mml[(g + 8) * 2] = m1;
        mml[(g + 8) * 2 + 1] = lq1;
      }
    }
    __threadfence_block();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(slot_cnt + slot, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == W - 1) {
      __threadfence_block();
      merge_piece(k);
      __syncwarp();
      if (lane == 0) {
        slot_cnt[slot] = 0;
        __threadfence_block();
        *reinterpret_cast<volatile int *>(slot_gen + slot) = gen + 1;
      }
      __syncwarp();
      if (k + S < n_pieces) issue_q(k + S);
    }
  };

  // ---- main loop -------------------------------------------------------------
  // prologue: positions 0 .. NS-2 in flight
  int inf0 = 0, inf1 = 0, inf2 = 0, inf3 = 0;  // unit info by stage (NS <= 4)
  auto keep_info = [&](int stage, int inf) {
    if (stage == 0) inf0 = inf;
    else if (stage == 1) inf1 = inf;
    else if (stage == 2) inf2 = inf;
    else inf3 = inf;
  };
  for (int j = 0; j < NS - 1 && j < n_w; ++j) keep_info(j, issue(j));

  int cb = 0, csegl = 0, cnu = 1, csc = 0;  // segment cursor of this warp's units
  int64_t cstart = 0, cend = 0;
  if (n_w > 0) {
    const Loc l0c = locate(lo + warp, cum, segcum, B, segs_per_seq);
    cb = l0c.b;
    csegl = l0c.segl;
    cnu = l0c.nunits;
    csc = l0c.sc;
    cstart = l0c.seg_start;
    cend = cstart + cnu;
  }
  uint32_t qa[KS][4];
  int cur = 0;
  bool have_q = false;
  bool failed = false;
  for (int j = 0; j < n_w; ++j) {
    // keep NS-1 units in flight: issue position j+NS-1 before computing j
    const int jn = j + NS - 1;
    if (jn < n_w) {
      if ((jn & 31) == 0) {  // rotate the lookup pipeline: B -> C, A -> B, new A
        stage_c();
        stage_b();
        stage_a((jn >> 5) + 2);
      }
      keep_info(jn % NS, issue(jn));
    }
    const int64_t u = lo + warp + int64_t(j) * W;
    while (u >= cend) {  // advance the segment cursor
      if (++csegl == segs_per_seq) {
        csegl = 0;
        do {
          ++cb;
        } while (cum[cb + 1] == cum[cb]);
        cnu = int(cum[cb + 1] - cum[cb]) / segs_per_seq;
      }
      ++csc;
      cstart = cend;
      cend = cstart + cnu;
    }
    const int k = csc - sc0;
    while (cur < k) {
      finalize(cur);
      ++cur;
      reset();
      have_q = false;
    }
    if (!have_q) {
      const bool q_in = ptx::mbar_wait_bounded(ptx::smem_u32(qbars + cur % S),
                                               uint32_t((cur / S) & 1), kLimitNs);
      if (!__all_sync(0xffffffffu, q_in)) {
        failed = true;
        break;
      }
      const T *qt = qslots + (cur % S) * 16 * RS;
      const int mi2 = lane >> 3, r = lane & 7;
      const int row = (mi2 & 1) * 8 + r;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        ptx::ldsm_x4(ptx::smem_u32(qt + row * RS + ks * 16 + (mi2 >> 1) * 8), qa[ks][0],
                     qa[ks][1], qa[ks][2], qa[ks][3]);
      }
      have_q = true;
    }
    const int st = j % NS;
    const int inf = st == 0 ? inf0 : st == 1 ? inf1 : st == 2 ? inf2 : inf3;
    const bool landed =
        ptx::mbar_wait_bounded(ptx::smem_u32(wbars + st), uint32_t((j / NS) & 1), kLimitNs);
    if (!__all_sync(0xffffffffu, landed)) {
      failed = true;
      break;
    }
    const uint32_t kt = ptx::smem_u32(wring + size_t(st) * 2 * TILE_B);
    const uint32_t vt = kt + TILE_B;
    auto sw = [](uint32_t tile, int tok, int d0) -> uint32_t {
      const int ch = d0 >> 3;
      const int pc = ch < (CPR & ~7) ? (ch ^ (tok & 7)) : ch;  // same rule as the stores
      return tile + tok * (D * 2) + (pc << 4);
    };
    if (inf & 1) {
      const int nvalid = inf >> 1;
      // S = Q K^T with two independent accumulation chains (even / odd k-steps)
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      float s2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      {
        const int mi2 = lane >> 3, r = lane & 7;
        const int tok = (mi2 >> 1) * 8 + r;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t b0, b1, b2, b3;
          ptx::ldsm_x4(sw(kt, tok, ks * 16 + (mi2 & 1) * 8), b0, b1, b2, b3);
          float(*acc)[4] = (ks & 1) ? s2 : s;
          MMA::run(acc[0], qa[ks], b0, b1);
          MMA::run(acc[1], qa[ks], b2, b3);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) s[nt][jj] += s2[nt][jj];
      }
      if (nvalid < kUnitTok) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int tok = nt * 8 + 2 * t + (jj & 1);
            s[nt][jj] = tok < nvalid ? s[nt][jj] : -INFINITY;
          }
      }
      // online softmax in the log2 domain; the scale (> 0) is folded into the
      // exponent, so the running max is kept on scaled values
      const float sc = p.scale_log2;
      float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
      float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0 * sc), mn1 = fmaxf(m1, mx1 * sc);
      const float a0 = ptx::fast_exp2(m0 - mn0), a1 = ptx::fast_exp2(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = ptx::fast_exp2(fmaf(s[nt][0], sc, -mn0));
        s[nt][1] = ptx::fast_exp2(fmaf(s[nt][1], sc, -mn0));
        s[nt][2] = ptx::fast_exp2(fmaf(s[nt][2], sc, -mn1));
        s[nt][3] = ptx::fast_exp2(fmaf(s[nt][3], sc, -mn1));
        ps0 += s[nt][0] + s[nt][1];
        ps1 += s[nt][2] + s[nt][3];
      }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
      if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
        for (int d = 0; d < ND; ++d) {
          o[d][0] *= a0;
          o[d][1] *= a0;
          o[d][2] *= a1;
          o[d][3] *= a1;
        }
      }
      uint32_t pa[4], pl[4];  // P = hi + lo (16-bit each)
      MMA::split(s[0][0], s[0][1], pa[0], pl[0]);
      MMA::split(s[0][2], s[0][3], pa[1], pl[1]);
      MMA::split(s[1][0], s[1][1], pa[2], pl[2]);
      MMA::split(s[1][2], s[1][3], pa[3], pl[3]);
      {
        const int mi2 = lane >> 3, r = lane & 7;
        const int tok = (mi2 & 1) * 8 + r;
#pragma unroll
        for (int jj = 0; jj < KS; ++jj) {
          uint32_t b0, b1, b2, b3;
          ptx::ldsm_x4_t(sw(vt, tok, jj * 16 + (mi2 >> 1) * 8), b0, b1, b2, b3);
          MMA::run(o[2 * jj], pa, b0, b1);
          MMA::run(o[2 * jj], pl, b0, b1);
          MMA::run(o[2 * jj + 1], pa, b2, b3);
          MMA::run(o[2 * jj + 1], pl, b2, b3);
        }
      }
    }
    __syncwarp();  // every lane is done with stage st before it is refilled
  }
  if (failed) {
    for (int st = 0; st < NS; ++st) {  // let copies still in flight land
      ptx::mbar_wait_bounded(ptx::smem_u32(wbars + st), 0, 2000000ull);
      ptx::mbar_wait_bounded(ptx::smem_u32(wbars + st), 1, 2000000ull);
    }
    if (lane == 0) {
      atomicOr(p.diag, int32_t(kDiagWaitTimeout));
      s_fail = 1;
    }
    return;
  }
  while (cur < n_pieces) {
    if (s_fail) break;
    finalize(cur);
    ++cur;
    reset();
  }
}

// Second pass: pieces of segments that straddle CTAs, merged by log-sum-exp.
template <typename T, int D>
__global__ void merge(const Params p, int P) {
  const int row = blockIdx.x;  // b * hq + h
  const int b = row / p.hq, h = row % p.hq;
  const int64_t *cum = p.cum_out;
  const int B = p.batch;
  const int nht = p.n_head_tiles, segs_per_seq = p.hkv * nht;
  const int64_t U = cum[B];
  if (cum[b + 1] == cum[b] || U == 0) return;
  const int kvh = int(int64_t(h) * p.hkv / p.hq);
  const int g_lo = int((int64_t(kvh) * p.hq + p.hkv - 1) / p.hkv);
  const int ht = (h - g_lo) / 16;
  const int hlo = g_lo + ht * 16;
  const int segl = kvh * nht + ht;
  const int nunits = int((cum[b + 1] - cum[b]) / segs_per_seq);
  const int64_t s_start = cum[b] + int64_t(segl) * nunits;
  const int cf = cta_of(s_start, U, P), cl = cta_of(s_start + nunits - 1, U, P);
  if (cf == cl) return;
  const int sc = p.segcum_out[b] + segl;
  const int hr = h - hlo;
  // CTAs cf..cl hold the pieces, except those whose slice is empty (more CTAs
  // than units): they wrote nothing and are skipped.
  auto has_piece = [&](int c) { return (int64_t(c) * U) / P != ((int64_t(c) + 1) * U) / P; };
  float M = -INFINITY;
  for (int c = cf; c <= cl; ++c) {
    if (has_piece(c)) M = fmaxf(M, p.part_lse[(int64_t(sc) + c) * p.g_max + hr]);
  }
  float wsum = 0.f;
  for (int c = cf; c <= cl; ++c) {
    if (has_piece(c)) wsum += ptx::fast_exp2(p.part_lse[(int64_t(sc) + c) * p.g_max + hr] - M);
  }
  const float inv = 1.f / wsum;
  T *dst = static_cast<T *>(p.out) + int64_t(row) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int c = cf; c <= cl; ++c) {
      if (!has_piece(c)) continue;
      const int64_t gi = int64_t(sc) + c;
      acc += p.part_o[(gi * p.g_max + hr) * D + d] *
             ptx::fast_exp2(p.part_lse[gi * p.g_max + hr] - M);
    }
    dst[d] = ptx::from_f32<T>(acc * inv);
  }
}

}  // namespace sk
}  // namespace dev
}  // namespace kcmm
