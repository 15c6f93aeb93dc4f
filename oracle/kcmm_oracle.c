/*
 * TEST INFRASTRUCTURE -- NOT PART OF THE PRODUCT.
 *
 * CPU oracle for the KV-cache hot path: a plain-C restatement of the
 * reference's arithmetic, used only by tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg as the checker.  Nothing in lattice_b200/
 * links, loads or calls it.
 *
 * Parity pins (see tests/test_oracle_*.py):
 *   - paged decode attention: ref src/cuda/kernels/kcmm_vllm_paged_attn.cu:40-101
 *     and the fp32 torch reference ref scripts/kcmm/kv_read_plan.py:735-781;
 *     checked against the reference kernel itself compiled for the host
 *     (oracle/_ref) and against KAT ref scripts/kcmm/non_default_stream_ffi_smoke.py:172-179.
 *   - RMSNorm: ref src/cuda/kernels/rms_norm.cu:14-35.
 *   - RoPE: ref src/cuda/kernels/rope.cu:13-52 ("reference" mode, base as a
 *     parameter) plus GPT-J and NeoX conventions.
 *   - device-slot KV write: ref src/cuda/kernels/kcmm_vllm_kv_write.cu:37-65.
 *   - block copies / swap layout: ref src/kcmm/tiering.rs:1414-1458, 1755-1798.
 *
 * Math is done in double where the reference accumulates in fp32, so the
 * oracle is at least as accurate as the fp32 reference path it stands for.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2 };

/* --- 16-bit float conversions (IEEE round-to-nearest-even) --------------- */

static inline float bf16_to_f32(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t v) {
  _Float16 h;
  memcpy(&h, &v, 2);
  return (float)h;
}

static inline uint16_t f32_to_f16(float f) {
  _Float16 h = (_Float16)f;
  uint16_t v;
  memcpy(&v, &h, 2);
  return v;
}

static inline double load_elem(int dt, const void *base, int64_t idx) {
  switch (dt) {
    case DT_F16: return f16_to_f32(((const uint16_t *)base)[idx]);
    case DT_BF16: return bf16_to_f32(((const uint16_t *)base)[idx]);
    default: return ((const float *)base)[idx];
  }
}

static inline void store_elem(int dt, void *base, int64_t idx, double v) {
  switch (dt) {
    case DT_F16: ((uint16_t *)base)[idx] = f32_to_f16((float)v); break;
    case DT_BF16: ((uint16_t *)base)[idx] = f32_to_bf16((float)v); break;
    default: ((float *)base)[idx] = (float)v; break;
  }
}

uint16_t oracle_f32_to_bf16(float f) { return f32_to_bf16(f); }
float oracle_bf16_to_f32(uint16_t v) { return bf16_to_f32(v); }

/* --- paged decode attention ------------------------------------------------
 * offsets[] are in 2-byte units (byte offset / 2) whatever the element type;
 * the element of token t, kv head kvh, dim i lives at byte
 *   offsets[blk]*2 + ((t % bs)*hkv*d + kvh*d + i) * esize.
 * seq_lens[b] <= 0 leaves out / out_f32 of sequence b untouched.
 */
void oracle_paged_attn(int dt, const void *q, void *out, float *out_f32, const void *va_k,
                       const void *va_v, const int32_t *tables, const int32_t *seq_lens,
                       const uint64_t *offsets, int batch, int hq, int hkv, int d, int bs,
                       int max_bps, float scale) {
  const int esize = dt == DT_F32 ? 4 : 2;
  #pragma omp parallel for schedule(dynamic, 1)
  for (int64_t bh = 0; bh < (int64_t)batch * hq; ++bh) {
    const int b = (int)(bh / hq), h = (int)(bh % hq);
    const int kvh = (int)((int64_t)h * hkv / hq);
    const int L = seq_lens[b];
    if (L <= 0) continue;
    double *logits = (double *)malloc(sizeof(double) * (size_t)L);
    double *acc = (double *)calloc((size_t)d, sizeof(double));
    double *qv = (double *)malloc(sizeof(double) * (size_t)d);
    for (int i = 0; i < d; ++i) qv[i] = load_elem(dt, q, bh * d + i);
    double mx = -INFINITY;
    for (int t = 0; t < L; ++t) {
      const int blk = tables[(int64_t)b * max_bps + t / bs];
      const uint8_t *kb = (const uint8_t *)va_k + offsets[blk] * 2 +
                          ((int64_t)(t % bs) * hkv * d + (int64_t)kvh * d) * esize;
      double s = 0.0;
      for (int i = 0; i < d; ++i) s += qv[i] * load_elem(dt, kb, i);
      s *= (double)scale;
      logits[t] = s;
      if (s > mx) mx = s;
    }
    double den = 0.0;
    for (int t = 0; t < L; ++t) {
      logits[t] = exp(logits[t] - mx);
      den += logits[t];
    }
    for (int t = 0; t < L; ++t) {
      const int blk = tables[(int64_t)b * max_bps + t / bs];
      const uint8_t *vb = (const uint8_t *)va_v + offsets[blk] * 2 +
                          ((int64_t)(t % bs) * hkv * d + (int64_t)kvh * d) * esize;
      const double p = logits[t] / den;
      for (int i = 0; i < d; ++i) acc[i] += p * load_elem(dt, vb, i);
    }
    for (int i = 0; i < d; ++i) {
      if (out_f32) out_f32[bh * d + i] = (float)acc[i];
      if (out) store_elem(dt, out, bh * d + i, acc[i]);
    }
    free(logits);
    free(acc);
    free(qv);
  }
}

/* --- chunked prefill: causal paged attention for a chunk of new tokens ---------
 * The reference has no prefill kernel (ref src/model/transformer.rs:50-65 runs
 * prefill as decode steps); each query row is the decode computation above
 * (ref kcmm_vllm_paged_attn.cu:40-101, GQA map h*hkv/hq) over keys
 * [0, position], position = ctx_lens[b] - chunk length + i.  q/out rows are
 * [total_tokens][hq][d]; rows whose token has mask[token] == 0 are skipped
 * (mask may be NULL). */
void oracle_paged_prefill(int dt, const void *q, float *out_f32, const void *va_k,
                          const void *va_v, const int32_t *tables, const int32_t *q_start,
                          const int32_t *ctx_lens, const uint64_t *offsets, const uint8_t *mask,
                          int batch, int hq, int hkv, int d, int bs, int max_bps, float scale) {
  const int esize = dt == DT_F32 ? 4 : 2;
  const int64_t total = q_start[batch];
  #pragma omp parallel for schedule(dynamic, 4)
  for (int64_t th = 0; th < total * hq; ++th) {
    const int64_t tok = th / hq;
    const int h = (int)(th % hq);
    if (mask && !mask[tok]) continue;
    int b = 0;
    while (b + 1 < batch && q_start[b + 1] <= tok) ++b;
    const int qlen = q_start[b + 1] - q_start[b];
    const int i = (int)(tok - q_start[b]);
    const int L = ctx_lens[b] - qlen + i + 1;  /* keys [0, position] */
    const int kvh = (int)((int64_t)h * hkv / hq);
    if (L <= 0) continue;
    double *logits = (double *)malloc(sizeof(double) * (size_t)L);
    double *acc = (double *)calloc((size_t)d, sizeof(double));
    double *qv = (double *)malloc(sizeof(double) * (size_t)d);
    for (int e = 0; e < d; ++e) qv[e] = load_elem(dt, q, th * d + e);
    double mx = -INFINITY;
    for (int t = 0; t < L; ++t) {
      const int blk = tables[(int64_t)b * max_bps + t / bs];
      const uint8_t *kb = (const uint8_t *)va_k + offsets[blk] * 2 +
                          ((int64_t)(t % bs) * hkv * d + (int64_t)kvh * d) * esize;
      double sc = 0.0;
      for (int e = 0; e < d; ++e) sc += qv[e] * load_elem(dt, kb, e);
      sc *= (double)scale;
      logits[t] = sc;
      if (sc > mx) mx = sc;
    }
    double den = 0.0;
    for (int t = 0; t < L; ++t) {
      logits[t] = exp(logits[t] - mx);
      den += logits[t];
    }
    for (int t = 0; t < L; ++t) {
      const int blk = tables[(int64_t)b * max_bps + t / bs];
      const uint8_t *vb = (const uint8_t *)va_v + offsets[blk] * 2 +
                          ((int64_t)(t % bs) * hkv * d + (int64_t)kvh * d) * esize;
      const double pr = logits[t] / den;
      for (int e = 0; e < d; ++e) acc[e] += pr * load_elem(dt, vb, e);
    }
    for (int e = 0; e < d; ++e) out_f32[th * d + e] = (float)acc[e];
    free(logits);
    free(acc);
    free(qv);
  }
}

/* --- RMSNorm (ref rms_norm.cu:14-35): y = ((x * (1/sqrt(mean(x^2)+eps))) * w) -- */
void oracle_rms_norm(int dt, const void *x, const void *w, void *y, int rows, int cols,
                     float eps) {
  #pragma omp parallel for
  for (int r = 0; r < rows; ++r) {
    double ss = 0.0;
    for (int c = 0; c < cols; ++c) {
      double v = load_elem(dt, x, (int64_t)r * cols + c);
      ss += v * v;
    }
    const float inv = 1.0f / sqrtf((float)(ss / cols) + eps);
    for (int c = 0; c < cols; ++c) {
      float v = (float)load_elem(dt, x, (int64_t)r * cols + c) * inv;
      store_elem(dt, y, (int64_t)r * cols + c, v * (float)load_elem(dt, w, c));
    }
  }
}

/* --- RoPE ----------------------------------------------------------------------
 * mode 0 "reference": pairs (2i, 2i+1), theta_i = 1/base^(2*floor(i/2)/d)
 *        (ref rope.cu:18 with base 10000 -> parameter);
 * mode 1 GPT-J: pairs (2i, 2i+1), theta_i = 1/base^(2i/d);
 * mode 2 NeoX:  pairs (i, i+d/2), theta_i = 1/base^(2i/d).
 * angle = (float)pos * theta in fp32 as the kernels form it; cos/sin in double.
 */
static void rope_table(int d, int mode, float base, int pos, float *cs, float *sn) {
  for (int i = 0; i < d / 2; ++i) {
    const float e = mode == 0 ? (float)(2 * (i / 2)) / (float)d : (float)(2 * i) / (float)d;
    const float theta = 1.0f / powf(base, e);
    const float ang = (float)pos * theta;
    cs[i] = (float)cos((double)ang);
    sn[i] = (float)sin((double)ang);
  }
}

static void rope_row(int dt, const void *src, void *dst, int64_t base_idx, int d, int mode,
                     const float *cs, const float *sn) {
  for (int i = 0; i < d / 2; ++i) {
    const int64_t a = mode == 2 ? base_idx + i : base_idx + 2 * i;
    const int64_t b = mode == 2 ? base_idx + i + d / 2 : base_idx + 2 * i + 1;
    const float x0 = (float)load_elem(dt, src, a), x1 = (float)load_elem(dt, src, b);
    store_elem(dt, dst, a, x0 * cs[i] - x1 * sn[i]);
    store_elem(dt, dst, b, x0 * sn[i] + x1 * cs[i]);
  }
}

/* In-place rotation of x[tokens][heads][d] at per-token positions. */
void oracle_rope(int dt, void *x, int tokens, int heads, int d, const int32_t *pos, float base,
                 int mode) {
  float *cs = (float *)malloc(sizeof(float) * (size_t)d);
  float *sn = cs + d / 2;
  for (int t = 0; t < tokens; ++t) {
    rope_table(d, mode, base, pos[t], cs, sn);
    for (int h = 0; h < heads; ++h) rope_row(dt, x, x, ((int64_t)t * heads + h) * d, d, mode, cs, sn);
  }
  free(cs);
}

/* --- device-slot KV write (ref kcmm_vllm_kv_write.cu:37-65) ------------------
 * 16-bit words; returns the status word the kernel would leave (first error
 * in row order: 1 = block id >= offsets_len, 2 = block marked free).
 */
int32_t oracle_slot_write(uint16_t *va_k, uint16_t *va_v, const int64_t *slots,
                          const uint64_t *offsets, const uint8_t *valid, int offsets_len,
                          const uint16_t *k_src, const uint16_t *v_src, int rows, int step,
                          int bs) {
  int32_t status = 0;
  for (int r = 0; r < rows; ++r) {
    const int64_t slot = slots[r];
    if (slot < 0) continue;
    const int64_t blk = slot / bs;
    if (blk >= offsets_len) {
      if (!status) status = 1;
      continue;
    }
    if (valid && !valid[blk]) {
      if (!status) status = 2;
      continue;
    }
    const int64_t dst = (int64_t)offsets[blk] + (slot % bs) * step;
    memcpy(va_k + dst, k_src + (int64_t)r * step, (size_t)step * 2);
    memcpy(va_v + dst, v_src + (int64_t)r * step, (size_t)step * 2);
  }
  return status;
}

/* --- fused RMSNorm + RoPE + append (bf16) -----------------------------------
 * The composition rms_norm -> rope -> slot write of ref
 * src/model/llama_transformer.rs:313-333 for one batch of decode tokens,
 * with per-token positions.
 */
int32_t oracle_fused_norm_rope_append(const uint16_t *x, const uint16_t *w, uint16_t *normed,
                                      int tokens, int hidden, float eps, uint16_t *q, int hq,
                                      const uint16_t *k, const uint16_t *v, const int32_t *pos,
                                      float base, int mode, const int64_t *slots,
                                      const uint64_t *offsets, const uint8_t *valid,
                                      int offsets_len, int hkv, int d, int bs, uint16_t *va_k,
                                      uint16_t *va_v) {
  oracle_rms_norm(DT_BF16, x, w, normed, tokens, hidden, eps);
  oracle_rope(DT_BF16, q, tokens, hq, d, pos, base, mode);
  const int step = hkv * d;
  uint16_t *krot = (uint16_t *)malloc((size_t)tokens * step * 2);
  memcpy(krot, k, (size_t)tokens * step * 2);
  oracle_rope(DT_BF16, krot, tokens, hkv, d, pos, base, mode);
  int32_t st = oracle_slot_write(va_k, va_v, slots, offsets, valid, offsets_len, krot, v, tokens,
                                 step, bs);
  free(krot);
  return st;
}

/* --- whole-block copies -------------------------------------------------------
 * regions[2L] host buffers standing for the K/V layer regions.
 * copy: block at src_off -> dst_off in every region (CoW fork).
 * swap out: host slot = [K0][V0]...[K(L-1)][V(L-1)] (ref tiering.rs:1414-1421).
 */
void oracle_copy_blocks(uint8_t **regions, int num_layers, const uint64_t *src_off,
                        const uint64_t *dst_off, int count, uint64_t block_bytes) {
  for (int i = 0; i < count; ++i)
    for (int r = 0; r < 2 * num_layers; ++r)
      memmove(regions[r] + dst_off[i], regions[r] + src_off[i], block_bytes);
}

void oracle_swap_blocks(uint8_t **regions, int num_layers, const uint64_t *va_off,
                        const uint64_t *host_off, int count, uint64_t block_bytes, uint8_t *host,
                        int dir) {
  for (int i = 0; i < count; ++i)
    for (int r = 0; r < 2 * num_layers; ++r) {
      uint8_t *dev = regions[r] + va_off[i];
      uint8_t *h = host + host_off[i] + (uint64_t)r * block_bytes;
      if (dir == 0) memcpy(h, dev, block_bytes);
      else memcpy(dev, h, block_bytes);
    }
}
