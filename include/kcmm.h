/*
 * kcmm.h -- C ABI of the B200 KV-cache manager (KCMM).
 *
 * This header is the drop-in boundary of the library `libkcmm.so` (also
 * reachable as `libbaseline_llm_os.so`, the name existing ctypes callers
 * load).  Every declaration in the first part keeps the name, argument
 * order, types and error behaviour of the Lattice reference ABI
 * (include/kcmm.h and src/kcmm/ffi.rs in Vitalrubbish/Lattice); the line
 * cited beside each one is the reference declaration it replaces.  The
 * second part ("B200 additions") holds new, additive exports that follow
 * the same conventions.
 *
 * Conventions shared by every function:
 *   - `int` results: 0 = success, -1 = failure.  Count/size results are 0
 *     on failure; pointer-sized VA results are 0 on failure.
 *   - A failure stores a message in the pool; read it with
 *     kcmm_get_last_error().  A NULL pool is a no-op / failure.
 *   - Every `uint64_t *_ptr` argument is a CUDA device virtual address
 *     (or a raw cudaStream_t for `stream_ptr`; 0 = legacy default stream).
 *     The caller owns those buffers and keeps them alive until the stream
 *     has executed the queued work.
 *   - KV pages live in per-layer K and V VA regions.  A block occupies
 *     `block_bytes = block_size * kv_heads * head_dim * 2` bytes in each
 *     region, laid out token-major: [block_size][kv_heads][head_dim] of
 *     16-bit elements (f16 or bf16 -- the pool stores bits, not a type).
 *   - All functions are thread-safe.
 */
#ifndef KCMM_H
#define KCMM_H

#ifdef __cplusplus
extern "C" {
#endif

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

/* ------------------------------------------------------------------------- */
/* Types                                                                     */
/* ------------------------------------------------------------------------- */

/** Opaque pool handle (ref include/kcmm.h:36). */
typedef struct kcmm_pool_t kcmm_pool_t;

/** Per-sequence eviction hints (ref include/kcmm.h:43-52). */
typedef enum {
    KCMM_HINT_MULTI_TURN     = 1,
    KCMM_HINT_NEAR_END       = 2,
    KCMM_HINT_SYSTEM_PROMPT  = 3,
    KCMM_HINT_HIGH_PRIORITY  = 4,
    KCMM_HINT_LOW_PRIORITY   = 5,
    KCMM_HINT_ATTENTION_SINK = 6,
    KCMM_HINT_HEAVY_HITTER   = 7,
    KCMM_HINT_EVICTABLE      = 8,
} kcmm_hint_t;

/** Per-block protection levels (ref include/kcmm.h:55-59). */
typedef enum {
    KCMM_PROTECT_NEVER_EVICT = 0,
    KCMM_PROTECT_PREFERRED   = 1,
    KCMM_EVICT_PREFERRED     = 2,
} kcmm_protection_t;

/** Where a block's bytes live (ref include/kcmm.h:62-68). */
typedef enum {
    KCMM_LOC_GPU_RESIDENT  = 0,
    KCMM_LOC_CPU_RESIDENT  = 1,
    KCMM_LOC_NVME_RESIDENT = 2,
    KCMM_LOC_EVICTING      = 3,
    KCMM_LOC_RESTORING     = 4,
} kcmm_block_location_t;

/**
 * Pool configuration (ref include/kcmm.h:81-144).  376 bytes on LP64; the
 * field order and offsets are part of the ABI (max_seq_len @336,
 * low_watermark_threshold @344, background_evict_interval_ms @352,
 * attention_sink_blocks @360, recent_window_blocks @368).  Zero (or, for the
 * watermark, non-positive) fields take defaults: block_size 16, max_blocks
 * 16384, prefetch_window 4, max_batch_blocks 64, watermark 0.2, interval
 * 100 ms, sink 1, window 4.  num_layers, kv_heads, head_dim, max_batch and
 * max_seq_len are required.
 */
typedef struct {
    size_t   block_size;
    size_t   max_blocks;
    char     cpu_cache_path[256];
    int32_t  tiering;
    int32_t  eviction_policy;           /* 0 = lru, 1 = lfu, 2 = fifo */
    size_t   prefetch_window;
    size_t   max_batch_blocks;
    size_t   device_ordinal;
    size_t   num_layers;
    size_t   kv_heads;
    size_t   head_dim;
    size_t   max_batch;
    size_t   max_seq_len;
    float    low_watermark_threshold;
    uint64_t background_evict_interval_ms;
    size_t   attention_sink_blocks;
    size_t   recent_window_blocks;
} kcmm_config_t;

/** Fragmentation / tier snapshot (ref include/kcmm.h:151-161). */
typedef struct {
    double   ifr;
    double   pme;
    double   bu;
    double   rfi;
    uint64_t gpu_blocks;
    uint64_t cpu_blocks;
    uint64_t nvme_blocks;
    uint64_t eviction_count;
    uint64_t restoration_count;
} kcmm_metrics_t;

/** Latency histogram in microseconds; buckets end at 100, 250, 500, 1000, 2500,
 *  5000, 10000 us and above (ref src/kcmm/metrics.rs:29-74). */
typedef struct {
    uint64_t count;
    uint64_t sum_us;
    uint64_t min_us;
    uint64_t max_us;
    uint64_t buckets[9];
} kcmm_latency_histogram_t;

/** The reference's extended KcmmMetrics (ref src/kcmm/metrics.rs:77-114), which its C
 *  ABI does not export: kcmm_metrics_t plus eviction observability. */
typedef struct {
    kcmm_metrics_t base;
    uint64_t evicted_blocks_total;
    uint64_t restored_blocks_total;
    uint64_t eviction_failures;
    uint64_t restoration_failures;
    uint64_t background_eviction_count;
    kcmm_latency_histogram_t eviction_latency;
    kcmm_latency_histogram_t restoration_latency;
} kcmm_metrics_ext_t;

/** Per-policy counters (ref src/kcmm/metrics.rs:14-20), keyed by the policy active
 *  when the operation ran. */
typedef struct {
    uint64_t eviction_count;
    uint64_t restoration_count;
    uint64_t evicted_blocks;
    uint64_t restored_blocks;
    double   avg_evict_batch_size;
} kcmm_policy_stats_t;

/** Pool statistics (ref include/kcmm.h:164-179). */
typedef struct {
    uint32_t blocks_in_use;
    uint32_t total_blocks;
    uint32_t total_physical_blocks;
    uint32_t free_physical_blocks;
    uint32_t active_sequences;
    uint32_t num_layers;
    uint32_t blocks_per_superblock;
    uint32_t superblock_count;
    uint32_t block_size;
    uint32_t max_blocks_per_seq;
    uint32_t block_bytes;
    int32_t  tiering_enabled;
    int32_t  sharing_enabled;
    float    physical_idle_ratio;
} kcmm_pool_stats_t;

/* ------------------------------------------------------------------------- */
/* Lifecycle and errors                                                      */
/* ------------------------------------------------------------------------- */

/** Create a pool; NULL on failure (ref include/kcmm.h:193). */
kcmm_pool_t *kcmm_pool_create(const kcmm_config_t *config);
/** Synchronise, unmap and release everything (ref include/kcmm.h:203). */
void kcmm_pool_destroy(kcmm_pool_t *pool);
/** Copy the last error into buf; bytes written or 0 (ref include/kcmm.h:218). */
size_t kcmm_get_last_error(kcmm_pool_t *pool, char *buf, size_t max_len);
/** Clear the last error (ref include/kcmm.h:225). */
void kcmm_clear_error(kcmm_pool_t *pool);

/* ------------------------------------------------------------------------- */
/* Block allocation and sequences                                            */
/* ------------------------------------------------------------------------- */

/** Allocate blocks in lockstep across all layers (ref include/kcmm.h:239). */
int kcmm_alloc_blocks(kcmm_pool_t *pool, uint32_t num_blocks, uint32_t *out_blocks);
/** Release blocks; a shared block is only released at refcount 0 (ref include/kcmm.h:249). */
int kcmm_free_blocks(kcmm_pool_t *pool, const uint32_t *blocks, uint32_t num);
/** Register a sequence; indices are never reused (ref include/kcmm.h:264). */
int kcmm_register_sequence(kcmm_pool_t *pool, const uint32_t *block_table,
                           uint32_t num_blocks, uint32_t *out_seq_idx);
/** Free a sequence's blocks and clear its table (ref include/kcmm.h:277). */
int kcmm_unregister_sequence(kcmm_pool_t *pool, uint32_t seq_idx);
/** Mark hot (ref include/kcmm.h:288). */
void kcmm_touch(kcmm_pool_t *pool, uint32_t seq_idx);
/** Mark cold (ref include/kcmm.h:299). */
void kcmm_cool(kcmm_pool_t *pool, uint32_t seq_idx);
/** Set token length (ref include/kcmm.h:308). */
void kcmm_update_seq_len(kcmm_pool_t *pool, uint32_t seq_idx, uint32_t len);
/** Token length or 0 (ref include/kcmm.h:317). */
uint32_t kcmm_get_seq_len(kcmm_pool_t *pool, uint32_t seq_idx);
/** Append one block id to a table (ref include/kcmm.h:327). */
int kcmm_append_block_to_sequence(kcmm_pool_t *pool, uint32_t seq_idx, uint32_t block_idx);
/** Copy a block table out (ref include/kcmm.h:340). */
int kcmm_get_block_table(kcmm_pool_t *pool, uint32_t seq_idx, uint32_t *out_table,
                         uint32_t max_blocks, uint32_t *out_count);

/* ------------------------------------------------------------------------- */
/* Block queries and VA accessors                                            */
/* ------------------------------------------------------------------------- */

/** Byte offset of a live block inside every layer region, else 0 (ref include/kcmm.h:355). */
uint64_t kcmm_get_block_va_offset(kcmm_pool_t *pool, uint32_t block_idx);
/** Offsets table indexed by block id, in 2-byte units, 0 if free (ref include/kcmm.h:369). */
int kcmm_get_all_block_offsets_f16(kcmm_pool_t *pool, uint64_t *out_offsets,
                                   uint32_t max_blocks, uint32_t *out_count);
/** In-use byte per block id (ref src/kcmm/ffi.rs:920). */
int kcmm_get_all_block_valid(kcmm_pool_t *pool, uint8_t *out_valid,
                             uint32_t max_blocks, uint32_t *out_count);
/** Location of a live block (ref include/kcmm.h:381). */
int kcmm_get_block_location(kcmm_pool_t *pool, uint32_t block_idx,
                            kcmm_block_location_t *out_location);
/** Byte offsets of a sequence's blocks (ref include/kcmm.h:394). */
int kcmm_get_block_table_va_offsets(kcmm_pool_t *pool, uint32_t seq_idx,
                                    uint64_t *out_offsets, uint32_t max_blocks,
                                    uint32_t *out_count);
/** K region base of a layer, 0 if out of range (ref include/kcmm.h:409). */
uint64_t kcmm_get_va_k(kcmm_pool_t *pool, uint32_t layer);
/** V region base of a layer, 0 if out of range (ref include/kcmm.h:418). */
uint64_t kcmm_get_va_v(kcmm_pool_t *pool, uint32_t layer);
/** Monotonic counter bumped by every in-use / mapping change (ref src/kcmm/ffi.rs:2143). */
uint64_t kcmm_block_state_epoch(kcmm_pool_t *pool);

/* ------------------------------------------------------------------------- */
/* KV append (reshape_and_cache)                                             */
/* ------------------------------------------------------------------------- */

/**
 * Write row b of k_src/v_src ([batch, kv_heads*head_dim], 16-bit) to
 * position positions[b] of sequence seq_indices[b]; legacy stream
 * (ref include/kcmm.h:438).
 */
int kcmm_append_kv_step(kcmm_pool_t *pool, uint32_t layer_idx,
                        const uint32_t *seq_indices, const uint32_t *positions,
                        uint32_t batch, uint64_t k_src_ptr, uint64_t v_src_ptr);
/** Same, addressed by host slot ids `block*block_size+offset`; slot<0 skipped (ref include/kcmm.h:459). */
int kcmm_append_kv_slots(kcmm_pool_t *pool, uint32_t layer_idx,
                         const int64_t *slot_mapping, uint32_t batch,
                         uint64_t k_src_ptr, uint64_t v_src_ptr);
/** Same on a caller stream (ref include/kcmm.h:475). */
int kcmm_append_kv_slots_on_stream(kcmm_pool_t *pool, uint32_t layer_idx,
                                   const int64_t *slot_mapping, uint32_t batch,
                                   uint64_t k_src_ptr, uint64_t v_src_ptr,
                                   uint64_t stream_ptr);
/**
 * Device-resident slot write (ref src/kcmm/ffi.rs:1399).  The optional
 * int32 status word is set once to 1 (block id >= block_offsets_f16_len)
 * or 2 (valid_blocks marks the block free); the caller zeroes it first.
 */
int kcmm_append_kv_device_slots_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t slot_mapping_ptr,
    uint64_t block_offsets_f16_ptr, uint64_t valid_blocks_ptr,
    uint32_t block_offsets_f16_len, uint32_t batch, uint64_t k_src_ptr,
    uint64_t v_src_ptr, uint64_t status_ptr, uint64_t stream_ptr);
/** Load the write kernel now (ref src/kcmm/ffi.rs:210). */
int kcmm_precompile_vllm_kv_write_f16(kcmm_pool_t *pool);

/* ------------------------------------------------------------------------- */
/* Paged decode attention                                                    */
/* ------------------------------------------------------------------------- */

/**
 * out[b,h,:] = softmax_t(scale * q[b,h,:].k_t) . v_t over t < seq_lens[b],
 * kv head = h*kv_heads/num_q_heads; f16 q/out [batch,num_q_heads,head_dim];
 * block_tables int32 [batch,max_blocks_per_seq]; seq_lens int32 [batch];
 * block_offsets_f16 u64 [n] in 2-byte units.  seq_lens[b] <= 0 leaves
 * out[b] untouched.  head_dim <= 256 and a multiple of 8; packed fields
 * <= 65535.  Launches on the legacy stream and synchronises
 * (ref include/kcmm.h:505).
 */
int kcmm_paged_attn_decode_f16(kcmm_pool_t *pool, uint32_t layer_idx,
                               uint64_t query_ptr, uint64_t out_ptr,
                               uint64_t block_tables_ptr, uint64_t seq_lens_ptr,
                               uint64_t block_offsets_f16_ptr,
                               uint32_t batch, uint32_t num_q_heads,
                               uint32_t kv_heads, uint32_t head_dim,
                               uint32_t block_size, uint32_t max_blocks_per_seq,
                               float scale);
/** Enqueue on a caller stream, no sync (ref include/kcmm.h:525). */
int kcmm_paged_attn_decode_f16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t out_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t num_q_heads,
    uint32_t kv_heads, uint32_t head_dim, uint32_t block_size,
    uint32_t max_blocks_per_seq, float scale, uint64_t stream_ptr);
/** Enqueue without selecting the pool's device first (ref include/kcmm.h:544). */
int kcmm_paged_attn_decode_f16_on_current_context_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t out_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t num_q_heads,
    uint32_t kv_heads, uint32_t head_dim, uint32_t block_size,
    uint32_t max_blocks_per_seq, float scale, uint64_t stream_ptr);
/** Load the decode kernels now (ref include/kcmm.h:559). */
int kcmm_precompile_paged_attn_decode_f16(kcmm_pool_t *pool);

/* ------------------------------------------------------------------------- */
/* Tiering                                                                   */
/* ------------------------------------------------------------------------- */

/** Evict up to count victim blocks to the host swap tier; number evicted (ref include/kcmm.h:577). */
uint32_t kcmm_evict_blocks(kcmm_pool_t *pool, uint32_t count);
/** Restore one block; new VA byte offset or 0 (ref include/kcmm.h:590). */
uint64_t kcmm_restore_evicted_block(kcmm_pool_t *pool, uint32_t block_idx);
/** Restore several blocks; resident ones are skipped (ref include/kcmm.h:603). */
int kcmm_restore_evicted_blocks(kcmm_pool_t *pool, const uint32_t *block_indices,
                                uint32_t count);
/** 1 if GPU-resident (ref include/kcmm.h:613). */
int kcmm_is_gpu_resident(kcmm_pool_t *pool, uint32_t block_idx);

/* ------------------------------------------------------------------------- */
/* Metrics, statistics, policy, hints                                        */
/* ------------------------------------------------------------------------- */

int kcmm_get_metrics(kcmm_pool_t *pool, kcmm_metrics_t *out);          /* ref include/kcmm.h:626 */
int kcmm_get_pool_stats(kcmm_pool_t *pool, kcmm_pool_stats_t *out);    /* ref include/kcmm.h:635 */
uint32_t kcmm_blocks_in_use(kcmm_pool_t *pool);                        /* ref include/kcmm.h:638 */
uint32_t kcmm_total_blocks(kcmm_pool_t *pool);                         /* ref include/kcmm.h:641 */
uint32_t kcmm_free_physical_blocks(kcmm_pool_t *pool);                 /* ref include/kcmm.h:644 */
int kcmm_has_free_blocks(kcmm_pool_t *pool);                           /* ref include/kcmm.h:647 */
uint32_t kcmm_active_sequences(kcmm_pool_t *pool);                     /* ref include/kcmm.h:650 */
/* Policy names: lru, lfu, fifo, arc, sink_window (ref src/kcmm/tiering.rs:877-895). */
int kcmm_set_eviction_policy(kcmm_pool_t *pool, const char *policy);   /* ref include/kcmm.h:664 */
uint32_t kcmm_get_eviction_policy(kcmm_pool_t *pool, char *out_policy,
                                  uint32_t max_len);                   /* ref include/kcmm.h:674 */
int kcmm_is_tiering_enabled(kcmm_pool_t *pool);                        /* ref include/kcmm.h:683 */
int kcmm_hint(kcmm_pool_t *pool, uint32_t seq_idx, kcmm_hint_t hint);  /* ref include/kcmm.h:704 */
int kcmm_protect(kcmm_pool_t *pool, uint32_t seq_idx, const uint32_t *block_ids,
                 uint32_t num_blocks, kcmm_protection_t level);        /* ref include/kcmm.h:722 */

/**
 * Share the first num_blocks blocks of src_seq with dst_seq: each block's
 * refcount rises by one, the ids are appended to dst_seq's table and
 * written to out_blocks.  (ref include/kcmm.h:744 -- a stub there.)
 */
int kcmm_share_prefix(kcmm_pool_t *pool, uint32_t src_seq, uint32_t dst_seq,
                      uint32_t num_blocks, uint32_t *out_blocks);

int kcmm_below_low_watermark(kcmm_pool_t *pool, float threshold);      /* ref include/kcmm.h:761 */
int kcmm_synchronize(kcmm_pool_t *pool);                               /* ref include/kcmm.h:771 */
uint32_t kcmm_get_block_size(kcmm_pool_t *pool);                       /* ref include/kcmm.h:778 */
uint32_t kcmm_get_max_blocks_per_seq(kcmm_pool_t *pool);               /* ref include/kcmm.h:781 */
uint32_t kcmm_get_block_bytes(kcmm_pool_t *pool);                      /* ref include/kcmm.h:784 */
uint32_t kcmm_get_num_layers(kcmm_pool_t *pool);                       /* ref include/kcmm.h:787 */
uint32_t kcmm_get_max_batch(kcmm_pool_t *pool);                        /* ref include/kcmm.h:790 */
uint32_t kcmm_get_max_seq_len(kcmm_pool_t *pool);                      /* ref include/kcmm.h:793 */

/* ========================================================================= */
/* B200 additions (no reference counterpart unless cited)                    */
/* ========================================================================= */

/**
 * bf16 twin of kcmm_paged_attn_decode_f16_on_stream: same tensor contract,
 * bf16 q/K/V/out, fp32 softmax and accumulation.  Replaces the f16-only
 * kernel behind ref src/kcmm/ffi.rs:1618 for bf16 models.
 */
int kcmm_paged_attn_decode_bf16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t out_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t num_q_heads,
    uint32_t kv_heads, uint32_t head_dim, uint32_t block_size,
    uint32_t max_blocks_per_seq, float scale, uint64_t stream_ptr);

/**
 * kcmm_paged_attn_decode_bf16_on_stream without any device allocation.  This
 * entry point has no reference counterpart.
 *
 * The regular entry point takes its split/merge scratch from a stream-ordered
 * memory pool.  This one uses a static 32 MiB per-device array instead.  It is
 * for callers that cannot allocate on the decode step: a KV pool sized to fill
 * HBM leaves the memory pool nothing to grow into, and a host with its own
 * allocator has no scratch buffer to pass.
 *
 * Launches needing more than 32 MiB of scratch return -1 with an error
 * message and launch nothing.  With Llama-3-8B heads that is above about 1000
 * sequences of up to 4096 tokens, or 500 of up to 8192.  The first
 * call on each device resolves the array's address and may load its module,
 * so make that call before any stream capture.  Calls on one device share the
 * array: overlapping calls (other streams or threads, unordered) race on it.
 * Same arguments and results as kcmm_paged_attn_decode_bf16_on_stream.
 */
int kcmm_paged_attn_decode_bf16_noalloc_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t out_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t num_q_heads,
    uint32_t kv_heads, uint32_t head_dim, uint32_t block_size,
    uint32_t max_blocks_per_seq, float scale, uint64_t stream_ptr);

/**
 * Causal chunked-prefill attention over the paged cache, on the tcgen05 tensor
 * cores.  The reference has no prefill kernel; its prefill loops decode steps
 * (ref src/model/transformer.rs:50-65).
 *
 * Sequence b contributes the query rows [qs[b], qs[b+1]) of query_ptr
 * ([total_tokens][num_q_heads][head_dim], 16-bit, 16-byte aligned), where
 * qs = query_start_loc_ptr (int32 [batch+1], device).  context_lens_ptr[b]
 * (int32, device) is the number of keys in the sequence's pages after the
 * chunk: the chunk's own K/V rows must already be written (append or fused
 * append).  Query row i of the chunk sits at position context_lens[b] - chunk
 * length + i and attends to keys [0, that position].  Block tables, offsets
 * and page layout are those of kcmm_paged_attn_decode_f16.  out_ptr has the
 * shape of query_ptr.
 *
 * Limits: head_dim 128, and num_q_heads / kv_heads must divide 128.
 * max_query_len bounds every chunk length.  Enqueues on stream_ptr and
 * returns; device-side problems (bad offsets, a context shorter than its
 * chunk) set kcmm_get_kernel_status bits.
 */
int kcmm_paged_prefill_bf16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t out_ptr,
    uint64_t block_tables_ptr, uint64_t query_start_loc_ptr, uint64_t context_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t max_query_len,
    uint32_t num_q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t block_size,
    uint32_t max_blocks_per_seq, float scale, uint64_t stream_ptr);

/*
 * Strided twins for views into a fused QKV projection output (the vLLM seam of
 * ref scripts/kcmm/kv_read_plan.py:830-838 and kv_write_mirror.py:536-537 copies
 * such views to compact tensors first).  Strides are in elements; head_dim (and
 * a token's kv_heads * head_dim row) must be contiguous.
 *   q[b][h][:]   at query_ptr + b*q_stride_token + h*q_stride_head
 *   out[b][h][:] at out_ptr   + b*out_stride_token + h*out_stride_head
 *   table row b  at block_tables_ptr + b*block_tables_row_stride  (int32 entries)
 * Head strides must be >= head_dim and the table row stride >= max_blocks_per_seq.
 * Otherwise as kcmm_paged_attn_decode_bf16_on_stream.
 */
int kcmm_paged_attn_decode_bf16_strided_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, int64_t q_stride_token,
    int64_t q_stride_head, uint64_t out_ptr, int64_t out_stride_token, int64_t out_stride_head,
    uint64_t block_tables_ptr, int64_t block_tables_row_stride, uint64_t seq_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t num_q_heads, uint32_t kv_heads,
    uint32_t head_dim, uint32_t block_size, uint32_t max_blocks_per_seq, float scale,
    uint64_t stream_ptr);
/** f16 twin of kcmm_paged_attn_decode_bf16_strided_on_stream. */
int kcmm_paged_attn_decode_f16_strided_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, int64_t q_stride_token,
    int64_t q_stride_head, uint64_t out_ptr, int64_t out_stride_token, int64_t out_stride_head,
    uint64_t block_tables_ptr, int64_t block_tables_row_stride, uint64_t seq_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t num_q_heads, uint32_t kv_heads,
    uint32_t head_dim, uint32_t block_size, uint32_t max_blocks_per_seq, float scale,
    uint64_t stream_ptr);
/**
 * kcmm_append_kv_device_slots_on_stream with source rows k_src_ptr + b*k_row_stride
 * and v_src_ptr + b*v_row_stride (elements; 0 = dense, else >= kv_heads*head_dim).
 */
int kcmm_append_kv_device_slots_strided_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t slot_mapping_ptr,
    uint64_t block_offsets_f16_ptr, uint64_t valid_blocks_ptr, uint32_t block_offsets_f16_len,
    uint32_t batch, uint64_t k_src_ptr, int64_t k_row_stride, uint64_t v_src_ptr,
    int64_t v_row_stride, uint64_t status_ptr, uint64_t stream_ptr);

/** f16 twin of kcmm_paged_prefill_bf16_on_stream. */
int kcmm_paged_prefill_f16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t out_ptr,
    uint64_t block_tables_ptr, uint64_t query_start_loc_ptr, uint64_t context_lens_ptr,
    uint64_t block_offsets_f16_ptr, uint32_t batch, uint32_t max_query_len,
    uint32_t num_q_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t block_size,
    uint32_t max_blocks_per_seq, float scale, uint64_t stream_ptr);

/** bf16 name for the device-slot write (the write copies 16-bit words, so it is the f16 kernel). */
int kcmm_append_kv_device_slots_bf16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t slot_mapping_ptr,
    uint64_t block_offsets_f16_ptr, uint64_t valid_blocks_ptr,
    uint32_t block_offsets_f16_len, uint32_t batch, uint64_t k_src_ptr,
    uint64_t v_src_ptr, uint64_t status_ptr, uint64_t stream_ptr);

/** Rotary conventions accepted by the fused append. */
typedef enum {
    /* Interleaved pairs (2i, 2i+1); pair i uses base^(-2*floor(i/2)/head_dim),
       the exact formula of ref src/cuda/kernels/rope.cu:18 (adjacent pairs share a frequency). */
    KCMM_ROPE_REFERENCE = 0,
    /* Interleaved pairs (2i, 2i+1) with base^(-2i/head_dim) (GPT-J). */
    KCMM_ROPE_GPTJ      = 1,
    /* Half-split pairs (i, i+head_dim/2) with base^(-2i/head_dim) (GPT-NeoX / Llama HF). */
    KCMM_ROPE_NEOX      = 2,
} kcmm_rope_mode_t;

/**
 * One pass of RMSNorm + rotary + KV append for num_tokens decode tokens
 * (the composition of ref src/cuda/kernels/rms_norm.cu, rope.cu and
 * kcmm_vllm_kv_write.cu as called at ref src/model/llama_transformer.rs:313-333):
 *   normed_out[t,:] = bf16((x[t,:] * rsqrt(mean(x^2) + eps)) * norm_weight)
 *   q[t] rotated in place at positions[t]
 *   K page slot slot_mapping[t] <- rotate(k[t]),  V page slot <- v[t]
 * x/normed_out [num_tokens, hidden]; q [num_tokens, num_q_heads, head_dim];
 * k/v [num_tokens, kv_heads, head_dim] (pool kv_heads/head_dim); positions
 * int32; slot_mapping int64 (<0 = padding: no cache write).  Status word as
 * for the device-slot write.  hidden a multiple of 8, head_dim even.
 */
int kcmm_fused_norm_rope_append_bf16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx,
    uint64_t x_ptr, uint64_t norm_weight_ptr, uint64_t normed_out_ptr,
    uint32_t hidden, float eps,
    uint64_t q_ptr, uint32_t num_q_heads, uint64_t k_ptr, uint64_t v_ptr,
    uint64_t positions_ptr, float rope_theta, uint32_t rope_mode,
    uint64_t slot_mapping_ptr, uint64_t block_offsets_f16_ptr,
    uint64_t valid_blocks_ptr, uint32_t block_offsets_f16_len,
    uint32_t num_tokens, uint64_t status_ptr, uint64_t stream_ptr);

/* --- reference counting and copy-on-write (refcount seam of
       ref scripts/kcmm/shadow_allocator.py:22-110, skeleton ref
       src/kcmm/sharing.rs:61-101) --- */

/** Add one owner to a live block. */
int kcmm_block_incref(kcmm_pool_t *pool, uint32_t block_idx);
/** Drop one owner; at zero the block is freed exactly as kcmm_free_blocks would. */
int kcmm_block_decref(kcmm_pool_t *pool, uint32_t block_idx);
/** Owner count of a live block, 0 if free or out of range. */
uint32_t kcmm_block_refcount(kcmm_pool_t *pool, uint32_t block_idx);
/** New sequence sharing every block of src_seq (each block incref'd). */
int kcmm_fork_sequence(kcmm_pool_t *pool, uint32_t src_seq, uint32_t *out_seq_idx);
/**
 * For each i: if block table entry logical_blocks[i] of seq_indices[i] has
 * refcount > 1, allocate a fresh block, copy its K and V pages for every
 * layer on stream_ptr (one launch for all i), decref the old block and
 * rewrite the table entry.  out_blocks[i] receives the block id now in the
 * table (unchanged when the block was not shared).
 */
int kcmm_cow_blocks_on_stream(kcmm_pool_t *pool, const uint32_t *seq_indices,
                              const uint32_t *logical_blocks, uint32_t count,
                              uint32_t *out_blocks, uint64_t stream_ptr);

/* --- host swap tier (data movement of ref src/kcmm/tiering.rs:1207-1798) --- */

/**
 * Move each listed GPU-resident block to the pinned host swap tier:
 * one kernel copies [K0][V0]...[K(L-1)][V(L-1)] of every block into its
 * host slot, the physical slot is returned to the allocator and the block
 * becomes CPU-resident (same block id).  Completes before returning.
 */
int kcmm_swap_out_blocks_on_stream(kcmm_pool_t *pool, const uint32_t *blocks,
                                   uint32_t count, uint64_t stream_ptr);
/**
 * Bring listed CPU-resident blocks back into freshly allocated physical
 * slots (new VA offset, same block id); GPU-resident ones are skipped.
 * Completes before returning.
 */
int kcmm_swap_in_blocks_on_stream(kcmm_pool_t *pool, const uint32_t *blocks,
                                  uint32_t count, uint64_t stream_ptr);

/**
 * Sticky device-side diagnostics of the pool's kernels, then cleared:
 * bit 0 = a bounded wait for a KV page gave up (no data arrived),
 * bit 1 = a block offset was misaligned or outside the layer region,
 * bit 2 = launch arguments the kernel found inconsistent (a prefill context
 *         shorter than its chunk; members of a shared-prefix group whose shared
 *         table entries differ).
 * Synchronises the pool's device.  -1 if the pool has no device.
 */
int32_t kcmm_get_kernel_status(kcmm_pool_t *pool);

/*
 * Decode attention over sequences that share a prefix of their pages (no
 * counterpart in the reference: its kernel reads every sequence's pages on its
 * own, also where kcmm_share_prefix / kcmm_fork_sequence made them the same
 * blocks).  Same arguments and result as kcmm_paged_attn_decode_bf16_on_stream,
 * plus groups of consecutive sequences:
 *   group_starts_ptr  device int32[n_groups + 1], ascending, 0 .. batch_size:
 *                     group g is the sequences [starts[g], starts[g+1]);
 *   prefix_lens_ptr   device int32[n_groups]: the first prefix_lens[g] tokens of
 *                     every member are the same blocks (same ids in the first
 *                     ceil(prefix_lens[g] / block_size) table entries).
 * The shared pages are read once per group (and kv head) for all members' query
 * rows together, each member's remaining tokens on their own, and the two
 * partial results merge through their log-sum-exp.  The prefix used is the
 * group's length capped by every member's context, in whole 16-token units.
 * At most max_group_size members of a group share (the rest attend alone); a
 * malformed group attends alone.  A member whose table differs from the first
 * member's inside the shared pages sets bit 2 of kcmm_get_kernel_status (the
 * result is then undefined for that group).  Needs num_q_heads a multiple of
 * num_kv_heads with at most 16 query heads per kv head, head_dim 64, 128 or 256,
 * and at most 8192 sequences; -1 otherwise.  Each call first resolves the groups
 * in one small kernel, so the attention kernels read two words per item.
 */
int kcmm_paged_attn_decode_shared_prefix_bf16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t output_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr, uint64_t block_offsets_ptr,
    uint32_t batch_size, uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
    uint32_t block_size, uint32_t max_blocks_per_seq, float scale, uint64_t group_starts_ptr,
    uint64_t prefix_lens_ptr, uint32_t n_groups, uint32_t max_group_size, uint64_t stream_ptr);
int kcmm_paged_attn_decode_shared_prefix_f16_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t output_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr, uint64_t block_offsets_ptr,
    uint32_t batch_size, uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
    uint32_t block_size, uint32_t max_blocks_per_seq, float scale, uint64_t group_starts_ptr,
    uint64_t prefix_lens_ptr, uint32_t n_groups, uint32_t max_group_size, uint64_t stream_ptr);

/* --- all-gather over NVLink peer memory (KV-head split, no reference counterpart) --- */

/*
 * The KV-head split of the decode (each GPU attends its own kv heads) needs every
 * rank's output on every rank; the reference plan uses ncclAllGather.  These
 * two calls do it with plain stores into peers' memory and per-CTA flags:
 *   dst_ptrs[r]    rank r's gathered buffer, mapped on this device (CUDA IPC or
 *                  P2P): two halves of world slices of nbytes, 2*world*nbytes in
 *                  all.  Epoch e writes slice `rank` of half (e & 1);
 *   signal_ptrs[r] rank r's signal array, kcmm_peer_signal_words(world) u64
 *                  flags, zeroed once; every call raises this rank's flags there
 *                  to `epoch`, which must grow by one per call on every rank.
 * kcmm_peer_wait_on_stream then waits (bounded, 1 s) until all ranks' flags in
 * this rank's signal array reached epoch; on a timeout it writes 1 to *status.
 * After the wait for epoch e, half (e & 1) of this rank's buffer holds every
 * rank's slice.
 * Ordering rule: on every rank, issue gather(e), wait(e), then every read of
 * half (e & 1), all before gather(e+1), in stream order.  A peer can be one
 * epoch ahead and writes the other half meanwhile; it writes half (e & 1) again
 * only at epoch e+2, after it has seen this rank's epoch e+1 flags.
 * nbytes must be a multiple of 16 and world <= 8.  -1 on invalid arguments.
 */
uint32_t kcmm_peer_signal_words(uint32_t world);
int kcmm_peer_allgather_on_stream(uint64_t src_ptr, uint64_t nbytes, const uint64_t *dst_ptrs,
                                  const uint64_t *signal_ptrs, uint32_t rank, uint32_t world,
                                  uint64_t epoch, uint64_t stream_ptr);
int kcmm_peer_wait_on_stream(uint64_t signal_ptr, uint32_t world, uint64_t epoch,
                             uint64_t status_ptr, uint64_t stream_ptr);

/*
 * The decode of kcmm_paged_attn_decode_{bf16,f16}_on_stream fused with the
 * all-gather above: the kernel that merges the split partials also stores every
 * finished output row into slot `rank` of half (epoch & 1) of every rank's
 * gathered buffer (gathered_ptrs[r], [2][world][batch][num_q_heads][head_dim]
 * 16-bit values, 16-byte aligned), then raises this rank's flags in
 * signal_ptrs[r] to `epoch`, under the same ordering rule and as
 * kcmm_peer_allgather_on_stream does, so no separate gather kernel runs.
 * `output_ptr` receives this rank's rows as usual.  Follow with
 * kcmm_peer_wait_on_stream.  Sequences of length 0 leave their rows untouched
 * everywhere.  Only the tensor-core decode path takes peers (head_dim 32, 64, 80,
 * 96, 112, 128, 160, 192 or 256 and block_size a multiple of 16); -1 otherwise.
 * Replaces the decode + ncclAllGather pair of the reference's KV-head split plan.
 */
int kcmm_paged_attn_decode_bf16_allgather_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t output_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr, uint64_t block_offsets_ptr,
    uint32_t batch_size, uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
    uint32_t block_size, uint32_t max_blocks_per_seq, float scale, const uint64_t *gathered_ptrs,
    const uint64_t *signal_ptrs, uint32_t rank, uint32_t world, uint64_t epoch,
    uint64_t stream_ptr);
int kcmm_paged_attn_decode_f16_allgather_on_stream(
    kcmm_pool_t *pool, uint32_t layer_idx, uint64_t query_ptr, uint64_t output_ptr,
    uint64_t block_tables_ptr, uint64_t seq_lens_ptr, uint64_t block_offsets_ptr,
    uint32_t batch_size, uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
    uint32_t block_size, uint32_t max_blocks_per_seq, float scale, const uint64_t *gathered_ptrs,
    const uint64_t *signal_ptrs, uint32_t rank, uint32_t world, uint64_t epoch,
    uint64_t stream_ptr);

/* --- extended metrics (Rust-only in the reference) --- */

/** Fill the extended metrics; -1 on NULL arguments. */
int kcmm_get_metrics_ext(kcmm_pool_t *pool, kcmm_metrics_ext_t *out);
/** Counters of one policy name; -1 when none were recorded for it. */
int kcmm_get_policy_stats(kcmm_pool_t *pool, const char *policy, kcmm_policy_stats_t *out);

/* --- background eviction and victim preview (no C counterpart in the reference) --- */

/**
 * Start the background eviction thread of ref src/kcmm/pool.rs:1308-1398 (Rust-only
 * there): every background_evict_interval_ms, while the free physical block ratio
 * is below low_watermark_threshold, swap out up to min(max_batch_blocks, 16)
 * blocks of inactive (cooled) sequences chosen by the eviction policy.  A no-op
 * when it runs already; -1 when tiering is disabled or the pool has no device.
 */
int kcmm_start_background_eviction(kcmm_pool_t *pool);
/** Stop the thread and wait for it; 0 also when it was not running. */
int kcmm_stop_background_eviction(kcmm_pool_t *pool);
/**
 * The victims kcmm_evict_blocks(pool, count) would take now, in eviction order,
 * without moving anything; returns how many were written to out_blocks
 * (at most max_out).  0 when tiering is disabled.
 */
uint32_t kcmm_preview_eviction_victims(kcmm_pool_t *pool, uint32_t count, uint32_t *out_blocks,
                                       uint32_t max_out);

/* --- device-resident step tables (no reference counterpart) --- */

/*
 * The block tables, sequence lengths and block offsets a decode step reads,
 * kept on the device between steps.  They replace the per-step host build and
 * per-layer upload of ref src/model/llama_transformer.rs:277-303 and :338-339
 * (offsets: kcmm_get_all_block_offsets_f16).  A sync uploads only what changed
 * since the previous sync: rows whose sequence or table changed, lengths that
 * differ, and offsets of the blocks the pool installed, freed or swapped in.
 * The contents equal the reference's host build: row b holds the first
 * max_blocks_per_seq entries of seq_indices[b]'s table, zeros after it.
 */
typedef struct kcmm_step_tables kcmm_step_tables_t;

typedef struct {
    uint64_t syncs;          /* sync calls */
    uint64_t table_entries;  /* 32-bit entries written (table entries and lengths) */
    uint64_t offset_entries; /* 64-bit offsets entries written */
    uint64_t bytes;          /* bytes copied host to device */
    uint64_t full_offsets;   /* syncs that wrote the whole offsets array */
} kcmm_step_tables_stats_t;

/** Device tables for up to max_batch rows on the pool's device; NULL on error. */
kcmm_step_tables_t *kcmm_step_tables_create(kcmm_pool_t *pool, uint32_t max_batch);
/** Synchronises the device, then frees the tables. */
void kcmm_step_tables_destroy(kcmm_step_tables_t *tables);
/**
 * Bring rows [0, batch) up to date for seq_indices[0..batch) (host array), and
 * the offsets for every block of the pool.  Enqueues one copy and one kernel
 * on stream_ptr when anything changed.  Syncs of one tables object must be
 * ordered on the device (one stream, or events between streams).  -1 on a bad
 * sequence index or batch > max_batch (message on the pool).
 */
int kcmm_step_tables_sync_on_stream(kcmm_step_tables_t *tables, const uint32_t *seq_indices,
                                    uint32_t batch, uint64_t stream_ptr);
/** Device int32 [max_batch, max_blocks_per_seq] block tables (block_tables_ptr of decode). */
uint64_t kcmm_step_tables_block_tables(const kcmm_step_tables_t *tables);
/** Device int32 [max_batch] sequence lengths (seq_lens_ptr of decode). */
uint64_t kcmm_step_tables_seq_lens(const kcmm_step_tables_t *tables);
/** Device u64 block offsets in 2-byte units; may move at a sync that grows it. */
uint64_t kcmm_step_tables_block_offsets(const kcmm_step_tables_t *tables);
/** Counters since creation; -1 on NULL arguments. */
int kcmm_step_tables_stats(const kcmm_step_tables_t *tables, kcmm_step_tables_stats_t *out);

/* --- library facts --- */

/** Build tag of the library ("kcmm-b200 <version> sm_100a"). */
const char *kcmm_build_info(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* KCMM_H */
