// Host-side launchers of the sm_100a kernels (defined in kernels/*.cu).
// Every launcher validates nothing itself: the ABI layer (ffi.cpp) checks
// arguments and reports errors; a launcher returns the cudaError_t of the
// launch (0 on success).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace kcmm {
namespace dev {

enum class Dtype : int { F16 = 0, BF16 = 1 };

// Sticky bits written into the pool's device diagnostic word.
enum DiagBits : int32_t {
  kDiagWaitTimeout = 1 << 0,   // an mbarrier wait gave up (no data arrived)
  kDiagBadOffset = 1 << 1,     // a block offset was misaligned or past the region
  kDiagBadLaunch = 1 << 2,
};

struct DecodeArgs {
  Dtype dtype;
  const void *q;
  void *out;
  const int32_t *block_tables;
  const int32_t *seq_lens;
  const uint64_t *block_offsets;  // 2-byte units
  const void *va_k;
  const void *va_v;
  uint64_t region_elems;  // size of one layer region in 2-byte units
  int batch, num_q_heads, kv_heads, head_dim, block_size, max_blocks_per_seq;
  float scale;
  int32_t *diag;
  // Optional caller-provided split-K scratch; when null the launcher takes it
  // from a stream-ordered memory pool (cudaMallocAsync) and frees it after use.
  float *scratch;
  size_t scratch_bytes;
  int force_splits;  // >0 overrides the split heuristic (tests)
  // Element strides of q and out (token, head; head_dim is contiguous) and of the
  // block-table rows; 0 = dense ([batch][Hq][D] and max_blocks_per_seq).
  int64_t q_stride_token, q_stride_head, out_stride_token, out_stride_head, tables_stride;
  // All-gather of the KV-head split (kernels/decode.cu, merge_gather_kernel):
  // peer_world > 0 writes every output row also to slot peer_rank of each
  // rank's gathered buffer peer_out[r] ([2][world][batch][Hq][D]; half
  // peer_epoch & 1) and raises this rank's flags in peer_sig[r] to peer_epoch
  // (host arrays of device addresses).
  const uint64_t *peer_out;
  const uint64_t *peer_sig;
  int peer_rank, peer_world;
  uint64_t peer_epoch;
};

// Bytes of split-K scratch decode_attention needs for these arguments
// (0 when no split is needed).
size_t decode_scratch_bytes(const DecodeArgs &a);
cudaError_t decode_attention(const DecodeArgs &a, cudaStream_t stream);
// Shared-prefix (cascade) decode (kernels/decode.cu): sequences
// [group_starts[g], group_starts[g+1]) share their first prefix_lens[g] tokens'
// pages (device arrays); at most max_group members of a group share, the rest
// attend alone.  Dense q / out / tables only; the strides and peer fields of `a`
// are ignored.  cudaErrorNotSupported outside head_dim 64 / 128 / 256, a block
// size that is a multiple of 16, or G > 16.
cudaError_t decode_attention_shared_prefix(const DecodeArgs &a, const int32_t *group_starts,
                                           const int32_t *prefix_lens, int n_groups,
                                           int max_group, cudaStream_t stream);
// decode_attention with its scratch in a static per-device array instead of a
// stream-ordered allocation (kernels/decode_noalloc.cu).  Returns
// cudaErrorInvalidValue when the launch needs more than
// decode_noalloc_scratch_limit() bytes; a.scratch is ignored.
size_t decode_noalloc_scratch_limit();
cudaError_t decode_attention_noalloc(const DecodeArgs &a, cudaStream_t stream);
// Force module load of every decode kernel (precompile entry points).
cudaError_t decode_preload();

struct PrefillArgs {
  Dtype dtype;
  const void *q;      // [total_q_tokens, num_q_heads, head_dim]
  void *out;          // same shape
  const int32_t *block_tables;  // [batch, max_blocks_per_seq]
  const int32_t *query_start;   // [batch + 1] prefix sum of chunk lengths
  const int32_t *context_lens;  // [batch] keys after the chunk (chunk included)
  const uint64_t *block_offsets;
  const void *va_k;
  const void *va_v;
  uint64_t region_elems;
  int batch, max_q_len, num_q_heads, kv_heads, head_dim, block_size, max_blocks_per_seq;
  float scale;
  int32_t *diag;
  // K and V TMA descriptors of the layer ({D, Hkv, tokens}, box {64, 1, 16}) or null,
  // and the V page-box descriptor ({64, tokens, D/64, Hkv}, box {64, 16, D/64, 1}) or null.
  const void *tensor_maps;
  const void *v_page_map;
};
// Causal chunked-prefill attention on the tcgen05 tensor cores
// (kernels/prefill.cu).  head_dim 128; num_q_heads / kv_heads must divide 128.
cudaError_t paged_prefill(const PrefillArgs &a, cudaStream_t stream);

// Device scratch kept per (device, stream) between calls (kernels/decode.cu), used by the
// decode split merge and the prefill tail split.  Calls on one stream share it in stream
// order.  Null while the stream is being captured or once the per-process stream cache is
// full; the caller then allocates for the call, or skips the split.
void *stream_scratch(cudaStream_t stream, size_t bytes);

// All-gather over NVLink peer memory (kernels/peer.cu).  dst[r] is rank r's
// gathered buffer (two halves of world slices of nbytes, P2P-accessible from
// this device; epoch e fills half e & 1), sig[r] rank r's signal array of
// world * kGatherBlocks u64 flags.
constexpr int kMaxPeers = 8;
constexpr int kGatherBlocks = 16;
cudaError_t peer_allgather(const void *src, uint64_t nbytes, void *const *dst,
                           unsigned long long *const *sig, int rank, int world,
                           unsigned long long epoch, cudaStream_t stream);
// Wait (bounded, 1 s) until every flag of this rank's signal array reaches epoch;
// a timeout writes 1 to *status.
cudaError_t peer_wait(const unsigned long long *sig, int world, unsigned long long epoch,
                      int32_t *status, cudaStream_t stream);

// Apply a packed step-table update list (kernels/tables.cu): 32-bit entries into
// i32 and 64-bit entries into o64.
cudaError_t apply_table_updates(const void *stage, int n32, int n64, size_t off64, int32_t *i32,
                                uint64_t *o64, cudaStream_t stream);

// Copy `rows` K and V rows of `row_elems` 16-bit elements from k_src/v_src
// (row r at r*row_elems) to va_k/va_v + dst_elems[r]; dst_elems[r] < 0 skips.
cudaError_t copy_rows(const void *k_src, const void *v_src, void *va_k, void *va_v,
                      const int64_t *dst_elems_host, int rows, int row_elems,
                      cudaStream_t stream);

struct SlotWriteArgs {
  void *va_k;
  void *va_v;
  const int64_t *slot_mapping;
  const uint64_t *block_offsets;
  const uint8_t *valid;  // may be null
  int offsets_len;
  int batch;
  int step_elems;
  int block_size;
  const void *k_src;
  const void *v_src;
  int32_t *status;  // may be null
  uint64_t region_elems;
  int64_t k_stride, v_stride;  // elements between source rows; 0 = step_elems
};
cudaError_t device_slot_write(const SlotWriteArgs &a, cudaStream_t stream);

struct FusedAppendArgs {
  const void *x;
  const void *norm_weight;
  void *normed_out;
  int hidden;
  float eps;
  void *q;
  int num_q_heads;
  const void *k;
  const void *v;
  const int32_t *positions;
  float rope_theta;
  int rope_mode;
  const int64_t *slot_mapping;
  const uint64_t *block_offsets;
  const uint8_t *valid;
  int offsets_len;
  int num_tokens;
  int kv_heads;
  int head_dim;
  int block_size;
  void *va_k;
  void *va_v;
  uint64_t region_elems;
  int32_t *status;
  // Rotary frequencies theta_i = 1 / base^e_i per pair index (head_dim/2 <= 128
  // entries), filled by the launcher from rope_theta, rope_mode and head_dim.
  float inv_freq[128];
};
cudaError_t fused_norm_rope_append(const FusedAppendArgs &a, cudaStream_t stream);

// Copy whole blocks: for each pair i and each of the 2*num_layers regions,
// block_bytes from region + src_off[i] to region + dst_off[i].
cudaError_t copy_blocks(const uint64_t *d_layer_bases, int num_layers, const uint64_t *src_off,
                        const uint64_t *dst_off, int count, uint64_t block_bytes,
                        cudaStream_t stream);

// Swap tier: gather blocks into host-mapped memory (dir=0) or scatter back
// (dir=1).  Host slot i holds [K0][V0]...[K(L-1)][V(L-1)].
cudaError_t swap_blocks(const uint64_t *d_layer_bases, int num_layers, const uint64_t *va_off,
                        const uint64_t *host_off, int count, uint64_t block_bytes,
                        uint8_t *host_base_dev, int dir, cudaStream_t stream);
// The same move through the copy engines.  The swap kernel packs blocks into
// (or unpacks them from) one half of a device staging buffer on the caller's
// stream; every run of consecutive host slots crosses the host link as one
// cudaMemcpyAsync between that half and `host` (the host view of the
// registered tier) on copy_stream.  The two halves alternate, so packing one
// chunk overlaps the copy of the previous one; events order the halves' reuse,
// and the caller's stream ends behind the last copy.
struct SwapStaging {
  uint8_t *buffer;  // device, `bytes` long, two halves
  uint64_t bytes;
  cudaStream_t copy_stream;
  cudaEvent_t ev_kernel[2], ev_copy[2];  // per half: last pack / unpack, last copy
};
cudaError_t swap_blocks_staged(const SwapStaging &st, const uint64_t *d_layer_bases,
                               int num_layers, const uint64_t *va_off, const uint64_t *host_off,
                               int count, uint64_t block_bytes, uint8_t *host, int dir,
                               cudaStream_t stream);

}  // namespace dev
}  // namespace kcmm
