// Paged decode attention that allocates no device memory.
//
// decode_attention takes its split/merge scratch from a stream-ordered pool
// (cudaMallocFromPoolAsync + cudaFreeAsync) unless the caller passes a buffer.
// Some callers can do neither:
//  * a server whose KV pool was sized to claim nearly all of HBM at start-up:
//    the stream-ordered pool's first growth is a fresh driver allocation that
//    can fail, or evict pages the pool relies on, in the middle of a step;
//  * a host that owns device memory through its own allocator (no torch, no
//    cudarc buffers on the decode path) and has no scratch buffer to hand in;
//  * a latency-bound step loop that must not take the allocator's locks or pay
//    a pool trim/grow inside the step.
// For them the scratch is one file-scope device array.  It lives in its own
// translation unit (its own module), so only processes that use this entry
// point pay its footprint.
//
// Contract:
//  * At most kNoAllocScratchBytes of scratch; larger launches are rejected
//    with cudaErrorInvalidValue before anything is launched.
//  * The array is per device (each device's context holds its own copy of the
//    module); its address is resolved with cudaGetSymbolAddress on the first
//    call made on each device.  Under lazy module loading that first call also
//    loads this module, so make it before any stream capture.
//  * The scratch needs no clearing: every partial row the merge pass reads is
//    written by the split pass of the same call, and the unit prefix arrays are
//    rewritten by every call.
//  * Calls on one device share the array, so two calls that overlap in time
//    (different streams, or host threads, without ordering between them) race
//    on it.  Serialise them: one stream, or events between streams.
#include <cuda_runtime.h>

#include <mutex>

#include "../launch.hpp"

namespace {
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB
}  // namespace

// One copy per device context; internal linkage, reached only through
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

namespace kcmm {
namespace dev {
namespace {

constexpr int kMaxDevices = 64;

cudaError_t scratch_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  static std::mutex mu;
  static void *addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    if (!p) return cudaErrorInvalidSymbol;
    addr[dev] = p;
  }
  *out = addr[dev];
  return cudaSuccess;
}

}  // namespace

size_t decode_noalloc_scratch_limit() { return kNoAllocScratchBytes; }

cudaError_t decode_attention_noalloc(const DecodeArgs &args, cudaStream_t stream) {
  const size_t need = decode_scratch_bytes(args);
  if (need > kNoAllocScratchBytes) return cudaErrorInvalidValue;
  void *scratch = nullptr;
  cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) return e;
  DecodeArgs a = args;
  a.scratch = static_cast<float *>(scratch);
  a.scratch_bytes = kNoAllocScratchBytes;
  return decode_attention(a, stream);
}

}  // namespace dev
}  // namespace kcmm
