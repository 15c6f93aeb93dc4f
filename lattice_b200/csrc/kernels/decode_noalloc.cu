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
//  * The array is per device context (each context holds its own copy of the
//    module); its address is resolved with cudaGetSymbolAddress by the first
//    call made in each context, and cached under the context's unique id
//    (cuCtxGetId).  A context that is destroyed and recreated (cudaDeviceReset,
//    a primary-context reset) gets a new id, so its first call resolves the
//    array again instead of reusing an address from the old module.  Under lazy
//    module loading that first call also loads this module, so make it before
//    any stream capture.
//  * The scratch needs no clearing: every partial row the merge pass reads is
//    written by the split pass of the same call, and the unit prefix arrays are
//    rewritten by every call.
//  * Calls on one device share the array, so two calls that overlap in time
//    (different streams, or host threads, without ordering between them) race
//    on it.  Serialise them: one stream, or events between streams.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

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

struct ContextApi {
  PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  PFN_cuCtxGetId_v12000 get_id = nullptr;
};

// Driver entry points for the context id (null when the driver lacks them; then
// every call resolves the address afresh).
const ContextApi &context_api() {
  static ContextApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 4000, cudaEnableDefault, &q) ==
            cudaSuccess && fn && q == cudaDriverEntryPointSuccess)
      api.get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && fn && q == cudaDriverEntryPointSuccess)
      api.get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
    if (!api.get_current || !api.get_id) api = ContextApi{};
  });
  return api;
}

// Unique id of the calling thread's current context, or 0 if there is none yet
// (or the driver cannot tell).
unsigned long long current_context_id() {
  const ContextApi &api = context_api();
  if (!api.get_current) return 0;
  CUcontext ctx = nullptr;
  if (api.get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  unsigned long long id = 0;
  if (api.get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

constexpr int kCachedContexts = 64;

cudaError_t scratch_address(void **out) {
  static std::mutex mu;
  static unsigned long long ids[kCachedContexts] = {};
  static void *addrs[kCachedContexts] = {};
  static int used = 0;
  unsigned long long id = current_context_id();
  if (id != 0) {
    std::lock_guard<std::mutex> g(mu);
    for (int i = 0; i < used; ++i) {
      if (ids[i] == id) {
        *out = addrs[i];
        return cudaSuccess;
      }
    }
  }
  // Set-up for this context: resolve the array's device address (this also makes
  // the primary context current if the thread had none).
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess) return e;
  if (!p) return cudaErrorInvalidSymbol;
  if (id == 0) id = current_context_id();
  if (id != 0) {
    std::lock_guard<std::mutex> g(mu);
    bool known = false;
    for (int i = 0; i < used; ++i) known = known || ids[i] == id;
    if (!known && used < kCachedContexts) {  // past the cap: resolved on every call
      ids[used] = id;
      addrs[used] = p;
      ++used;
    }
  }
  *out = p;
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
