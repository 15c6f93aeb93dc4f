// All-gather over NVLink peer memory, for the KV-head split of the decode
// (each rank attends its own kv heads; every rank needs all heads' outputs).
//
// A rank's gathered buffer holds two halves of world slices of `nbytes`; epoch
// e fills half e & 1, and slice r of a half comes from rank r.  peer_allgather
// copies this rank's slice into slot `rank` of that half of every rank's buffer
// (its own included) with plain stores through CUDA IPC mappings, then raises
// its flags in every rank's signal array:
//   signal[r][src * kGatherBlocks + blk] = epoch   (u64, system scope, release)
// one flag per CTA and rank, written by thread r after the CTA barrier and a
// system-scope fence.  peer_wait spins, bounded, until every flag of its own
// signal array has reached `epoch`; the gathered buffer is then complete.  A
// wait that runs out writes 1 to `status` and returns (no trap), so a missing
// rank is reported instead of hanging the GPU.
//
// Why two halves: once a rank's wait for epoch e has passed, it may start
// epoch e+1 while a slower peer is still reading epoch e's rows.  Epoch e+1
// goes to the other half, and a rank can only reach epoch e+2 (the same half
// again) after its wait for e+1 saw every peer's e+1 flags.  A peer raises
// those after everything it ordered before its epoch e+1 gather on its stream,
// including its reads of epoch e.  So with gather(e) -> wait(e) -> reads of
// half e & 1 -> gather(e+1) in stream order on every rank, no half is
// overwritten while a rank may still read it.
//
// No TMA and no multicast: remote memory is only ever the target of ordinary
// stores, and flags are read from this GPU's own memory.
#include <cuda_runtime.h>

#include <cstdint>

#include "../launch.hpp"
#include "pdl.cuh"
#include "ptx.cuh"

namespace kcmm {
namespace dev {
namespace {

constexpr uint64_t kPeerWaitLimitNs = 1000000000ull;  // 1 s

struct GatherArgs {
  const uint4 *src;
  uint64_t n16;  // 16-byte chunks per slice
  uint4 *dst[kMaxPeers];
  unsigned long long *sig[kMaxPeers];
  int rank, world;
  unsigned long long epoch;
};

__global__ void __launch_bounds__(512) peer_allgather_kernel(const GatherArgs a) {
  ptx::grid_dependency_wait();  // the slice is the previous kernel's output
  ptx::launch_dependents();
  const uint64_t per = (a.n16 + gridDim.x - 1) / gridDim.x;
  const uint64_t lo = uint64_t(blockIdx.x) * per;
  const uint64_t hi = lo + per < a.n16 ? lo + per : a.n16;
  const uint64_t base = ((a.epoch & 1ull) * uint64_t(a.world) + uint64_t(a.rank)) * a.n16;
  for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const uint4 v = a.src[i];
    for (int r = 0; r < a.world; ++r) a.dst[r][base + i] = v;
  }
  // The CTA barrier orders every thread's peer stores before the flag threads'
  // system-scope fence and release store (cumulativity: the pattern of a
  // cooperative grid barrier), so one fence per flag replaces one per thread.
  __syncthreads();
  if (threadIdx.x < a.world) {
    __threadfence_system();
    unsigned long long *f = a.sig[threadIdx.x] + a.rank * kGatherBlocks + blockIdx.x;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(a.epoch) : "memory");
  }
}

__global__ void peer_wait_kernel(const unsigned long long *sig, int world,
                                 unsigned long long epoch, int32_t *status) {
  ptx::grid_dependency_wait();
  ptx::launch_dependents();
  const int n = world * kGatherBlocks;
  bool ok = true;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint64_t t0 = ptx::globaltimer_ns();
    for (;;) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(sig + i) : "memory");
      if (v >= epoch) break;
      if (ptx::globaltimer_ns() - t0 > kPeerWaitLimitNs) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  if (!ok && status) atomicExch(status, 1);
  __threadfence_system();
}

}  // namespace

cudaError_t peer_allgather(const void *src, uint64_t nbytes, void *const *dst,
                           unsigned long long *const *sig, int rank, int world,
                           unsigned long long epoch, cudaStream_t stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || nbytes % 16 != 0)
    return cudaErrorInvalidValue;
  GatherArgs a = {};
  a.src = static_cast<const uint4 *>(src);
  a.n16 = nbytes / 16;
  for (int r = 0; r < world; ++r) {
    a.dst[r] = static_cast<uint4 *>(dst[r]);
    a.sig[r] = sig[r];
  }
  a.rank = rank;
  a.world = world;
  a.epoch = epoch;
  return launch_pdl(peer_allgather_kernel, dim3(kGatherBlocks), dim3(512), 0, stream, a);
}

cudaError_t peer_wait(const unsigned long long *sig, int world, unsigned long long epoch,
                      int32_t *status, cudaStream_t stream) {
  if (world < 1 || world > kMaxPeers) return cudaErrorInvalidValue;
  return launch_pdl(peer_wait_kernel, dim3(1), dim3(128), 0, stream, sig, world, epoch, status);
}

}  // namespace dev
}  // namespace kcmm
