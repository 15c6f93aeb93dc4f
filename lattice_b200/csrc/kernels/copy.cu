// Whole-block copies for sm_100a: copy-on-write forks and the host swap tier.
//
// A block occupies block_bytes at the same offset of every one of the
// 2*num_layers K/V regions.  Both kernels take one CTA per (block, region)
// and move the block with 16-byte accesses.
//   * copy_blocks: device -> device (CoW fork of a shared block; the
//     reference has only a refcount seam, ref scripts/kcmm/shadow_allocator.py).
//   * swap_blocks_staged (the default swap path): the swap kernel packs a
//     chunk of blocks into half of a device staging buffer, in host-slot
//     layout, and the copy engines move each run of consecutive host slots
//     with one cudaMemcpyAsync; the two halves alternate so packing overlaps
//     the previous chunk's copy (restores run the same steps backwards).  The
//     reference also stages (ref src/kcmm/tiering.rs:1207-1798: a gather
//     kernel, one D2H per layer and a CPU memcpy scatter); here one copy
//     covers every layer of a run of blocks and nothing is scattered on the CPU.
//   * swap_blocks: device <-> pinned host memory mapped into the device
//     address space; the kernel reads/writes the host bytes directly
//     (KCMM_SWAP_IMPL=sm).
//   Host slot layout: [K0][V0][K1][V1]...[K(L-1)][V(L-1)], each block_bytes
//   (ref src/kcmm/tiering.rs:1414-1421).
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "../launch.hpp"

namespace kcmm {
namespace dev {
namespace {

constexpr int kPairsPerLaunch = 240;  // 2 x 8 B x 240 < 4 KB of parameters

struct BlockPairs {
  const uint64_t *bases;  // [2L] region bases on the device
  uint8_t *host;          // swap tier (device view), swap only
  uint64_t block_bytes;
  int count;
  int dir;  // swap: 0 = device -> host, 1 = host -> device
  uint64_t a[kPairsPerLaunch];
  uint64_t b[kPairsPerLaunch];
};

__device__ __forceinline__ void copy_bytes(uint8_t *dst, const uint8_t *src, uint64_t n) {
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | n) & 15) == 0;
  if (vec) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    const uint64_t m = n / 16;
    uint64_t i = threadIdx.x;
    // four independent 16 B loads in flight per thread
    for (; i + 3 * blockDim.x < m; i += 4 * blockDim.x) {
      uint4 v0 = s[i], v1 = s[i + blockDim.x], v2 = s[i + 2 * blockDim.x], v3 = s[i + 3 * blockDim.x];
      d[i] = v0;
      d[i + blockDim.x] = v1;
      d[i + 2 * blockDim.x] = v2;
      d[i + 3 * blockDim.x] = v3;
    }
    for (; i < m; i += blockDim.x) d[i] = s[i];
  } else {
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}

// grid = (count, 2L): copy block a[i] -> b[i] in region blockIdx.y.
__global__ void copy_blocks_kernel(const BlockPairs p) {
  const int i = blockIdx.x, r = blockIdx.y;
  uint8_t *base = reinterpret_cast<uint8_t *>(p.bases[r]);
  copy_bytes(base + p.b[i], base + p.a[i], p.block_bytes);
}

// grid = (count, 2L): a[i] = block VA offset, b[i] = host slot offset.
__global__ void swap_blocks_kernel(const BlockPairs p) {
  const int i = blockIdx.x, r = blockIdx.y;
  uint8_t *dev = reinterpret_cast<uint8_t *>(p.bases[r]) + p.a[i];
  uint8_t *host = p.host + p.b[i] + uint64_t(r) * p.block_bytes;
  if (p.dir == 0) {
    copy_bytes(host, dev, p.block_bytes);
  } else {
    copy_bytes(dev, host, p.block_bytes);
  }
}

template <typename K>
cudaError_t launch_pairs(K kernel, const uint64_t *bases, uint8_t *host, int num_layers,
                         const uint64_t *a, const uint64_t *b, int count, uint64_t block_bytes,
                         int dir, cudaStream_t stream) {
  for (int base = 0; base < count; base += kPairsPerLaunch) {
    BlockPairs p;
    p.bases = bases;
    p.host = host;
    p.block_bytes = block_bytes;
    p.count = std::min(kPairsPerLaunch, count - base);
    p.dir = dir;
    for (int i = 0; i < p.count; ++i) {
      p.a[i] = a[base + i];
      p.b[i] = b[base + i];
    }
    dim3 grid(p.count, 2 * num_layers);
    kernel<<<grid, 256, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t copy_blocks(const uint64_t *d_layer_bases, int num_layers, const uint64_t *src_off,
                        const uint64_t *dst_off, int count, uint64_t block_bytes,
                        cudaStream_t stream) {
  return launch_pairs(copy_blocks_kernel, d_layer_bases, nullptr, num_layers, src_off, dst_off,
                      count, block_bytes, 0, stream);
}

cudaError_t swap_blocks(const uint64_t *d_layer_bases, int num_layers, const uint64_t *va_off,
                        const uint64_t *host_off, int count, uint64_t block_bytes,
                        uint8_t *host_base_dev, int dir, cudaStream_t stream) {
  return launch_pairs(swap_blocks_kernel, d_layer_bases, host_base_dev, num_layers, va_off,
                      host_off, count, block_bytes, dir, stream);
}

cudaError_t swap_blocks_staged(const SwapStaging &st, const uint64_t *d_layer_bases,
                               int num_layers, const uint64_t *va_off, const uint64_t *host_off,
                               int count, uint64_t block_bytes, uint8_t *host, int dir,
                               cudaStream_t stream) {
  const uint64_t slot = uint64_t(2) * num_layers * block_bytes;
  const uint64_t half_bytes = st.bytes / 2;
  if (half_bytes < slot || !st.copy_stream) return cudaErrorInvalidValue;
  const int per = int(half_bytes / slot);
  std::vector<uint64_t> local(size_t(std::min(per, count)));
  for (size_t j = 0; j < local.size(); ++j) local[j] = j * slot;
  const cudaMemcpyKind kind = dir == 0 ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
  cudaStream_t cs = st.copy_stream;
  // The copy stream starts behind everything already queued on the caller's stream.
  cudaError_t e = cudaEventRecord(st.ev_kernel[0], stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, st.ev_kernel[0], 0);
  if (e == cudaSuccess) e = cudaEventRecord(st.ev_copy[0], cs);
  if (e == cudaSuccess) e = cudaEventRecord(st.ev_copy[1], cs);
  if (e == cudaSuccess) e = cudaEventRecord(st.ev_kernel[1], stream);
  for (int base = 0, chunk = 0; e == cudaSuccess && base < count; base += per, ++chunk) {
    const int n = std::min(per, count - base);
    const int h = chunk & 1;
    uint8_t *half = st.buffer + uint64_t(h) * half_bytes;
    // one cudaMemcpyAsync per run of consecutive host slots, on the copy stream
    auto copy_runs = [&]() -> cudaError_t {
      int j0 = 0;
      while (j0 < n) {
        int j1 = j0 + 1;
        while (j1 < n && host_off[base + j1] == host_off[base + j1 - 1] + slot) ++j1;
        uint8_t *hp = host + host_off[base + j0];
        uint8_t *dp = half + uint64_t(j0) * slot;
        const uint64_t bytes = uint64_t(j1 - j0) * slot;
        cudaError_t r = dir == 0 ? cudaMemcpyAsync(hp, dp, bytes, kind, cs)
                                 : cudaMemcpyAsync(dp, hp, bytes, kind, cs);
        if (r != cudaSuccess) return r;
        j0 = j1;
      }
      return cudaSuccess;
    };
    if (dir == 0) {
      // pack on the caller's stream once the half's previous copy has left it
      e = cudaStreamWaitEvent(stream, st.ev_copy[h], 0);
      if (e == cudaSuccess)
        e = launch_pairs(swap_blocks_kernel, d_layer_bases, half, num_layers, va_off + base,
                         local.data(), n, block_bytes, 0, stream);
      if (e == cudaSuccess) e = cudaEventRecord(st.ev_kernel[h], stream);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, st.ev_kernel[h], 0);
      if (e == cudaSuccess) e = copy_runs();
      if (e == cudaSuccess) e = cudaEventRecord(st.ev_copy[h], cs);
    } else {
      // fill the half once its previous unpack has read it
      e = cudaStreamWaitEvent(cs, st.ev_kernel[h], 0);
      if (e == cudaSuccess) e = copy_runs();
      if (e == cudaSuccess) e = cudaEventRecord(st.ev_copy[h], cs);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, st.ev_copy[h], 0);
      if (e == cudaSuccess)
        e = launch_pairs(swap_blocks_kernel, d_layer_bases, half, num_layers, va_off + base,
                         local.data(), n, block_bytes, 1, stream);
      if (e == cudaSuccess) e = cudaEventRecord(st.ev_kernel[h], stream);
    }
  }
  // the caller's stream ends behind the last copy
  if (e == cudaSuccess) e = cudaEventRecord(st.ev_copy[0], cs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, st.ev_copy[0], 0);
  return e;
}

}  // namespace dev
}  // namespace kcmm
