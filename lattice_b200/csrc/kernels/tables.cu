// Scatter kernel of the device-resident step tables (step_tables.cpp): applies one
// packed update list [idx32 n32][val32 n32][idx64 n64][pad to 8][val64 n64] to the
// 32-bit array (block tables, then sequence lengths) and the 64-bit block-offset
// array.  One launch per sync; a grid-stride loop over both lists.
#include <cuda_runtime.h>

#include <cstdint>

#include "../launch.hpp"
#include "pdl.cuh"
#include "ptx.cuh"

namespace kcmm {
namespace dev {
namespace {

__global__ void apply_updates_kernel(const unsigned char *stage, int n32, int n64, size_t off64,
                                     int32_t *i32, uint64_t *o64) {
  // The previous kernel on the stream may still read the tables: write after it.
  ptx::grid_dependency_wait();
  ptx::launch_dependents();
  const uint32_t *idx32 = reinterpret_cast<const uint32_t *>(stage);
  const int32_t *val32 = reinterpret_cast<const int32_t *>(stage) + n32;
  const uint32_t *idx64 = reinterpret_cast<const uint32_t *>(stage) + 2 * size_t(n32);
  const uint64_t *val64 = reinterpret_cast<const uint64_t *>(stage + off64);
  const int total = n32 + n64;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    if (i < n32) {
      i32[idx32[i]] = val32[i];
    } else {
      const int k = i - n32;
      o64[idx64[k]] = val64[k];
    }
  }
}

}  // namespace

cudaError_t apply_table_updates(const void *stage, int n32, int n64, size_t off64, int32_t *i32,
                                uint64_t *o64, cudaStream_t stream) {
  const int total = n32 + n64;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = std::min((total + threads - 1) / threads, 1184);
  return launch_pdl(apply_updates_kernel, dim3(blocks), dim3(threads), 0, stream,
                    static_cast<const unsigned char *>(stage), n32, n64, off64, i32, o64);
}

}  // namespace dev
}  // namespace kcmm
