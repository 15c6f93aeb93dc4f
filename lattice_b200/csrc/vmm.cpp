// Physical memory backends for the per-layer K/V regions.
//
// The CUDA backend restates ref src/cache/cuda_vmm.rs:56-170: reserve a VA
// range, then back it 2 MiB at a time with cuMemCreate(PINNED, device) +
// cuMemMap + cuMemSetAccess(RW).  The driver entry points are fetched through
// cudaGetDriverEntryPoint so the library has no link-time dependency on
// libcuda (it loads in a container without a GPU driver).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <sys/mman.h>

#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "kcmm_internal.hpp"

namespace kcmm {
namespace {

struct DriverApi {
  PFN_cuTensorMapEncodeTiled_v12000 encode_tiled = nullptr;
  PFN_cuMemAddressReserve_v10020 reserve = nullptr;
  PFN_cuMemAddressFree_v10020 address_free = nullptr;
  PFN_cuMemCreate_v10020 create = nullptr;
  PFN_cuMemRelease_v10020 release = nullptr;
  PFN_cuMemMap_v10020 map = nullptr;
  PFN_cuMemUnmap_v10020 unmap = nullptr;
  PFN_cuMemSetAccess_v10020 set_access = nullptr;
};

template <typename F>
void fetch(const char *sym, F *out) {
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion(sym, &fn, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess) {
    throw Error(std::string("driver entry point unavailable: ") + sym);
  }
  *out = reinterpret_cast<F>(fn);
}

const DriverApi &driver() {
  static DriverApi api;
  static std::once_flag once;
  static std::string failure;
  std::call_once(once, [] {
    try {
      fetch("cuTensorMapEncodeTiled", &api.encode_tiled);
      fetch("cuMemAddressReserve", &api.reserve);
      fetch("cuMemAddressFree", &api.address_free);
      fetch("cuMemCreate", &api.create);
      fetch("cuMemRelease", &api.release);
      fetch("cuMemMap", &api.map);
      fetch("cuMemUnmap", &api.unmap);
      fetch("cuMemSetAccess", &api.set_access);
    } catch (const Error &e) {
      failure = e.what();
    }
  });
  if (!failure.empty()) throw Error(failure);
  return api;
}

void check(CUresult r, const char *what) {
  if (r != CUDA_SUCCESS) {
    throw Error(std::string(what) + " failed: CUresult " + std::to_string(int(r)));
  }
}

class CudaVmm final : public Vmm {
 public:
  explicit CudaVmm(int device) : device_(device) {
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaFree(nullptr);  // create the primary context
    if (e != cudaSuccess) {
      throw Error(std::string("CUDA device ") + std::to_string(device) +
                  " unavailable: " + cudaGetErrorString(e));
    }
    (void)driver();
  }
  ~CudaVmm() override { release_all(); }

  uint64_t reserve(size_t bytes) override {
    CUdeviceptr p = 0;
    check(driver().reserve(&p, bytes, kSuperblockBytes, 0, 0), "cuMemAddressReserve");
    reservations_.push_back({uint64_t(p), bytes});
    return uint64_t(p);
  }

  void create_and_map(uint64_t va, size_t bytes) override {
    CUmemAllocationProp prop = {};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = device_;
    CUmemGenericAllocationHandle h = 0;
    check(driver().create(&h, bytes, &prop, 0), "cuMemCreate");
    CUresult r = driver().map(CUdeviceptr(va), bytes, 0, h, 0);
    if (r != CUDA_SUCCESS) {
      driver().release(h);
      check(r, "cuMemMap");
    }
    CUmemAccessDesc acc = {};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = device_;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    r = driver().set_access(CUdeviceptr(va), bytes, &acc, 1);
    if (r != CUDA_SUCCESS) {
      driver().unmap(CUdeviceptr(va), bytes);
      driver().release(h);
      check(r, "cuMemSetAccess");
    }
    mappings_.push_back({va, bytes, h});
  }

  void release_all() noexcept override {
    if (mappings_.empty() && reservations_.empty()) return;
    cudaSetDevice(device_);
    cudaDeviceSynchronize();
    for (auto &m : mappings_) {
      driver().unmap(CUdeviceptr(m.va), m.bytes);
      driver().release(m.handle);
    }
    mappings_.clear();
    for (auto &r : reservations_) driver().address_free(CUdeviceptr(r.first), r.second);
    reservations_.clear();
  }
  bool is_device() const override { return true; }
  const char *name() const override { return "cuda-vmm"; }

 private:
  struct Mapping {
    uint64_t va;
    size_t bytes;
    CUmemGenericAllocationHandle handle;
  };
  int device_;
  std::vector<Mapping> mappings_;
  std::vector<std::pair<uint64_t, size_t>> reservations_;
};

class HostVmm final : public Vmm {
 public:
  HostVmm() {
    if (const char *s = std::getenv("KCMM_HOST_VMM_FAIL_AFTER")) fail_after_ = std::atol(s);
  }
  ~HostVmm() override { release_all(); }
  uint64_t reserve(size_t bytes) override {
    void *p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE,
                   MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
    if (p == MAP_FAILED) throw Error("host reserve failed");
    regions_.push_back({uint64_t(p), bytes});
    return uint64_t(p);
  }
  void create_and_map(uint64_t va, size_t bytes) override {
    if (fail_after_ >= 0 && created_ >= fail_after_) {
      throw Error("cuMemCreate failed: CUresult 2 (injected by KCMM_HOST_VMM_FAIL_AFTER)");
    }
    // as cuMemMap does, refuse a range outside every reservation
    bool inside = false;
    for (const auto &r : regions_) inside = inside || (va >= r.first && va + bytes <= r.first + r.second);
    if (!inside) throw Error("cuMemMap failed: CUresult 1 (range outside the reserved region)");
    ++created_;
  }
  void release_all() noexcept override {
    for (auto &r : regions_) munmap(reinterpret_cast<void *>(r.first), r.second);
    regions_.clear();
  }
  bool is_device() const override { return false; }
  const char *name() const override { return "host"; }

 private:
  std::vector<std::pair<uint64_t, size_t>> regions_;
  long fail_after_ = -1;
  long created_ = 0;
};

}  // namespace

std::unique_ptr<Vmm> make_cuda_vmm(int device) { return std::make_unique<CudaVmm>(device); }

bool encode_kv_tensor_map(void *out, uint64_t base, uint64_t tokens, int kv_heads, int head_dim) {
  // 3-D view of a layer region: {head_dim, kv_heads, tokens} of 16-bit words;
  // box {64, 1, 16} = 16 tokens x 64 dims of one head, 128B-swizzled in smem.
  if (head_dim % 64 != 0 || tokens == 0 || tokens > (uint64_t(1) << 32)) return false;
  cuuint64_t dims[3] = {cuuint64_t(head_dim), cuuint64_t(kv_heads), cuuint64_t(tokens)};
  cuuint64_t strides[2] = {cuuint64_t(head_dim) * 2, cuuint64_t(head_dim) * 2 * kv_heads};
  cuuint32_t box[3] = {64, 1, 16};
  cuuint32_t estr[3] = {1, 1, 1};
  const DriverApi *api = nullptr;
  try {
    api = &driver();
  } catch (const Error &) {
    return false;
  }
  CUresult r = api->encode_tiled(
      static_cast<CUtensorMap *>(out), CU_TENSOR_MAP_DATA_TYPE_UINT16, 3,
      reinterpret_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}
bool encode_kv_page_tensor_map(void *out, uint64_t base, uint64_t tokens, int kv_heads,
                               int head_dim) {
  if (head_dim % 64 != 0 || head_dim / 64 > 8 || tokens == 0 || tokens > (uint64_t(1) << 32))
    return false;
  const cuuint64_t row = cuuint64_t(kv_heads) * head_dim * 2;  // bytes per token row
  cuuint64_t dims[4] = {64, cuuint64_t(tokens), cuuint64_t(head_dim / 64), cuuint64_t(kv_heads)};
  cuuint64_t strides[3] = {row, 128, cuuint64_t(head_dim) * 2};
  cuuint32_t box[4] = {64, 16, cuuint32_t(head_dim / 64), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const DriverApi *api = nullptr;
  try {
    api = &driver();
  } catch (const Error &) {
    return false;
  }
  CUresult r = api->encode_tiled(
      static_cast<CUtensorMap *>(out), CU_TENSOR_MAP_DATA_TYPE_UINT16, 4,
      reinterpret_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

std::unique_ptr<Vmm> make_host_vmm() { return std::make_unique<HostVmm>(); }

}  // namespace kcmm
