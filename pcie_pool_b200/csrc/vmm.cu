#include "vmm.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <unistd.h>

#include <map>
#include <mutex>
#include <stdexcept>
#include <string>

namespace ppb {
namespace {

// Driver entry points, resolved through the runtime (no link against libcuda).
struct VmmApi {
  CUresult (*create)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long) = nullptr;
  CUresult (*release)(CUmemGenericAllocationHandle) = nullptr;
  CUresult (*export_fd)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType, unsigned long long) = nullptr;
  CUresult (*import_fd)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType) = nullptr;
  CUresult (*reserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
  CUresult (*free_va)(CUdeviceptr, size_t) = nullptr;
  CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
  CUresult (*unmap)(CUdeviceptr, size_t) = nullptr;
  CUresult (*set_access)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t) = nullptr;
  CUresult (*granularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags) = nullptr;
};

template <class F>
void resolve(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr) {
    cudaGetLastError();
    throw std::runtime_error(std::string("CUDA driver does not provide ") + name);
  }
  fn = reinterpret_cast<F>(p);
}

const VmmApi& api() {
  static VmmApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    resolve("cuMemCreate", a.create);
    resolve("cuMemRelease", a.release);
    resolve("cuMemExportToShareableHandle", a.export_fd);
    resolve("cuMemImportFromShareableHandle", a.import_fd);
    resolve("cuMemAddressReserve", a.reserve);
    resolve("cuMemAddressFree", a.free_va);
    resolve("cuMemMap", a.map);
    resolve("cuMemUnmap", a.unmap);
    resolve("cuMemSetAccess", a.set_access);
    resolve("cuMemGetAllocationGranularity", a.granularity);
  });
  return a;
}

void check(CUresult rc, const char* what) {
  if (rc != CUDA_SUCCESS) throw std::runtime_error(std::string(what) + " failed with CUresult " + std::to_string(rc));
}

CUmemAllocationProp props(int device) {
  CUmemAllocationProp p{};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

struct Mapping {
  CUmemGenericAllocationHandle handle;
  uint64_t size;
};
std::mutex g_mu;
std::map<uint64_t, Mapping> g_maps;

// Reserve address space, map the handle into it and open it to `device`.
uint64_t map_handle(CUmemGenericAllocationHandle h, uint64_t size, int device) {
  const VmmApi& a = api();
  CUdeviceptr va = 0;
  check(a.reserve(&va, size, 0, 0, 0), "cuMemAddressReserve");
  CUresult rc = a.map(va, size, 0, h, 0);
  if (rc != CUDA_SUCCESS) {
    a.free_va(va, size);
    check(rc, "cuMemMap");
  }
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  rc = a.set_access(va, size, &acc, 1);
  if (rc != CUDA_SUCCESS) {
    a.unmap(va, size);
    a.free_va(va, size);
    check(rc, "cuMemSetAccess");
  }
  return static_cast<uint64_t>(va);
}

}  // namespace

uint64_t vmm_granularity(int device) {
  cudaFree(nullptr);  // the driver needs an initialised runtime on some paths
  const CUmemAllocationProp p = props(device);
  size_t g = 0;
  check(api().granularity(&g, &p, CU_MEM_ALLOC_GRANULARITY_MINIMUM), "cuMemGetAllocationGranularity");
  return static_cast<uint64_t>(g);
}

VmmBuffer vmm_alloc(int device, uint64_t bytes) {
  if (bytes == 0) throw std::invalid_argument("vmm_alloc: empty allocation");
  const uint64_t g = vmm_granularity(device);
  const uint64_t size = (bytes + g - 1) / g * g;
  const CUmemAllocationProp p = props(device);
  const VmmApi& a = api();
  CUmemGenericAllocationHandle h = 0;
  check(a.create(&h, size, &p, 0), "cuMemCreate");
  int fd = -1;
  CUresult rc = a.export_fd(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (rc != CUDA_SUCCESS) {
    a.release(h);
    check(rc, "cuMemExportToShareableHandle");
  }
  uint64_t ptr = 0;
  try {
    ptr = map_handle(h, size, device);
  } catch (...) {
    close(fd);
    a.release(h);
    throw;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_maps[ptr] = Mapping{h, size};
  return VmmBuffer{ptr, size, fd, device};
}

VmmBuffer vmm_import(int fd, int device, uint64_t size) {
  if (fd < 0 || size == 0) throw std::invalid_argument("vmm_import: needs a descriptor and a size");
  const uint64_t g = vmm_granularity(device);
  if (size % g != 0) throw std::invalid_argument("vmm_import: size must be a multiple of the granularity");
  const VmmApi& a = api();
  CUmemGenericAllocationHandle h = 0;
  check(a.import_fd(&h, reinterpret_cast<void*>(static_cast<intptr_t>(fd)), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
        "cuMemImportFromShareableHandle");
  uint64_t ptr = 0;
  try {
    ptr = map_handle(h, size, device);
  } catch (...) {
    a.release(h);
    throw;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_maps[ptr] = Mapping{h, size};
  return VmmBuffer{ptr, size, -1, device};
}

void vmm_release(uint64_t ptr) {
  Mapping m{};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(ptr);
    if (it == g_maps.end()) throw std::invalid_argument("vmm_release: not a VMM mapping of this process");
    m = it->second;
    g_maps.erase(it);
  }
  const VmmApi& a = api();
  a.unmap(static_cast<CUdeviceptr>(ptr), m.size);
  a.free_va(static_cast<CUdeviceptr>(ptr), m.size);
  a.release(m.handle);
}

}  // namespace ppb
