// Virtual-memory arenas: a device address range that stays reserved for the life of the process
// while its physical memory is mapped in and out.
//
// The rollout engine's KV cache lives in one arena. Releasing the engine's memory for training
// unmaps and frees the physical pages; resuming maps fresh pages at the SAME virtual addresses,
// so the CUDA graphs captured for decode (which bake in the cache's addresses) stay valid
// across release / resume and are captured once per process instead of once per rollout.
//
// Reference role: torch_memory_saver's pause / resume of tagged allocations (the reference
// releases SGLang's KV cache and weights around training the same way, keeping addresses).
//
// Driver entry points are resolved through cudaGetDriverEntryPoint (no link-time libcuda).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace {

struct VmmApi {
  CUresult (*reserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
  CUresult (*free_va)(CUdeviceptr, size_t) = nullptr;
  CUresult (*create)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*,
                     unsigned long long) = nullptr;
  CUresult (*release)(CUmemGenericAllocationHandle) = nullptr;
  CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle,
                  unsigned long long) = nullptr;
  CUresult (*unmap)(CUdeviceptr, size_t) = nullptr;
  CUresult (*set_access)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t) = nullptr;
  CUresult (*granularity)(size_t*, const CUmemAllocationProp*,
                          CUmemAllocationGranularity_flags) = nullptr;
  bool ok = false;
};

template <typename F>
bool resolve(const char* name, F* fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr)
    return false;
  *fn = reinterpret_cast<F>(p);
  return true;
}

const VmmApi& api() {
  static VmmApi a = [] {
    VmmApi v;
    v.ok = resolve("cuMemAddressReserve", &v.reserve) && resolve("cuMemAddressFree", &v.free_va) &&
           resolve("cuMemCreate", &v.create) && resolve("cuMemRelease", &v.release) &&
           resolve("cuMemMap", &v.map) && resolve("cuMemUnmap", &v.unmap) &&
           resolve("cuMemSetAccess", &v.set_access) &&
           resolve("cuMemGetAllocationGranularity", &v.granularity);
    return v;
  }();
  return a;
}

CUmemAllocationProp device_prop(int device) {
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  return prop;
}

}  // namespace

// Allocation granularity of `device` (sizes passed to the functions below are multiples of it).
extern "C" int mb_vmm_granularity(int device, size_t* gran) {
  const VmmApi& a = api();
  if (!a.ok) return -1;
  CUmemAllocationProp prop = device_prop(device);
  return a.granularity(gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) == CUDA_SUCCESS ? 0 : -2;
}

// Reserves `bytes` (a granularity multiple) of device virtual address space.
extern "C" int mb_vmm_reserve(size_t bytes, unsigned long long* ptr) {
  const VmmApi& a = api();
  if (!a.ok) return -1;
  CUdeviceptr p = 0;
  if (a.reserve(&p, bytes, 0, 0, 0) != CUDA_SUCCESS) return -2;
  *ptr = static_cast<unsigned long long>(p);
  return 0;
}

extern "C" int mb_vmm_free(unsigned long long ptr, size_t bytes) {
  const VmmApi& a = api();
  if (!a.ok) return -1;
  return a.free_va(static_cast<CUdeviceptr>(ptr), bytes) == CUDA_SUCCESS ? 0 : -2;
}

// Backs [ptr, ptr + bytes) with new physical memory of `device` (read / write from it).
extern "C" int mb_vmm_map(unsigned long long ptr, size_t bytes, int device,
                          unsigned long long* handle) {
  const VmmApi& a = api();
  if (!a.ok) return -1;
  CUmemAllocationProp prop = device_prop(device);
  CUmemGenericAllocationHandle h = 0;
  if (a.create(&h, bytes, &prop, 0) != CUDA_SUCCESS) return -3;  // out of memory
  if (a.map(static_cast<CUdeviceptr>(ptr), bytes, 0, h, 0) != CUDA_SUCCESS) {
    a.release(h);
    return -4;
  }
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  if (a.set_access(static_cast<CUdeviceptr>(ptr), bytes, &acc, 1) != CUDA_SUCCESS) {
    a.unmap(static_cast<CUdeviceptr>(ptr), bytes);
    a.release(h);
    return -5;
  }
  *handle = static_cast<unsigned long long>(h);
  return 0;
}

// Unmaps [ptr, ptr + bytes) and frees its physical memory (the address range stays reserved).
// The caller synchronises the device first: no kernel may still be reading the range.
extern "C" int mb_vmm_unmap(unsigned long long ptr, size_t bytes, unsigned long long handle) {
  const VmmApi& a = api();
  if (!a.ok) return -1;
  if (a.unmap(static_cast<CUdeviceptr>(ptr), bytes) != CUDA_SUCCESS) return -2;
  return a.release(static_cast<CUmemGenericAllocationHandle>(handle)) == CUDA_SUCCESS ? 0 : -3;
}

// Page-locks [ptr, ptr + bytes) of ordinary host memory so that copies from / to it run as
// asynchronous DMA (used to pin the host-resident optimizer state chunk by chunk in the
// background instead of one long cudaHostAlloc before the first optimizer step).
extern "C" int mb_host_register(void* ptr, size_t bytes) {
  return cudaHostRegister(ptr, bytes, cudaHostRegisterDefault) == cudaSuccess ? 0 : -1;
}

extern "C" int mb_host_unregister(void* ptr) {
  return cudaHostUnregister(ptr) == cudaSuccess ? 0 : -1;
}
