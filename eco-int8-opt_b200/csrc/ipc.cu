// Mapping of the data-parallel exchange buffers between the processes of one
// node with CUDA IPC memory handles (cudaIpcGetMemHandle / cudaIpcOpenMemHandle).
//
// Every rank allocates its own copy of an exchange buffer (ordinary device
// memory from the caller's allocator), exports the allocation that contains
// it, and opens the other ranks' allocations; a peer's copy is then an
// ordinary device pointer that kernels store to over NVLink.  Only unicast
// peer mappings are made: no NVLink multicast object is created or bound, so
// a rank that ends early leaves nothing bound on the other GPUs.
#include <cuda.h>

#include <cstring>

#include "abi.cuh"

namespace {

typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  }
  return fn;
}

}  // namespace

extern "C" int eco_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  ECO_REQUIRE(ptr && handle && offset, ECO_ERR_ARG, "eco_ipc_export: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == ECO_IPC_HANDLE_BYTES, "IPC handle size");
  AddrRangeFn fn = addr_range_fn();
  if (!fn) return eco_fail(ECO_ERR_LAUNCH, "eco_ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return eco_fail(ECO_ERR_ARG, "eco_ipc_export: not device memory (%d)", (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return eco_fail(ECO_ERR_LAUNCH, "eco_ipc_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  std::memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return ECO_OK;
}

extern "C" int eco_ipc_open(const void* handle, void** base) {
  ECO_REQUIRE(handle && base, ECO_ERR_ARG, "eco_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return eco_fail(ECO_ERR_LAUNCH, "eco_ipc_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  }
  *base = p;
  return ECO_OK;
}

extern "C" int eco_ipc_close(void* base) {
  ECO_REQUIRE(base, ECO_ERR_ARG, "eco_ipc_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return eco_fail(ECO_ERR_LAUNCH, "eco_ipc_close: %s", cudaGetErrorString(e));
  }
  return ECO_OK;
}
