// Copy-engine transfers between the GPUs of one node, for the head-sharded hybrid layer's
// exchange: CUDA IPC handles of device allocations (exported by one rank, mapped by the
// others) and asynchronous copies into the mapped memory. The copies run on the GPUs' copy
// engines over NVLink and occupy no SMs, so the exchange overlaps the attention kernel, which
// fills every SM. No kernels here.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstring>
#include <mutex>

#include "../../include/pbk.h"

namespace {
int status_of(cudaError_t e) { return e == cudaSuccess ? PBK_OK : PBK_ERR_LAUNCH; }

// cuMemGetAddressRange through the runtime's driver entry point (no link-time dependency on
// the driver library, so the library still loads on hosts without a GPU).
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}
}  // namespace

extern "C" {

int pbk_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return PBK_ERR_INVALID;
  CUdeviceptr base = 0;
  size_t size = 0;
  const AddressRangeFn range = address_range_fn();
  if (range == nullptr) return PBK_ERR_DEVICE;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return PBK_ERR_INVALID;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return status_of(e);
  static_assert(sizeof(cudaIpcMemHandle_t) == PBK_IPC_HANDLE_BYTES, "handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return PBK_OK;
}

int pbk_ipc_open(const void* handle, void** base) {
  if (handle == nullptr || base == nullptr) return PBK_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return status_of(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
}

int pbk_ipc_close(void* base) {
  if (base == nullptr) return PBK_ERR_INVALID;
  return status_of(cudaIpcCloseMemHandle(base));
}

int pbk_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return PBK_OK;
  if (dst == nullptr || src == nullptr) return PBK_ERR_INVALID;
  return status_of(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
