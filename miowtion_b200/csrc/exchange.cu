// Plumbing of the head-parallel exchange on the copy engines (no counterpart
// in the reference, which runs one clip per GPU): CUDA IPC handles of device
// buffers, so that one process can address another GPU's buffer, and a
// strided 2-D device copy, which the copy engines execute without using SMs
// (the persistent attention kernel holds every SM).
#include <cuda.h>
#include <string.h>

#include "common.cuh"

namespace veda {
namespace {

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange from the driver (the library links the CUDA runtime
// statically and not the driver): the start of the allocation that holds a
// pointer, which an IPC handle refers to.
int allocation_base(const void* ptr, uintptr_t* base) {
  static GetAddressRangeFn fn = nullptr;
  if (fn == nullptr) {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t err = cudaGetDriverEntryPoint(
        "cuMemGetAddressRange", &sym, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess ||
        sym == nullptr)
      return set_error(VEDA_ERR_CUDA,
                       "cuMemGetAddressRange is not available");
    fn = reinterpret_cast<GetAddressRangeFn>(sym);
  }
  CUdeviceptr b = 0;
  size_t size = 0;
  if (fn(&b, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(VEDA_ERR_INVALID,
                     "the pointer is not inside a device allocation");
  *base = static_cast<uintptr_t>(b);
  return VEDA_OK;
}

}  // namespace
}  // namespace veda

using namespace veda;

extern "C" int veda_ipc_handle(const void* ptr, void* handle,
                               int64_t* offset) {
  VEDA_REQUIRE(ptr != nullptr && handle != nullptr && offset != nullptr,
               "ptr, handle and offset are required");
  uintptr_t base = 0;
  const int rc = allocation_base(ptr, &base);
  if (rc != VEDA_OK) return rc;
  cudaIpcMemHandle_t h;
  VEDA_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(cudaIpcMemHandle_t) == VEDA_IPC_HANDLE_BYTES,
                "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - base);
  return VEDA_OK;
}

extern "C" int veda_ipc_open(const void* handle, void** base) {
  VEDA_REQUIRE(handle != nullptr && base != nullptr,
               "handle and base are required");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  VEDA_CUDA(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  return VEDA_OK;
}

extern "C" int veda_ipc_close(void* base) {
  VEDA_REQUIRE(base != nullptr, "base is required");
  VEDA_CUDA(cudaIpcCloseMemHandle(base));
  return VEDA_OK;
}

extern "C" int veda_copy_2d(void* dst, int64_t dst_pitch, const void* src,
                            int64_t src_pitch, int64_t width, int64_t height,
                            void* stream) {
  VEDA_REQUIRE(dst != nullptr && src != nullptr, "dst and src are required");
  VEDA_REQUIRE(width >= 0 && height >= 0 && dst_pitch >= width &&
                   src_pitch >= width,
               "need 0 <= width <= both pitches and height >= 0");
  if (width == 0 || height == 0) return VEDA_OK;
  VEDA_CUDA(cudaMemcpy2DAsync(dst, static_cast<size_t>(dst_pitch), src,
                              static_cast<size_t>(src_pitch),
                              static_cast<size_t>(width),
                              static_cast<size_t>(height),
                              cudaMemcpyDeviceToDevice, as_stream(stream)));
  return VEDA_OK;
}
