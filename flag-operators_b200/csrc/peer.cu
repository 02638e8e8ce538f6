// Peer-memory plumbing for the kernels that exchange data over NVLink: export a
// device buffer of this process as a CUDA IPC handle (plus its offset inside
// the allocation that holds it, since the caller's allocator may sub-allocate),
// and map another process's buffer into this process's current device.  Plain
// cudaIpc mappings: no multicast object is created, and the kernels access the
// mapped memory with ordinary loads and stores.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace fo {
namespace {

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  }
  return fn;
}

}  // namespace
}  // namespace fo

using namespace fo;

extern "C" int fo_peer_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int fo_peer_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  clear_error();
  FO_CHECK_ARG(ptr && handle_out && offset_out, "fo_peer_export: null pointer");
  AddressRangeFn range = address_range_fn();
  if (!range) {
    set_error("fo_peer_export: the driver's cuMemGetAddressRange is not available");
    return FO_ECUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("fo_peer_export: %p is not device memory of this process", ptr);
    return FO_EINVAL;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    set_error("fo_peer_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return FO_ECUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return FO_OK;
}

extern "C" int fo_peer_open(const void* handle, int64_t offset, void** ptr_out) {
  clear_error();
  FO_CHECK_ARG(handle && ptr_out && offset >= 0, "fo_peer_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("fo_peer_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return FO_ECUDA;
  }
  *ptr_out = static_cast<char*>(base) + offset;
  return FO_OK;
}

extern "C" int fo_peer_close(void* ptr, int64_t offset) {
  clear_error();
  FO_CHECK_ARG(ptr && offset >= 0, "fo_peer_close: bad argument");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) {
    set_error("fo_peer_close: cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
    return FO_ECUDA;
  }
  return FO_OK;
}

extern "C" int fo_peer_can_access(int device, int peer_device, int* ok) {
  clear_error();
  FO_CHECK_ARG(ok, "fo_peer_can_access: null pointer");
  int v = 0;
  if (device == peer_device) {
    v = 1;
  } else if (cudaDeviceCanAccessPeer(&v, device, peer_device) != cudaSuccess) {
    set_error("fo_peer_can_access: cudaDeviceCanAccessPeer(%d, %d) failed", device, peer_device);
    return FO_ECUDA;
  }
  *ok = v;
  return FO_OK;
}
