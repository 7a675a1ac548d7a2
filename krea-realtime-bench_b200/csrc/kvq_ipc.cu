// Mapping another process's device buffer into this one (CUDA IPC), for the
// head-sharded attention whose epilogue stores every output row into all
// ranks' output buffers over NVLink. Host code only; the reference is single
// GPU and has no counterpart.
//
// A tensor from a caching allocator usually sits inside a larger cudaMalloc
// block, and an IPC handle names a whole block, so the exporter sends the
// block's handle plus the tensor's byte offset within it.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "kvq_common.cuh"

namespace kvq {
namespace {

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

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
}  // namespace kvq

using namespace kvq;

static_assert(sizeof(cudaIpcMemHandle_t) == KVQ_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int kvq_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  clear_error();
  KVQ_REQUIRE(ptr && handle && offset, KVQ_ERR_ARG, "NULL argument");
  AddressRangeFn fn = address_range_fn();
  KVQ_REQUIRE(fn != nullptr, KVQ_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  KVQ_REQUIRE(r == CUDA_SUCCESS, KVQ_ERR_CUDA, "cuMemGetAddressRange failed with %d (not device memory?)", (int)r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  KVQ_REQUIRE(e == cudaSuccess, KVQ_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return KVQ_OK;
}

extern "C" int kvq_ipc_import(const void* handle, int64_t offset, void** base, void** ptr) {
  clear_error();
  KVQ_REQUIRE(handle && base && ptr && offset >= 0, KVQ_ERR_ARG, "bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  KVQ_REQUIRE(e == cudaSuccess, KVQ_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *base = b;
  *ptr = static_cast<char*>(b) + offset;
  return KVQ_OK;
}

extern "C" int kvq_ipc_close(void* base) {
  clear_error();
  KVQ_REQUIRE(base, KVQ_ERR_ARG, "NULL base");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  KVQ_REQUIRE(e == cudaSuccess, KVQ_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return KVQ_OK;
}
