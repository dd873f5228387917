// Peer-memory plumbing of the gathered Linears (pp_peer.h): CUDA IPC
// mapping of device buffers between the processes of one node, and the
// bounded wait for every rank's epoch.  No counterpart in the reference,
// which runs one model per process on one GPU.
#include <cuda.h>

#include "pp_common.cuh"
#include "pp_host.h"
#include "pp_peer.h"

namespace pp {
namespace {

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
    tried = true;
  }
  return fn;
}

// Polls until flag[q] - epoch >= 0 (wrap-safe) for every rank q < world,
// one thread per rank, for at most about a second; a rank that never
// arrives sets *status = 3 and the kernel ends.  The epoch count is written
// by this rank's previous launch, so it is read after the dependency wait.
constexpr int kWaitPolls = 1 << 24;

__global__ void gather_wait_kernel(const uint32_t* flags, int world, const uint32_t* epoch, int* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int q = threadIdx.x;
  if (q >= world) return;
  const uint32_t e = *epoch;
  for (int i = 0; i < kWaitPolls; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + q) : "memory");
    if ((int32_t)(v - e) >= 0) return;
    __nanosleep(64);
  }
  atomicExch(status, 3);
}

}  // namespace
}  // namespace pp

extern "C" {

int pp_ipc_handle(const void* ptr, void* handle, size_t* offset) {
  if (!ptr || !handle || !offset) {
    pp::set_error("pp_ipc_handle: NULL argument");
    return PP_ERR_INVALID;
  }
  pp::AddressRangeFn fn = pp::address_range_fn();
  if (!fn) {
    pp::set_error("cuMemGetAddressRange is not available from the driver");
    return PP_ERR_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    pp::set_error("cuMemGetAddressRange failed for %p", ptr);
    return PP_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    pp::set_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return PP_ERR_CUDA;
  }
  static_assert(sizeof(h) == PP_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (size_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return PP_OK;
}

int pp_ipc_open(const void* handle, void** base) {
  if (!handle || !base) {
    pp::set_error("pp_ipc_open: NULL argument");
    return PP_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    pp::set_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return PP_ERR_CUDA;
  }
  return PP_OK;
}

int pp_ipc_close(void* base) {
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    pp::set_error("cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
    return PP_ERR_CUDA;
  }
  return PP_OK;
}

int pp_gather_wait(const uint32_t* flags, int world, const uint32_t* epoch, int* status, void* stream) {
  if (world < 1 || world > pp::kMaxPeers || !flags || !epoch || !status) {
    pp::set_error("pp_gather_wait: world must be 1..%d and pointers non-NULL", pp::kMaxPeers);
    return PP_ERR_INVALID;
  }
  return pp::launch_kernel("gather_wait_kernel", pp::launch_overlap(), pp::gather_wait_kernel, dim3(1), dim3(32),
                           0, reinterpret_cast<cudaStream_t>(stream), flags, world, epoch, status);
}

}  // extern "C"
