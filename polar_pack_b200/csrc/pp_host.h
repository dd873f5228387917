// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <utility>

#include "../../include/polar_pack_b200.h"

namespace pp {

// Thread-local message for pp_last_error().
void set_error(const char* fmt, ...);

// Returns PP_OK, or records the CUDA error and returns PP_ERR_CUDA.
int check_launch(const char* what);

int device_sm_count(int device);
int current_device();

// Shared memory the driver reserves at the start of every CTA's window
// (the dynamic region of a kernel without static shared memory starts
// there); 0 if the query fails.
int reserved_smem(int device);

// 2D tensor map over a row-major uint32 matrix (dim0 contiguous), box
// box0 x box1, 128-byte swizzle, zero fill out of bounds.  Requires a
// 16-byte aligned base, stride1_bytes % 16 == 0 and box0 * 4 <= 128.
int encode_tmap_u32_2d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t stride1_bytes,
                       uint32_t box0, uint32_t box1);

// General 2D tiled tensor map (dim0 contiguous), zero fill out of bounds.
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                   uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle);

// Raises a kernel's dynamic shared memory limit to the device's opt-in
// maximum minus the kernel's static shared memory, once per device, and
// returns that limit in *max_dynamic.
template <typename K>
int ensure_smem_attr(K kernel, bool* done_flags, int* limits, int* max_dynamic) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) {
    set_error("no current CUDA device");
    return PP_ERR_CUDA;
  }
  if (!done_flags[dev]) {
    int optin = 0;
    cudaFuncAttributes fa{};
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kernel);
    const int lim = optin - (int)fa.sharedSizeBytes;
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    if (e != cudaSuccess) {
      set_error("shared memory attribute set-up: %s", cudaGetErrorString(e));
      return PP_ERR_CUDA;
    }
    limits[dev] = lim;
    done_flags[dev] = true;
  }
  *max_dynamic = limits[dev];
  return PP_OK;
}

// Launch overlap (programmatic dependent launch) for the kernels that
// support it, switched by pp_set_launch_overlap().
bool launch_overlap();

// cudaLaunchKernelEx with programmatic stream serialisation when
// `overlap` is set; records launch errors.
template <typename... KArgs, typename... Args>
int launch_kernel(const char* what, bool overlap, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("%s: %s", what, cudaGetErrorString(e));
    return PP_ERR_CUDA;
  }
  return check_launch(what);
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace pp
