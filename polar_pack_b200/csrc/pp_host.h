// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/polar_pack_b200.h"

namespace pp {

// Thread-local message for pp_last_error().
void set_error(const char* fmt, ...);

// Returns PP_OK, or records the CUDA error and returns PP_ERR_CUDA.
int check_launch(const char* what);

int device_sm_count(int device);
int current_device();

// Kernel attribute set-up done once per device (dynamic shared memory).
template <typename K>
int ensure_smem_attr(K kernel, int bytes, bool* done_flags) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return PP_ERR_CUDA;
  if (!done_flags[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute(max dynamic smem %d): %s", bytes, cudaGetErrorString(e));
      return PP_ERR_CUDA;
    }
    done_flags[dev] = true;
  }
  return PP_OK;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace pp
