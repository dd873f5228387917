// Error reporting, device queries and small utility kernels of the C-ABI.
#include "pp_host.h"

#include <cuda_fp16.h>

#include <cstring>

namespace pp {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return PP_ERR_CUDA;
  }
  return PP_OK;
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int device_sm_count(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 0;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    cache[device] = n;
  }
  return cache[device];
}

// Writes zeros into an (R, C) FP16 matrix with arbitrary element strides.
__global__ void fill_zero_f16(__half* p, int64_t R, int64_t C, int64_t ldr, int64_t ldc) {
  const int64_t total = R * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / C, c = i % C;
    p[r * ldr + c * ldc] = __float2half_rn(0.0f);
  }
}

int zero_f16(void* p, int64_t R, int64_t C, int64_t ldr, int64_t ldc, cudaStream_t s) {
  if (R <= 0 || C <= 0) return PP_OK;
  const int64_t total = R * C;
  const int blocks = (int)(total < 4096 * 256 ? cdiv(total, 256) : 4096);
  fill_zero_f16<<<blocks, 256, 0, s>>>(reinterpret_cast<__half*>(p), R, C, ldr, ldc);
  return check_launch("fill_zero_f16");
}

}  // namespace pp

extern "C" {

const char* pp_last_error(void) { return pp::g_err; }

int pp_version(void) { return PP_VERSION; }

int pp_device_sm_count(int device) { return pp::device_sm_count(device); }

}  // extern "C"
