// Error reporting, device queries and small utility kernels of the C-ABI.
#include "pp_host.h"

#include <cuda_fp16.h>

#include <atomic>
#include <cstring>

namespace pp {

static std::atomic<int> g_launch_overlap{0};

bool launch_overlap() { return g_launch_overlap.load(std::memory_order_relaxed) != 0; }

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

int reserved_smem(int device) {
  static int cache[64];
  static bool done[64];
  if (device < 0 || device >= 64) return 0;
  if (!done[device]) {
    int r = 0;
    if (cudaDeviceGetAttribute(&r, cudaDevAttrReservedSharedMemoryPerBlock, device) != cudaSuccess) {
      cudaGetLastError();
      r = 0;
    }
    cache[device] = r;
    done[device] = true;
  }
  return cache[device];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    tried = true;
  }
  return fn;
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t dim0, uint64_t dim1,
                   uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return PP_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {dim0, dim1};
  const cuuint64_t strides[1] = {stride1_bytes};
  const cuuint32_t box[2] = {box0, box1};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for dims %llu x %llu stride %llu", (int)r,
              (unsigned long long)dim0, (unsigned long long)dim1, (unsigned long long)stride1_bytes);
    return PP_ERR_CUDA;
  }
  return PP_OK;
}

int encode_tmap_u32_2d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1, uint64_t stride1_bytes,
                       uint32_t box0, uint32_t box1) {
  return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, base, dim0, dim1, stride1_bytes, box0, box1,
                        CU_TENSOR_MAP_SWIZZLE_128B);
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

int pp_set_launch_overlap(int enable) {
  const int old = pp::g_launch_overlap.exchange(enable ? 1 : 0);
  return old;
}

}  // extern "C"
