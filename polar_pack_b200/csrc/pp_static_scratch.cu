// pp_quad_gemm_static_scratch: pp_quad_gemm with its split-K scratch in a
// file-scope device array instead of a caller-provided workspace.
//
// For callers that cannot call cudaMalloc: plugin hosts that hand the
// library only tensor pointers while their own pool owns all device memory
// (they have no allocator to offer for a workspace), and code paths that
// must not allocate because cudaMalloc can synchronise the device.  This
// entry point allocates nothing; the scratch is module memory created when
// the library is loaded.
//
// Limit: kStaticScratchBytes (1 MiB) per device.  A plan that needs more
// is rejected with PP_ERR_WORKSPACE before anything is enqueued.  1 MiB
// covers the file layout (codes K-contiguous) at every batch size and the
// kernel layout (N-contiguous) up to M = 6 on a 148-SM device.
//
// All calls on a device share the one array, so two calls that can run at
// the same time (on different streams, or from different host threads)
// race on it and corrupt each other's results; such callers must
// serialise them.
//
// The host cannot pass g_quad_scratch itself to a kernel: in host code the
// name is a host-side stand-in, not a device address.  The first call on a
// device therefore looks the address up with cudaGetSymbolAddress while
// that device is current and keeps it for later calls; that first call
// should come before any stream capture on the device.
#include <mutex>

#include "pp_common.cuh"
#include "pp_engine.cuh"  // kCounterBytes: the counter block at the front of the scratch
#include "pp_host.h"

namespace pp {
namespace {

constexpr size_t kStaticScratchBytes = size_t(1) << 20;

static __device__ __align__(256) unsigned char g_quad_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64];
bool g_scratch_known[64];

// Device address of g_quad_scratch on the current device, looked up once
// per device while that device is current.
int static_scratch(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) {
    set_error("no current CUDA device");
    return PP_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_known[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_quad_scratch);
    if (e != cudaSuccess) {
      set_error("cudaGetSymbolAddress of the static scratch failed: %s", cudaGetErrorString(e));
      return PP_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
    g_scratch_known[dev] = true;
  }
  *out = g_scratch_addr[dev];
  return PP_OK;
}

}  // namespace
}  // namespace pp

extern "C" {

int pp_quad_gemm_static_scratch(const void* a, int64_t lda_m, int64_t lda_k, const uint32_t* codes, int64_t ldc_k,
                                int64_t ldc_n, const void* const luts[7], const float scales[4],
                                void* const out[4], int64_t ldo_m, int64_t ldo_n, int64_t M, int64_t N,
                                int64_t K, void* stream) {
  size_t need = 0;
  int rc = pp_quad_gemm_workspace_bytes(M, N, K, ldc_k, ldc_n, &need);
  if (rc) return rc;
  if (need > pp::kStaticScratchBytes) {
    pp::set_error("this problem needs %zu bytes of split-K scratch; the static scratch holds %zu",
                  need, pp::kStaticScratchBytes);
    return PP_ERR_WORKSPACE;
  }
  void* ws = nullptr;
  size_t ws_bytes = 0;
  if (need > 0) {
    if ((rc = pp::static_scratch(&ws))) return rc;
    ws_bytes = pp::kStaticScratchBytes;
    // The arrival counters (and the status word) at the front of the
    // scratch must start at zero.  Kernels leave them zero, but a call that
    // was cut short, or a racing call, may not have.
    const size_t clear = need < pp::kCounterBytes ? need : pp::kCounterBytes;
    const cudaError_t e = cudaMemsetAsync(ws, 0, clear, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
      pp::set_error("clearing the static scratch failed: %s", cudaGetErrorString(e));
      return PP_ERR_CUDA;
    }
  }
  return pp_quad_gemm(a, lda_m, lda_k, codes, ldc_k, ldc_n, luts, scales, out, ldo_m, ldo_n, M, N, K, ws, ws_bytes,
                      stream);
}

}  // extern "C"
