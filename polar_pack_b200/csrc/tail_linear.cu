// Plain FP16 Linear over per-model weight rows: the rows of a `.quadpack`
// Linear that lie past the coded range (the per-model FP16 tails).
//
// The reference writes every weight of model k beyond the shortest model's
// length as raw FP16 (quaternion_packer.py:118-126) and copies it back as
// is when restoring (201-210); a Linear whose flat range reaches past
// n_min therefore takes those rows from the tail of each model that is long
// enough.  The kernel computes, for every model k whose weight pointer is
// set,
//
//   out_k[m][r] = fp16( sum_i x_k[m][i] * W_k[r][i] )     (FP32 accumulate)
//
// with x_k = x + k * ldx_model (ldx_model = 0: one activation matrix for all
// models).  Tail rows start wherever the Linear's range crosses n_min, so
// the rows need not be aligned: each warp takes one row and reads it with
// 2-byte loads, 32 consecutive elements per warp instruction.  Tails hold a
// small share of a stream's weights; this kernel is bound by HBM latency,
// not tuned for bandwidth.
#include <cuda_fp16.h>

#include "pp_common.cuh"
#include "pp_host.h"

namespace pp {
namespace {

struct F16LinParams {
  const __half* x;
  int64_t ldx_m, ldx_model;
  const __half* w[4];
  int64_t ldw;
  __half* out[4];
  int64_t ldo_m, ldo_n;
  int M, R, K;
};

constexpr int kRowsPerBlock = 8;  // one warp per row
constexpr int kBatchPass = 8;     // batch rows accumulated per pass over a weight row

__global__ void __launch_bounds__(kRowsPerBlock * 32) f16_linear_kernel(const F16LinParams p) {
  const int model = blockIdx.y;
  const __half* w = p.w[model];
  if (w == nullptr) return;
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if (r >= p.R) return;
  const __half* wr = w + r * p.ldw;
  const __half* xm = p.x + (int64_t)model * p.ldx_model;
  for (int m0 = 0; m0 < p.M; m0 += kBatchPass) {
    float acc[kBatchPass];
#pragma unroll
    for (int j = 0; j < kBatchPass; ++j) acc[j] = 0.f;
    for (int i = lane; i < p.K; i += 32) {
      const float wv = __half2float(wr[i]);
#pragma unroll
      for (int j = 0; j < kBatchPass; ++j)
        if (m0 + j < p.M) acc[j] = fmaf(wv, __half2float(xm[(int64_t)(m0 + j) * p.ldx_m + i]), acc[j]);
    }
#pragma unroll
    for (int j = 0; j < kBatchPass; ++j) {
      float v = acc[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && m0 + j < p.M) p.out[model][(int64_t)(m0 + j) * p.ldo_m + r * p.ldo_n] = __float2half_rn(v);
    }
  }
}

}  // namespace
}  // namespace pp

extern "C" {

int pp_f16_linear(const void* x, int64_t ldx_m, int64_t ldx_model, int64_t M, int64_t K,
                  const void* const w[4], int64_t ldw, int64_t R, void* const out[4], int64_t ldo_m,
                  int64_t ldo_n, void* stream) {
  if (M < 0 || K < 0 || R < 0 || !w || !out) {
    pp::set_error("pp_f16_linear: negative shape or NULL weight / output array");
    return PP_ERR_INVALID;
  }
  if (M > INT32_MAX || K > INT32_MAX || R > INT32_MAX) {
    pp::set_error("pp_f16_linear: M, K and R must fit in 32 bits");
    return PP_ERR_INVALID;
  }
  pp::F16LinParams p{};
  int any = 0;
  for (int k = 0; k < 4; ++k) {
    p.w[k] = reinterpret_cast<const __half*>(w[k]);
    p.out[k] = reinterpret_cast<__half*>(out[k]);
    if (w[k] && !out[k]) {
      pp::set_error("pp_f16_linear: out[%d] is NULL for a model with weights", k);
      return PP_ERR_INVALID;
    }
    any |= w[k] != nullptr;
  }
  if (M == 0 || R == 0 || !any) return PP_OK;
  if (K > 0 && (!x || ldw < K)) {
    pp::set_error("pp_f16_linear: x is NULL or ldw < K");
    return PP_ERR_INVALID;
  }
  p.x = reinterpret_cast<const __half*>(x);
  p.ldx_m = ldx_m;
  p.ldx_model = ldx_model;
  p.ldw = ldw;
  p.ldo_m = ldo_m;
  p.ldo_n = ldo_n;
  p.M = (int)M;
  p.R = (int)R;
  p.K = (int)K;
  const int64_t gx = pp::cdiv(R, pp::kRowsPerBlock);
  if (gx > INT32_MAX) {
    pp::set_error("pp_f16_linear: too many rows");
    return PP_ERR_INVALID;
  }
  pp::f16_linear_kernel<<<dim3((unsigned)gx, 4), pp::kRowsPerBlock * 32, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return pp::check_launch("f16_linear_kernel");
}

}  // extern "C"
