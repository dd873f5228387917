// `.dualpack` streams on the GPU: the restore of both models' weights and a
// Linear computed straight from the file layout.
//
// File layout (reference polar_bitpack.py:26-29, 79-91, 160-172): pair p of
// the two models is one 16-bit code stored big-endian, amp << phase_bits |
// phase; FP16 group maxima, one per group of `group_size` pairs, with groups
// restarting at every chunk of `chunk_size` pairs; ascending uint32 plug
// positions with the exact FP16 amplitude of each plugged pair.
//
// Restore (polar_bitpack.py:220-247):
//   amp = float32( amp_norm[aq] * scale[g] )        amp_norm[a] = expm1(a / levels * ln(1 + mu)) / mu
//   amp = float32(plug_value)                         at plugged positions
//   w1  = float32( amp * cos(ang[ph]) ),  w2 = float32( amp * sin(ang[ph]) ),  ang = ph / 2^phase_bits * 2pi - pi
// in float64 arithmetic.  The kernels take the float64 tables (amp_norm,
// cos, sin) as the host computes them, so each product here is the same
// IEEE float64 product rounded the same way: the restore is bit-exact.
//
// The Linear (out N, in K; pairs [offset + n K, offset + n K + K) form row n)
// uses FP16 weights W_j = fp16(w_j), the form the reference installs into
// its models (polar_packer.py:309-310):  y_j[m][n] = fp16(sum_k x[m][k] W_j[n][k]),
// FP32 accumulation.  Plugged pairs have their amplitude field cleared at load
// time (amp_norm[0] = 0, so they decode to zeros) and enter as a per-row list
// of exact FP16 weights that the row's warp adds after the dense part.
#include <cuda_fp16.h>

#include "pp_common.cuh"
#include "pp_host.h"

namespace pp {
namespace {

struct DualStream {
  const uint8_t* codes;    // 2 bytes per pair, big-endian
  const __half* scales;    // group maxima
  int64_t chunk, group;    // chunk_size, group_size (groups restart per chunk)
  int phase_bits;
};

__device__ __forceinline__ int64_t group_of(const DualStream& s, int64_t p) {
  const int64_t per_chunk = (s.chunk + s.group - 1) / s.group;
  const int64_t c = p / s.chunk;
  return c * per_chunk + (p - c * s.chunk) / s.group;
}

__device__ __forceinline__ uint32_t code_at(const uint8_t* codes, int64_t p) {
  return ((uint32_t)codes[2 * p] << 8) | codes[2 * p + 1];
}

struct UnpackParams {
  DualStream s;
  const double* amp_norm;  // [2^amp_bits]
  const double* cos_t;     // [2^phase_bits]
  const double* sin_t;
  int64_t start, n;        // pairs [start, start + n)
  float* w1;               // [n] (NULL: not written)
  float* w2;
  __half* h1;              // [n] FP16 of w1 / w2 (NULL: not written)
  __half* h2;
};

__global__ void dual_unpack_kernel(const UnpackParams p) {
  const uint32_t amask = (1u << (16 - p.s.phase_bits)) - 1u, pmask = (1u << p.s.phase_bits) - 1u;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < p.n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = p.start + i;
    const uint32_t u = code_at(p.s.codes, pos);
    const uint32_t aq = (u >> p.s.phase_bits) & amask, ph = u & pmask;
    const float amp = (float)(p.amp_norm[aq] * (double)__half2float(p.s.scales[group_of(p.s, pos)]));
    const float a = (float)((double)amp * p.cos_t[ph]), b = (float)((double)amp * p.sin_t[ph]);
    if (p.w1) p.w1[i] = a;
    if (p.w2) p.w2[i] = b;
    if (p.h1) p.h1[i] = __float2half_rn(a);
    if (p.h2) p.h2[i] = __float2half_rn(b);
  }
}

struct PlugParams {
  const uint8_t* codes;
  int phase_bits;
  const double* cos_t;
  const double* sin_t;
  const uint32_t* pidx;    // plug positions (uint32, relative to base_lo32 modulo 2^32)
  const __half* pval;      // exact FP16 amplitudes
  int64_t np;
  uint32_t base_lo32;      // low 32 bits of the restored range's first position
  int64_t start;           // the range's first position (true, 64-bit)
  int64_t n;
  float* w1;
  float* w2;
  __half* h1;
  __half* h2;
};

// Plugged positions: the amplitude replaced by the plug value, then the same
// products as the restore.
__global__ void dual_unpack_plugs_kernel(const PlugParams p) {
  const uint32_t pmask = (1u << p.phase_bits) - 1u;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < p.np; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = (int64_t)(uint32_t)(p.pidx[e] - p.base_lo32);
    if (i >= p.n) continue;
    const uint32_t ph = code_at(p.codes, p.start + i) & pmask;
    const float amp = __half2float(p.pval[e]);
    const float a = (float)((double)amp * p.cos_t[ph]), b = (float)((double)amp * p.sin_t[ph]);
    if (p.w1) p.w1[i] = a;
    if (p.w2) p.w2[i] = b;
    if (p.h1) p.h1[i] = __float2half_rn(a);
    if (p.h2) p.h2[i] = __float2half_rn(b);
  }
}

constexpr int kDualLinWarps = 8;
constexpr int kDualLinMaxM = 4;

struct LinParams {
  DualStream s;
  const float* amp_norm;   // FP32 tables of the Linear: [2^amp_bits] and (cos, sin) [2^phase_bits]
  const float2* cs;
  int table_n;             // 2^phase_bits
  int amp_n;               // 2^amp_bits
  int64_t offset;          // first pair of the Linear
  const __half* x;         // [M][K], row stride ldx
  int64_t ldx;
  int M, N, K;
  // plug list per row: entries [row_ptr[n], row_ptr[n + 1]) of (col, w1, w2)
  const int* row_ptr;
  const int* pcol;
  const __half2* pw;       // (W1, W2) FP16
  __half* y1;              // [M][ldy]
  __half* y2;
  int64_t ldy;
};

// One warp per output row; the CTA stages x in shared memory (any row start
// alignment), then each lane decodes 16-byte words (8 pairs) of its row.
__global__ void __launch_bounds__(kDualLinWarps * 32) dual_file_linear_kernel(const LinParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* amp_s = reinterpret_cast<float*>(smem);
  float2* cs_s = reinterpret_cast<float2*>(smem + (size_t)p.amp_n * 4);
  __half* xs = reinterpret_cast<__half*>(smem + (size_t)p.amp_n * 4 + (size_t)p.table_n * 8);
  for (int i = threadIdx.x; i < p.amp_n; i += blockDim.x) amp_s[i] = p.amp_norm[i];
  for (int i = threadIdx.x; i < p.table_n; i += blockDim.x) cs_s[i] = p.cs[i];
  for (int i = threadIdx.x; i < p.M * p.K; i += blockDim.x) {
    const int m = i / p.K, k = i - m * p.K;
    xs[i] = p.x[m * p.ldx + k];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t amask = (uint32_t)p.amp_n - 1u, pmask = (uint32_t)p.table_n - 1u;
  for (int64_t n = (int64_t)blockIdx.x * kDualLinWarps + warp; n < p.N; n += (int64_t)gridDim.x * kDualLinWarps) {
    const int64_t r0 = p.offset + n * p.K, r1 = r0 + p.K;
    const int64_t w0 = r0 >> 3, w1 = (r1 + 7) >> 3;  // 16-byte words covering the row
    float acc1[kDualLinMaxM], acc2[kDualLinMaxM];
#pragma unroll
    for (int m = 0; m < kDualLinMaxM; ++m) acc1[m] = acc2[m] = 0.f;
    for (int64_t w = w0 + lane; w < w1; w += 32) {
      const uint4 q = ldg_stream(p.s.codes + 16 * w);
      const float sc = __half2float(p.s.scales[group_of(p.s, 8 * w)]);  // one group per 8-aligned run
      const uint32_t words[4] = {__byte_perm(q.x, 0, 0x2301), __byte_perm(q.y, 0, 0x2301),
                                 __byte_perm(q.z, 0, 0x2301), __byte_perm(q.w, 0, 0x2301)};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t pos = 8 * w + j;
        if (pos < r0 || pos >= r1) continue;
        const uint32_t u = (words[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
        const float amp = amp_s[(u >> p.s.phase_bits) & amask] * sc;
        const float2 c = cs_s[u & pmask];
        const float a = __half2float(__float2half_rn(amp * c.x)), b = __half2float(__float2half_rn(amp * c.y));
        const int k = (int)(pos - r0);
#pragma unroll
        for (int m = 0; m < kDualLinMaxM; ++m)
          if (m < p.M) {
            const float xv = __half2float(xs[m * p.K + k]);
            acc1[m] = fmaf(xv, a, acc1[m]);
            acc2[m] = fmaf(xv, b, acc2[m]);
          }
      }
    }
    for (int e = p.row_ptr[n] + lane; e < p.row_ptr[n + 1]; e += 32) {
      const int k = p.pcol[e];
      const float2 wv = __half22float2(p.pw[e]);
#pragma unroll
      for (int m = 0; m < kDualLinMaxM; ++m)
        if (m < p.M) {
          const float xv = __half2float(xs[m * p.K + k]);
          acc1[m] = fmaf(xv, wv.x, acc1[m]);
          acc2[m] = fmaf(xv, wv.y, acc2[m]);
        }
    }
#pragma unroll
    for (int m = 0; m < kDualLinMaxM; ++m) {
      float a = acc1[m], b = acc2[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
      }
      if (lane == 0 && m < p.M) {
        p.y1[m * p.ldy + n] = __float2half_rn(a);
        p.y2[m * p.ldy + n] = __float2half_rn(b);
      }
    }
  }
}

int check_stream(const uint8_t* codes, const void* scales, int64_t chunk, int64_t group, int phase_bits) {
  if (!codes || !scales || chunk <= 0 || group <= 0 || phase_bits < 1 || phase_bits > 15) {
    set_error("dual stream: codes and scales must be set, chunk and group sizes positive, 1 <= phase_bits <= 15");
    return PP_ERR_INVALID;
  }
  return PP_OK;
}

}  // namespace
}  // namespace pp

extern "C" {

int pp_dual_unpack(const uint8_t* codes, const void* scales, int64_t chunk_size, int64_t group_size, int phase_bits,
                   const double* amp_norm, const double* cos_t, const double* sin_t, const uint32_t* plug_idx,
                   const void* plug_vals, int64_t n_plugs, uint32_t base_lo32, int64_t start, int64_t n, float* w1,
                   float* w2, void* h1, void* h2, void* stream) {
  int rc = pp::check_stream(codes, scales, chunk_size, group_size, phase_bits);
  if (rc) return rc;
  if (!amp_norm || !cos_t || !sin_t || start < 0 || n < 0 || n_plugs < 0 || (n_plugs > 0 && (!plug_idx || !plug_vals))) {
    pp::set_error("pp_dual_unpack: tables must be set, start, n and n_plugs non-negative, plugs set when counted");
    return PP_ERR_INVALID;
  }
  if (n == 0) return PP_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  pp::UnpackParams p{{codes, reinterpret_cast<const __half*>(scales), chunk_size, group_size, phase_bits},
                     amp_norm, cos_t, sin_t, start, n, w1, w2,
                     reinterpret_cast<__half*>(h1), reinterpret_cast<__half*>(h2)};
  const int64_t blocks = pp::cdiv(n, 256) < 4096 ? pp::cdiv(n, 256) : 4096;
  pp::dual_unpack_kernel<<<(unsigned)blocks, 256, 0, s>>>(p);
  if ((rc = pp::check_launch("dual_unpack_kernel"))) return rc;
  if (n_plugs == 0) return PP_OK;
  pp::PlugParams q{codes, phase_bits, cos_t, sin_t, plug_idx, reinterpret_cast<const __half*>(plug_vals), n_plugs,
                   base_lo32, start, n, w1, w2, reinterpret_cast<__half*>(h1), reinterpret_cast<__half*>(h2)};
  const int64_t pb = pp::cdiv(n_plugs, 256) < 4096 ? pp::cdiv(n_plugs, 256) : 4096;
  pp::dual_unpack_plugs_kernel<<<(unsigned)pb, 256, 0, s>>>(q);
  return pp::check_launch("dual_unpack_plugs_kernel");
}

int pp_dual_file_linear(const uint8_t* codes, const void* scales, int64_t chunk_size, int64_t group_size,
                        int phase_bits, const float* amp_norm, const void* cos_sin, int64_t offset,
                        const int* row_ptr, const int* plug_col, const void* plug_w, const void* x, int64_t ldx,
                        int64_t M, int64_t N, int64_t K, void* y1, void* y2, int64_t ldy, void* stream) {
  int rc = pp::check_stream(codes, scales, chunk_size, group_size, phase_bits);
  if (rc) return rc;
  if (chunk_size % 8 || group_size % 8) {
    pp::set_error("pp_dual_file_linear: chunk and group sizes must be multiples of 8 (one group per 16-byte word)");
    return PP_ERR_INVALID;
  }
  if (!amp_norm || !cos_sin || !row_ptr || !x || !y1 || !y2 || offset < 0 || M < 0 || N < 0 || K < 0 ||
      M > pp::kDualLinMaxM || N > INT32_MAX || K > INT32_MAX || ldx < K || ldy < N || !pp::aligned(codes, 16) ||
      !pp::aligned(cos_sin, 8)) {
    pp::set_error("pp_dual_file_linear: tables, plug rows, x and outputs must be set; 0 <= M <= %d; "
                  "16-byte aligned codes", pp::kDualLinMaxM);
    return PP_ERR_INVALID;
  }
  if (M == 0 || N == 0) return PP_OK;
  const int amp_n = 1 << (16 - phase_bits), table_n = 1 << phase_bits;
  const size_t smem = (size_t)amp_n * 4 + (size_t)table_n * 8 + (size_t)M * K * 2;
  int dev_max = 0;
  cudaDeviceGetAttribute(&dev_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, pp::current_device());
  if (smem > (size_t)dev_max) {
    pp::set_error("pp_dual_file_linear: tables and x need %zu bytes of shared memory, more than %d", smem, dev_max);
    return PP_ERR_INVALID;
  }
  cudaFuncSetAttribute(pp::dual_file_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  pp::LinParams p{};
  p.s = {codes, reinterpret_cast<const __half*>(scales), chunk_size, group_size, phase_bits};
  p.amp_norm = amp_norm;
  p.cs = reinterpret_cast<const float2*>(cos_sin);
  p.table_n = table_n;
  p.amp_n = amp_n;
  p.offset = offset;
  p.x = reinterpret_cast<const __half*>(x);
  p.ldx = ldx;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.row_ptr = row_ptr;
  p.pcol = plug_col;
  p.pw = reinterpret_cast<const __half2*>(plug_w);
  p.y1 = reinterpret_cast<__half*>(y1);
  p.y2 = reinterpret_cast<__half*>(y2);
  p.ldy = ldy;
  const int sms = pp::device_sm_count(pp::current_device());
  const int64_t want = pp::cdiv(N, pp::kDualLinWarps);
  const int64_t grid = want < (int64_t)(sms > 0 ? sms : 148) * 4 ? want : (int64_t)(sms > 0 ? sms : 148) * 4;
  pp::dual_file_linear_kernel<<<(unsigned)grid, pp::kDualLinWarps * 32, smem,
                                reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return pp::check_launch("dual_file_linear_kernel");
}

}  // extern "C"
