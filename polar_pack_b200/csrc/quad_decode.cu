// Quad-pack decode-only kernels: FP16 weight restore and plug-table indexing.
//
//  * quad_decode_kernel  -- (R, C) codes -> four (R, C) FP16 matrices with the
//    same replicated shared-memory tables and FP16 chain as the GEMV.
//  * quad_plug_scatter   -- overwrite plugged positions with the plug table's
//    FP16 4-tuples (optionally scaled), the in-memory merge of
//    quaternion_packer.py:187-193.
//  * quad_plug_windows / quad_plug_zero -- load-time preparation of a
//    Linear's plug table for the fused kernel: index of the first plug of
//    every (row, 64-column window), and the norm byte of plugged codes set to
//    zero so that they decode to exact zeros in the main loop.
//  * unit_plug_size / unit_plug_scan / unit_plug_fill -- load-time copy of
//    a Linear's plug table in unit-major order (one segment per 8-row x
//    64-column work unit), which the GEMV streams beside the codes.
#include "pp_common.cuh"
#include "pp_host.h"

namespace pp {

struct QuadDecodeParams {
  const uint32_t* codes;
  int64_t ldc_r, ldc_c, R, C;
  const __half* luts[7];
  float scale[4];
  int scaled;
  __half* out[4];
  int64_t ldo_r, ldo_c;
};

__global__ void __launch_bounds__(512, 1) quad_decode_kernel(const QuadDecodeParams p) {
  // tables at the first 64 KiB boundary of the window (the host requests
  // 64 KiB of slack), table stage right after them
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(pp_smem);
  const uint32_t lut_saddr = (base + 0xFFFFu) & ~0xFFFFu;
  uint8_t* lut = pp_smem + (lut_saddr - base);
  build_quad_lut(lut, reinterpret_cast<uint32_t*>(lut + kQuadLutBytes), p.luts);
  __syncthreads();
  const uint32_t lb0 = lut_saddr | ((threadIdx.x & 31) * 4u);
  const uint32_t lb1 = (lut_saddr + 65536u) | ((threadIdx.x & 31) * 4u);
  const int64_t total = p.R * p.C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / p.C, c = i - r * p.C;
    const uint32_t code = __ldg(p.codes + r * p.ldc_r + c * p.ldc_c);
    const QuadDec d = decode_quad<true>(code, lb0, lb1, 0u, 0u);
    __half w[4] = {__low2half(u2h(d.p1)), __low2half(u2h(d.p2)), __low2half(u2h(d.p3)),
                   __high2half(u2h(d.p3))};
    const int64_t o = r * p.ldo_r + c * p.ldo_c;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half v = w[k];
      if (p.scaled) v = __float2half_rn(__half2float(v) * p.scale[k]);
      p.out[k][o] = v;
    }
  }
}

struct QuadScatterParams {
  const uint32_t* plug_idx;
  const uint2* plug_vals;
  int64_t p_lo, p_hi, n;
  uint32_t base;
  float scale[4];
  int scaled;
  __half* out[4];
};

__global__ void quad_plug_scatter(const QuadScatterParams p) {
  for (int64_t j = p.p_lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < p.p_hi;
       j += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t loc = __ldg(p.plug_idx + j) - p.base;
    if ((int64_t)loc >= p.n) continue;
    const uint2 v = __ldg(p.plug_vals + j);
    const uint16_t h[4] = {(uint16_t)(v.x & 0xFFFF), (uint16_t)(v.x >> 16), (uint16_t)(v.y & 0xFFFF),
                           (uint16_t)(v.y >> 16)};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half x = __ushort_as_half(h[k]);
      if (p.scaled) x = __float2half_rn(__half2float(x) * p.scale[k]);
      p.out[k][loc] = x;
    }
  }
}

__global__ void fill_zero_u32(uint32_t* p, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = 0u;
}

struct PlugPrepParams {
  uint32_t* codes;  // the Linear's (N, K) codes, row stride ldw
  int64_t ldw;
  const uint32_t* plug_idx;
  int64_t p_lo, p_hi;
  uint32_t base;
  int64_t N, K, W;
  uint32_t* wbase;  // [N*W + 1]
  int* bad;
};

// wbase[w] = number of plug entries of this Linear whose position is below
// the start of window w = (row, win): row*K + 64*win; wbase[N*W] = P.
// Lower bound by binary search over the (ascending) slice.
__global__ void quad_plug_windows_kernel(const PlugPrepParams p) {
  const int64_t nw = p.N * p.W;
  const int64_t P = p.p_hi - p.p_lo;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w <= nw;
       w += (int64_t)gridDim.x * blockDim.x) {
    uint64_t target;
    if (w == nw) {
      target = (uint64_t)p.N * (uint64_t)p.K;
    } else {
      const int64_t row = w / p.W, win = w - row * p.W;
      target = (uint64_t)row * (uint64_t)p.K + (uint64_t)win * 64u;
    }
    int64_t lo = 0, hi = P;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      const uint64_t loc = (uint32_t)(__ldg(p.plug_idx + p.p_lo + mid) - p.base);
      if (loc < target) lo = mid + 1;
      else hi = mid;
    }
    p.wbase[w] = (uint32_t)lo;
  }
}

// Zero the norm byte of every plugged code (it then decodes to exact zeros)
// and count entries that are out of range or out of order.
__global__ void quad_plug_zero_kernel(const PlugPrepParams p) {
  const uint64_t span = (uint64_t)p.N * (uint64_t)p.K;
  for (int64_t j = p.p_lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < p.p_hi;
       j += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t loc = __ldg(p.plug_idx + j) - p.base;
    bool ok = (uint64_t)loc < span;
    if (ok && j > p.p_lo) {
      const uint32_t prev = __ldg(p.plug_idx + j - 1) - p.base;
      if ((uint64_t)prev < span && prev >= loc) ok = false;
    }
    if (!ok) {
      if (p.bad) atomicAdd(p.bad, 1);
      continue;
    }
    const uint64_t row = loc / (uint64_t)p.K, k = loc % (uint64_t)p.K;
    p.codes[row * p.ldw + k] &= 0x00FFFFFFu;
  }
}

namespace {
bool g_decode_attr[64];
int g_decode_limit[64];

int grid_for(int64_t n, int threads) {
  const int64_t b = cdiv(n, threads);
  return (int)(b < 65535 ? (b > 0 ? b : 1) : 65535);
}
}  // namespace

static int quad_decode_impl(const uint32_t* codes, int64_t ldc_r, int64_t ldc_c, int64_t R, int64_t C,
                            const void* const luts[7], const float* scales, void* const out[4],
                            int64_t ldo_r, int64_t ldo_c, cudaStream_t s) {
  if (R < 0 || C < 0 || !luts || !out) {
    set_error("invalid arguments to quad decode");
    return PP_ERR_INVALID;
  }
  if (R == 0 || C == 0) return PP_OK;
  if (!codes) {
    set_error("codes is NULL");
    return PP_ERR_INVALID;
  }
  QuadDecodeParams prm{};
  prm.codes = codes;
  prm.ldc_r = ldc_r;
  prm.ldc_c = ldc_c;
  prm.R = R;
  prm.C = C;
  for (int i = 0; i < 7; ++i) {
    if (!luts[i]) {
      set_error("luts[%d] is NULL", i);
      return PP_ERR_INVALID;
    }
    prm.luts[i] = reinterpret_cast<const __half*>(luts[i]);
  }
  for (int i = 0; i < 4; ++i) {
    if (!out[i]) {
      set_error("out[%d] is NULL", i);
      return PP_ERR_INVALID;
    }
    prm.out[i] = reinterpret_cast<__half*>(out[i]);
    prm.scale[i] = scales ? scales[i] : 1.f;
  }
  prm.scaled = scales ? 1 : 0;
  prm.ldo_r = ldo_r;
  prm.ldo_c = ldo_c;
  constexpr int smem = (int)kQuadLutBytes + 65536 + 4096;
  int max_smem = 0;
  int rc = ensure_smem_attr(quad_decode_kernel, g_decode_attr, g_decode_limit, &max_smem);
  if (rc) return rc;
  const int sms = device_sm_count(current_device());
  const int64_t want = cdiv(R * C, 512);
  const int grid = (int)(want < sms ? want : sms);
  quad_decode_kernel<<<grid > 0 ? grid : 1, 512, smem, s>>>(prm);
  return check_launch("quad_decode_kernel");
}

}  // namespace pp

namespace pp {

// The 128 KiB shared-memory image of the replicated quad tables (the same
// bytes quad_lut_fanout writes): thread i writes 16-byte chunk i.
struct QuadLutPtrs {
  const __half* luts[7];
};

__global__ void __launch_bounds__(256) quad_prepare_tables_kernel(const QuadLutPtrs p, uint8_t* tables) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= 4 * 256 * 8) return;
  const int t = idx >> 11, e = (idx >> 3) & 255, part = idx & 7;
  const uint32_t w = quad_table_word(p.luts, t, e);
  *reinterpret_cast<uint4*>(tables + lut_off(t) + (uint32_t)e * 256u + (uint32_t)part * 16u) = make_uint4(w, w, w, w);
}

}  // namespace pp

extern "C" {

int pp_quad_tables_bytes(size_t* bytes) {
  if (!bytes) {
    pp::set_error("bytes must not be NULL");
    return PP_ERR_INVALID;
  }
  *bytes = pp::kQuadLutBytes;
  return PP_OK;
}

int pp_quad_prepare_tables(const void* const luts[7], void* tables, void* stream) {
  if (!luts || !tables || !pp::aligned(tables, 16)) {
    pp::set_error("luts and a 16-byte aligned tables buffer are required");
    return PP_ERR_INVALID;
  }
  pp::QuadLutPtrs prm{};
  for (int i = 0; i < 7; ++i) {
    if (!luts[i]) {
      pp::set_error("luts[%d] is NULL", i);
      return PP_ERR_INVALID;
    }
    prm.luts[i] = reinterpret_cast<const __half*>(luts[i]);
  }
  pp::quad_prepare_tables_kernel<<<32, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      prm, reinterpret_cast<uint8_t*>(tables));
  return pp::check_launch("quad_prepare_tables_kernel");
}

int pp_quad_decode(const uint32_t* codes, int64_t ldc_r, int64_t ldc_c, int64_t R, int64_t C,
                   const void* const luts[7], const float* scales, void* const out[4], int64_t ldo_r,
                   int64_t ldo_c, void* stream) {
  return pp::quad_decode_impl(codes, ldc_r, ldc_c, R, C, luts, scales, out, ldo_r, ldo_c,
                              reinterpret_cast<cudaStream_t>(stream));
}

int pp_quad_unpack(const uint32_t* codes, int64_t n, const uint32_t* plug_idx, const void* plug_vals,
                   int64_t p_lo, int64_t p_hi, uint32_t base_lo32, const void* const luts[7],
                   const float* scales, void* const out[4], void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n < 0 || p_lo < 0 || p_hi < p_lo) {
    pp::set_error("invalid arguments to quad unpack");
    return PP_ERR_INVALID;
  }
  int rc = pp::quad_decode_impl(codes, 0, 1, 1, n, luts, scales, out, 0, 1, s);
  if (rc) return rc;
  if (p_hi == p_lo || n == 0) return PP_OK;
  if (!plug_idx || !plug_vals || !pp::aligned(plug_vals, 8)) {
    pp::set_error("plug_idx / plug_vals missing or plug_vals not 8-byte aligned");
    return PP_ERR_INVALID;
  }
  pp::QuadScatterParams sp{};
  sp.plug_idx = plug_idx;
  sp.plug_vals = reinterpret_cast<const uint2*>(plug_vals);
  sp.p_lo = p_lo;
  sp.p_hi = p_hi;
  sp.n = n;
  sp.base = base_lo32;
  for (int i = 0; i < 4; ++i) {
    sp.out[i] = reinterpret_cast<__half*>(out[i]);
    sp.scale[i] = scales ? scales[i] : 1.f;
  }
  sp.scaled = scales ? 1 : 0;
  pp::quad_plug_scatter<<<pp::grid_for(p_hi - p_lo, 256), 256, 0, s>>>(sp);
  return pp::check_launch("quad_plug_scatter");
}

int pp_quad_prepare_plugs(uint32_t* codes, int64_t ldw, const uint32_t* plug_idx, int64_t p_lo, int64_t p_hi,
                          uint32_t base_lo32, int64_t N, int64_t K, uint32_t* plug_window_base, int* bad_count,
                          void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (N < 0 || K <= 0 || p_lo < 0 || p_hi < p_lo || ldw < K || !plug_window_base || (N > 0 && !codes)) {
    pp::set_error("invalid arguments to quad prepare plugs");
    return PP_ERR_INVALID;
  }
  if (p_hi > p_lo && !plug_idx) {
    pp::set_error("plug_idx is NULL");
    return PP_ERR_INVALID;
  }
  const int64_t W = pp::cdiv(K, 64);
  pp::PlugPrepParams prm{codes, ldw, plug_idx, p_lo, p_hi, base_lo32, N, K, W, plug_window_base, bad_count};
  pp::quad_plug_windows_kernel<<<pp::grid_for(N * W + 1, 256), 256, 0, s>>>(prm);
  int rc = pp::check_launch("quad_plug_windows_kernel");
  if (rc || p_hi == p_lo) return rc;
  pp::quad_plug_zero_kernel<<<pp::grid_for(p_hi - p_lo, 256), 256, 0, s>>>(prm);
  return pp::check_launch("quad_plug_zero_kernel");
}

}  // extern "C"

namespace pp {

// Plug-table correction of one file-layout Linear, as a CSR sparse product:
//   corr[q][m][n] = sum over plug entries j of row n of  pv_j[q] * x[m][k_j]
// (FP32).  The fused kernel decodes plugged codes to exact zeros (their norm
// byte was cleared by pp_quad_prepare_plugs) and adds corr before the
// per-model scale and the FP16 store, so the result equals the product with
// the plug values substituted, up to FP32 summation order.  The warp sums
// lane totals in a fixed butterfly order, so results are deterministic.
struct PlugCorrParams {
  const __half* x;
  int64_t ldx_m;
  const uint32_t* plug_idx;  // this Linear's slice
  const uint2* plug_vals;
  const uint32_t* wbase;     // [N*W + 1]
  uint32_t base_lo32;
  int M, N, K, W;
  float* corr;               // corr[q * ldq + m * N + n]
  int64_t ldq;               // model stride of corr (M * N for a dense [4][M][N] buffer)
  __half* xt;                // M > 1: scratch for x transposed, K x 128 halves
};  // (declared identically in quad_gemv.cu)

// A warp owns RPW consecutive rows, whose entries are one contiguous range
// of the sorted plug table; lanes take every 32nd entry, U per lane in
// flight.  Two rows per warp when rows are short halves the warps, so the
// largest layers fit one wave; long rows keep one row per warp.
template <int MB, int RPW, int U>
__global__ void __launch_bounds__(256) quad_plug_corr_kernel(const PlugCorrParams p) {
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
  const int nrows = row0 < p.N ? (p.N - row0 < RPW ? p.N - row0 : RPW) : 0;
  if (nrows == 0) {
    pdl_wait();
    return;
  }
  // row pointers: lane r holds the first entry of row row0 + r (r <= nrows)
  uint32_t rp = 0u;
  if (lane <= nrows) rp = __ldg(p.wbase + (int64_t)(row0 + lane) * p.W);
  uint32_t rs[RPW + 1];
#pragma unroll
  for (int r = 0; r <= RPW; ++r) rs[r] = __shfl_sync(0xffffffffu, rp, r <= nrows ? r : nrows);
  const uint32_t j0 = rs[0], j1 = rs[nrows];
  float acc[RPW][MB][4];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[r][m][q] = 0.f;
  for (uint32_t jb = j0; jb < j1; jb += 32u * U) {
    // the plug arrays are weights: loads of a batch are issued before the wait
    uint32_t kk[U];
    uint2 vv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = jb + (uint32_t)lane + 32u * u;
      kk[u] = 0u;
      vv[u] = make_uint2(0u, 0u);
      if (j < j1) {
        kk[u] = __ldg(p.plug_idx + j);
        vv[u] = __ldg(p.plug_vals + j);
      }
    }
    pdl_wait();  // activations may come from the previous kernel
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t j = jb + (uint32_t)lane + 32u * u;
      if (j >= j1) continue;
      const float pv[4] = {__half2float(__ushort_as_half((uint16_t)(vv[u].x & 0xFFFF))),
                           __half2float(__ushort_as_half((uint16_t)(vv[u].x >> 16))),
                           __half2float(__ushort_as_half((uint16_t)(vv[u].y & 0xFFFF))),
                           __half2float(__ushort_as_half((uint16_t)(vv[u].y >> 16)))};
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        if (RPW == 1 || (j >= rs[r] && j < rs[r + 1])) {
          const uint32_t k = kk[u] - (p.base_lo32 + (uint32_t)(row0 + r) * (uint32_t)p.K);
#pragma unroll
          for (int m = 0; m < MB; ++m) {
            if (m < p.M) {
              const float xv = __half2float(p.x[(int64_t)m * p.ldx_m + k]);
#pragma unroll
              for (int q = 0; q < 4; ++q) acc[r][m][q] = fmaf(pv[q], xv, acc[r][m][q]);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v = acc[r][m][q];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m][q] = v;
      }
  pdl_wait();  // the previous kernel may still read the correction buffer
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < RPW; ++r)
      if (r < nrows)
#pragma unroll
        for (int m = 0; m < MB; ++m)
          if (m < p.M)
#pragma unroll
            for (int q = 0; q < 4; ++q) p.corr[(int64_t)q * p.ldq + (int64_t)m * p.N + row0 + r] = acc[r][m][q];
  }
}

// Batched rows (M > 1): the correction is a sparse (N x K) times dense
// (K x M) product.  x is first transposed into scratch, xt[k * ldt + m], so
// the M activations of one plug column are one contiguous row.  WPR warps
// share a row, each a contiguous range of its entries.  A warp loads 32
// entries at a time (lane l entry l, one coalesced load; the next 32 are
// loaded before the current ones are used) and hands them out by shuffle:
// its lanes form EG = 32 / MPAD groups of MPAD lanes, lane l of a group
// holding the FP16 pairs of batch rows 2l + {0, 1} + 64 i (i < MPL), and
// group g takes the entries g, g + EG, ...  A lane issues the activation
// loads (one 4-byte pair per row pair) of up to 16 / MPL entries before it
// uses the first, and applies an entry with eight FP16 x FP16 + FP32 FMAs
// per row pair (the product is exact, one rounding, as fmaf on the
// converted values).  The row's warps are summed in warp order through
// shared memory and the groups in a fixed butterfly, so results are
// deterministic.
//
// The transpose: a CTA takes 64 columns k of all M rows (coalesced row
// reads into shared memory) and writes their xt rows (coalesced along m).
__global__ void __launch_bounds__(256) transpose_x_kernel(const __half* x, int64_t ldx_m, int M, int K, __half* xt,
                                                          int ldt) {
  __shared__ uint16_t tile[128][66];  // [m][k], M <= 128
  pdl_launch_dependents();
  pdl_wait();  // activations may come from the previous kernel
  const int k0 = blockIdx.x * 64, kl = threadIdx.x & 63;
  const uint16_t* xs = reinterpret_cast<const uint16_t*>(x);
  for (int m = threadIdx.x >> 6; m < M; m += 4)
    tile[m][kl] = k0 + kl < K ? xs[(int64_t)m * ldx_m + k0 + kl] : (uint16_t)0;
  __syncthreads();
  uint16_t* xo = reinterpret_cast<uint16_t*>(xt);
  const int kn = K - k0 < 64 ? K - k0 : 64;
  for (int i = threadIdx.x; i < kn * M; i += 256) {
    const int k = i / M, m = i - k * M;
    xo[(int64_t)(k0 + k) * ldt + m] = tile[m][k];
  }
}

// acc[q] += value q * x.lo, acc[4 + q] += value q * x.hi: FP16 operands,
// FP32 accumulation
__device__ __forceinline__ void corr_fma8(float (&acc)[8], uint32_t v01, uint32_t v23, uint32_t xpair) {
  asm("{\n .reg .f16 v0, v1, v2, v3, xl, xh;\n"
      " mov.b32 {v0, v1}, %8;\n mov.b32 {v2, v3}, %9;\n mov.b32 {xl, xh}, %10;\n"
      " fma.rn.f32.f16 %0, v0, xl, %0;\n fma.rn.f32.f16 %1, v1, xl, %1;\n"
      " fma.rn.f32.f16 %2, v2, xl, %2;\n fma.rn.f32.f16 %3, v3, xl, %3;\n"
      " fma.rn.f32.f16 %4, v0, xh, %4;\n fma.rn.f32.f16 %5, v1, xh, %5;\n"
      " fma.rn.f32.f16 %6, v2, xh, %6;\n fma.rn.f32.f16 %7, v3, xh, %7;\n}"
      : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
        "+f"(acc[7])
      : "r"(v01), "r"(v23), "r"(xpair));
}

template <int MPAD, int MPL, int WPR>
__global__ void __launch_bounds__(256) quad_plug_corr_t_kernel(const PlugCorrParams p, int ldt) {
  constexpr int EG = 32 / MPAD, RPC = 8 / WPR;
  constexpr int EPL = MPAD;                                 // entries per lane group and chunk
  constexpr int BATCH = EPL < 16 / MPL ? EPL : 16 / MPL;    // activation loads in flight per lane
  __shared__ float red[8][MPL][8][32];
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, eg = lane / MPAD, ml = lane % MPAD;
  const int row = blockIdx.x * RPC + warp / WPR, wr = warp % WPR;
  const int ldp = ldt / 2;  // row pairs per xt row
  const uint32_t* xs = reinterpret_cast<const uint32_t*>(p.xt) + ml;
  float acc[MPL][8];
#pragma unroll
  for (int i = 0; i < MPL; ++i)
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[i][q] = 0.f;
  if (row < p.N) {
    const uint32_t j0 = __ldg(p.wbase + (int64_t)row * p.W), j1 = __ldg(p.wbase + (int64_t)(row + 1) * p.W);
    const uint32_t a = j0 + (uint32_t)((uint64_t)(j1 - j0) * wr / WPR);
    const uint32_t b = j0 + (uint32_t)((uint64_t)(j1 - j0) * (wr + 1) / WPR);
    const uint32_t rowbase = p.base_lo32 + (uint32_t)row * (uint32_t)p.K;
    // entry a + lane of the first chunk; past the range: zero values, column 0
    uint32_t nk = 0u;
    uint2 nv = make_uint2(0u, 0u);
    if (a + (uint32_t)lane < b) {
      nk = __ldg(p.plug_idx + a + lane) - rowbase;
      nv = __ldg(p.plug_vals + a + lane);
    }
    pdl_wait();  // xt is written by the transpose launched just before
    for (uint32_t jb = a; jb < b; jb += 32u) {
      const uint32_t kk = nk;
      const uint2 vv = nv;
      const uint32_t jn = jb + 32u + (uint32_t)lane;
      nk = 0u;
      nv = make_uint2(0u, 0u);
      if (jn < b) {
        nk = __ldg(p.plug_idx + jn) - rowbase;
        nv = __ldg(p.plug_vals + jn);
      }
#pragma unroll
      for (int e0 = 0; e0 < EPL; e0 += BATCH) {
        uint32_t kb[BATCH], xw[BATCH][MPL];
#pragma unroll
        for (int t = 0; t < BATCH; ++t) kb[t] = __shfl_sync(0xffffffffu, kk, (e0 + t) * EG + eg);
#pragma unroll
        for (int t = 0; t < BATCH; ++t)
#pragma unroll
          for (int i = 0; i < MPL; ++i) xw[t][i] = __ldg(xs + kb[t] * (uint32_t)ldp + 32 * i);
#pragma unroll
        for (int t = 0; t < BATCH; ++t) {
          const int src = (e0 + t) * EG + eg;
          const uint32_t v01 = __shfl_sync(0xffffffffu, vv.x, src), v23 = __shfl_sync(0xffffffffu, vv.y, src);
#pragma unroll
          for (int i = 0; i < MPL; ++i) corr_fma8(acc[i], v01, v23, xw[t][i]);
        }
      }
    }
  } else {
    pdl_wait();
  }
  if (WPR > 1) {
#pragma unroll
    for (int i = 0; i < MPL; ++i)
#pragma unroll
      for (int q = 0; q < 8; ++q) red[warp][i][q][lane] = acc[i][q];
    __syncthreads();
    if (wr != 0) return;
#pragma unroll
    for (int i = 0; i < MPL; ++i)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float v = red[warp][i][q][lane];
#pragma unroll
        for (int w = 1; w < WPR; ++w) v += red[warp + w][i][q][lane];
        acc[i][q] = v;
      }
  }
#pragma unroll
  for (int o = MPAD; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < MPL; ++i)
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[i][q] += __shfl_xor_sync(0xffffffffu, acc[i][q], o);
  if (eg != 0 || row >= p.N) return;
#pragma unroll
  for (int i = 0; i < MPL; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = 64 * i + 2 * ml + h;
      if (m < p.M)
#pragma unroll
        for (int q = 0; q < 4; ++q) p.corr[(int64_t)q * p.ldq + (int64_t)m * p.N + row] = acc[i][4 * h + q];
    }
}

// Warps per row for about 64 entries per warp, 1..8, from the row length:
// the packer caps plugs at 5% of the codes, so a row holds about K / 20.
// (The count itself lives on the device; the choice only affects speed.)
template <int MPAD, int MPL>
int launch_corr_t(const PlugCorrParams& prm, cudaStream_t s) {
  const int ldt = 2 * MPAD * MPL;
  int rc = launch_kernel("transpose_x_kernel", launch_overlap(), transpose_x_kernel,
                         dim3((unsigned)cdiv(prm.K, 64)), dim3(256), 0, s, prm.x, prm.ldx_m, prm.M, prm.K, prm.xt,
                         ldt);
  if (rc) return rc;
  const int64_t per_row = prm.K / 20;
  const bool ov = launch_overlap();
  if (per_row >= 384)
    return launch_kernel("quad_plug_corr_t_kernel", ov, quad_plug_corr_t_kernel<MPAD, MPL, 8>,
                         dim3((unsigned)prm.N), dim3(256), 0, s, prm, ldt);
  if (per_row >= 192)
    return launch_kernel("quad_plug_corr_t_kernel", ov, quad_plug_corr_t_kernel<MPAD, MPL, 4>,
                         dim3((unsigned)cdiv(prm.N, 2)), dim3(256), 0, s, prm, ldt);
  if (per_row >= 96)
    return launch_kernel("quad_plug_corr_t_kernel", ov, quad_plug_corr_t_kernel<MPAD, MPL, 2>,
                         dim3((unsigned)cdiv(prm.N, 4)), dim3(256), 0, s, prm, ldt);
  return launch_kernel("quad_plug_corr_t_kernel", ov, quad_plug_corr_t_kernel<MPAD, MPL, 1>,
                       dim3((unsigned)cdiv(prm.N, 8)), dim3(256), 0, s, prm, ldt);
}

int launch_plug_corr(const PlugCorrParams& prm, cudaStream_t s) {
  const int warps = 8;
  const bool ov = launch_overlap();
  if (prm.M > 1 && prm.xt) {
    if (prm.M > 128) {
      set_error("plug correction: at most 128 batch rows per launch");
      return PP_ERR_INVALID;
    }
    // MPAD lanes of row pairs per entry: 2 * MPAD * MPL >= M
    if (prm.M <= 4) return launch_corr_t<2, 1>(prm, s);
    if (prm.M <= 8) return launch_corr_t<4, 1>(prm, s);
    if (prm.M <= 16) return launch_corr_t<8, 1>(prm, s);
    if (prm.M <= 32) return launch_corr_t<16, 1>(prm, s);
    if (prm.M <= 64) return launch_corr_t<32, 1>(prm, s);
    return launch_corr_t<32, 2>(prm, s);
  }
  if (prm.M == 1) {
    if (prm.K <= 4096) {  // short rows: two per warp
      const int grid = (int)cdiv(prm.N, warps * 2);
      return launch_kernel("quad_plug_corr_kernel", ov, quad_plug_corr_kernel<1, 2, 8>, dim3(grid), dim3(warps * 32),
                           0, s, prm);
    }
    const int grid = (int)cdiv(prm.N, warps);
    return launch_kernel("quad_plug_corr_kernel", ov, quad_plug_corr_kernel<1, 1, 8>, dim3(grid), dim3(warps * 32),
                         0, s, prm);
  }
  const int grid = (int)cdiv(prm.N, warps);
  if (prm.M <= 8)
    return launch_kernel("quad_plug_corr_kernel", ov, quad_plug_corr_kernel<8, 1, 4>, dim3(grid), dim3(warps * 32), 0,
                         s, prm);
  return launch_kernel("quad_plug_corr_kernel", ov, quad_plug_corr_kernel<16, 1, 4>, dim3(grid), dim3(warps * 32), 0,
                       s, prm);
}

}  // namespace pp

// ------------------------------------------------------------ unit plugs --
// Unit-major plug stream of one file-layout Linear (N, K) for the fused
// correction of quad_gemv.cu.  Unit u = t * W + kc (W = ceil(K / 64))
// covers rows 8t..8t+7 and columns 64kc..64kc+63.  Its segment starts at
// byte off[u], a multiple of 16, and holds its n plug entries in table
// order (row-major, k ascending):
//   bytes [0, 32)          eight u32, one per tile row r:
//                          start_r | end_r << 10 | n << 20
//                          (entries [start_r, end_r) belong to row 8t + r)
//   bytes [32, 32 + 8n)    the entries' FP16x4 values (as in plug_vals)
//   bytes [32 + 8n, 32+9n) the entries' columns k - 64kc
// then zeros up to the next multiple of 16.  off[U] = total bytes.  One
// 32-bit read gives a lane its row's range and the segment's size.
namespace pp {

struct UnitPlugParams {
  const uint32_t* plug_idx;  // this Linear's slice
  const uint2* plug_vals;
  const uint32_t* wbase;     // [N*W + 1] (quad_plug_windows_kernel)
  uint32_t base;
  int64_t N, K, W, U;
  uint8_t* out;
  uint32_t* off;             // [U + 1]
};

__host__ __device__ inline uint32_t unit_plug_seg_bytes(uint32_t n) { return (32u + 9u * n + 15u) & ~15u; }

__global__ void unit_plug_size_kernel(const UnitPlugParams p) {
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u <= p.U; u += (int64_t)gridDim.x * blockDim.x) {
    if (u == p.U) {
      p.off[u] = 0u;
      continue;
    }
    const int64_t t = u / p.W, kc = u - t * p.W;
    uint32_t n = 0;
    for (int r = 0; r < 8; ++r) {
      const int64_t row = 8 * t + r;
      if (row < p.N) n += __ldg(p.wbase + row * p.W + kc + 1) - __ldg(p.wbase + row * p.W + kc);
    }
    p.off[u] = unit_plug_seg_bytes(n);
  }
}

// In-place exclusive scan of off[0..n) by one CTA of 1024 threads, each
// owning a contiguous chunk.
__global__ void __launch_bounds__(1024) unit_plug_scan_kernel(uint32_t* off, int64_t n) {
  __shared__ uint32_t part[1024];
  const int tid = threadIdx.x;
  const int64_t chunk = (n + 1023) / 1024;
  const int64_t i0 = tid * chunk < n ? tid * chunk : n, i1 = i0 + chunk < n ? i0 + chunk : n;
  uint32_t sum = 0;
  for (int64_t i = i0; i < i1; ++i) sum += off[i];
  part[tid] = sum;
  __syncthreads();
  for (int d = 1; d < 1024; d <<= 1) {  // Hillis-Steele inclusive scan
    const uint32_t v = tid >= d ? part[tid - d] : 0u;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  uint32_t run = part[tid] - sum;
  for (int64_t i = i0; i < i1; ++i) {
    const uint32_t v = off[i];
    off[i] = run;
    run += v;
  }
}

// One warp per unit: lanes 0..7 own the tile rows (their entry ranges),
// then all lanes copy each row's entries.
__global__ void unit_plug_fill_kernel(const UnitPlugParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t u = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); u < p.U; u += nwarps) {
    const int64_t t = u / p.W, kc = u - t * p.W;
    const int64_t row = 8 * t + lane;
    uint32_t a = 0, cnt = 0;
    if (lane < 8 && row < p.N) {
      a = __ldg(p.wbase + row * p.W + kc);
      cnt = __ldg(p.wbase + row * p.W + kc + 1) - a;
    }
    uint32_t h = cnt;  // inclusive scan over lanes 0..7
#pragma unroll
    for (int d = 1; d < 8; d <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, h, d);
      if (lane >= d) h += v;
    }
    const uint32_t n = __shfl_sync(0xffffffffu, h, 7);
    uint8_t* seg = p.out + __ldg(p.off + u);
    const uint32_t len = __ldg(p.off + u + 1) - __ldg(p.off + u);
    if (lane < 8) reinterpret_cast<uint32_t*>(seg)[lane] = (h - cnt) | (h << 10) | (n << 20);
    for (int r = 0; r < 8; ++r) {
      const uint32_t ar = __shfl_sync(0xffffffffu, a, r);
      const uint32_t cr = __shfl_sync(0xffffffffu, cnt, r);
      const uint32_t e0 = __shfl_sync(0xffffffffu, h, r) - cr;
      const uint32_t rowbase = p.base + (uint32_t)(8 * t + r) * (uint32_t)p.K + (uint32_t)(64 * kc);
      for (uint32_t j = lane; j < cr; j += 32) {
        const uint32_t e = e0 + j;
        reinterpret_cast<uint2*>(seg + 32)[e] = __ldg(p.plug_vals + ar + j);
        seg[32 + 8 * n + e] = (uint8_t)(__ldg(p.plug_idx + ar + j) - rowbase);
      }
    }
    for (uint32_t b = 32 + 9 * n + lane; b < len; b += 32) seg[b] = 0;
  }
}

}  // namespace pp

extern "C" {

int pp_quad_unit_plugs_bytes(int64_t N, int64_t K, int64_t n_plugs, size_t* stream_bytes, int64_t* n_offsets) {
  if (N < 0 || K < 0 || n_plugs < 0 || !stream_bytes || !n_offsets) {
    pp::set_error("invalid arguments to quad unit plugs bytes");
    return PP_ERR_INVALID;
  }
  const int64_t U = pp::cdiv(N, 8) * pp::cdiv(K, 64);
  // a segment takes at most 32 + 9n + 15 bytes
  *stream_bytes = pp::align_up((size_t)U * 47u + (size_t)n_plugs * 9u, 256);
  *n_offsets = U + 1;
  return PP_OK;
}

int pp_quad_prepare_unit_plugs(const uint32_t* plug_idx, const void* plug_vals, int64_t n_plugs, uint32_t base_lo32,
                               const uint32_t* plug_window_base, int64_t N, int64_t K, void* unit_plugs,
                               size_t unit_plugs_bytes, uint32_t* unit_plug_off, void* stream) {
  size_t need = 0;
  int64_t noff = 0;
  int rc = pp_quad_unit_plugs_bytes(N, K, n_plugs, &need, &noff);
  if (rc) return rc;
  if (N == 0 || K == 0) {
    pp::set_error("empty Linear");
    return PP_ERR_INVALID;
  }
  if (!plug_window_base || !unit_plugs || !unit_plug_off || (n_plugs > 0 && (!plug_idx || !plug_vals)) ||
      !pp::aligned(unit_plugs, 16) || !pp::aligned(unit_plug_off, 4) || (plug_vals && !pp::aligned(plug_vals, 8))) {
    pp::set_error("unit plugs: NULL or misaligned pointer (stream 16-byte, values 8-byte aligned)");
    return PP_ERR_INVALID;
  }
  if (unit_plugs_bytes < need) {
    pp::set_error("unit plug stream of %zu bytes required, got %zu", need, unit_plugs_bytes);
    return PP_ERR_WORKSPACE;
  }
  if (need > 0xFFFFFFF0ull) {
    pp::set_error("unit plug stream above 4 GiB (32-bit offsets)");
    return PP_ERR_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t W = pp::cdiv(K, 64);
  pp::UnitPlugParams prm{plug_idx, reinterpret_cast<const uint2*>(plug_vals), plug_window_base, base_lo32, N, K,
                         W, noff - 1, reinterpret_cast<uint8_t*>(unit_plugs), unit_plug_off};
  pp::unit_plug_size_kernel<<<pp::grid_for(noff, 256), 256, 0, s>>>(prm);
  if ((rc = pp::check_launch("unit_plug_size_kernel"))) return rc;
  pp::unit_plug_scan_kernel<<<1, 1024, 0, s>>>(unit_plug_off, noff);
  if ((rc = pp::check_launch("unit_plug_scan_kernel"))) return rc;
  pp::unit_plug_fill_kernel<<<pp::grid_for((noff - 1) * 32, 256), 256, 0, s>>>(prm);
  return pp::check_launch("unit_plug_fill_kernel");
}

}  // extern "C"
