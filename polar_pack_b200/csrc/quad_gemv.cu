// Quad-pack fused dequant GEMV/GEMM for batch <= 16 on sm_100a.
//
// One HBM pass over the uint32 codes feeds four matrix products (one per
// packed model).  Per code: one 128-bit streaming load (shared by 4 codes),
// four conflict-free shared-memory table reads, three FP16x2 multiplies
// (the reference's FP16 chain), two byte permutes into tensor-core
// fragments.  The dot products run on mma.sync m16n8k16 with FP32
// accumulators: A = decoded weights (rows 0-7 model j, rows 8-15 model
// j+1 of eight output features), B = activations (columns = batch rows).
//
// Two code layouts have fast paths:
//   NK ("file" layout, K contiguous): a work unit is 8 rows x 64 columns;
//      lane (g, c) owns row g, columns 16*s + 4*c + {0..3}, s = 0..3.
//   KN (kernel layout (K, N), N contiguous): a unit is 16 k x 32 features;
//      lane (g, c) owns features 4*g + {0..3} of rows 2c, 2c+1, 2c+8, 2c+9.
// The logical K order inside one mma is a permutation of the physical
// order; the activation fragment uses the same permutation.
//
// Work partition and the deterministic split-K reduction: pp_engine.cuh.
#include "pp_common.cuh"
#include "pp_engine.cuh"
#include "pp_host.h"

namespace pp {

int zero_f16(void* p, int64_t R, int64_t C, int64_t ldr, int64_t ldc, cudaStream_t s);

// Warps per CTA: the KN tile keeps 4x more accumulators per lane, so it
// trades warps for registers (NB = number of 8-row batch tiles).
__host__ __device__ constexpr int quad_warps(bool nk, int nb) { return nk ? 16 : (nb == 1 ? 12 : 8); }

struct QuadParams {
  const __half* x;
  int64_t ldx_m, ldx_k;
  const uint32_t* codes;
  int64_t ldc;  // NK: stride between rows n; KN: stride between rows k
  const __half* luts[7];
  float scale[4];
  __half* out[4];
  int64_t ldo_m, ldo_n;
  int M, N, K;
  // plug tables (NK only)
  const uint2* plug_vals;
  const unsigned long long* pmask;
  const uint32_t* pbase;
  int W;
  Partition part;
  int xvec;
};

struct QuadBuf {
  uint4 q[4];
};

template <bool NK, int NB, bool PLUG>
struct QuadOp {
  static constexpr int kWarps = quad_warps(NK, NB);
  static constexpr int kTileW = NK ? 8 : 32;  // output features per tile
  static constexpr int kT = NK ? 1 : 4;       // mma pairs per 16-k step
  static constexpr int kNOut = 4;
  static constexpr int kNBat = 8 * NB;
  static constexpr int kSlot = kNOut * kNBat * kTileW;
  using Buf = QuadBuf;

  const QuadParams& p;
  const uint8_t* lut;
  int g, c;
  uint32_t laneoff;
  float acc[kT][NB][2][4];

  __device__ __forceinline__ QuadOp(const QuadParams& p_, const uint8_t* lut_)
      : p(p_), lut(lut_), g((threadIdx.x & 31) >> 2), c(threadIdx.x & 3),
        laneoff((threadIdx.x & 31) * 4u) {}

  __device__ __forceinline__ int M() const { return p.M; }
  __device__ __forceinline__ int64_t N() const { return p.N; }

  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int t = 0; t < kT; ++t)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[t][nb][h][j] = 0.f;
  }

  __device__ __forceinline__ void load(Buf& b, int64_t tile, int kc) const {
    if constexpr (NK) {
      const int64_t row = tile * 8 + g;
      const int kb = kc * 64 + 4 * c;
      const uint32_t* base = p.codes + row * p.ldc + kb;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        if (row < p.N && kb + 16 * s < p.K) b.q[s] = ldg_stream(base + 16 * s);
        else b.q[s] = make_uint4(0, 0, 0, 0);
      }
    } else {
      const int64_t f = tile * 32 + 4 * g;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int k = kc * 16 + 2 * c + (r & 1) + 8 * (r >> 1);
        if (f < p.N && k < p.K) b.q[r] = ldg_stream(p.codes + (int64_t)k * p.ldc + f);
        else b.q[r] = make_uint4(0, 0, 0, 0);
      }
    }
  }

  __device__ __forceinline__ uint32_t xpair(int bat, int k) const {
    // activations (bat, k) and (bat, k+1) as one half2 word, zero outside
    if (bat >= p.M) return 0u;
    const __half* row = p.x + (int64_t)bat * p.ldx_m;
    if (p.xvec && k + 1 < p.K) return ldg_u32(row + k);
    uint32_t lo = 0, hi = 0;
    if (k < p.K) lo = ldg_u16(row + (int64_t)k * p.ldx_k);
    if (k + 1 < p.K) hi = ldg_u16(row + (int64_t)(k + 1) * p.ldx_k);
    return lo | (hi << 16);
  }

  __device__ __forceinline__ uint2 xquad(int bat, int k) const {
    // activations (bat, k..k+3); the NK path guarantees K % 4 == 0
    if (bat >= p.M || k >= p.K) return make_uint2(0u, 0u);
    const __half* row = p.x + (int64_t)bat * p.ldx_m;
    if (p.xvec) return ldg_u2(row + k);
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = ldg_u16(row + (int64_t)(k + i) * p.ldx_k);
    return make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
  }

  __device__ __forceinline__ void compute(const Buf& b, int64_t tile, int kc) {
    if constexpr (NK) {
      const int kbase = kc * 64;
      const int64_t row = tile * 8 + g;
      unsigned long long pm = 0ull;
      uint32_t pb = 0u;
      if constexpr (PLUG) {
        if (row < p.N) {
          const int64_t wi = row * p.W + kc;
          pm = __ldg(p.pmask + wi);
          if (pm) pb = __ldg(p.pbase + wi);
        }
      }
      const bool full_k = kbase + 64 <= p.K;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int kp = kbase + 16 * s + 4 * c;
        QuadDec d[4];
        d[0] = decode_quad(b.q[s].x, lut, laneoff);
        d[1] = decode_quad(b.q[s].y, lut, laneoff);
        d[2] = decode_quad(b.q[s].z, lut, laneoff);
        d[3] = decode_quad(b.q[s].w, lut, laneoff);
        if constexpr (PLUG) {
          const uint32_t nib = (uint32_t)(pm >> (16 * s + 4 * c)) & 0xFu;
          if (nib) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if ((nib >> e) & 1u) {
                const int bit = 16 * s + 4 * c + e;
                const uint32_t j = pb + (uint32_t)__popcll(pm & ((1ull << bit) - 1ull));
                const uint2 v = __ldg(p.plug_vals + j);
                d[e].p1 = v.x;        // low half = model 0
                d[e].p2 = v.x >> 16;  // low half = model 1
                d[e].p3 = v.y;        // (model 2, model 3)
              }
            }
          }
        }
        uint32_t a01[4] = {lo_pair(d[0].p1, d[1].p1), lo_pair(d[0].p2, d[1].p2),
                           lo_pair(d[2].p1, d[3].p1), lo_pair(d[2].p2, d[3].p2)};
        uint32_t a23[4] = {lo_pair(d[0].p3, d[1].p3), hi_pair(d[0].p3, d[1].p3),
                           lo_pair(d[2].p3, d[3].p3), hi_pair(d[2].p3, d[3].p3)};
        if (!full_k && kp >= p.K) {
#pragma unroll
          for (int i = 0; i < 4; ++i) a01[i] = a23[i] = 0u;
        }
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const uint2 xb = xquad(nb * 8 + g, kp);
          mma_16816(acc[0][nb][0], a01[0], a01[1], a01[2], a01[3], xb.x, xb.y);
          mma_16816(acc[0][nb][1], a23[0], a23[1], a23[2], a23[3], xb.x, xb.y);
        }
      }
    } else {
      const int kbase = kc * 16;
      const bool full_k = kbase + 16 <= p.K;
      uint32_t b0[NB], b1[NB];
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        b0[nb] = xpair(nb * 8 + g, kbase + 2 * c);
        b1[nb] = xpair(nb * 8 + g, kbase + 2 * c + 8);
      }
      bool rv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) rv[r] = full_k || (kbase + 2 * c + (r & 1) + 8 * (r >> 1) < p.K);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        QuadDec d[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint32_t code = t == 0 ? b.q[r].x : t == 1 ? b.q[r].y : t == 2 ? b.q[r].z : b.q[r].w;
          d[r] = decode_quad(code, lut, laneoff);
          if (!rv[r]) d[r] = QuadDec{0u, 0u, 0u};
        }
        const uint32_t a01[4] = {lo_pair(d[0].p1, d[1].p1), lo_pair(d[0].p2, d[1].p2),
                                 lo_pair(d[2].p1, d[3].p1), lo_pair(d[2].p2, d[3].p2)};
        const uint32_t a23[4] = {lo_pair(d[0].p3, d[1].p3), hi_pair(d[0].p3, d[1].p3),
                                 lo_pair(d[2].p3, d[3].p3), hi_pair(d[2].p3, d[3].p3)};
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          mma_16816(acc[t][nb][0], a01[0], a01[1], a01[2], a01[3], b0[nb], b1[nb]);
          mma_16816(acc[t][nb][1], a23[0], a23[1], a23[2], a23[3], b0[nb], b1[nb]);
        }
      }
    }
  }

  // Fragment register j of mma half h: model 2h + (j>>1), batch 8nb+2c+(j&1);
  // feature-in-tile g (NK) or 4g + t (KN).
  __device__ __forceinline__ void write_partial(float* red) const {
#pragma unroll
    for (int t = 0; t < kT; ++t) {
      const int fi = NK ? g : 4 * g + t;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int model = 2 * h + (j >> 1);
            const int bat = nb * 8 + 2 * c + (j & 1);
            red[(model * kNBat + bat) * kTileW + fi] = acc[t][nb][h][j];
          }
    }
  }

  __device__ __forceinline__ void store(int model, int bat, int64_t f, float v) const {
    p.out[model][(int64_t)bat * p.ldo_m + f * p.ldo_n] = __float2half_rn(v * p.scale[model]);
  }
};

template <bool NK, int NB, bool PLUG>
constexpr int quad_red_bytes() {
  return QuadOp<NK, NB, PLUG>::kWarps * QuadOp<NK, NB, PLUG>::kSlot * 4;
}

template <bool NK, int NB, bool PLUG>
__global__ void __launch_bounds__(quad_warps(NK, NB) * 32, 1) quad_gemv_kernel(const QuadParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ int s_flag;
  float* red = reinterpret_cast<float*>(smem + kQuadLutBytes);
  build_quad_lut(smem, reinterpret_cast<uint32_t*>(red), p.luts);
  __syncthreads();
  QuadOp<NK, NB, PLUG> op(p, smem);
  run_partition(op, p.part, red, &s_flag);
}

// Generic fallback for layouts the vector paths do not take (unaligned or
// strided codes).  One thread per (feature, batch row); plain table reads.
struct QuadGenericParams {
  const __half* x;
  int64_t ldx_m, ldx_k;
  const uint32_t* codes;
  int64_t ldc_k, ldc_n;
  const __half* luts[7];
  float scale[4];
  __half* out[4];
  int64_t ldo_m, ldo_n;
  int64_t M, N, K;
};

__global__ void quad_generic_kernel(const QuadGenericParams p) {
  __shared__ uint32_t tab[4][256];
  for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
    const int t = i >> 8, e = i & 255;
    uint32_t v;
    if (t == 0) {
      const uint32_t r = ldg_u16(reinterpret_cast<const uint16_t*>(p.luts[0]) + e);
      v = r | (r << 16);
    } else {
      v = (uint32_t)ldg_u16(reinterpret_cast<const uint16_t*>(p.luts[2 * t - 1]) + e) |
          ((uint32_t)ldg_u16(reinterpret_cast<const uint16_t*>(p.luts[2 * t]) + e) << 16);
    }
    tab[t][e] = v;
  }
  __syncthreads();
  const int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t m = blockIdx.y;
  if (n >= p.N || m >= p.M) return;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t k = 0; k < p.K; ++k) {
    const uint32_t code = p.codes[k * p.ldc_k + n * p.ldc_n];
    const __half2 p1 = __hmul2_rn(u2h(tab[0][code >> 24]), u2h(tab[1][(code >> 16) & 255]));
    const __half2 p2 = __hmul2_rn(__high2half2(p1), u2h(tab[2][(code >> 8) & 255]));
    const __half2 p3 = __hmul2_rn(__high2half2(p2), u2h(tab[3][code & 255]));
    const float xv = __half2float(p.x[m * p.ldx_m + k * p.ldx_k]);
    acc[0] = fmaf(xv, __low2float(p1), acc[0]);
    acc[1] = fmaf(xv, __low2float(p2), acc[1]);
    acc[2] = fmaf(xv, __low2float(p3), acc[2]);
    acc[3] = fmaf(xv, __high2float(p3), acc[3]);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) p.out[k][m * p.ldo_m + n * p.ldo_n] = __float2half_rn(acc[k] * p.scale[k]);
}

// ------------------------------------------------------------------ host --
namespace {

PartitionPlan quad_plan(bool nk, int64_t Mc, int64_t N, int64_t K, int sms) {
  const int nb = Mc > 8 ? 2 : 1;
  const int tile_w = nk ? 8 : 32, unit_k = nk ? 64 : 16;
  return plan_partition(cdiv(N, tile_w), cdiv(K, unit_k), quad_warps(nk, nb), sms, 4, Mc, tile_w);
}

bool g_attr_done[6][64];

template <bool NK, int NB, bool PLUG>
int launch_quad(const QuadParams& prm, int grid, int idx, cudaStream_t s) {
  auto kern = quad_gemv_kernel<NK, NB, PLUG>;
  constexpr int smem = (int)kQuadLutBytes + quad_red_bytes<NK, NB, PLUG>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  int rc = ensure_smem_attr(kern, smem, g_attr_done[idx]);
  if (rc) return rc;
  kern<<<grid, quad_warps(NK, NB) * 32, smem, s>>>(prm);
  return check_launch("quad_gemv_kernel");
}

int launch_plan(const PartitionPlan& pl, bool nk, int nb, QuadParams prm, void* ws, bool plug,
                cudaStream_t s) {
  prm.part.units = pl.units;
  prm.part.upt = (int)pl.upt;
  prm.part.counters = reinterpret_cast<int*>(ws);
  prm.part.slots = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + pl.counters_bytes);
  if (nk) {
    if (plug) return nb == 1 ? launch_quad<true, 1, true>(prm, pl.grid, 0, s)
                             : launch_quad<true, 2, true>(prm, pl.grid, 1, s);
    return nb == 1 ? launch_quad<true, 1, false>(prm, pl.grid, 2, s) : launch_quad<true, 2, false>(prm, pl.grid, 3, s);
  }
  return nb == 1 ? launch_quad<false, 1, false>(prm, pl.grid, 4, s) : launch_quad<false, 2, false>(prm, pl.grid, 5, s);
}

bool quad_vector_ok(bool nk, const uint32_t* codes, int64_t ldc_k, int64_t ldc_n, int64_t N, int64_t K) {
  if (!aligned(codes, 16)) return false;
  if (nk) return ldc_k == 1 && ldc_n % 4 == 0 && K % 4 == 0 && ldc_n >= K;
  return ldc_n == 1 && ldc_k % 4 == 0 && N % 4 == 0 && ldc_k >= N;
}

int check_common(const void* const luts[7], const float scales[4], void* const out[4], int64_t M,
                 int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) {
    set_error("negative shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
    return PP_ERR_INVALID;
  }
  if (N > INT32_MAX || K > INT32_MAX) {
    set_error("N and K must fit in 32 bits");
    return PP_ERR_INVALID;
  }
  if (!luts || !scales || !out) {
    set_error("luts, scales and out must not be NULL");
    return PP_ERR_INVALID;
  }
  for (int i = 0; i < 7; ++i)
    if (!luts[i]) {
      set_error("luts[%d] is NULL", i);
      return PP_ERR_INVALID;
    }
  for (int i = 0; i < 4; ++i)
    if (!out[i] && M > 0 && N > 0) {
      set_error("out[%d] is NULL", i);
      return PP_ERR_INVALID;
    }
  return PP_OK;
}

size_t quad_ws_bytes(bool nk, int64_t M, int64_t N, int64_t K) {
  const int sms = device_sm_count(current_device());
  const int64_t Mc = M < 16 ? M : 16;
  if (Mc <= 0) return 0;
  return quad_plan(nk, Mc, N, K, sms > 0 ? sms : 148).total();
}

}  // namespace

static int quad_run(const void* a, int64_t lda_m, int64_t lda_k, const uint32_t* codes, int64_t ldc_k,
                    int64_t ldc_n, const void* plug_vals, const uint64_t* pmask, const uint32_t* pbase,
                    const void* const luts[7], const float scales[4], void* const out[4], int64_t ldo_m,
                    int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* ws, size_t ws_bytes,
                    cudaStream_t s, bool file_layout) {
  int rc = check_common(luts, scales, out, M, N, K);
  if (rc) return rc;
  if (M == 0 || N == 0) return PP_OK;
  if (K == 0) {
    for (int i = 0; i < 4; ++i)
      if ((rc = zero_f16(out[i], M, N, ldo_m, ldo_n, s))) return rc;
    return PP_OK;
  }
  if (!a || !codes) {
    set_error("a and codes must not be NULL");
    return PP_ERR_INVALID;
  }
  const bool plug = file_layout && plug_vals != nullptr;
  if (plug && (!pmask || !pbase || !aligned(plug_vals, 8))) {
    set_error("plug_mask/plug_base missing or plug_vals not 8-byte aligned");
    return PP_ERR_INVALID;
  }
  const bool nk = file_layout || (ldc_k == 1 && ldc_n != 1);
  const bool vec = quad_vector_ok(nk, codes, ldc_k, ldc_n, N, K);
  if (!vec) {
    if (plug) {
      set_error("file-layout codes need 16-byte alignment, K %% 4 == 0 and row stride %% 4 == 0");
      return PP_ERR_INVALID;
    }
    QuadGenericParams g{};
    g.x = reinterpret_cast<const __half*>(a);
    g.ldx_m = lda_m;
    g.ldx_k = lda_k;
    g.codes = codes;
    g.ldc_k = ldc_k;
    g.ldc_n = ldc_n;
    for (int i = 0; i < 7; ++i) g.luts[i] = reinterpret_cast<const __half*>(luts[i]);
    for (int i = 0; i < 4; ++i) {
      g.scale[i] = scales[i];
      g.out[i] = reinterpret_cast<__half*>(out[i]);
    }
    g.ldo_m = ldo_m;
    g.ldo_n = ldo_n;
    g.M = M;
    g.N = N;
    g.K = K;
    for (int64_t m0 = 0; m0 < M; m0 += 65535) {
      QuadGenericParams gg = g;
      gg.x += m0 * lda_m;
      for (int i = 0; i < 4; ++i) gg.out[i] += m0 * ldo_m;
      gg.M = (M - m0) < 65535 ? (M - m0) : 65535;
      dim3 grid((unsigned)cdiv(N, 128), (unsigned)gg.M);
      quad_generic_kernel<<<grid, 128, 0, s>>>(gg);
      if ((rc = check_launch("quad_generic_kernel"))) return rc;
    }
    return PP_OK;
  }
  const int sms = device_sm_count(current_device());
  if (sms <= 0) {
    set_error("cannot query the SM count of the current device");
    return PP_ERR_CUDA;
  }
  QuadParams prm{};
  prm.ldx_m = lda_m;
  prm.ldx_k = lda_k;
  prm.codes = codes;
  prm.ldc = nk ? ldc_n : ldc_k;
  for (int i = 0; i < 7; ++i) prm.luts[i] = reinterpret_cast<const __half*>(luts[i]);
  for (int i = 0; i < 4; ++i) prm.scale[i] = scales[i];
  prm.ldo_m = ldo_m;
  prm.ldo_n = ldo_n;
  prm.N = (int)N;
  prm.K = (int)K;
  prm.plug_vals = reinterpret_cast<const uint2*>(plug_vals);
  prm.pmask = reinterpret_cast<const unsigned long long*>(pmask);
  prm.pbase = pbase;
  prm.W = (int)cdiv(K, 64);
  const size_t need = quad_plan(nk, M < 16 ? M : 16, N, K, sms).total();
  if (ws_bytes < need || (need && !ws) || !aligned(ws, 256)) {
    set_error("workspace of %zu bytes (256-byte aligned, zero-filled) required, got %zu", need, ws_bytes);
    return PP_ERR_WORKSPACE;
  }
  // batch rows in chunks of 16: each chunk is one launch over the codes
  for (int64_t m0 = 0; m0 < M; m0 += 16) {
    const int64_t Mc = (M - m0) < 16 ? (M - m0) : 16;
    const PartitionPlan pl = quad_plan(nk, Mc, N, K, sms);
    prm.x = reinterpret_cast<const __half*>(a) + m0 * lda_m;
    for (int i = 0; i < 4; ++i) prm.out[i] = reinterpret_cast<__half*>(out[i]) + m0 * ldo_m;
    prm.M = (int)Mc;
    const int xalign = nk ? 8 : 4;
    prm.xvec = (lda_k == 1 && aligned(prm.x, xalign) && (lda_m * 2) % xalign == 0) ? 1 : 0;
    if ((rc = launch_plan(pl, nk, Mc > 8 ? 2 : 1, prm, ws, plug, s))) return rc;
  }
  return PP_OK;
}

}  // namespace pp

extern "C" {

int pp_quad_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t ldc_k, int64_t ldc_n,
                                 size_t* bytes) {
  if (!bytes || M < 0 || N < 0 || K < 0) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  const bool nk = ldc_k == 1 && ldc_n != 1;
  *bytes = pp::quad_ws_bytes(nk, M, N, K);
  return PP_OK;
}

int pp_quad_gemm(const void* a, int64_t lda_m, int64_t lda_k, const uint32_t* codes, int64_t ldc_k,
                 int64_t ldc_n, const void* const luts[7], const float scales[4], void* const out[4],
                 int64_t ldo_m, int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* workspace,
                 size_t workspace_bytes, void* stream) {
  return pp::quad_run(a, lda_m, lda_k, codes, ldc_k, ldc_n, nullptr, nullptr, nullptr, luts, scales, out,
                      ldo_m, ldo_n, M, N, K, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream), false);
}

int pp_quad_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, size_t* bytes) {
  if (!bytes || M < 0 || N < 0 || K < 0) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  *bytes = pp::quad_ws_bytes(true, M, N, K);
  return PP_OK;
}

int pp_quad_linear(const void* x, int64_t ldx_m, int64_t ldx_k, const uint32_t* codes, int64_t ldw,
                   const void* plug_vals, const uint64_t* plug_mask, const uint32_t* plug_base,
                   const void* const luts[7], const float scales[4], void* const out[4], int64_t ldo_m,
                   int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                   void* stream) {
  return pp::quad_run(x, ldx_m, ldx_k, codes, 1, ldw, plug_vals, plug_mask, plug_base, luts, scales, out,
                      ldo_m, ldo_n, M, N, K, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream), true);
}

}  // extern "C"
