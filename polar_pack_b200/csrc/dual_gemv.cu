// Dual-pack (2 models, 16-bit polar codes) fused dequant GEMV/GEMM, sm_100a.
//
// Kernel layout (K, N) int16, N contiguous.  A work unit is 16 k x 64
// features: lane (g, c) loads 8 codes (128 bits) of features 8g..8g+7 for
// rows 2c, 2c+1, 2c+8, 2c+9.  Per code: two conflict-free shared-memory
// table reads (FP32 amplitude level, half2 (cos, sin)), one FP32 product
// with the group scale and two with cos / sin -- the reference's rounding
// points -- then one cvt packs two FP32 weights into an FP16 pair that is
// directly an mma fragment register.  One m16n8k16 per feature column
// carries both models (rows 0-7 model 1, rows 8-15 model 2).
//
// Work partition and the deterministic split-K reduction: pp_engine.cuh.
#include "pp_common.cuh"
#include "pp_engine.cuh"
#include "pp_host.h"

namespace pp {

int zero_f16(void* p, int64_t R, int64_t C, int64_t ldr, int64_t ldc, cudaStream_t s);

// dual_tma.cu: batch 1 on the TMA engine
bool dual_tma_ok(int64_t M, int64_t N, int64_t K, int64_t gs, const void* x, int64_t ldx_k, const int16_t* codes,
                 int64_t ldp_k, int64_t ldp_n, const void* bmax);
int launch_dual_tma(const void* x, const int16_t* codes, int64_t ldp_k, const void* bmax, const void* amp_lut,
                    const void* cos_lut, const void* sin_lut, void* out1, void* out2, int64_t ldo_n, int64_t N,
                    int64_t K, void* ws, size_t ws_bytes, int sms, cudaStream_t s);

// Warps per CTA, bounded by shared memory: 136 KiB of tables plus two
// partial slots per warp.
__host__ __device__ constexpr int dual_warps(int nb) { return nb == 1 ? 10 : 5; }

struct DualParams {
  const __half* x;
  int64_t ldx_m, ldx_k;
  const int16_t* codes;
  int64_t ldc;  // stride between rows k
  const __half* bmax;
  int gs;
  const __half *amp_lut, *cos_lut, *sin_lut;
  __half* out[2];
  int64_t ldo_m, ldo_n;
  int M, N, K;
  Partition part;
  int xvec;
};

struct DualBuf {
  uint4 q[4];
  float sc[4];
};

template <int NB>
struct DualOp {
  static constexpr int kWarps = dual_warps(NB);
  static constexpr int kTileW = 64;
  static constexpr int kNOut = 2;
  static constexpr int kNBat = 8 * NB;
  using Buf = DualBuf;

  const DualParams& p;
  int g, c;
  uint32_t laneoff;
  int Mv, Nv, Kv;
  int64_t ldc;
  const __half* xrow[NB];  // this lane's activation row per batch tile (clamped)
  bool xok[NB];
  float acc[8][NB][4];

  __device__ __forceinline__ DualOp(const DualParams& p_)
      : p(p_), g((threadIdx.x & 31) >> 2), c(threadIdx.x & 3),
        laneoff((threadIdx.x & 31) * 4u), Mv(p_.M), Nv(p_.N), Kv(p_.K), ldc(p_.ldc) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int bat = nb * 8 + g;
      xok[nb] = bat < Mv;
      xrow[nb] = p.x + (int64_t)(xok[nb] ? bat : 0) * p.ldx_m;
    }
  }

  __device__ __forceinline__ int M() const { return Mv; }
  __device__ __forceinline__ int N() const { return Nv; }

  __device__ __forceinline__ void prefetch(int tile, int kc) const {
    // 16 rows x 128 bytes (64 int16 codes): lane l touches row l & 15, half l >> 4
    const int lane = threadIdx.x & 31;
    const int k = kc * 16 + (lane & 15);
    const int f = tile * 64 + 32 * (lane >> 4);
    if (k < Kv && f < Nv) prefetch_l2(p.codes + (int64_t)k * ldc + f);
  }

  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[t][nb][j] = 0.f;
  }

  __device__ __forceinline__ void load(Buf& b, int tile, int kc) const {
    const int f = tile * 64 + 8 * g;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int k = kc * 16 + 2 * c + (r & 1) + 8 * (r >> 1);
      if (f < Nv && k < Kv) {
        b.q[r] = ldg_stream(p.codes + (int64_t)k * ldc + f);
        b.sc[r] = __half2float(__ushort_as_half(ldg_u16(p.bmax + ((int64_t)k * Nv + f) / p.gs)));
      } else {
        b.q[r] = make_uint4(0, 0, 0, 0);
        b.sc[r] = 0.f;
      }
    }
  }

  __device__ __forceinline__ uint32_t xpair(int nb, int k) const {
    uint32_t v;
    if (k + 1 < Kv) {
      v = ldg_u32(xrow[nb] + k);
    } else {
      v = k < Kv ? (uint32_t)ldg_u16(xrow[nb] + k) : 0u;
    }
    return xok[nb] ? v : 0u;
  }

  // (B1, B2) of the low and high code of word w, FP32, reference rounding
  __device__ __forceinline__ void decode2(uint32_t w, float s, float& b1l, float& b2l, float& b1h,
                                          float& b2h) const {
    const uint32_t al = ((w >> 3) & 0x1F80u) | laneoff;
    const uint32_t ah = ((w >> 19) & 0x1F80u) | laneoff;
    const uint32_t pl = ((w << 7) & 0x1FF80u) | laneoff;
    const uint32_t ph = ((w >> 9) & 0x1FF80u) | laneoff;
    const float ampl = __fmul_rn(*reinterpret_cast<const float*>(pp_smem + al), s);
    const float amph = __fmul_rn(*reinterpret_cast<const float*>(pp_smem + ah), s);
    const __half2 csl = u2h(*reinterpret_cast<const uint32_t*>(pp_smem + kDualAmpBytes + pl));
    const __half2 csh = u2h(*reinterpret_cast<const uint32_t*>(pp_smem + kDualAmpBytes + ph));
    b1l = __fmul_rn(ampl, __low2float(csl));
    b2l = __fmul_rn(ampl, __high2float(csl));
    b1h = __fmul_rn(amph, __low2float(csh));
    b2h = __fmul_rn(amph, __high2float(csh));
  }

  __device__ __forceinline__ void compute(const Buf& b, int tile, int kc) {
    const int kbase = kc * 16;
    uint32_t b0[NB], b1[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      b0[nb] = xpair(nb, kbase + 2 * c);
      b1[nb] = xpair(nb, kbase + 2 * c + 8);
    }
    // rows beyond K: scale 0 gives +-0 weights, activations are 0 there too
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float w1l[4], w2l[4], w1h[4], w2h[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint32_t w = j == 0 ? b.q[r].x : j == 1 ? b.q[r].y : j == 2 ? b.q[r].z : b.q[r].w;
        decode2(w, b.sc[r], w1l[r], w2l[r], w1h[r], w2h[r]);
      }
      // feature t = 2j (low codes) and t = 2j + 1 (high codes)
      const uint32_t al0 = h2u(__floats2half2_rn(w1l[0], w1l[1]));
      const uint32_t al1 = h2u(__floats2half2_rn(w2l[0], w2l[1]));
      const uint32_t al2 = h2u(__floats2half2_rn(w1l[2], w1l[3]));
      const uint32_t al3 = h2u(__floats2half2_rn(w2l[2], w2l[3]));
      const uint32_t ah0 = h2u(__floats2half2_rn(w1h[0], w1h[1]));
      const uint32_t ah1 = h2u(__floats2half2_rn(w2h[0], w2h[1]));
      const uint32_t ah2 = h2u(__floats2half2_rn(w1h[2], w1h[3]));
      const uint32_t ah3 = h2u(__floats2half2_rn(w2h[2], w2h[3]));
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        mma_16816(acc[2 * j][nb], al0, al1, al2, al3, b0[nb], b1[nb]);
        mma_16816(acc[2 * j + 1][nb], ah0, ah1, ah2, ah3, b0[nb], b1[nb]);
      }
    }
  }

  // Fragment register j: model (j >> 1), batch 8nb + 2c + (j & 1), feature 8g + t.
  __device__ __forceinline__ void write_partial(float* slot, int M) const {
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int bat = nb * 8 + 2 * c + (j & 1);
          if (bat < M) slot[((j >> 1) * M + bat) * kTileW + 8 * g + t] = acc[t][nb][j];
        }
  }

  __device__ __forceinline__ void store_tile(int tile) const {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int f = tile * 64 + 8 * g + t;
      if (f >= Nv) continue;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int bat = nb * 8 + 2 * c + (j & 1);
          if (bat < Mv) store(j >> 1, bat, f, acc[t][nb][j]);
        }
    }
  }

  __device__ __forceinline__ void store(int model, int bat, int f, float v) const {
    p.out[model][(int64_t)bat * p.ldo_m + (int64_t)f * p.ldo_n] = __float2half_rn(v);
  }
};

inline size_t dual_smem_bytes(int nb, int64_t M) {
  const size_t r = red_bytes(dual_warps(nb), 2, M, 64);
  return kDualLutBytes + (r > 8192 ? r : 8192);
}

template <int NB>
__global__ void __launch_bounds__(dual_warps(NB) * 32, 1) dual_gemv_kernel(const DualParams p) {
  __shared__ int s_flag;
  float* red = reinterpret_cast<float*>(pp_smem + kDualLutBytes);
  build_dual_lut(pp_smem, reinterpret_cast<uint32_t*>(red), p.amp_lut, p.cos_lut, p.sin_lut);
  __syncthreads();
  DualOp<NB> op(p);
  run_partition(op, p.part, red, &s_flag);
}

// ------------------------------------------------ generic and decode ----
struct DualGenericParams {
  const __half* x;
  int64_t ldx_m, ldx_k;
  const int16_t* codes;
  int64_t ldc_k, ldc_n;
  const __half* bmax;
  int64_t gs;
  const __half *amp_lut, *cos_lut, *sin_lut;
  __half* out[2];
  int64_t ldo_m, ldo_n;  // for decode: (ldo_k, ldo_n)
  int64_t M, N, K;
};

__device__ __forceinline__ void dual_decode_one(const DualGenericParams& p, int64_t k, int64_t n, float& b1,
                                                float& b2) {
  const int32_t u = (int32_t)p.codes[k * p.ldc_k + n * p.ldc_n] + 32768;
  const int aq = (u >> 10) & 63, ph = u & 1023;
  const float amp = __fmul_rn(__half2float(p.amp_lut[aq]), __half2float(p.bmax[(k * p.N + n) / p.gs]));
  b1 = __fmul_rn(amp, __half2float(p.cos_lut[ph]));
  b2 = __fmul_rn(amp, __half2float(p.sin_lut[ph]));
}

__global__ void dual_generic_kernel(const DualGenericParams p) {
  const int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t m = blockIdx.y;
  if (n >= p.N || m >= p.M) return;
  float a1 = 0.f, a2 = 0.f;
  for (int64_t k = 0; k < p.K; ++k) {
    float b1, b2;
    dual_decode_one(p, k, n, b1, b2);
    const float xv = __half2float(p.x[m * p.ldx_m + k * p.ldx_k]);
    a1 = fmaf(xv, __half2float(__float2half_rn(b1)), a1);
    a2 = fmaf(xv, __half2float(__float2half_rn(b2)), a2);
  }
  p.out[0][m * p.ldo_m + n * p.ldo_n] = __float2half_rn(a1);
  p.out[1][m * p.ldo_m + n * p.ldo_n] = __float2half_rn(a2);
}

__global__ void dual_decode_kernel(const DualGenericParams p) {
  const int64_t total = p.K * p.N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = i / p.N, n = i - k * p.N;
    float b1, b2;
    dual_decode_one(p, k, n, b1, b2);
    p.out[0][k * p.ldo_m + n * p.ldo_n] = __float2half_rn(b1);
    p.out[1][k * p.ldo_m + n * p.ldo_n] = __float2half_rn(b2);
  }
}

namespace {

PartitionPlan dual_plan(int64_t Mc, int64_t N, int64_t K, int sms) {
  const int nb = Mc > 8 ? 2 : 1;
  return plan_partition(cdiv(N, 64), cdiv(K, 16), dual_warps(nb), sms, 2, Mc, 64);
}

bool g_dual_attr[2][64];
int g_dual_limit[2][64];

template <int NB>
int launch_dual(const DualParams& prm, int grid, cudaStream_t s) {
  auto kern = dual_gemv_kernel<NB>;
  int max_smem = 0;
  int rc = ensure_smem_attr(kern, g_dual_attr[NB - 1], g_dual_limit[NB - 1], &max_smem);
  if (rc) return rc;
  const size_t smem = dual_smem_bytes(NB, prm.M);
  if (smem > (size_t)max_smem) {
    set_error("shared memory plan of %zu bytes exceeds the per-CTA limit %d", smem, max_smem);
    return PP_ERR_INVALID;
  }
  kern<<<grid, dual_warps(NB) * 32, smem, s>>>(prm);
  return check_launch("dual_gemv_kernel");
}

bool dual_vector_ok(const int16_t* codes, int64_t ldp_k, int64_t ldp_n, int64_t N, int64_t gs) {
  return aligned(codes, 16) && ldp_n == 1 && ldp_k % 8 == 0 && ldp_k >= N && N % 8 == 0 && gs % 8 == 0;
}

}  // namespace

static int dual_run(const void* a, int64_t lda_m, int64_t lda_k, const int16_t* packed, int64_t ldp_k,
                    int64_t ldp_n, const void* bmax, int64_t gs, const void* amp_lut, const void* cos_lut,
                    const void* sin_lut, void* out1, void* out2, int64_t ldo_m, int64_t ldo_n, int64_t M,
                    int64_t N, int64_t K, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (M < 0 || N < 0 || K < 0 || gs <= 0) {
    set_error("invalid shape or group size");
    return PP_ERR_INVALID;
  }
  if (N > INT32_MAX || K > INT32_MAX) {
    set_error("N and K must fit in 32 bits");
    return PP_ERR_INVALID;
  }
  if (M == 0 || N == 0) return PP_OK;
  if (!out1 || !out2) {
    set_error("outputs must not be NULL");
    return PP_ERR_INVALID;
  }
  int rc;
  if (K == 0) {
    if ((rc = zero_f16(out1, M, N, ldo_m, ldo_n, s))) return rc;
    return zero_f16(out2, M, N, ldo_m, ldo_n, s);
  }
  if (!a || !packed || !bmax || !amp_lut || !cos_lut || !sin_lut) {
    set_error("a NULL tensor argument");
    return PP_ERR_INVALID;
  }
  const bool xcontig = lda_k == 1 && aligned(a, 4) && (lda_m * 2) % 4 == 0;
  if (!xcontig || !dual_vector_ok(packed, ldp_k, ldp_n, N, gs)) {
    DualGenericParams g{};
    g.x = reinterpret_cast<const __half*>(a);
    g.ldx_m = lda_m;
    g.ldx_k = lda_k;
    g.codes = packed;
    g.ldc_k = ldp_k;
    g.ldc_n = ldp_n;
    g.bmax = reinterpret_cast<const __half*>(bmax);
    g.gs = gs;
    g.amp_lut = reinterpret_cast<const __half*>(amp_lut);
    g.cos_lut = reinterpret_cast<const __half*>(cos_lut);
    g.sin_lut = reinterpret_cast<const __half*>(sin_lut);
    g.out[0] = reinterpret_cast<__half*>(out1);
    g.out[1] = reinterpret_cast<__half*>(out2);
    g.ldo_m = ldo_m;
    g.ldo_n = ldo_n;
    g.N = N;
    g.K = K;
    for (int64_t m0 = 0; m0 < M; m0 += 65535) {
      DualGenericParams gg = g;
      gg.x += m0 * lda_m;
      gg.out[0] += m0 * ldo_m;
      gg.out[1] += m0 * ldo_m;
      gg.M = (M - m0) < 65535 ? (M - m0) : 65535;
      dim3 grid((unsigned)cdiv(N, 128), (unsigned)gg.M);
      dual_generic_kernel<<<grid, 128, 0, s>>>(gg);
      if ((rc = check_launch("dual_generic_kernel"))) return rc;
    }
    return PP_OK;
  }
  const int sms = device_sm_count(current_device());
  if (sms <= 0) {
    set_error("cannot query the SM count of the current device");
    return PP_ERR_CUDA;
  }
  if (cdiv(N, 64) * cdiv(K, 16) >= (int64_t)INT32_MAX) {
    set_error("matrix too large for one launch (more than 2^31 work units)");
    return PP_ERR_INVALID;
  }
  const size_t need = dual_plan(M < 16 ? M : 16, N, K, sms).total();
  if (ws_bytes < need || (need && !ws) || !aligned(ws, 256)) {
    set_error("workspace of %zu bytes (256-byte aligned, zero-filled) required, got %zu", need, ws_bytes);
    return PP_ERR_WORKSPACE;
  }
  if (dual_tma_ok(M, N, K, gs, a, lda_k, packed, ldp_k, ldp_n, bmax))
    return launch_dual_tma(a, packed, ldp_k, bmax, amp_lut, cos_lut, sin_lut, out1, out2, ldo_n, N, K, ws, ws_bytes,
                           sms, s);
  DualParams prm{};
  prm.ldx_m = lda_m;
  prm.ldx_k = lda_k;
  prm.codes = packed;
  prm.ldc = ldp_k;
  prm.bmax = reinterpret_cast<const __half*>(bmax);
  prm.gs = (int)gs;
  prm.amp_lut = reinterpret_cast<const __half*>(amp_lut);
  prm.cos_lut = reinterpret_cast<const __half*>(cos_lut);
  prm.sin_lut = reinterpret_cast<const __half*>(sin_lut);
  prm.ldo_m = ldo_m;
  prm.ldo_n = ldo_n;
  prm.N = (int)N;
  prm.K = (int)K;
  for (int64_t m0 = 0; m0 < M; m0 += 16) {
    const int64_t Mc = (M - m0) < 16 ? (M - m0) : 16;
    const PartitionPlan pl = dual_plan(Mc, N, K, sms);
    prm.x = reinterpret_cast<const __half*>(a) + m0 * lda_m;
    prm.out[0] = reinterpret_cast<__half*>(out1) + m0 * ldo_m;
    prm.out[1] = reinterpret_cast<__half*>(out2) + m0 * ldo_m;
    prm.M = (int)Mc;
    prm.xvec = 1;
    prm.part.units = (int)pl.units;
    prm.part.upt = (int)pl.upt;
    prm.part.counters = reinterpret_cast<int*>(ws);
    prm.part.slots = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + pl.counters_bytes);
    rc = Mc <= 8 ? launch_dual<1>(prm, pl.grid, s) : launch_dual<2>(prm, pl.grid, s);
    if (rc) return rc;
  }
  return PP_OK;
}

}  // namespace pp

extern "C" {

int pp_dual_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t ldp_k, int64_t ldp_n,
                                 size_t* bytes) {
  (void)ldp_k;
  (void)ldp_n;
  if (!bytes || M < 0 || N < 0 || K < 0) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  const int sms = pp::device_sm_count(pp::current_device());
  const int64_t Mc = M < 16 ? M : 16;
  *bytes = Mc > 0 ? pp::dual_plan(Mc, N, K, sms > 0 ? sms : 148).total() : 0;
  return PP_OK;
}

int pp_dual_gemm(const void* a, int64_t lda_m, int64_t lda_k, const int16_t* packed, int64_t ldp_k,
                 int64_t ldp_n, const void* bmax, int64_t group_size, const void* amp_lut, const void* cos_lut,
                 const void* sin_lut, void* out1, void* out2, int64_t ldo_m, int64_t ldo_n, int64_t M,
                 int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  return pp::dual_run(a, lda_m, lda_k, packed, ldp_k, ldp_n, bmax, group_size, amp_lut, cos_lut, sin_lut,
                      out1, out2, ldo_m, ldo_n, M, N, K, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream));
}

int pp_dual_decode(const int16_t* packed, int64_t ldp_k, int64_t ldp_n, int64_t K, int64_t N,
                   const void* bmax, int64_t group_size, const void* amp_lut, const void* cos_lut,
                   const void* sin_lut, void* out1, void* out2, int64_t ldo_k, int64_t ldo_n, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (K < 0 || N < 0 || group_size <= 0) {
    pp::set_error("invalid arguments to dual decode");
    return PP_ERR_INVALID;
  }
  if (K == 0 || N == 0) return PP_OK;
  if (!packed || !bmax || !amp_lut || !cos_lut || !sin_lut || !out1 || !out2) {
    pp::set_error("a NULL tensor argument");
    return PP_ERR_INVALID;
  }
  pp::DualGenericParams g{};
  g.codes = packed;
  g.ldc_k = ldp_k;
  g.ldc_n = ldp_n;
  g.bmax = reinterpret_cast<const __half*>(bmax);
  g.gs = group_size;
  g.amp_lut = reinterpret_cast<const __half*>(amp_lut);
  g.cos_lut = reinterpret_cast<const __half*>(cos_lut);
  g.sin_lut = reinterpret_cast<const __half*>(sin_lut);
  g.out[0] = reinterpret_cast<__half*>(out1);
  g.out[1] = reinterpret_cast<__half*>(out2);
  g.ldo_m = ldo_k;
  g.ldo_n = ldo_n;
  g.N = N;
  g.K = K;
  const int64_t blocks = pp::cdiv(K * N, 256);
  pp::dual_decode_kernel<<<(int)(blocks < 8192 ? blocks : 8192), 256, 0, s>>>(g);
  return pp::check_launch("dual_decode_kernel");
}

}  // extern "C"
