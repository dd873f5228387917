// Dual-pack (2 models, 16-bit polar codes) fused dequant GEMV at batch 1 on
// the TMA engine of pp_engine.cuh, sm_100a.
//
// Same decode as dual_gemv.cu (two conflict-free table reads per code, the
// group scale, FP32 products at the reference's rounding points, one cvt
// per FP16 pair, one m16n8k16 per feature column carrying both models),
// but each warp streams its units through its own TMA ring like the quad
// kernel.  A unit is 16 rows k x 64 features of int16 codes: 16 rows of
// 128 bytes, one tensor-map box with 128-byte swizzle.  The group scales of
// those rows come by a second tensor map over bmax viewed as (K, N/32):
// a box of 8 groups x 16 rows whose x is rounded down to a multiple of 8
// groups (16 bytes, the TMA alignment rule), landing in a 256-byte side
// slot beside the ring slot on the same mbarrier.  A lane reads its 4
// scales from there by the unit's tile.
//
// Taken for M == 1, group size 32, N % 256 == 0 (16-byte scale rows) and
// 16-byte aligned codes, scales and activations; other shapes run on the
// register engine of dual_gemv.cu.
#include "pp_common.cuh"
#include "pp_engine.cuh"
#include "pp_host.h"

namespace pp {

constexpr int kDualTWarps = 16;
constexpr int kDualTStages = 2;
constexpr uint32_t kDualTUnit = 2048u;  // 16 rows x 128 bytes of codes
constexpr uint32_t kDualTSide = 256u;   // 16 rows x 16 bytes of scales

// shared-memory layout from the dynamic base (1 KiB aligned)
constexpr uint32_t kDualTRing = kDualLutBytes;  // 136 KiB of tables first
constexpr uint32_t kDualTSideOff = kDualTRing + kDualTWarps * kDualTStages * kDualTUnit;
constexpr uint32_t kDualTBars = kDualTSideOff + kDualTWarps * kDualTStages * kDualTSide;
constexpr uint32_t kDualTTables = kDualTBars + kDualTWarps * kDualTStages * 8u;
constexpr uint32_t kDualTScratch = kDualTTables + 512u;
// partial slots: two per warp of 2 models x 64 features (batch 1), which
// also stage the 4352-byte table words before the first barrier
constexpr uint32_t kDualTScratchBytes = kDualTWarps * 2u * 2u * 64u * 4u;
constexpr uint32_t kDualTSmem = kDualTScratch + kDualTScratchBytes;
static_assert(kDualTScratchBytes >= (64 + 1024) * 4, "the scratch stages the table words");
static_assert(kDualTRing % 1024 == 0, "128-byte swizzled boxes need 1 KiB aligned slots");

struct DualTParams {
  CUtensorMap tcodes;  // (N, K) 16-bit view of the codes, box 64 x 16, 128-byte swizzle
  CUtensorMap tscale;  // (N/32, K) FP16 view of bmax, box 8 x 16, no swizzle
  const __half* x;
  const __half *amp_lut, *cos_lut, *sin_lut;
  __half* out[2];
  int64_t ldo_n;
  int N, K;
  Partition part;
  int cta_start[kMaxCtaTable + 1];
};

struct DualTBuf {
  uint4 q[4];
  float sc[4];
};

struct DualTOp {
  static constexpr int kWarps = kDualTWarps;
  static constexpr int kTileW = 64;
  static constexpr int kNOut = 2;
  static constexpr int kNBat = 8;
  static constexpr int kUnitBytes = (int)kDualTUnit;
  static constexpr int kPrefetch = 0;
  static constexpr bool kGather16 = false;
  using Buf = DualTBuf;

  const DualTParams& p;
  int g, c;
  uint32_t laneoff;
  uint32_t roff[4];  // this lane's 16-byte code chunks in a ring slot
  uint32_t ring, sring;  // this warp's ring and side slots
  int Nv, Kv;
  float acc[8][4];

  __device__ __forceinline__ DualTOp(const DualTParams& p_, uint32_t ring_, uint32_t side_)
      : p(p_), g((threadIdx.x & 31) >> 2), c(threadIdx.x & 3), laneoff((threadIdx.x & 31) * 4u), ring(ring_),
        sring(side_), Nv(p_.N), Kv(p_.K) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      // lane (g, c): features 8g..8g+7 (chunk g) of rows 2c, 2c+1, 2c+8, 2c+9
      const int row = 2 * c + (s & 1) + 8 * (s >> 1);
      roff[s] = (uint32_t)(row * 128 + ((g ^ (row & 7)) << 4));
    }
  }

  __device__ __forceinline__ int M() const { return 1; }
  __device__ __forceinline__ int N() const { return Nv; }

  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[t][j] = 0.f;
  }

  // One unit by TMA (one lane): the 16 x 64 code box and the 16 x 8 scale
  // box (x rounded down to 8 groups) on the slot's barrier.
  static __device__ __forceinline__ void issue(const DualTParams& q, uint32_t slot, uint32_t bar, uint32_t sslot,
                                               int tile, int kc) {
    mbar_expect_tx(bar, kDualTUnit + kDualTSide);
    tma_load_2d(slot, &q.tcodes, tile * 64, kc * 16, bar);
    tma_load_2d(sslot, &q.tscale, (tile * 2) & ~7, kc * 16, bar);
  }

  // Codes of ring slot s and the lane's four row scales from its side slot:
  // group 2 (tile mod 4) + (g >> 2) of the 8-group box, rows as the codes.
  __device__ __forceinline__ void read(Buf& b, uint32_t slot, int s, int tile) const {
#pragma unroll
    for (int r = 0; r < 4; ++r) b.q[r] = lds128(slot + roff[r]);
    const uint32_t sb = sring + (uint32_t)s * kDualTSide + 2u * (uint32_t)(2 * (tile & 3) + (g >> 2));
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = 2 * c + (r & 1) + 8 * (r >> 1);
      b.sc[r] = __half2float(__ushort_as_half((uint16_t)lds_u16(sb + 16u * (uint32_t)row)));
    }
  }

  __device__ __forceinline__ void prefetch(int, int) const {}
  __device__ __forceinline__ void side(int, int, int) {}
  __device__ __forceinline__ void end_chunk() {}

  // batch 1: lanes g = 0 feed the activations, the other batch columns are
  // zero; columns k >= K read as zero
  __device__ __forceinline__ uint32_t xpair(int k) const {
    if (g != 0) return 0u;
    if (k + 1 < Kv) return ld_u32(p.x + k);
    return k < Kv ? (uint32_t)ld_u16(p.x + k) : 0u;
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

  // rows beyond K arrive with code and scale 0 (zero weights)
  __device__ __forceinline__ void compute(const Buf& b, int, int kc) {
    const int kbase = kc * 16;
    const uint32_t b0 = xpair(kbase + 2 * c), b1 = xpair(kbase + 2 * c + 8);
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
      mma_16816(acc[2 * j], al0, al1, al2, al3, b0, b1);
      mma_16816(acc[2 * j + 1], ah0, ah1, ah2, ah3, b0, b1);
    }
  }

  // Fragment register j: model (j >> 1), batch column 2c + (j & 1), feature 8g + t.
  __device__ __forceinline__ void write_partial(float* slot, int) const {
    if (c != 0) return;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      slot[0 * kTileW + 8 * g + t] = acc[t][0];
      slot[1 * kTileW + 8 * g + t] = acc[t][2];
    }
  }

  __device__ __forceinline__ void store_tile(int tile) const {
    if (c != 0) return;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int f = tile * 64 + 8 * g + t;
      if (f >= Nv) continue;
      store(0, 0, f, acc[t][0]);
      store(1, 0, f, acc[t][2]);
    }
  }

  __device__ __forceinline__ void store(int model, int, int f, float v) const {
    p.out[model][(int64_t)f * p.ldo_n] = __float2half_rn(v);
  }
  __device__ __forceinline__ float corr_at(int, int, int) const { return 0.f; }
  __device__ __forceinline__ void store_raw(int model, int bat, int f, float v) const { store(model, bat, f, v); }
};

// Table words are staged and the per-CTA tables filled before the first
// barrier; then lane 0 of every warp initialises its ring and issues its
// first units, whose copies overlap the table fan-out; after the second
// barrier every warp streams and reduces on its own.
__global__ void __launch_bounds__(kDualTWarps * 32, 1) dual_tma_kernel(const __grid_constant__ DualTParams p) {
  constexpr int NW = kDualTWarps;
  if (threadIdx.x == 0) {  // the first copies need the tensor maps
    prefetch_tmap(&p.tcodes);
    prefetch_tmap(&p.tscale);
  }
  pdl_launch_dependents();
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(pp_smem);
  int* status = p.part.counters + (kMaxGrid - 1);
  const int cu0 = p.cta_start[blockIdx.x], cu1 = p.cta_start[blockIdx.x + 1];
  if (cu0 >= cu1) return;  // uniform over the CTA
  Partition pt = p.part;
  pt.cta_start = p.cta_start;
  pt.cta = blockIdx.x;
  pt.ncta = gridDim.x;
  int* ti = reinterpret_cast<int*>(pp_smem + kDualTTables);
  const CtaTables tb{ti, ti + (NW + 1), ti + 2 * (NW + 1)};
  cta_tables_init<NW>(tb, cu0, cu1, p.part.upt);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wu0 = warp_start<NW>(cu0, cu1, warp), wu1 = warp_start<NW>(cu0, cu1, warp + 1);
  const uint32_t ring = base + kDualTRing + (uint32_t)warp * kDualTStages * kDualTUnit;
  const uint32_t side = base + kDualTSideOff + (uint32_t)warp * kDualTStages * kDualTSide;
  TmaRing rg;
  if (wu0 < wu1) {
    rg.ring = ring;
    rg.bars = base + kDualTBars + 8u * (uint32_t)(warp * kDualTStages);
    rg.S = kDualTStages;
    rg.P = kDualTStages;  // side slot i belongs to ring slot i
    rg.next.init(wu0, wu1, p.part.upt);
  }
  uint32_t* stage = reinterpret_cast<uint32_t*>(pp_smem + kDualTScratch);
  dual_lut_stage(stage, p.amp_lut, p.cos_lut, p.sin_lut);
  __syncthreads();
  auto issue = [&](uint32_t slot, uint32_t bar, int sp, int tile, int kc) {
    DualTOp::issue(p, slot, bar, side + (uint32_t)sp * kDualTSide, tile, kc);
  };
  if (wu0 < wu1 && lane == 0) {
    rg.prologue(issue, kDualTUnit);
  }
  dual_lut_fanout(pp_smem, stage);
  __syncthreads();  // tables complete; the stage is free for the partial slots
  // everything above reads only weights; activations, the workspace and the
  // outputs may belong to the previous kernel of the stream
  pdl_wait();
  if (wu0 >= wu1) return;
  float* red = reinterpret_cast<float*>(pp_smem + kDualTScratch);
  DualTOp op(p, ring, side);
  tma_stream(op, issue, rg, pt, tb, red, warp, wu0, wu1, cu0, cu1, status);
}

// ------------------------------------------------------------------ host --
bool dual_tma_ok(int64_t M, int64_t N, int64_t K, int64_t gs, const void* x, int64_t ldx_k, const int16_t* codes,
                 int64_t ldp_k, int64_t ldp_n, const void* bmax) {
  return M == 1 && gs == 32 && N % 256 == 0 && K > 0 && ldp_n == 1 && ldp_k % 8 == 0 && ldp_k >= N &&
         aligned(codes, 16) && aligned(bmax, 16) && ldx_k == 1 && aligned(x, 4) &&
         cdiv(N, 64) * cdiv(K, 16) < (int64_t)INT32_MAX;
}

namespace {
bool g_dt_attr[64];
int g_dt_limit[64];
}  // namespace

// Plan and launch; the workspace holds the counter block and the
// cross-CTA slots (its size is that of the register engine's plan, which
// never has fewer CTAs).
int launch_dual_tma(const void* x, const int16_t* codes, int64_t ldp_k, const void* bmax, const void* amp_lut,
                    const void* cos_lut, const void* sin_lut, void* out1, void* out2, int64_t ldo_n, int64_t N,
                    int64_t K, void* ws, size_t ws_bytes, int sms, cudaStream_t s) {
  int max_smem = 0;
  int rc = ensure_smem_attr(dual_tma_kernel, g_dt_attr, g_dt_limit, &max_smem);
  if (rc) return rc;
  if ((uint32_t)max_smem < kDualTSmem) {
    set_error("the dual TMA kernel needs %u bytes of shared memory, the limit is %d", kDualTSmem, max_smem);
    return PP_ERR_INVALID;
  }
  DualTParams prm{};
  if ((rc = encode_tmap_2d(&prm.tcodes, CU_TENSOR_MAP_DATA_TYPE_UINT16, codes, (uint64_t)N, (uint64_t)K,
                           (uint64_t)ldp_k * 2, 64, 16, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = encode_tmap_2d(&prm.tscale, CU_TENSOR_MAP_DATA_TYPE_UINT16, bmax, (uint64_t)(N / 32), (uint64_t)K,
                           (uint64_t)(N / 32) * 2, 8, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  prm.x = reinterpret_cast<const __half*>(x);
  prm.amp_lut = reinterpret_cast<const __half*>(amp_lut);
  prm.cos_lut = reinterpret_cast<const __half*>(cos_lut);
  prm.sin_lut = reinterpret_cast<const __half*>(sin_lut);
  prm.out[0] = reinterpret_cast<__half*>(out1);
  prm.out[1] = reinterpret_cast<__half*>(out2);
  prm.ldo_n = ldo_n;
  prm.N = (int)N;
  prm.K = (int)K;
  const int cap = sms < kMaxCtaTable ? sms : kMaxCtaTable;
  PartitionPlan pl = plan_partition(cdiv(N, 64), cdiv(K, 16), kDualTWarps, cap, 2, 1, 64);
  plan_cta_starts(pl, prm.cta_start, 32);
  if (ws_bytes < pl.total() || !ws || !aligned(ws, 256)) {
    set_error("workspace of %zu bytes (256-byte aligned, zero-filled) required, got %zu", pl.total(), ws_bytes);
    return PP_ERR_WORKSPACE;
  }
  for (int c = 0; c < pl.grid; ++c)  // warp split in 32-bit arithmetic (warp_start)
    if ((int64_t)(prm.cta_start[c + 1] - prm.cta_start[c]) * kDualTWarps >= INT32_MAX) {
      set_error("matrix too large for one launch (units per thread block)");
      return PP_ERR_INVALID;
    }
  prm.part.units = (int)pl.units;
  prm.part.upt = (int)pl.upt;
  prm.part.counters = reinterpret_cast<int*>(ws);
  prm.part.slots = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + pl.counters_bytes);
  return launch_kernel("dual_tma_kernel", launch_overlap(), dual_tma_kernel, dim3(pl.grid),
                       dim3(kDualTWarps * 32), (size_t)max_smem, s, prm);
}

}  // namespace pp
