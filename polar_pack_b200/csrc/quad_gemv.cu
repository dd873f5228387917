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
// Plug correction fused into the stream (file layout, batch 1): each unit's
// plug entries come as one segment of a unit-major plug stream (built at
// load time by pp_quad_prepare_unit_plugs, quad_decode.cu), copied into a
// slot beside the unit's ring slot on the same mbarrier.  Plugged codes
// decode to zeros; lane (g, c) adds value * x[k] of the plug entries of its
// tile row with index = c mod 4 into four FP32 sums, which the row's four
// lanes combine into the accumulators before the tile is stored or reduced.
//
// Work partition and the deterministic split-K reduction: pp_engine.cuh.
#include "pp_common.cuh"
#include "pp_engine.cuh"
#include "pp_host.h"
#include "pp_peer.h"
#include "quad_layout.h"

namespace pp {

static_assert(kQuadTableBytes == kQuadLutBytes, "table size shared with the layout planner");

int zero_f16(void* p, int64_t R, int64_t C, int64_t ldr, int64_t ldc, cudaStream_t s);

// quad_decode.cu: CSR plug-table correction of one file-layout Linear
struct PlugCorrParams {
  const __half* x;
  int64_t ldx_m;
  const uint32_t* plug_idx;
  const uint2* plug_vals;
  const uint32_t* wbase;
  uint32_t base_lo32;
  int M, N, K, W;
  float* corr;
  int64_t ldq;
  __half* xt;  // M > 1: scratch for x transposed, K x 128 halves
};
int launch_plug_corr(const PlugCorrParams& prm, cudaStream_t s);

// workspace for the transposed activations of the batched plug correction
inline size_t xt_bytes(int64_t K) { return ((size_t)K * 128 * 2 + 255) / 256 * 256; }

// quad_tc.cu: batched tensor-core path (file layout, prepared tables)
bool quad_tc_ok(int64_t M, int64_t N, int64_t K, const uint32_t* codes, int64_t ldw, const void* x, int64_t ldx_m,
                int64_t ldx_k);
size_t quad_tc_slots_bytes(int64_t M, int64_t N, int64_t K, int sms);
int launch_quad_tc(const void* x, int64_t ldx_m, const uint32_t* codes, int64_t ldw, const void* tables,
                   const float scales[4], void* const out[4], int64_t ldo_m, int64_t ldo_n, const float* corr,
                   int64_t corr_q, int64_t Mc, int64_t N, int64_t K, int* counters, float* slots,
                   const void* uplugs, const uint32_t* uplug_off, cudaStream_t s);
constexpr int64_t kTcLaunchRows = 128;

// Warps per CTA.  Shared memory holds the 128 KiB tables, each warp's TMA
// ring (2 KiB per slot) and two partial slots per warp.  The batch-1 file
// layout runs 16 warps of two ring slots (more warps hide the decode
// latencies better than deeper rings); the KN tile keeps 4x more
// accumulators and partials per warp, and two batch tiles double them
// again, so those variants use fewer warps (NB = 8-row batch tiles).
__host__ __device__ constexpr int quad_warps(bool nk, int nb) { return nk ? (nb == 1 ? 16 : 8) : (nb == 1 ? 8 : 4); }

struct QuadParams {
  CUtensorMap tmap;  // 2D map over the codes, 128-byte swizzle (first: 64-byte aligned)
  const __half* x;
  int64_t ldx_m, ldx_k;
  const uint32_t* codes;
  int64_t ldc;  // NK: stride between rows n; KN: stride between rows k
  const __half* luts[7];
  const uint8_t* tables;  // prepared 128 KiB table image (NULL: build from luts)
  float scale[4];
  __half* out[4];
  int64_t ldo_m, ldo_n;
  int M, N, K;
  // plug-table correction [4][M][N] FP32 added before the scale (NULL: none)
  const float* corr;
  Partition part;
  int stages;           // TMA ring slots per warp
  uint32_t smem_bytes;  // dynamic shared memory of the launch
  // shared-memory layout planned on the host for a dynamic region at
  // layout_base (the kernel recomputes it if its base differs)
  QuadLayout layout;
  uint32_t layout_base;
  // fused plug correction: unit-major plug stream, its unit byte offsets
  // (units + 1) and the plug slot size (a multiple of 16)
  const uint8_t* uplugs;
  const uint32_t* uplug_off;
  uint32_t pcap;
  // outputs gathered into every rank's buffer (batch 1; world 0: none)
  PeerGather gather;
  // epilogue (NULL: none): y = fp16(s_k * acc + bias_k[n]), then
  // y = fp16(y + resid_k[m][n]) (resid with the output strides, may be out)
  const __half* bias[4];
  const __half* resid[4];
  // DIAG, optional (NULL: none): the four activation rows interleaved,
  // xil[4 * k + q] = x_q[k]; a plug entry's four activations are one load
  const __half* xil;
  int cta_start[kMaxCtaTable + 1];  // unit start of every CTA (plan_cta_starts)
};

struct QuadBuf {
  uint4 q[4];
};

// Plug slot of the fused plug correction (one more per warp than ring
// slots): a segment of up to (512 - 32) / 9 = 53 entries is staged; larger
// ones are read from HBM by the lanes.
constexpr uint32_t kPlugCap = 512u;

// NK: file layout.  DIRECT: tables at a 64 KiB-aligned shared address (see
// decode_quad).  PLUG: fused plug correction (NK, NB == 1, batch 1).
// DIAG: one activation row per model (NK, NB == 1, M == 1): x has four rows,
// model q multiplies row q and writes row 0 of out[q].  The four rows feed
// mma batch columns 0-3; model q's result is column q of its fragment rows
// (the other columns hold products nobody stores), and the plug terms, which
// need x_q, collect in four separate per-lane sums.
template <bool NK, int NB, bool DIRECT, bool PLUG = false, bool DIAG = false>
struct QuadOp {
  static_assert(!PLUG || (NK && NB == 1), "fused plugs: file layout, one batch tile");
  static_assert(!DIAG || (NK && NB == 1), "per-model activations: file layout, one batch tile");
  static constexpr int kWarps = quad_warps(NK, NB);
  static constexpr int kTileW = NK ? 8 : 32;  // output features per tile
  static constexpr int kT = NK ? 1 : 4;       // mma pairs per 16-k step
  static constexpr int kNOut = 4;
  static constexpr int kNBat = 8 * NB;
  static constexpr int kUnitBytes = 2048;
  static constexpr int kPrefetch = 0;  // units of a chunk prefetched into L2 ahead of the ring (0: none)
  using Buf = QuadBuf;

  const QuadParams& p;
  int g, c;
  int pr;  // NK: physical row of mma row g inside the 8-row tile (see read())
  uint32_t lb0, lb1, add0, add1;  // table addressing (decode_quad)
  uint32_t roff[4];               // this lane's 16-byte reads inside a ring slot (see read())
  int Mv, Nv, Kv;
  int64_t ldc, ldx_m;
  const uint32_t* codes;
  const __half* x;
  const __half* xrow[NB];  // this lane's activation row per batch tile (clamped); NK: + 4c
  float acc[kT][NB][2][4];
  // PLUG: this warp's plug slots (shared address); the lane's first two
  // entries of the current unit (values and raw FP16 activations), loaded
  // by side() and applied after the decode
  uint32_t pring = 0u;
  uint2 pv0, pv1;
  uint32_t px;
  // DIAG + PLUG: per-model plug sums of this lane's entries and the two
  // entries' activations of every model (x_q[col0] | x_q[col1] << 16)
  float pacc[4];
  uint32_t pxq[4];

  __device__ __forceinline__ QuadOp(const QuadParams& p_, uint32_t lut_saddr)
      : p(p_), g((threadIdx.x & 31) >> 2), c(threadIdx.x & 3),
        pr((((threadIdx.x & 31) >> 2) >> 1) | ((((threadIdx.x & 31) >> 2) & 1) << 2)),
        lb0((DIRECT ? lut_saddr : 0u) | ((threadIdx.x & 31) * 4u)),
        lb1((DIRECT ? lut_saddr + 65536u : 0u) | ((threadIdx.x & 31) * 4u)), add0(DIRECT ? 0u : lut_saddr),
        add1(DIRECT ? 0u : lut_saddr + 65536u),
        Mv(p_.M), Nv(p_.N), Kv(p_.K), ldc(p_.ldc), ldx_m(p_.ldx_m), codes(p_.codes), x(p_.x) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int bat = nb * 8 + g;
      const int rows = DIAG ? 4 : Mv;  // DIAG: activation row q = model q
      xrow[nb] = x + (int64_t)(bat < rows ? bat : 0) * ldx_m + (NK ? 4 * c : 0);
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if constexpr (NK) {
        const int j = 4 * (s & 1) + c;
        roff[s] = (uint32_t)((s >> 1) * 1024 + pr * 128 + ((j ^ pr) << 4));
      } else {
        const int row = 2 * c + (s & 1) + 8 * (s >> 1);
        roff[s] = (uint32_t)(row * 128 + ((g ^ (row & 7)) << 4));
      }
    }
  }

  __device__ __forceinline__ int M() const { return Mv; }
  __device__ __forceinline__ int N() const { return Nv; }

  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int t = 0; t < kT; ++t)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[t][nb][h][j] = 0.f;
    if constexpr (DIAG && PLUG) {
#pragma unroll
      for (int q = 0; q < 4; ++q) pacc[q] = 0.f;
    }
  }

  __device__ __forceinline__ void begin(int, int) {}
  __device__ __forceinline__ void preload(int, int) {}

  __device__ __forceinline__ void plug_init(uint32_t ring) { pring = ring; }

  // One unit by TMA into a 2 KiB ring slot (one lane).  NK: 8
  // rows x 64 codes as two 8 x 32 boxes (128-byte rows, 128-byte swizzle);
  // KN: 16 rows x 32 features, one box.  Out-of-range elements arrive as
  // zeros.  ARRIVE: arrive on the barrier expecting the unit plus `extra`
  // bytes of side copies; else only raise its transaction count by the
  // unit, leaving the arrival to a later side copy.
  template <bool ARRIVE = true>
  static __device__ __forceinline__ void issue(const QuadParams& q, uint32_t slot, uint32_t bar, int tile, int kc,
                                               uint32_t extra = 0u) {
    if (ARRIVE) mbar_expect_tx(bar, kUnitBytes + extra);
    else mbar_expect_tx_only(bar, kUnitBytes);
    if constexpr (NK) {
      tma_load_2d(slot, &q.tmap, kc * 64, tile * 8, bar);
      tma_load_2d(slot + 1024u, &q.tmap, kc * 64 + 32, tile * 8, bar);
    } else {
      tma_load_2d(slot, &q.tmap, tile * 32, kc * 16, bar);
    }
  }

  // L2 prefetch of unit (tile, kc): the same boxes as issue()
  __device__ __forceinline__ void prefetch(int tile, int kc) const {
    if constexpr (NK) {
      tma_prefetch_2d(&p.tmap, kc * 64, tile * 8);
      tma_prefetch_2d(&p.tmap, kc * 64 + 32, tile * 8);
    } else {
      tma_prefetch_2d(&p.tmap, tile * 32, kc * 16);
    }
  }

  // 16-byte chunk j of box row r sits at r*128 + 16*(j ^ (r & 7)) (128-byte
  // swizzle).  NK: lane (g, c) needs row pr, chunk 4*(s&1) + c of box s>>1;
  // mma row g maps to tile row pr = (g>>1) | ((g&1)<<2), so the two rows of
  // a quarter-warp differ in bit 2 and their chunks never share banks.
  // KN: lane (g, c) needs chunk g of rows 2c, 2c+1, 2c+8, 2c+9.
  __device__ __forceinline__ void read(Buf& b, uint32_t slot, int = 0, int = 0) const {
#pragma unroll
    for (int s = 0; s < 4; ++s) b.q[s] = lds128(slot + roff[s]);
  }


  // Activation fragments.  Batch columns >= M read row 0 (clamped): their
  // mma output column is never stored.  FULL units lie wholly below K and
  // load without checks; in the last K chunk, columns k >= K read as zero.
  template <bool FULL>
  __device__ __forceinline__ uint32_t xpair(int nb, int k) const {
    if (FULL || k + 1 < Kv) return ld_u32(xrow[nb] + k);
    return k < Kv ? (uint32_t)ld_u16(xrow[nb] + k) : 0u;
  }

  // NK: activations (bat, kbase + 16s + 4c .. +3) from xrow (which holds
  // the + 4c); the NK path guarantees K % 4 == 0
  template <bool FULL>
  __device__ __forceinline__ uint2 xquad(int nb, int kbase, int s) const {
    if (FULL || kbase + 16 * s + 4 * c < Kv) return ld_u2(xrow[nb] + kbase + 16 * s);
    return make_uint2(0u, 0u);
  }

  // PLUG: plug entries of unit u (column chunk kc) from plug slot sp.  The
  // segment starts with eight u32 header words, one per tile row r:
  // start_r | end_r << 10 | n << 20; then n FP16x4 values and n column
  // bytes (k - 64 kc).  It is staged whole when 32 + 9n <= kPlugCap, else
  // read from HBM.  Lane (g, c) takes the entries of tile row pr whose index
  // within the row is c mod 4.  Its first two are loaded here with their
  // activations and applied after the unit's decode (plug_finish), which
  // hides the load latency; further ones (rows of more than 8 entries) are
  // applied now.  The terms go to the lane's accumulators of batch column
  // 2c, which hold zeros for c > 0 (the PLUG kernel runs batch 1 and feeds
  // zero activations to the other columns); end_chunk sums the row's four
  // lanes.
  __device__ __forceinline__ void side(int sp, int u, int kc) {
    if constexpr (PLUG) {
      const uint32_t ps = pring + (uint32_t)sp * kPlugCap;
      const uint32_t h = lds_u32(ps + 4u * (uint32_t)pr);
      const uint32_t lo = h & 1023u, hi = (h >> 10) & 1023u, n = h >> 20;
      const __half* xk = x + kc * 64;
      const uint32_t e0 = lo + (uint32_t)c, e1 = e0 + 4u;
      pv0 = pv1 = make_uint2(0u, 0u);
      px = 0u;  // the two entries' columns; plug_x() loads their activations
      if (32u + 9u * n <= kPlugCap) {
        const uint32_t vb = ps + 32u, kb = ps + 32u + 8u * n;
        if (e0 < hi) {
          pv0 = lds_u2(vb + 8u * e0);
          px = lds_u8(kb + e0);
        }
        if (e1 < hi) {
          pv1 = lds_u2(vb + 8u * e1);
          px |= lds_u8(kb + e1) << 16;
        }
        for (uint32_t e = e1 + 4u; e < hi; e += 4u) plug_term(lds_u2(vb + 8u * e), xk, lds_u8(kb + e));
      } else {
        const uint8_t* gs = p.uplugs + __ldg(p.uplug_off + u);
        for (uint32_t e = e0; e < hi; e += 4u)
          plug_term(__ldg(reinterpret_cast<const uint2*>(gs + 32u + 8u * e)), xk, __ldg(gs + 32u + 8u * n + e));
      }
    }
  }

  // PLUG: the activations of the unit's first two plug entries of this lane
  // (columns from side(); an empty entry has value zero and reads column 0),
  // loaded at the start of the unit's compute so the decode hides them
  __device__ __forceinline__ void plug_x(int kc) {
    if constexpr (PLUG) {
      const __half* xk = x + kc * 64;
      if constexpr (DIAG) {
        if (p.xil) {  // uniform: the two entries' four activations, one 8-byte load each
          const __half* xi = p.xil + (int64_t)kc * 64 * 4;
          const uint2 a = ld_u2(xi + 4u * (px & 0xFFu)), b = ld_u2(xi + 4u * (px >> 16));
          pxq[0] = lo_pair(a.x, b.x);
          pxq[1] = hi_pair(a.x, b.x);
          pxq[2] = lo_pair(a.y, b.y);
          pxq[3] = hi_pair(a.y, b.y);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            pxq[q] = (uint32_t)ld_u16(xk + q * ldx_m + (px & 0xFFu)) |
                     ((uint32_t)ld_u16(xk + q * ldx_m + (px >> 16)) << 16);
        }
      } else {
        px = (uint32_t)ld_u16(xk + (px & 0xFFu)) | ((uint32_t)ld_u16(xk + (px >> 16)) << 16);
      }
    }
  }

  __device__ __forceinline__ void plug_finish() {
    if constexpr (PLUG) {
      if constexpr (DIAG) {
        plug_fma4(pv0, pxq, 0);
        plug_fma4(pv1, pxq, 16);
      } else {
        plug_fma(pv0, px & 0xFFFFu);
        plug_fma(pv1, px >> 16);
      }
    }
  }

  // one plug entry (values v, column col of the unit at xk) applied now
  __device__ __forceinline__ void plug_term(uint2 v, const __half* xk, uint32_t col) {
    if constexpr (DIAG) {
      uint32_t xq[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) xq[q] = ld_u16(xk + q * ldx_m + col);
      plug_fma4(v, xq, 0);
    } else {
      plug_fma(v, ld_u16(xk + col));
    }
  }

  // DIAG: pacc[q] += value q * x_q (the FP16 activation in bits sh..sh+15
  // of xq[q]), FP16 operands and one FP32 rounding, as in plug_fma
  __device__ __forceinline__ void plug_fma4(uint2 v, const uint32_t (&xq)[4], int sh) {
    asm("{\n .reg .f16 v0, v1, v2, v3, x0, x1, x2, x3;\n .reg .b16 t;\n"
        " mov.b32 {v0, v1}, %4;\n mov.b32 {v2, v3}, %5;\n"
        " mov.b32 {x0, t}, %6;\n mov.b32 {x1, t}, %7;\n mov.b32 {x2, t}, %8;\n mov.b32 {x3, t}, %9;\n"
        " fma.rn.f32.f16 %0, v0, x0, %0;\n fma.rn.f32.f16 %1, v1, x1, %1;\n"
        " fma.rn.f32.f16 %2, v2, x2, %2;\n fma.rn.f32.f16 %3, v3, x3, %3;\n}"
        : "+f"(pacc[0]), "+f"(pacc[1]), "+f"(pacc[2]), "+f"(pacc[3])
        : "r"(v.x), "r"(v.y), "r"(xq[0] >> sh), "r"(xq[1] >> sh), "r"(xq[2] >> sh), "r"(xq[3] >> sh));
  }

  // acc(model q, batch column 2c) += value q * x with the FP16 operands
  // taken as they are (their product is exact in FP32) and one FP32
  // rounding, as cvt + fmaf would.
  __device__ __forceinline__ void plug_fma(uint2 v, uint32_t xbits) {
    asm("{\n .reg .f16 v0, v1, v2, v3, xh;\n"
        " mov.b32 {v0, v1}, %4;\n mov.b32 {v2, v3}, %5;\n mov.b32 {xh, _}, %6;\n"
        " fma.rn.f32.f16 %0, v0, xh, %0;\n fma.rn.f32.f16 %1, v1, xh, %1;\n"
        " fma.rn.f32.f16 %2, v2, xh, %2;\n fma.rn.f32.f16 %3, v3, xh, %3;\n}"
        : "+f"(acc[0][0][0][0]), "+f"(acc[0][0][0][2]), "+f"(acc[0][0][1][0]), "+f"(acc[0][0][1][2])
        : "r"(v.x), "r"(v.y), "r"(xbits));
  }

  // PLUG: the four lanes of each row sum their batch column 2c (a fixed
  // butterfly): lane c = 0 then holds the product plus every plug term of
  // the row in batch column 0 (fragment register 2 (q & 1) of half q >> 1
  // for model q).
  __device__ __forceinline__ void end_chunk() {
    if constexpr (PLUG && DIAG) {
      // the row's four lanes sum each model's plug terms; lane c = q >> 1
      // holds model q's result (column q) in register (q & 1) * 3 of half q >> 1
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v = pacc[q];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (c == (q >> 1)) acc[0][0][q >> 1][(q & 1) * 3] += v;
        pacc[q] = 0.f;
      }
    } else if constexpr (PLUG) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          float v = acc[0][0][h][j];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          acc[0][0][h][j] = v;
        }
    }
  }

  __device__ __forceinline__ void compute(const Buf& b, int tile, int kc) {
    plug_x(kc);
    if (kc * (NK ? 64 : 16) + (NK ? 64 : 16) <= Kv) compute_unit<true>(b, kc);
    else compute_unit<false>(b, kc);
    plug_finish();
  }

  template <bool FULL>
  __device__ __forceinline__ void compute_unit(const Buf& b, int kc) {
    if constexpr (NK) {
      const int kbase = kc * 64;
      uint2 xb[4][NB];
#pragma unroll
      for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
          // PLUG (batch 1): only lanes g = 0 feed activations; the other
          // batch columns stay zero for side()'s plug terms.  DIAG: batch
          // columns 4-7 are never stored, lanes g >= 4 load nothing
          xb[s][nb] = ((PLUG && !DIAG && g != 0) || (DIAG && g >= 4)) ? make_uint2(0u, 0u)
                                                                       : xquad<FULL>(nb, kbase, s);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int kp = kbase + 16 * s + 4 * c;
        QuadDec d[4];
        d[0] = decode_quad<DIRECT>(b.q[s].x, lb0, lb1, add0, add1);
        d[1] = decode_quad<DIRECT>(b.q[s].y, lb0, lb1, add0, add1);
        d[2] = decode_quad<DIRECT>(b.q[s].z, lb0, lb1, add0, add1);
        d[3] = decode_quad<DIRECT>(b.q[s].w, lb0, lb1, add0, add1);
        uint32_t a01[4] = {lo_pair(d[0].p1, d[1].p1), lo_pair(d[0].p2, d[1].p2),
                           lo_pair(d[2].p1, d[3].p1), lo_pair(d[2].p2, d[3].p2)};
        uint32_t a23[4] = {lo_pair(d[0].p3, d[1].p3), hi_pair(d[0].p3, d[1].p3),
                           lo_pair(d[2].p3, d[3].p3), hi_pair(d[2].p3, d[3].p3)};
        if (!FULL && kp >= Kv) {
#pragma unroll
          for (int i = 0; i < 4; ++i) a01[i] = a23[i] = 0u;
        }
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          mma_16816(acc[0][nb][0], a01[0], a01[1], a01[2], a01[3], xb[s][nb].x, xb[s][nb].y);
          mma_16816(acc[0][nb][1], a23[0], a23[1], a23[2], a23[3], xb[s][nb].x, xb[s][nb].y);
        }
      }
    } else {
      const int kbase = kc * 16;
      uint32_t b0[NB], b1[NB];
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        b0[nb] = xpair<FULL>(nb, kbase + 2 * c);
        b1[nb] = xpair<FULL>(nb, kbase + 2 * c + 8);
      }
      bool rv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) rv[r] = FULL || (kbase + 2 * c + (r & 1) + 8 * (r >> 1) < Kv);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        QuadDec d[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint32_t code = t == 0 ? b.q[r].x : t == 1 ? b.q[r].y : t == 2 ? b.q[r].z : b.q[r].w;
          d[r] = decode_quad<DIRECT>(code, lb0, lb1, add0, add1);
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
  __device__ __forceinline__ void write_partial(float* slot, int M) {
#pragma unroll
    for (int t = 0; t < kT; ++t) {
      const int fi = NK ? pr : 4 * g + t;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int bat = nb * 8 + 2 * c + (j & 1);
            if constexpr (DIAG) {  // model q's result is batch column q: stored as batch row 0
              if (bat == 2 * h + (j >> 1)) slot[(2 * h + (j >> 1)) * kTileW + fi] = acc[t][nb][h][j];
            } else if (bat < M) {
              slot[((2 * h + (j >> 1)) * M + bat) * kTileW + fi] = acc[t][nb][h][j];
            }
          }
    }
  }

  // Batch-1 gather with 16-byte stores: an 8-row tile is 8 consecutive
  // elements of each model's block, so one store per model and rank
  // replaces eight 2-byte stores (each a separate NVLink write to a peer).
  static constexpr bool kGather16 = NK && NB == 1;
  __device__ __forceinline__ bool gather16(int tile) const {
    return !DIAG && p.gather.world && p.gather.vec && tile * 8 + 8 <= Nv && !p.bias[0] && !p.resid[0];
  }
  // lane = element (model lane >> 3, row lane & 7) of tile `tile`; v is the
  // sum before the plug correction and the scale
  __device__ __forceinline__ void gather_store16(int tile, float v) const {
    const int lane = threadIdx.x & 31, q = lane >> 3;
    const uint32_t hv = __half_as_ushort(__float2half_rn((v + corr_at(q, 0, tile * 8 + (lane & 7))) * p.scale[q]));
    const uint32_t pair = hv | (__shfl_down_sync(0xffffffffu, hv, 1) << 16);
    const uint32_t p1 = __shfl_down_sync(0xffffffffu, pair, 2);
    const uint32_t p2 = __shfl_down_sync(0xffffffffu, pair, 4);
    const uint32_t p3 = __shfl_down_sync(0xffffffffu, pair, 6);
    if ((lane & 7) == 0) {
      const int64_t o = (int64_t)q * p.gather.ld + p.gather.row0 + (int64_t)tile * 8;
      const uint4 w = make_uint4(pair, p1, p2, p3);
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r < p.gather.world) *reinterpret_cast<uint4*>(p.gather.out[r] + o) = w;
    }
  }

  // The plug corrections of a batch tile are loaded before its outputs are
  // stored: otherwise each load would wait for the store before it (the
  // compiler cannot rule out that they alias).
  __device__ __forceinline__ void store_tile(int tile) {
    if constexpr (kGather16) {
      if (gather16(tile)) {  // warp-uniform
        // lane (g, 0) holds row pr(g)'s four model sums; row r is on lane
        // 4 g_r with g_r = ((r & 3) << 1) | (r >> 2)
        const int lane = threadIdx.x & 31, q = lane >> 3, r = lane & 7;
        const int src = 4 * (((r & 3) << 1) | (r >> 2));
        // (the value a shuffle passes is the source lane's: fetch all four
        // models, then choose by this lane's model)
        const float m0 = __shfl_sync(0xffffffffu, acc[0][0][0][0], src);
        const float m1 = __shfl_sync(0xffffffffu, acc[0][0][0][2], src);
        const float m2 = __shfl_sync(0xffffffffu, acc[0][0][1][0], src);
        const float m3 = __shfl_sync(0xffffffffu, acc[0][0][1][2], src);
        gather_store16(tile, q == 0 ? m0 : q == 1 ? m1 : q == 2 ? m2 : m3);
        return;
      }
    }
    if constexpr (DIAG) {
      const int f = tile * kTileW + pr;
      if (f >= Nv) return;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (2 * c + (j & 1) == 2 * h + (j >> 1)) store(2 * h + (j >> 1), 0, f, acc[0][0][h][j]);
    } else {
      store_tile_rows(tile);
    }
  }

  __device__ __forceinline__ void store_tile_rows(int tile) {
#pragma unroll
    for (int t = 0; t < kT; ++t) {
      const int f = tile * kTileW + (NK ? pr : 4 * g + t);
      if (f >= Nv) continue;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        float cv[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int bat = nb * 8 + 2 * c + (j & 1);
            cv[h][j] = (p.corr && bat < Mv) ? __ldcg(p.corr + ((int64_t)(2 * h + (j >> 1)) * Mv + bat) * Nv + f) : 0.f;
          }
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int bat = nb * 8 + 2 * c + (j & 1);
            if (bat < Mv) store_raw(2 * h + (j >> 1), bat, f, acc[t][nb][h][j] + cv[h][j]);
          }
      }
    }
  }

  __device__ __forceinline__ float corr_at(int model, int bat, int f) const {
    return p.corr ? __ldcg(p.corr + ((int64_t)model * Mv + bat) * Nv + f) : 0.f;
  }

  __device__ __forceinline__ void store(int model, int bat, int f, float v) const {
    store_raw(model, bat, f, v + corr_at(model, bat, f));
  }

  // v already includes the plug correction
  __device__ __forceinline__ void store_raw(int model, int bat, int f, float v) const {
    const __half* bias = p.bias[model];
    const __half* resid = p.resid[model];
    __half h = __float2half_rn(v * p.scale[model] + (bias ? __half2float(bias[f]) : 0.f));
    if (resid) h = __float2half_rn(__half2float(h) + __half2float(resid[(int64_t)bat * p.ldo_m + (int64_t)f * p.ldo_n]));
    if (p.gather.world) {  // batch 1: element (model, row0 + f) of every rank's buffer
      const int64_t o = (int64_t)model * p.gather.ld + p.gather.row0 + f;
#pragma unroll
      for (int q = 0; q < kMaxPeers; ++q)
        if (q < p.gather.world) p.gather.out[q][o] = h;
      return;
    }
    p.out[model][(int64_t)bat * p.ldo_m + (int64_t)f * p.ldo_n] = h;
  }
};

// PLUG: lane 0 copies the plug segment of unit u into plug slot s, at most
// pcap bytes, with the offsets from the warp's table.  Returns its bytes.
__device__ __forceinline__ uint32_t plug_bytes(const QuadParams& p, uint32_t ptab, int wu0, int u, uint32_t* off) {
  const uint32_t o0 = lds_u32(ptab + 4u * (uint32_t)(u - wu0));
  const uint32_t len = lds_u32(ptab + 4u * (uint32_t)(u - wu0 + 1)) - o0;
  *off = o0;
  return len < kPlugCap ? len : kPlugCap;
}

template <bool NK, int NB, bool DIRECT, bool PLUG, bool DIAG>
__device__ __forceinline__ void quad_body(const QuadParams& p, const Partition& pt, const QuadLayout& L, TmaRing& rg,
                                          const CtaTables& tb, int cu0, int cu1, int wu0, int wu1, int* status) {
  using Op = QuadOp<NK, NB, DIRECT, PLUG, DIAG>;
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(pp_smem);
  float* red = reinterpret_cast<float*>(pp_smem + (L.scratch - base));
  const int warp = threadIdx.x >> 5;
  Op op(p, L.lut);
  if constexpr (PLUG) {
    const uint32_t pring = L.plug + (uint32_t)(warp * (p.stages + 1)) * kPlugCap;
    const uint32_t ptab = L.ptab + (uint32_t)warp * (kPlugTabEntries * 4u);
    op.plug_init(pring);
    const int upt = pt.upt;
    tma_stream(op, [&](uint32_t slot, uint32_t bar, int s, int tile, int kc) {
      uint32_t off;
      const uint32_t pb = plug_bytes(p, ptab, wu0, tile * upt + kc, &off);
      Op::template issue<true>(p, slot, bar, tile, kc, pb);
      bulk_load(pring + (uint32_t)s * kPlugCap, p.uplugs + off, pb, bar);  // s: side slot
    }, rg, pt, tb, red, warp, wu0, wu1, cu0, cu1, status);
  } else {
    tma_stream(op, [&](uint32_t slot, uint32_t bar, int, int tile, int kc) { Op::issue(p, slot, bar, tile, kc); },
               rg, pt, tb, red, warp, wu0, wu1, cu0, cu1, status);
  }
}

// Partial-sum scratch of a CTA: two slots per warp.
__host__ __device__ inline uint32_t quad_scratch_bytes(bool nk, int nb, int M) {
  return (uint32_t)red_bytes(quad_warps(nk, nb), 4, M, nk ? 8 : 32);
}

// Tables either come prepared (thread 0 bulk-copies the 128 KiB image, which
// every thread then waits for on one mbarrier) or are built here (the table
// words, their loads issued first, are staged before the first barrier and
// fanned out after it).  Before the first barrier the per-CTA int tables
// are filled; after it lane 0 of every warp initialises its ring and issues
// its first S units, whose copies overlap the table build or copy.  Then
// every warp streams and reduces on its own; there is no closing barrier.
template <bool NK, int NB, bool PLUG, bool DIAG>
__device__ __forceinline__ int* quad_gemv_run(const QuadParams& p, int cta, int ncta) {
  constexpr int NW = quad_warps(NK, NB);
  // the first code copies need the tensor map: fetch it while the
  // parameters and per-CTA tables are read
  if (threadIdx.x == 0) prefetch_tmap(&p.tmap);
  pdl_launch_dependents();
  const bool prepared = p.tables != nullptr;
  uint32_t v[kLutWordsPerThread];
  if (!prepared) quad_lut_load(v, p.luts);
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(pp_smem);
  int* status = p.part.counters + (kMaxGrid - 1);
  const QuadLayout L = base == p.layout_base
                           ? p.layout
                           : quad_layout(base, p.smem_bytes, NW, p.stages, quad_scratch_bytes(NK, NB, p.M), true,
                                         PLUG ? p.pcap : 0u);
  if (!L.ok) {  // the host plans for this never to happen
    if (threadIdx.x == 0) atomicExch(status, 2);
    return nullptr;
  }
  const int cu0 = p.cta_start[cta], cu1 = p.cta_start[cta + 1];
  if (cu0 >= cu1) return nullptr;  // uniform over the CTA
  const uint32_t tbar = L.flag;  // mbarrier of the prepared-table copies
  if (prepared && threadIdx.x == 0) {
    mbar_init(tbar, 1);
    fence_mbar_init();
    mbar_expect_tx(tbar, kQuadLutBytes);
    for (uint32_t off = 0; off < kQuadLutBytes; off += 16384u) bulk_load(L.lut + off, p.tables + off, 16384u, tbar);
  }
  Partition pt = p.part;
  pt.cta_start = p.cta_start;
  pt.cta = cta;
  pt.ncta = ncta;
  int* ti = reinterpret_cast<int*>(pp_smem + (L.tables - base));
  const CtaTables tb{ti, ti + (NW + 1), ti + 2 * (NW + 1)};
  cta_tables_init<NW>(tb, cu0, cu1, p.part.upt);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wu0 = warp_start<NW>(cu0, cu1, warp), wu1 = warp_start<NW>(cu0, cu1, warp + 1);
  // PLUG: the plug-stream offsets of units wu0..wu1 (the host keeps
  // wu1 - wu0 < kPlugTabEntries), loaded now, stored after the CTA barrier
  uint32_t po0 = 0u, po1 = 0u;
  if constexpr (PLUG) {
    const int nu = wu1 - wu0;
    if (nu > 0 && lane <= nu) po0 = __ldg(p.uplug_off + wu0 + lane);
    if (nu > 0 && lane + 32 <= nu) po1 = __ldg(p.uplug_off + wu0 + lane + 32);
  }
  TmaRing rg;
  if (wu0 < wu1) {
    const uint32_t rw = (uint32_t)p.stages * 2048u;
    rg.ring = warp < L.splitw ? L.ringA + (uint32_t)warp * rw : L.ringB + (uint32_t)(warp - L.splitw) * rw;
    rg.bars = L.bars + 8u * (uint32_t)(warp * p.stages);
    rg.S = p.stages;
    rg.P = PLUG ? p.stages + 1 : p.stages;
    rg.next.init(wu0, wu1, p.part.upt);
  }
  // lane 0 of each warp initialises its ring and issues its first units
  // before the barrier (the rings overlap nothing written before it).
  // PLUG: codes only for now; the plug copies, which need the offsets,
  // arrive on the same barriers after the CTA barrier
  if (wu0 < wu1 && (threadIdx.x & 31) == 0) {
    rg.prologue([&](uint32_t slot, uint32_t bar, int, int tile, int kc) {
      QuadOp<NK, NB, false>::template issue<!PLUG>(p, slot, bar, tile, kc);
    }, 2048u);
  }
  uint32_t* stage = reinterpret_cast<uint32_t*>(pp_smem + (L.scratch - base));
  if (!prepared) quad_lut_stage(stage, v);
  __syncthreads();
  // PLUG: the plug copies of the prologue units go out as soon as the
  // warp's unit offsets have arrived, before the table wait
  if constexpr (PLUG) {
    if (wu0 < wu1) {
      const uint32_t ptab = L.ptab + (uint32_t)warp * (kPlugTabEntries * 4u);
      const int nu = wu1 - wu0;
      if (lane <= nu) sts_u32(ptab + 4u * (uint32_t)lane, po0);
      if (lane + 32 <= nu) sts_u32(ptab + 4u * (uint32_t)(lane + 32), po1);
      __syncwarp();
      if (lane == 0) {  // the plug copies of the prologue units, in the same order
        const uint32_t pring = L.plug + (uint32_t)(warp * (p.stages + 1)) * kPlugCap;
        UnitSeq q;
        q.init(wu0, wu1, p.part.upt);
        for (int i = 0; i < p.stages && q.seg < 3; ++i) {
          uint32_t off;
          const uint32_t pb = plug_bytes(p, ptab, wu0, q.t * p.part.upt + q.kc, &off);
          const uint32_t bar = rg.bars + 8u * (uint32_t)i;
          mbar_expect_tx(bar, pb);
          bulk_load(pring + (uint32_t)i * kPlugCap, p.uplugs + off, pb, bar);
          q.advance();
        }
      }
    }
  }
  if (prepared) {
    mbar_wait_bounded(tbar, 0u, status);
  } else {
    quad_lut_fanout(pp_smem + (L.lut - base), stage);
    __syncthreads();
  }
  // everything above reads only weights; activations, the workspace and the
  // outputs may belong to the previous kernel of the stream
  pdl_wait();
  if (wu0 >= wu1) return tb.cnt + 2 * NW;
  if (L.direct) quad_body<NK, NB, true, PLUG, DIAG>(p, pt, L, rg, tb, cu0, cu1, wu0, wu1, status);
  else quad_body<NK, NB, false, PLUG, DIAG>(p, pt, L, rg, tb, cu0, cu1, wu0, wu1, status);
  return tb.cnt + 2 * NW;
}

// Every warp leaves quad_gemv_run, whatever path it took, and then takes
// part in the gather's completion signal.
template <bool NK, int NB, bool PLUG, bool DIAG = false>
__global__ void __launch_bounds__(quad_warps(NK, NB) * 32, 1) quad_gemv_kernel(const __grid_constant__ QuadParams p) {
  int* const cta_arrivals = quad_gemv_run<NK, NB, PLUG, DIAG>(p, blockIdx.x, gridDim.x);
  if (p.gather.world) gather_signal(p.gather, cta_arrivals, quad_warps(NK, NB));
}

// Several independent Linears in one launch: member j runs on CTAs
// [first_cta[j], first_cta[j + 1]) with its own parameters, partition and
// workspace, exactly as a launch of its own would, so the members' fixed
// costs (launch, table copy, first code copies, tail) overlap instead of
// adding up.  With a gather, every member stores into the same buffers and
// the launch publishes once (the completion count spans the whole grid).
constexpr int kMaxGroup = 8;

struct QuadGroupParams {
  int count;
  int first_cta[kMaxGroup + 1];
  QuadParams m[kMaxGroup];
};

template <bool NK, int NB, bool PLUG, bool DIAG>
__global__ void __launch_bounds__(quad_warps(NK, NB) * 32, 1)
    quad_group_kernel(const __grid_constant__ QuadGroupParams g) {
  int j = 0;
  while (j + 1 < g.count && (int)blockIdx.x >= g.first_cta[j + 1]) ++j;
  const QuadParams& p = g.m[j];
  int* const cta_arrivals =
      quad_gemv_run<NK, NB, PLUG, DIAG>(p, (int)blockIdx.x - g.first_cta[j], g.first_cta[j + 1] - g.first_cta[j]);
  if (p.gather.world) gather_signal(p.gather, cta_arrivals, quad_warps(NK, NB));
}

// Generic fallback for layouts the vector paths do not take (unaligned or
// strided codes).  One thread per (feature, batch row); plain table reads.
struct QuadGenericParams {
  const __half* x;
  int64_t ldx_m, ldx_k;
  const uint32_t* codes;
  int64_t ldc_k, ldc_n;
  const __half* luts[7];
  const uint8_t* tables;  // prepared image (NULL: read luts)
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
    if (p.tables) {  // lane copy 0 of entry e of table t
      v = __ldg(reinterpret_cast<const uint32_t*>(p.tables + lut_off(t) + (uint32_t)e * 256u));
    } else if (t == 0) {
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

// Imbalance (units on the most loaded CTA above the mean) accepted to keep
// every tile inside one CTA; about the time of the cross-CTA reduction.
constexpr int64_t kAlignSlackUnits = 32;

PartitionPlan quad_plan(bool nk, int64_t Mc, int64_t N, int64_t K, int sms, int* starts = nullptr) {
  const int nb = Mc > 8 ? 2 : 1;
  const int tile_w = nk ? 8 : 32, unit_k = nk ? 64 : 16;
  const int cap = sms < kMaxCtaTable ? sms : kMaxCtaTable;
  PartitionPlan pl = plan_partition(cdiv(N, tile_w), cdiv(K, unit_k), quad_warps(nk, nb), cap, 4, Mc, tile_w);
  if (pl.units > 0) {
    int tmp[kMaxCtaTable + 1];
    plan_cta_starts(pl, starts ? starts : tmp, kAlignSlackUnits);
  }
  return pl;
}

bool g_attr_done[8][64];
int g_attr_limit[8][64];



// Deepest ring (up to 4 slots per consumer) with the tables at a 64 KiB
// boundary for a dynamic region at the reserved-memory offset, else the
// deepest that fits with the tables at the base.  Both must also fit with
// the tables at the base, which the kernel falls back to if the runtime
// base differs.  Returns 0 if nothing fits.
int quad_stages(int nw, uint32_t redb, uint32_t reserved, uint32_t size, uint32_t pcap = 0u) {
  int plain = 0;
  for (int S = 4; S >= 1; --S) {
    if (!quad_layout(reserved, size, nw, S, redb, false, pcap).ok) continue;
    if (!plain) plain = S;
    if (S >= 2 && quad_layout(reserved, size, nw, S, redb, true, pcap).direct) return S;
  }
  return plain;
}

template <bool NK, int NB, bool PLUG>
int launch_quad(QuadParams& prm, int grid, int idx, cudaStream_t s) {
  constexpr int NW = quad_warps(NK, NB);
  auto kern = quad_gemv_kernel<NK, NB, PLUG>;
  int max_smem = 0;
  int rc = ensure_smem_attr(kern, g_attr_done[idx], g_attr_limit[idx], &max_smem);
  if (rc) return rc;
  const uint32_t redb = quad_scratch_bytes(NK, NB, prm.M);
  prm.pcap = PLUG ? kPlugCap : 0u;
  const int stages =
      quad_stages(NW, redb, (uint32_t)reserved_smem(current_device()), (uint32_t)max_smem, prm.pcap);
  if (stages == 0) {
    set_error("no shared memory layout fits the per-CTA limit %d", max_smem);
    return PP_ERR_INVALID;
  }
  prm.stages = stages;
  prm.smem_bytes = (uint32_t)max_smem;
  prm.layout_base = (uint32_t)reserved_smem(current_device());
  prm.layout = quad_layout(prm.layout_base, prm.smem_bytes, NW, stages, redb, true, prm.pcap);
  if (prm.gather.world) {  // completion count of this launch: the counter below the status word
    prm.gather.ctas = grid;
    prm.gather.vec = (prm.gather.ld % 8 == 0 && prm.gather.row0 % 8 == 0) ? 1 : 0;
    for (int q = 0; q < prm.gather.world; ++q)
      if (!aligned(prm.gather.out[q], 16)) prm.gather.vec = 0;
    prm.gather.done = reinterpret_cast<uint32_t*>(prm.part.counters + (kMaxGrid - 2));
  }
  return launch_kernel("quad_gemv_kernel", launch_overlap(), kern, dim3(grid), dim3(NW * 32), (size_t)max_smem, s,
                       prm);
}

// Workspace: [counter block 4 KiB][plug correction 4 x 16 x N floats][partial slots]
inline size_t corr_bytes(int64_t N) { return align_up((size_t)4 * 16 * N * sizeof(float), 256); }

int launch_plan(const PartitionPlan& pl, bool nk, int64_t Mc, QuadParams prm, void* ws, size_t corr_sz,
                cudaStream_t s, bool fused_plugs = false) {
  prm.part.units = (int)pl.units;
  prm.part.upt = (int)pl.upt;
  prm.part.counters = reinterpret_cast<int*>(ws);
  prm.part.slots = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + pl.counters_bytes + corr_sz);
  if (fused_plugs) return launch_quad<true, 1, true>(prm, pl.grid, 4, s);
  const int nb = Mc > 8 ? 2 : 1;
  if (nk)
    return nb == 1 ? launch_quad<true, 1, false>(prm, pl.grid, 0, s) : launch_quad<true, 2, false>(prm, pl.grid, 1, s);
  return nb == 1 ? launch_quad<false, 1, false>(prm, pl.grid, 2, s) : launch_quad<false, 2, false>(prm, pl.grid, 3, s);
}

// The fused plug correction runs when the batch is one row, every warp's
// unit range fits its offset table and the layout with plug slots fits.
bool fused_plugs_ok(const PartitionPlan& pl, const int* starts, int64_t Mc) {
  if (Mc != 1) return false;
  constexpr int NW = quad_warps(true, 1);
  for (int c = 0; c < pl.grid; ++c) {
    const int64_t r = (int64_t)starts[c + 1] - starts[c];
    if ((r + NW - 1) / NW >= (int64_t)kPlugTabEntries) return false;
  }
  int lim = 0;
  if (ensure_smem_attr(quad_gemv_kernel<true, 1, true>, g_attr_done[4], g_attr_limit[4], &lim)) return false;
  return quad_stages(NW, quad_scratch_bytes(true, 1, 1), (uint32_t)reserved_smem(current_device()), (uint32_t)lim,
                     kPlugCap) > 0;
}

bool quad_vector_ok(bool nk, const uint32_t* codes, int64_t ldc_k, int64_t ldc_n, int64_t N, int64_t K) {
  if (!aligned(codes, 16)) return false;
  if (nk) return ldc_k == 1 && ldc_n % 4 == 0 && K % 4 == 0 && ldc_n >= K;
  return ldc_n == 1 && ldc_k % 4 == 0 && N % 4 == 0 && ldc_k >= N;
}

int check_common(const void* const luts[7], const void* tables, const float scales[4], void* const out[4],
                 int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) {
    set_error("negative shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
    return PP_ERR_INVALID;
  }
  if (N > INT32_MAX || K > INT32_MAX) {
    set_error("N and K must fit in 32 bits");
    return PP_ERR_INVALID;
  }
  if (!scales || !out || (!luts && !tables)) {
    set_error("luts (or prepared tables), scales and out must not be NULL");
    return PP_ERR_INVALID;
  }
  if (tables && !aligned(tables, 16)) {
    set_error("prepared tables must be 16-byte aligned");
    return PP_ERR_INVALID;
  }
  if (!tables)
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

// Tensor-core path workspace: [counter block][plug correction 4 x Mc x N][split-K slots]
inline size_t tc_corr_bytes(int64_t M, int64_t N) {
  const int64_t Mc = M < kTcLaunchRows ? M : kTcLaunchRows;
  return align_up((size_t)4 * Mc * N * sizeof(float), 256);
}

// Fused plug correction over row chunks of a batch-1 Linear too large for
// one launch's offset tables: each chunk is a launch over rows [n0, n0 +
// rows) whose warps hold at most 63 units.  Every chunk is planned first;
// if one does not fit, nothing is launched and *done stays false.
int launch_fused_chunks(const QuadParams& base, const uint32_t* codes, int64_t ldw, int64_t ldo_n, int64_t N,
                        int64_t K, int sms, const uint8_t* uplugs, const uint32_t* uplug_off, void* ws, size_t csz,
                        cudaStream_t s, bool* done) {
  *done = false;
  const int64_t W = cdiv(K, 64);
  const int64_t cap = (int64_t)sms * quad_warps(true, 1) * ((int64_t)kPlugTabEntries - 1) * 9 / 10;
  const int64_t rows = cap / W * 8;
  if (rows <= 0) return PP_OK;
  int starts[kMaxCtaTable + 1];
  for (int64_t n0 = 0; n0 < N; n0 += rows) {
    const int64_t Nc = N - n0 < rows ? N - n0 : rows;
    if (!fused_plugs_ok(quad_plan(true, 1, Nc, K, sms, starts), starts, 1)) return PP_OK;
  }
  for (int64_t n0 = 0; n0 < N; n0 += rows) {
    const int64_t Nc = N - n0 < rows ? N - n0 : rows;
    QuadParams c = base;
    c.N = (int)Nc;
    c.codes = codes + n0 * ldw;
    int rc = encode_tmap_u32_2d(&c.tmap, c.codes, (uint64_t)K, (uint64_t)Nc, (uint64_t)ldw * 4, 32, 8);
    if (rc) return rc;
    for (int i = 0; i < 4; ++i) c.out[i] = base.out[i] + n0 * ldo_n;
    c.gather.row0 = base.gather.row0 + n0;
    c.corr = nullptr;
    c.uplugs = uplugs;
    c.uplug_off = uplug_off + (n0 / 8) * W;
    const PartitionPlan pl = quad_plan(true, 1, Nc, K, sms, c.cta_start);
    if ((rc = launch_plan(pl, true, 1, c, ws, csz, s, true))) return rc;
  }
  *done = true;
  return PP_OK;
}

size_t quad_ws_bytes(bool nk, int64_t M, int64_t N, int64_t K, bool plug) {
  const int sms = device_sm_count(current_device());
  const int64_t Mc = M < 16 ? M : 16;
  if (Mc <= 0) return 0;
  const size_t xt = plug && M > 1 ? xt_bytes(K) : 0;
  size_t need = quad_plan(nk, Mc, N, K, sms > 0 ? sms : 148).total() + (plug ? corr_bytes(N) : 0) + xt;
  if (nk && M > 16) {  // the batched tensor-core path (taken with prepared tables)
    const size_t tc = kCounterBytes + (plug ? tc_corr_bytes(M, N) : 0) +
                      quad_tc_slots_bytes(M, N, K, sms > 0 ? sms : 148) + xt;
    need = tc > need ? tc : need;
  }
  return need;
}

}  // namespace

static int quad_run(const void* a, int64_t lda_m, int64_t lda_k, const uint32_t* codes, int64_t ldc_k,
                    int64_t ldc_n, const uint32_t* plug_idx, const void* plug_vals, const uint32_t* wbase,
                    uint32_t base_lo32, const uint8_t* uplugs, const uint32_t* uplug_off,
                    const void* const luts[7], const void* tables, const float scales[4], void* const out[4],
                    int64_t ldo_m, int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* ws, size_t ws_bytes,
                    cudaStream_t s, bool file_layout, const PeerGather* gather = nullptr) {
  int rc = check_common(luts, tables, scales, out, M, N, K);
  if (rc) return rc;
  if (gather && (M != 1 || K == 0 || N == 0)) {
    set_error("a gathered Linear needs batch 1 and a non-empty (N, K)");
    return PP_ERR_INVALID;
  }
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
  if (plug && (!plug_idx || !wbase || !aligned(plug_vals, 8))) {
    set_error("plug_idx / plug_window_base missing or plug_vals not 8-byte aligned");
    return PP_ERR_INVALID;
  }
  if (uplugs && (!plug || !uplug_off || !aligned(uplugs, 16) || !aligned(uplug_off, 4))) {
    set_error("unit plugs need the plug table too, their offsets, and 16-byte alignment");
    return PP_ERR_INVALID;
  }
  const bool nk = file_layout || (ldc_k == 1 && ldc_n != 1);
  // activation rows must be contiguous and aligned for the vector loads
  const bool xcontig = lda_k == 1 && aligned(a, nk ? 8 : 4) && (lda_m * 2) % (nk ? 8 : 4) == 0;
  const bool vec = xcontig && quad_vector_ok(nk, codes, ldc_k, ldc_n, N, K);
  if (!vec && gather) {
    set_error("a gathered Linear needs the vector path (aligned codes and activations)");
    return PP_ERR_INVALID;
  }
  if (!vec) {
    if (plug) {
      set_error("file-layout Linear needs 16-byte aligned codes, K %% 4 == 0, row stride %% 4 == 0 and "
                "contiguous 8-byte aligned activation rows");
      return PP_ERR_INVALID;
    }
    QuadGenericParams g{};
    g.x = reinterpret_cast<const __half*>(a);
    g.ldx_m = lda_m;
    g.ldx_k = lda_k;
    g.codes = codes;
    g.ldc_k = ldc_k;
    g.ldc_n = ldc_n;
    for (int i = 0; i < 7; ++i) g.luts[i] = luts ? reinterpret_cast<const __half*>(luts[i]) : nullptr;
    g.tables = reinterpret_cast<const uint8_t*>(tables);
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
  if (tables && nk && quad_tc_ok(M, N, K, codes, ldc_n, a, lda_m, lda_k)) {
    // batched tensor-core path: every code decoded once for up to 128 batch
    // rows.  With the unit plug stream and more than 32 rows the plug values
    // are substituted into the decoded tiles; otherwise a separate kernel
    // computes an FP32 correction, whose cost grows with the rows while the
    // substitution's is fixed (2048 x 11008: 132 vs 140 us at 32 rows,
    // 182 vs 154 us at 64).
    auto in_tile = [&](int64_t Mc) { return plug && uplugs != nullptr && Mc > 32; };
    const int64_t last = M % kTcLaunchRows ? M % kTcLaunchRows : kTcLaunchRows;  // rows of the last launch
    const bool sep = plug && (!in_tile(M < kTcLaunchRows ? M : kTcLaunchRows) || !in_tile(last));
    const size_t csz = sep ? tc_corr_bytes(M, N) : 0;
    const size_t ssz = quad_tc_slots_bytes(M, N, K, sms);
    const size_t need = kCounterBytes + csz + ssz + (sep ? xt_bytes(K) : 0);
    if (ws_bytes < need || !ws || !aligned(ws, 256)) {
      set_error("workspace of %zu bytes (256-byte aligned, zero-filled) required, got %zu", need, ws_bytes);
      return PP_ERR_WORKSPACE;
    }
    int* counters = reinterpret_cast<int*>(ws);
    float* corr = sep ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kCounterBytes) : nullptr;
    float* slots = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kCounterBytes + csz);
    __half* xt = sep ? reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(ws) + kCounterBytes + csz + ssz)
                     : nullptr;
    for (int64_t m0 = 0; m0 < M; m0 += kTcLaunchRows) {
      const int64_t Mc = (M - m0) < kTcLaunchRows ? (M - m0) : kTcLaunchRows;
      const __half* xc = reinterpret_cast<const __half*>(a) + m0 * lda_m;
      void* oc[4];
      for (int i = 0; i < 4; ++i) oc[i] = reinterpret_cast<__half*>(out[i]) + m0 * ldo_m;
      const bool tile_plugs = in_tile(Mc);
      if (plug && !tile_plugs) {  // all rows of the launch in one correction
        PlugCorrParams cp{xc, lda_m, plug_idx, reinterpret_cast<const uint2*>(plug_vals), wbase, base_lo32,
                          (int)Mc, (int)N, (int)K, (int)cdiv(K, 64), corr, Mc * N, xt};
        if ((rc = launch_plug_corr(cp, s))) return rc;
      }
      if ((rc = launch_quad_tc(xc, lda_m, codes, ldc_n, tables, scales, oc, ldo_m, ldo_n,
                               plug && !tile_plugs ? corr : nullptr, Mc * N, Mc, N, K, counters, slots,
                               tile_plugs ? uplugs : nullptr, tile_plugs ? uplug_off : nullptr, s)))
        return rc;
    }
    return PP_OK;
  }
  QuadParams prm{};
  if (gather) prm.gather = *gather;
  prm.ldx_m = lda_m;
  prm.ldx_k = lda_k;
  prm.codes = codes;
  prm.ldc = nk ? ldc_n : ldc_k;
  for (int i = 0; i < 7; ++i) prm.luts[i] = luts ? reinterpret_cast<const __half*>(luts[i]) : nullptr;
  prm.tables = reinterpret_cast<const uint8_t*>(tables);
  for (int i = 0; i < 4; ++i) prm.scale[i] = scales[i];
  prm.ldo_m = ldo_m;
  prm.ldo_n = ldo_n;
  prm.N = (int)N;
  prm.K = (int)K;
  if (cdiv(N, nk ? 8 : 32) * cdiv(K, nk ? 64 : 16) >= (int64_t)INT32_MAX) {
    set_error("matrix too large for one launch (more than 2^31 work units)");
    return PP_ERR_INVALID;
  }
  // codes as a 2D tensor for TMA: NK rows n of K codes, KN rows k of N codes
  if ((rc = nk ? encode_tmap_u32_2d(&prm.tmap, codes, (uint64_t)K, (uint64_t)N, (uint64_t)ldc_n * 4, 32, 8)
               : encode_tmap_u32_2d(&prm.tmap, codes, (uint64_t)N, (uint64_t)K, (uint64_t)ldc_k * 4, 32, 16)))
    return rc;
  const size_t csz = plug ? corr_bytes(N) : 0;
  const size_t plan_bytes = quad_plan(nk, M < 16 ? M : 16, N, K, sms).total();
  const size_t need = plan_bytes + csz + (plug && M > 1 ? xt_bytes(K) : 0);
  if (ws_bytes < need || (need && !ws) || !aligned(ws, 256)) {
    set_error("workspace of %zu bytes (256-byte aligned, zero-filled) required, got %zu", need, ws_bytes);
    return PP_ERR_WORKSPACE;
  }
  float* corr = plug ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kCounterBytes) : nullptr;
  __half* xt = plug && M > 1 ? reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(ws) + plan_bytes + csz)
                             : nullptr;
  // batch rows in chunks of 16: each chunk is one launch over the codes
  for (int64_t m0 = 0; m0 < M; m0 += 16) {
    const int64_t Mc = (M - m0) < 16 ? (M - m0) : 16;
    const PartitionPlan pl = quad_plan(nk, Mc, N, K, sms, prm.cta_start);
    for (int c = 0; c < pl.grid; ++c)  // warp split in 32-bit arithmetic (warp_start)
      if ((int64_t)(prm.cta_start[c + 1] - prm.cta_start[c]) * quad_warps(nk, Mc > 8 ? 2 : 1) >= INT32_MAX) {
        set_error("matrix too large for one launch (units per thread block)");
        return PP_ERR_INVALID;
      }
    prm.x = reinterpret_cast<const __half*>(a) + m0 * lda_m;
    for (int i = 0; i < 4; ++i) prm.out[i] = reinterpret_cast<__half*>(out[i]) + m0 * ldo_m;
    prm.M = (int)Mc;
    prm.corr = corr;
    if (uplugs && fused_plugs_ok(pl, prm.cta_start, Mc)) {
      prm.corr = nullptr;
      prm.uplugs = uplugs;
      prm.uplug_off = uplug_off;
      if ((rc = launch_plan(pl, nk, Mc, prm, ws, csz, s, true))) return rc;
      continue;
    }
    if (uplugs && Mc == 1) {  // too long for one launch's offset tables: row chunks
      bool done = false;
      if ((rc = launch_fused_chunks(prm, codes, ldc_n, ldo_n, N, K, sms, uplugs, uplug_off, ws, csz, s, &done)))
        return rc;
      if (done) continue;
    }
    if (plug) {
      PlugCorrParams cp{prm.x, lda_m, plug_idx, reinterpret_cast<const uint2*>(plug_vals), wbase, base_lo32,
                        (int)Mc, (int)N, (int)K, (int)cdiv(K, 64), corr, Mc * N, xt};
      if ((rc = launch_plug_corr(cp, s))) return rc;
    }
    if ((rc = launch_plan(pl, nk, Mc, prm, ws, csz, s))) return rc;
  }
  return PP_OK;
}

// ------------------------------------------------------------ grouped --
namespace {

bool g_group_attr_done[128];  // [0, 64): shared activations, [64, 128): per-model rows, by device
int g_group_attr_limit[128];

struct GroupPlan {
  int count = 0, grid = 0;
  bool one_launch = false;
  int first_cta[kMaxGroup + 1];
  size_t ws_off[kMaxGroup + 1];  // workspace region of member j: [ws_off[j], ws_off[j + 1])
  PartitionPlan pl[kMaxGroup];
  int starts[kMaxGroup][kMaxCtaTable + 1];
};

// Member j takes CTAs in proportion to its units (at least one), planned as
// a launch of its own on that many SMs.  One launch needs every member to be
// a batch-1 fused-plug Linear on the vector path whose warps' unit ranges
// fit their offset tables; otherwise the members run one after another.
int plan_group(int count, const pp_quad_linear_desc* d, int sms, GroupPlan* g) {
  g->count = count;
  g->one_launch = count >= 1 && count <= kMaxGroup;
  int64_t units[kMaxGroup] = {0}, total = 0;
  for (int j = 0; j < count && g->one_launch; ++j) {
    const pp_quad_linear_desc& m = d[j];
    const bool xok = m.x && m.ldx_k == 1 && aligned(m.x, 8) && (m.ldx_m * 2) % 8 == 0 && m.flags == d[0].flags &&
                     (m.flags & ~PP_QUAD_PER_MODEL_X) == 0;
    if (m.M != 1 || m.N <= 0 || m.K <= 0 || !m.tables || !m.unit_plugs || !m.unit_plug_off || !m.plug_vals ||
        !m.plug_idx || !m.plug_window_base || !xok || !quad_vector_ok(true, m.codes, 1, m.ldw, m.N, m.K) ||
        m.N > INT32_MAX || m.K > INT32_MAX) {
      g->one_launch = false;
      break;
    }
    units[j] = cdiv(m.N, 8) * cdiv(m.K, 64);
    total += units[j];
  }
  if (g->one_launch && total > 0) {
    int cap[kMaxGroup], used = 0;
    for (int j = 0; j < count; ++j) {
      cap[j] = (int)((int64_t)sms * units[j] / total);
      if (cap[j] < 1) cap[j] = 1;
      used += cap[j];
    }
    while (used > sms) {  // take back from the largest share
      int big = 0;
      for (int j = 1; j < count; ++j)
        if (cap[j] > cap[big]) big = j;
      if (cap[big] <= 1) break;
      --cap[big];
      --used;
    }
    while (used < sms) {  // hand out what rounding left, to the members with the most units per CTA
      int best = 0;
      for (int j = 1; j < count; ++j)
        if (units[j] * cap[best] > units[best] * cap[j]) best = j;
      ++cap[best];
      ++used;
    }
    g->first_cta[0] = 0;
    g->ws_off[0] = 0;
    for (int j = 0; j < count; ++j) {
      const pp_quad_linear_desc& m = d[j];
      g->pl[j] = quad_plan(true, 1, m.N, m.K, cap[j] < kMaxCtaTable ? cap[j] : kMaxCtaTable, g->starts[j]);
      if (!fused_plugs_ok(g->pl[j], g->starts[j], 1)) {
        g->one_launch = false;
        break;
      }
      g->first_cta[j + 1] = g->first_cta[j] + g->pl[j].grid;
      g->ws_off[j + 1] = g->ws_off[j] + align_up(g->pl[j].total(), 256);
    }
    if (g->one_launch) g->grid = g->first_cta[count];
    if (g->one_launch && used > sms) g->one_launch = false;
  } else {
    g->one_launch = false;
  }
  return PP_OK;
}

int group_run(int count, const pp_quad_linear_desc* d, const PeerGather* gather, const int64_t* gather_row0,
              void* ws, size_t ws_bytes, cudaStream_t s) {
  if (count < 0 || (count > 0 && !d)) {
    set_error("group: count must be >= 0 and descriptors non-NULL");
    return PP_ERR_INVALID;
  }
  if (count == 0) return PP_OK;
  const int sms = device_sm_count(current_device());
  if (sms <= 0) {
    set_error("cannot query the SM count of the current device");
    return PP_ERR_CUDA;
  }
  GroupPlan g;
  plan_group(count, d, sms, &g);
  bool extra = false;  // flags or an epilogue: the one-launch path only
  for (int j = 0; j < count; ++j) {
    extra |= d[j].flags != 0;
    for (int k = 0; k < 4; ++k) extra |= d[j].bias[k] != nullptr || d[j].resid[k] != nullptr;
  }
  if (!g.one_launch) {
    if (gather || extra) {
      set_error("a gathered group, per-model activations and epilogues need every member on the one-launch path "
                "(batch 1, unit plugs, vector path, same flags, at most %d members, fits its SM share)", kMaxGroup);
      return PP_ERR_INVALID;
    }
    for (int j = 0; j < count; ++j) {  // one after another, sharing the workspace
      const pp_quad_linear_desc& m = d[j];
      int rc = pp_quad_linear_fused(m.x, m.ldx_m, m.ldx_k, m.codes, m.ldw, m.plug_idx, m.plug_vals,
                                    m.plug_window_base, m.base_lo32, m.unit_plugs, m.unit_plug_off, m.tables,
                                    m.scales, m.out, m.ldo_m, m.ldo_n, m.M, m.N, m.K, ws, ws_bytes, s);
      if (rc) return rc;
    }
    return PP_OK;
  }
  if (ws_bytes < g.ws_off[count] || !ws || !aligned(ws, 256)) {
    set_error("workspace of %zu bytes (256-byte aligned, zero-filled) required, got %zu", g.ws_off[count], ws_bytes);
    return PP_ERR_WORKSPACE;
  }
  const bool diag = (d[0].flags & PP_QUAD_PER_MODEL_X) != 0;
  auto kern = diag ? quad_group_kernel<true, 1, true, true> : quad_group_kernel<true, 1, true, false>;
  int max_smem = 0;
  int rc = diag ? ensure_smem_attr(kern, g_group_attr_done + 64, g_group_attr_limit + 64, &max_smem)
                : ensure_smem_attr(kern, g_group_attr_done, g_group_attr_limit, &max_smem);
  if (rc) return rc;
  constexpr int NW = quad_warps(true, 1);
  const uint32_t redb = quad_scratch_bytes(true, 1, 1);
  const int stages = quad_stages(NW, redb, (uint32_t)reserved_smem(current_device()), (uint32_t)max_smem, kPlugCap);
  if (stages == 0) {
    set_error("no shared memory layout fits the per-CTA limit %d", max_smem);
    return PP_ERR_INVALID;
  }
  static thread_local QuadGroupParams gp;  // ~12 KB: kept off the stack
  gp = QuadGroupParams{};
  gp.count = count;
  for (int j = 0; j <= count; ++j) gp.first_cta[j] = g.first_cta[j];
  uint8_t* wsb = reinterpret_cast<uint8_t*>(ws);
  for (int j = 0; j < count; ++j) {
    const pp_quad_linear_desc& m = d[j];
    void* const unused_out[4] = {m.codes ? const_cast<uint32_t*>(m.codes) : nullptr, nullptr, nullptr, nullptr};
    void* const probe[4] = {unused_out[0], unused_out[0], unused_out[0], unused_out[0]};
    // a gathered member writes the gather buffers, not out[]
    if ((rc = check_common(nullptr, m.tables, m.scales, gather ? probe : m.out, m.M, m.N, m.K))) return rc;
    if (!aligned(m.plug_vals, 8) || !aligned(m.unit_plugs, 16) || !aligned(m.unit_plug_off, 4) ||
        !aligned(m.x_il, 8)) {
      set_error("group member %d: plug_vals and x_il must be 8-byte, unit plugs 16-byte aligned", j);
      return PP_ERR_INVALID;
    }
    QuadParams& prm = gp.m[j];
    if ((rc = encode_tmap_u32_2d(&prm.tmap, m.codes, (uint64_t)m.K, (uint64_t)m.N, (uint64_t)m.ldw * 4, 32, 8)))
      return rc;
    prm.x = reinterpret_cast<const __half*>(m.x);
    prm.ldx_m = m.ldx_m;
    prm.ldx_k = m.ldx_k;
    prm.codes = m.codes;
    prm.ldc = m.ldw;
    prm.tables = reinterpret_cast<const uint8_t*>(m.tables);
    for (int i = 0; i < 4; ++i) {
      prm.scale[i] = m.scales[i];
      prm.out[i] = reinterpret_cast<__half*>(m.out[i]);
    }
    prm.ldo_m = m.ldo_m;
    prm.ldo_n = m.ldo_n;
    for (int i = 0; i < 4; ++i) {
      prm.bias[i] = reinterpret_cast<const __half*>(m.bias[i]);
      prm.resid[i] = reinterpret_cast<const __half*>(m.resid[i]);
    }
    prm.xil = diag ? reinterpret_cast<const __half*>(m.x_il) : nullptr;
    prm.M = 1;
    prm.N = (int)m.N;
    prm.K = (int)m.K;
    prm.corr = nullptr;
    prm.uplugs = reinterpret_cast<const uint8_t*>(m.unit_plugs);
    prm.uplug_off = m.unit_plug_off;
    prm.pcap = kPlugCap;
    prm.part.units = (int)g.pl[j].units;
    prm.part.upt = (int)g.pl[j].upt;
    prm.part.counters = reinterpret_cast<int*>(wsb + g.ws_off[j]);
    prm.part.slots = reinterpret_cast<float*>(wsb + g.ws_off[j] + g.pl[j].counters_bytes);
    for (int c = 0; c <= g.pl[j].grid; ++c) prm.cta_start[c] = g.starts[j][c];
    prm.stages = stages;
    prm.smem_bytes = (uint32_t)max_smem;
    prm.layout_base = (uint32_t)reserved_smem(current_device());
    prm.layout = quad_layout(prm.layout_base, prm.smem_bytes, NW, stages, redb, true, kPlugCap);
    if (gather) {
      prm.gather = *gather;
      prm.gather.row0 = gather_row0[j];
      prm.gather.ctas = g.grid;  // one completion count over the whole launch
      prm.gather.vec = (prm.gather.ld % 8 == 0 && prm.gather.row0 % 8 == 0) ? 1 : 0;
      for (int q = 0; q < prm.gather.world; ++q)
        if (!aligned(prm.gather.out[q], 16)) prm.gather.vec = 0;
      prm.gather.done = reinterpret_cast<uint32_t*>(reinterpret_cast<int*>(wsb) + (kMaxGrid - 2));
    }
  }
  return launch_kernel("quad_group_kernel", launch_overlap(), kern, dim3(g.grid), dim3(NW * 32), (size_t)max_smem,
                       s, gp);
}

}  // namespace

}  // namespace pp

extern "C" {

int pp_quad_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t ldc_k, int64_t ldc_n,
                                 size_t* bytes) {
  if (!bytes || M < 0 || N < 0 || K < 0) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  const bool nk = ldc_k == 1 && ldc_n != 1;
  *bytes = pp::quad_ws_bytes(nk, M, N, K, false);
  return PP_OK;
}

int pp_quad_gemm(const void* a, int64_t lda_m, int64_t lda_k, const uint32_t* codes, int64_t ldc_k,
                 int64_t ldc_n, const void* const luts[7], const float scales[4], void* const out[4],
                 int64_t ldo_m, int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* workspace,
                 size_t workspace_bytes, void* stream) {
  return pp::quad_run(a, lda_m, lda_k, codes, ldc_k, ldc_n, nullptr, nullptr, nullptr, 0u, nullptr, nullptr, luts,
                      nullptr, scales,
                      out, ldo_m, ldo_n, M, N, K, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream), false);
}

int pp_quad_gemm_prepared(const void* a, int64_t lda_m, int64_t lda_k, const uint32_t* codes, int64_t ldc_k,
                          int64_t ldc_n, const void* tables, const float scales[4], void* const out[4],
                          int64_t ldo_m, int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* workspace,
                          size_t workspace_bytes, void* stream) {
  if (!tables) {
    pp::set_error("tables must not be NULL");
    return PP_ERR_INVALID;
  }
  return pp::quad_run(a, lda_m, lda_k, codes, ldc_k, ldc_n, nullptr, nullptr, nullptr, 0u, nullptr, nullptr,
                      nullptr, tables, scales, out, ldo_m, ldo_n, M, N, K, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream), false);
}

int pp_quad_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, size_t* bytes) {
  if (!bytes || M < 0 || N < 0 || K < 0) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  *bytes = pp::quad_ws_bytes(true, M, N, K, true);
  return PP_OK;
}

int pp_quad_linear(const void* x, int64_t ldx_m, int64_t ldx_k, const uint32_t* codes, int64_t ldw,
                   const uint32_t* plug_idx, const void* plug_vals, const uint32_t* plug_window_base,
                   uint32_t base_lo32, const void* const luts[7], const float scales[4], void* const out[4],
                   int64_t ldo_m, int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* workspace,
                   size_t workspace_bytes, void* stream) {
  return pp::quad_run(x, ldx_m, ldx_k, codes, 1, ldw, plug_idx, plug_vals, plug_window_base, base_lo32, nullptr,
                      nullptr, luts, nullptr, scales, out, ldo_m, ldo_n, M, N, K, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream), true);
}

int pp_quad_linear_prepared(const void* x, int64_t ldx_m, int64_t ldx_k, const uint32_t* codes, int64_t ldw,
                            const uint32_t* plug_idx, const void* plug_vals, const uint32_t* plug_window_base,
                            uint32_t base_lo32, const void* tables, const float scales[4], void* const out[4],
                            int64_t ldo_m, int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!tables) {
    pp::set_error("tables must not be NULL");
    return PP_ERR_INVALID;
  }
  return pp::quad_run(x, ldx_m, ldx_k, codes, 1, ldw, plug_idx, plug_vals, plug_window_base, base_lo32, nullptr,
                      nullptr, nullptr, tables, scales, out, ldo_m, ldo_n, M, N, K, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream), true);
}

int pp_quad_linear_fused(const void* x, int64_t ldx_m, int64_t ldx_k, const uint32_t* codes, int64_t ldw,
                         const uint32_t* plug_idx, const void* plug_vals, const uint32_t* plug_window_base,
                         uint32_t base_lo32, const void* unit_plugs, const uint32_t* unit_plug_off,
                         const void* tables, const float scales[4], void* const out[4], int64_t ldo_m,
                         int64_t ldo_n, int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (!tables || (unit_plugs && (!unit_plug_off || !plug_vals))) {
    pp::set_error("tables must not be NULL; unit plugs need their offsets and the plug table");
    return PP_ERR_INVALID;
  }
  return pp::quad_run(x, ldx_m, ldx_k, codes, 1, ldw, plug_idx, plug_vals, plug_window_base, base_lo32,
                      reinterpret_cast<const uint8_t*>(unit_plugs), unit_plug_off, nullptr, tables, scales, out,
                      ldo_m, ldo_n, M, N, K, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream),
                      true);
}

int pp_quad_linear_group_workspace_bytes(int count, const pp_quad_linear_desc* descs, size_t* bytes) {
  if (!bytes || count < 0 || (count > 0 && !descs)) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  *bytes = 0;
  if (count == 0) return PP_OK;
  const int sms = pp::device_sm_count(pp::current_device());
  pp::GroupPlan g;
  pp::plan_group(count, descs, sms > 0 ? sms : 148, &g);
  if (g.one_launch) {
    *bytes = g.ws_off[count];
    return PP_OK;
  }
  for (int j = 0; j < count; ++j) {  // members one after another
    const size_t b = pp::quad_ws_bytes(true, descs[j].M, descs[j].N, descs[j].K, true);
    if (b > *bytes) *bytes = b;
  }
  return PP_OK;
}

int pp_quad_linear_group_single_launch(int count, const pp_quad_linear_desc* descs) {
  if (count < 1 || count > pp::kMaxGroup || !descs) return 0;
  const int sms = pp::device_sm_count(pp::current_device());
  pp::GroupPlan g;
  pp::plan_group(count, descs, sms > 0 ? sms : 148, &g);
  return g.one_launch ? 1 : 0;
}

int pp_quad_linear_group(int count, const pp_quad_linear_desc* descs, void* workspace, size_t workspace_bytes,
                         void* stream) {
  return pp::group_run(count, descs, nullptr, nullptr, workspace, workspace_bytes,
                       reinterpret_cast<cudaStream_t>(stream));
}

int pp_quad_linear_group_gather(int count, const pp_quad_linear_desc* descs, int world, void* const gather_out[],
                                int64_t gather_ld, const int64_t* gather_row0, uint32_t* const gather_flag[],
                                uint32_t* gather_epoch, void* workspace, size_t workspace_bytes, void* stream) {
  if (world < 1 || world > pp::kMaxPeers || !gather_out || !gather_flag || !gather_epoch || !gather_row0 ||
      count < 1 || !descs) {
    pp::set_error("group gather: world must be 1..%d, buffers, flags, rows and epoch non-NULL, count >= 1",
                  pp::kMaxPeers);
    return PP_ERR_INVALID;
  }
  pp::PeerGather g{};
  for (int q = 0; q < world; ++q) {
    if (!gather_out[q] || !gather_flag[q] || !pp::aligned(gather_out[q], 2) || !pp::aligned(gather_flag[q], 4)) {
      pp::set_error("gather buffer or flag of rank %d is NULL or misaligned", q);
      return PP_ERR_INVALID;
    }
    g.out[q] = reinterpret_cast<__half*>(gather_out[q]);
    g.flag[q] = gather_flag[q];
  }
  for (int j = 0; j < count; ++j)
    if (gather_ld < descs[j].N || gather_row0[j] < 0) {
      pp::set_error("group gather: member %d needs ld >= N and row0 >= 0", j);
      return PP_ERR_INVALID;
    }
  g.ld = gather_ld;
  g.epoch = gather_epoch;
  g.world = world;
  return pp::group_run(count, descs, &g, gather_row0, workspace, workspace_bytes,
                       reinterpret_cast<cudaStream_t>(stream));
}

int pp_quad_linear_gather(const void* x, int64_t ldx_k, const uint32_t* codes, int64_t ldw,
                          const uint32_t* plug_idx, const void* plug_vals, const uint32_t* plug_window_base,
                          uint32_t base_lo32, const void* unit_plugs, const uint32_t* unit_plug_off,
                          const void* tables, const float scales[4], int world, void* const gather_out[],
                          int64_t gather_ld, int64_t gather_row0, uint32_t* const gather_flag[],
                          uint32_t* gather_epoch, int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (!tables || (unit_plugs && (!unit_plug_off || !plug_vals))) {
    pp::set_error("tables must not be NULL; unit plugs need their offsets and the plug table");
    return PP_ERR_INVALID;
  }
  if (world < 1 || world > pp::kMaxPeers || !gather_out || !gather_flag || !gather_epoch || gather_ld < N ||
      gather_row0 < 0) {
    pp::set_error("gather: world must be 1..%d, buffers, flags and epoch non-NULL, ld >= N, row0 >= 0",
                  pp::kMaxPeers);
    return PP_ERR_INVALID;
  }
  pp::PeerGather g{};
  for (int q = 0; q < world; ++q) {
    if (!gather_out[q] || !gather_flag[q] || !pp::aligned(gather_out[q], 2) || !pp::aligned(gather_flag[q], 4)) {
      pp::set_error("gather buffer or flag of rank %d is NULL or misaligned", q);
      return PP_ERR_INVALID;
    }
    g.out[q] = reinterpret_cast<__half*>(gather_out[q]);
    g.flag[q] = gather_flag[q];
  }
  g.ld = gather_ld;
  g.row0 = gather_row0;
  g.epoch = gather_epoch;
  g.world = world;
  // the ordinary output pointers are not written when gathering; the checks want them set
  void* out[4];
  for (int i = 0; i < 4; ++i) out[i] = g.out[0] + (int64_t)i * gather_ld + gather_row0;
  return pp::quad_run(x, K, ldx_k, codes, 1, ldw, plug_idx, plug_vals, plug_window_base, base_lo32,
                      reinterpret_cast<const uint8_t*>(unit_plugs), unit_plug_off, nullptr, tables, scales, out, 1,
                      1, 1, N, K, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), true, &g);
}

}  // extern "C"
