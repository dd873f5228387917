// The operations of a decoder step that sit between the packed Linears, for
// the four models of a `.quadpack` decoding one token each: embedding row
// gather, RMSNorm, grouped-query decode attention over the KV cache with the
// rotary embedding and the cache append of the token fused in, SwiGLU.  Every launch handles the four
// models' rows (row m belongs to model m).  The reference serves these models
// through Hugging Face Qwen2 modules (polar_inference.py:224-229 calls
// model.generate); the arithmetic follows those modules' FP16 steps:
//   RMSNorm   y = fp16(w * fp16(x * rsqrt(mean(x^2) + eps)))   (FP32 statistics)
//   RoPE      q' = fp16(fp16(q * cos) + fp16(rotate_half(q) * sin)), cos/sin FP16
//   attention softmax(q k^T * scale) v with FP32 scores, sums and weights
//   SwiGLU    y = fp16(fp16(silu(g)) * u)                       (silu in FP32)
// The position of the token is read from device memory, so a captured CUDA
// graph of the step can be replayed for every position.  Every kernel is
// launched with launch overlap (programmatic dependent launch) and lets the
// next launch of its stream start at once (griddepcontrol): before
// griddepcontrol.wait a kernel reads only what no launch of the step writes
// (norm weights; for attention the position and the cache rows of earlier
// tokens, whose copies into shared memory start there), and a packed Linear
// launched after it streams its tables and first codes meanwhile.
#include <cuda_fp16.h>
#include <math.h>

#include "pp_common.cuh"
#include "pp_host.h"

namespace pp {
namespace {

constexpr int kModels = 4;

// An optional wait for a gathered buffer (the row-sharded Linears of several
// GPUs store their outputs into every rank's buffer and publish an epoch per
// launch, pp_peer.h): before reading the buffer, thread 0 of every block
// polls until each rank's flag word has reached this rank's epoch count, at
// most about a second; a rank that never publishes sets *status to 3 and the
// block goes on.  flags == NULL: no wait.
struct GatherWait {
  const uint32_t* flags;  // this rank's flag array of the buffer, one word per rank
  const uint32_t* epoch;  // this rank's launches into the buffer
  int* status;
  int world;
};

__device__ __forceinline__ void gather_wait_block(const GatherWait& w) {
  if (w.flags == nullptr) return;
  if (threadIdx.x == 0) {
    const uint32_t e = *w.epoch;
    for (int q = 0; q < w.world; ++q) {
      int i = 0;
      for (; i < (1 << 24); ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(w.flags + q) : "memory");
        if ((int32_t)(v - e) >= 0) break;
        __nanosleep(64);
      }
      if (i == (1 << 24) && w.status) atomicExch(w.status, 3);
    }
  }
  __syncthreads();
}

inline GatherWait make_wait(const uint32_t* flags, int world, const uint32_t* epoch, int* status) {
  return GatherWait{flags, epoch, status, world};
}

struct EmbedParams {
  const int* tokens;          // [4] token id per model (device)
  const __half* table[kModels];  // [vocab][H] per model
  __half* h;                  // [4][ldh]
  int64_t ldh;
  int H, vocab;
  int* status;                // token out of range: 4 and a zero row
};

__global__ void embed_kernel(const EmbedParams p) {
  pdl_launch_dependents();  // the next packed Linear may start its weight-only prologue
  pdl_wait();
  const int m = blockIdx.x;
  const int tok = p.tokens[m];
  const bool ok = tok >= 0 && tok < p.vocab;
  if (!ok && threadIdx.x == 0 && p.status) atomicExch(p.status, 4);
  const __half* src = p.table[m] + (int64_t)(ok ? tok : 0) * p.H;
  for (int i = threadIdx.x; i < p.H; i += blockDim.x) p.h[m * p.ldh + i] = ok ? src[i] : __float2half(0.f);
}

struct NormParams {
  GatherWait wait;
  const __half* x;
  int64_t ldx;
  const __half* w[kModels];
  __half* y;
  int64_t ldy;
  __half* y_il;  // optional interleaved copy: y_il[4 * i + m] = y[m][i]
  int H;
  float eps;
};

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];  // same order in every thread
  return s;
}

__device__ __forceinline__ uint2 pack4(const __half (&v)[kModels]) {
  return make_uint2((uint32_t)__half_as_ushort(v[0]) | ((uint32_t)__half_as_ushort(v[1]) << 16),
                    (uint32_t)__half_as_ushort(v[2]) | ((uint32_t)__half_as_ushort(v[3]) << 16));
}

constexpr int kNormThreads = 512;
constexpr int kNormPer = 8;  // elements a thread keeps in registers (rows up to 4096)

// CTA m normalises model m's row (one CTA per model keeps the four
// reductions in parallel; the interleaved copy is written element by element).
__global__ void rmsnorm_kernel(const NormParams p) {
  __shared__ float red[32];
  pdl_launch_dependents();  // the next packed Linear may start its weight-only prologue
  const int m = blockIdx.x;
  const __half* w = m == 0 ? p.w[0] : m == 1 ? p.w[1] : m == 2 ? p.w[2] : p.w[3];
  float wv[kNormPer];  // the norm weights do not depend on the previous launch
#pragma unroll
  for (int j = 0; j < kNormPer; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    wv[j] = i < p.H ? __half2float(w[i]) : 0.f;
  }
  pdl_wait();
  gather_wait_block(p.wait);
  const __half* x = p.x + m * p.ldx;
  float xv[kNormPer];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormPer; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    xv[j] = i < p.H ? __half2float(x[i]) : 0.f;
    ss = fmaf(xv[j], xv[j], ss);
  }
  for (int i = threadIdx.x + kNormPer * kNormThreads; i < p.H; i += kNormThreads) {
    const float v = __half2float(x[i]);
    ss = fmaf(v, v, ss);
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)p.H + p.eps);
  __half* y = p.y + m * p.ldy;
  __half* yil = p.y_il;
#pragma unroll
  for (int j = 0; j < kNormPer; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < p.H) {
      const __half v = __float2half_rn(wv[j] * __half2float(__float2half_rn(xv[j] * r)));
      y[i] = v;
      if (yil) yil[4 * i + m] = v;
    }
  }
  for (int i = threadIdx.x + kNormPer * kNormThreads; i < p.H; i += kNormThreads) {
    const __half n = __float2half_rn(__half2float(x[i]) * r);
    const __half v = __float2half_rn(__half2float(w[i]) * __half2float(n));
    y[i] = v;
    if (yil) yil[4 * i + m] = v;
  }
}

constexpr int kHeadDim = 128;                 // 4 dimensions per lane where a warp holds one head
constexpr int kAttnWarps = 8;                 // warps per CTA; each walks 32-position tiles
constexpr int kTile = 32;                     // cache positions per warp tile
constexpr int kRowBytes = kHeadDim * 2 + 16;  // padded shared row: ldmatrix without bank conflicts
constexpr int kPRowBytes = (kTile + 8) * 2;   // probabilities row (one head, the tile's positions)
constexpr int kPartStride = kHeadDim + 4;     // floats per partial: acc, max, sum, 2 unused (16-byte rows)
constexpr int kCombineBatch = 16;             // partials whose loads the combine issues together

// Shared memory of the attention CTA with NT tiles of 8 query heads:
// the group's rotated queries, then per warp its key and value tile rows,
// its probabilities and its barrier.
template <int NT>
struct AttnSmem {
  static constexpr int kQ = 0;
  static constexpr int kWarp0 = NT * 8 * kRowBytes;
  static constexpr int kK = 0;
  static constexpr int kV = kTile * kRowBytes;
  static constexpr int kP = 2 * kTile * kRowBytes;
  static constexpr int kBar = kP + NT * 8 * kPRowBytes;
  static constexpr int kWarpBytes = (kBar + 8 + 15) / 16 * 16;
  static constexpr int kBytes = kWarp0 + kAttnWarps * kWarpBytes;
};

struct AttnParams {
  GatherWait wait;
  const __half* qkv;      // [4][ldq]: the token's nq query, nkv key and nkv value heads (not rotated)
  int64_t ldq;
  const __half* cos_t;    // [max_pos][hd] FP16 rotation tables (both halves)
  const __half* sin_t;
  __half* kc[kModels];    // [max_pos][nkv][hd] per model: rotated keys
  __half* vc[kModels];
  const int* pos;         // the token's position: keys 0..pos are attended
  __half* out;            // [4][ldo]: nq heads x hd
  int64_t ldo;
  __half* out_il;         // optional interleaved copy: out_il[4 * i + m] = out[m][i]
  float* part;            // [4][nq][splits * kAttnWarps][kPartStride] partials (acc, max, sum)
  int* cnt;               // [4][nkv] split arrivals (zero between launches)
  int* status;            // position outside the cache: 5; a tile that never arrived: 1
  int nq, nkv, splits, max_pos;
  float scale;
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void sts_u2(uint32_t saddr, uint2 v) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(saddr), "r"(v.x), "r"(v.y) : "memory");
}

__device__ __forceinline__ void sts_zero16(uint32_t saddr) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(saddr), "r"(0u) : "memory");
}

__device__ __forceinline__ void sts_u16(uint32_t saddr, __half v) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(saddr), "h"(__half_as_ushort(v)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Rotary embedding of the four dimensions 4l..4l+3 a lane holds of a head
// (v: those dimensions, FP32 of FP16; c, s: the same dimensions of the
// position's cos / sin rows): the pair of dimension d < hd/2 is d + hd/2,
// held by lane l ^ 16.  q' = fp16(fp16(q cos) + fp16(rotate_half(q) sin)).
__device__ __forceinline__ uint2 rope4(const uint2 x, const uint2 c, const uint2 s, int lane) {
  const float2 x01 = __half22float2(u2h(x.x)), x23 = __half22float2(u2h(x.y));
  const float2 c01 = __half22float2(u2h(c.x)), c23 = __half22float2(u2h(c.y));
  const float2 s01 = __half22float2(u2h(s.x)), s23 = __half22float2(u2h(s.y));
  const float v[4] = {x01.x, x01.y, x23.x, x23.y};
  const float cv[4] = {c01.x, c01.y, c23.x, c23.y}, sv[4] = {s01.x, s01.y, s23.x, s23.y};
  float r[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float o = __shfl_xor_sync(0xffffffffu, v[j], 16);
    const float rot = lane < 16 ? -o : o;  // rotate_half: (-x2, x1)
    r[j] = __half2float(__float2half_rn(__half2float(__float2half_rn(v[j] * cv[j])) +
                                        __half2float(__float2half_rn(rot * sv[j]))));
  }
  return make_uint2(h2u(__floats2half2_rn(r[0], r[1])), h2u(__floats2half2_rn(r[2], r[3])));
}

// Starts the copies of one warp tile: the cache rows t0.. before the token
// (the token's own row is written by the kernel), 256 bytes per key row
// and per value row, into the warp's padded shared rows.
__device__ __forceinline__ void attn_issue_tile(uint32_t ks, uint32_t vs, uint32_t bar, const __half* kg,
                                                const __half* vg, int64_t stride, int t0, int pos, int lane) {
  const int rows = max(0, min(kTile, pos - t0));
  if (lane == 0) mbar_expect_tx(bar, (uint32_t)rows * 4u * kHeadDim);
  __syncwarp();
  if (lane < rows) {
    bulk_load(ks + lane * kRowBytes, kg + (int64_t)(t0 + lane) * stride, 2 * kHeadDim, bar);
    bulk_load(vs + lane * kRowBytes, vg + (int64_t)(t0 + lane) * stride, 2 * kHeadDim, bar);
  }
}

// Split-K grouped-query decode attention on the tensor cores, with the
// rotary embedding and the KV-cache append of the token fused in.
//
// CTA (split, kv head, model) owns positions [s0, s1), split into 32-position
// tiles dealt to its 8 warps.  A tile's key and value rows arrive in shared
// memory by bulk copies that start before the kernel waits for the previous
// launch: the cache rows before the token do not depend on it.  Every warp
// serves all NT*8 query heads of the kv head at once (queries padded with
// zero heads):
//   S^T = K Q^T   m16n8k16, M = 16 positions, N = 8 heads, K = head_dim
//   online softmax per head (FP32), probabilities rounded to FP16
//   O^T += V^T P^T   M = 16 dimensions, N = 8 heads, K = 16 positions
// Each warp writes one partial (acc, max, sum) per head; the CTA whose
// arrival completes its (model, kv head) combines the partials in a fixed
// order (deterministic).  The warp whose tile holds the token rotates its
// key, writes key and value into the caches and into its tile rows, and
// zero-fills the rows after it.
template <int NT>
__global__ void __launch_bounds__(kAttnWarps * 32) decode_attention_kernel(const AttnParams p) {
  using S = AttnSmem<NT>;
  __shared__ int last;
  pdl_launch_dependents();  // the next packed Linear may start its weight-only prologue
  const int split = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
  const int group = p.nq / p.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(pp_smem);
  const uint32_t qs = base + S::kQ;
  const uint32_t wbase = base + S::kWarp0 + warp * S::kWarpBytes;
  const uint32_t ks = wbase + S::kK, vs = wbase + S::kV, ps = wbase + S::kP, bar = wbase + S::kBar;

  // the position is set before the step and the cache rows before it were
  // written by earlier steps: both are read before waiting for the previous launch
  const int pos = *p.pos;
  const bool pos_ok = pos >= 0 && pos < p.max_pos;
  const int len = pos + 1;
  const int chunk = pos_ok ? ((len + p.splits - 1) / p.splits + kTile - 1) / kTile * kTile : 0;
  const int s0 = split * chunk, s1 = min(len, s0 + chunk);
  const int64_t stride = (int64_t)p.nkv * kHeadDim;
  const __half* kg = p.kc[m] + kvh * kHeadDim;
  const __half* vg = p.vc[m] + kvh * kHeadDim;
  if (lane == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  int t0 = s0 + warp * kTile;
  if (pos_ok && t0 < s1) attn_issue_tile(ks, vs, bar, kg, vg, stride, t0, pos, lane);
  uint2 cr = make_uint2(0, 0), sr = make_uint2(0, 0);
  if (pos_ok) {
    cr = *reinterpret_cast<const uint2*>(p.cos_t + (int64_t)pos * kHeadDim + 4 * lane);
    sr = *reinterpret_cast<const uint2*>(p.sin_t + (int64_t)pos * kHeadDim + 4 * lane);
  }
  pdl_wait();
  if (!pos_ok) {
    if (threadIdx.x == 0 && split == 0 && kvh == 0 && m == 0 && p.status) atomicExch(p.status, 5);
    return;
  }
  gather_wait_block(p.wait);
  const __half* row = p.qkv + m * p.ldq;

  // the group's queries, rotated, as FP16 rows of shared memory (padding heads zero)
  for (int h = warp; h < NT * 8; h += kAttnWarps) {
    uint2 q = make_uint2(0, 0);
    if (h < group) q = rope4(*reinterpret_cast<const uint2*>(row + (kvh * group + h) * kHeadDim + 4 * lane), cr, sr, lane);
    sts_u2(qs + h * kRowBytes + 8 * lane, q);
  }
  __syncthreads();
  uint32_t qb[NT][8][2];  // B fragments of Q^T: k = dimensions, n = heads
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t r[4];
      ldsm_x4(r, qs + (nt * 8 + (lane & 7)) * kRowBytes + (32 * j + (lane >> 3) * 8) * 2);
      qb[nt][2 * j][0] = r[0];
      qb[nt][2 * j][1] = r[1];
      qb[nt][2 * j + 1][0] = r[2];
      qb[nt][2 * j + 1][1] = r[3];
    }

  float o[8][NT][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) o[i][nt][r] = 0.f;
  float mrun[NT][2], lsum[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      mrun[nt][j] = -INFINITY;
      lsum[nt][j] = 0.f;
    }
  bool any = false;
  uint32_t phase = 0;
  for (; t0 < s1; t0 += kAttnWarps * kTile) {
    if (any) {  // the slot's previous rows were read into registers: reuse it
      __syncwarp();
      fence_proxy_async_smem();
      attn_issue_tile(ks, vs, bar, kg, vg, stride, t0, pos, lane);
    }
    any = true;
    if (!mbar_wait_bounded(bar, phase, p.status)) break;
    phase ^= 1u;
    if (pos < t0 + kTile) {  // the token's tile: append the token, zero the rows after it
      const int r0 = pos - t0;
      const uint2 kr = rope4(*reinterpret_cast<const uint2*>(row + (p.nq + kvh) * kHeadDim + 4 * lane), cr, sr, lane);
      const uint2 vr = *reinterpret_cast<const uint2*>(row + (p.nq + p.nkv + kvh) * kHeadDim + 4 * lane);
      *reinterpret_cast<uint2*>(p.kc[m] + (int64_t)pos * stride + kvh * kHeadDim + 4 * lane) = kr;
      *reinterpret_cast<uint2*>(p.vc[m] + (int64_t)pos * stride + kvh * kHeadDim + 4 * lane) = vr;
      sts_u2(ks + r0 * kRowBytes + 8 * lane, kr);
      sts_u2(vs + r0 * kRowBytes + 8 * lane, vr);
      for (int i = lane; i < (kTile - 1 - r0) * 16; i += 32) {
        const uint32_t off = (r0 + 1 + (i >> 4)) * kRowBytes + (i & 15) * 16;
        sts_zero16(ks + off);
        sts_zero16(vs + off);
      }
      __syncwarp();
    }
    // S^T = K Q^T: s[mt][nt] rows = positions 16mt.., columns = heads 8nt..
    float s[2][NT][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) s[mt][nt][r] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4];
        ldsm_x4(a, ks + (16 * mt + (lane & 15)) * kRowBytes + (16 * kk + (lane >> 4) * 8) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(s[mt][nt], a[0], a[1], a[2], a[3], qb[nt][kk][0], qb[nt][kk][1]);
      }
    // online softmax per head; a thread holds heads 8nt + 2(lane&3) + j at
    // positions t0 + 16mt + (lane>>2) + 8hh
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float mx = -INFINITY;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int t = t0 + 16 * mt + (lane >> 2) + 8 * hh;
            const float v = t <= pos ? s[mt][nt][2 * hh + j] * p.scale : -INFINITY;
            s[mt][nt][2 * hh + j] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(mrun[nt][j], mx);  // finite: position t0 <= pos is in the tile
        const float corr = expf(mrun[nt][j] - mn);
        mrun[nt][j] = mn;
        float ls = lsum[nt][j] * corr;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i][nt][j] *= corr;
          o[i][nt][2 + j] *= corr;
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float e = expf(s[mt][nt][2 * hh + j] - mn);
            ls += e;
            s[mt][nt][2 * hh + j] = e;
          }
        lsum[nt][j] = ls;
      }
    // P to shared memory as [head][position] FP16, then as B fragments (k = positions)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r)
          sts_u16(ps + (nt * 8 + 2 * (lane & 3) + (r & 1)) * kPRowBytes + (16 * mt + (lane >> 2) + 8 * (r >> 1)) * 2,
                  __float2half_rn(s[mt][nt][r]));
    __syncwarp();
    uint32_t pb[NT][2][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t r[4];
      ldsm_x4(r, ps + (nt * 8 + (lane & 7)) * kPRowBytes + (lane >> 3) * 16);
      pb[nt][0][0] = r[0];
      pb[nt][0][1] = r[1];
      pb[nt][1][0] = r[2];
      pb[nt][1][1] = r[3];
    }
    // O^T += V^T P^T: o[i][nt] rows = dimensions 16i.., columns = heads 8nt..
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t a[4];
        ldsm_x4_t(a, vs + (16 * kk + (lane & 7) + ((lane >> 4) & 1) * 8) * kRowBytes + (16 * i + ((lane >> 3) & 1) * 8) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816(o[i][nt], a[0], a[1], a[2], a[3], pb[nt][kk][0], pb[nt][kk][1]);
      }
    __syncwarp();  // P and the tile rows are read before the next tile reuses them
  }

  // the warp's partial per head
  const int P = p.splits * kAttnWarps;
  const int pidx = split * kAttnWarps + warp;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float ls = lsum[nt][j];
      ls += __shfl_xor_sync(0xffffffffu, ls, 4);
      ls += __shfl_xor_sync(0xffffffffu, ls, 8);
      ls += __shfl_xor_sync(0xffffffffu, ls, 16);
      const int hq = nt * 8 + 2 * (lane & 3) + j;
      if (hq >= group) continue;
      float* rec = p.part + ((int64_t)(m * p.nq + kvh * group + hq) * P + pidx) * kPartStride;
      if (any) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          rec[16 * i + (lane >> 2)] = o[i][nt][j];
          rec[16 * i + (lane >> 2) + 8] = o[i][nt][2 + j];
        }
      }
      if (lane < 4) {
        rec[kHeadDim] = any ? mrun[nt][j] : -INFINITY;
        rec[kHeadDim + 1] = any ? ls : 0.f;
      }
    }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(p.cnt + m * p.nkv + kvh, 1) == p.splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // combine: warp w takes heads w, w + 8, ...; the lanes merge the maxima
  // and sums over the partials, then each lane's four dimensions over the
  // partials, kCombineBatch partials' loads at a time (fixed order: deterministic)
  // only the first min(8, chunk / 32) warps of a split can hold a tile:
  // the combine walks those Pe partials (c -> split c / wpc, warp c % wpc)
  const int wpc = min(kAttnWarps, chunk / kTile);
  const int Pe = p.splits * wpc;
  for (int hq = warp; hq < group; hq += kAttnWarps) {
    const int qh = kvh * group + hq;
    const float* pb_ = p.part + (int64_t)(m * p.nq + qh) * P * kPartStride;
    auto rec = [&](int c) { return pb_ + ((c / wpc) * kAttnWarps + c % wpc) * kPartStride; };
    float M = -INFINITY, L = 0.f;
    for (int sp = lane; sp < Pe; sp += 32) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(rec(sp) + kHeadDim));
      if (ml.x != -INFINITY) {
        const float mn = fmaxf(M, ml.x);
        L = L * expf(M - mn) + ml.y * expf(ml.x - mn);
        M = mn;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float M2 = __shfl_xor_sync(0xffffffffu, M, off), L2 = __shfl_xor_sync(0xffffffffu, L, off);
      const float mn = fmaxf(M, M2);
      L = (M == -INFINITY ? 0.f : L * expf(M - mn)) + (M2 == -INFINITY ? 0.f : L2 * expf(M2 - mn));
      M = mn;
    }
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    for (int sp0 = 0; sp0 < Pe; sp0 += kCombineBatch) {
      float w[kCombineBatch];
      float4 a[kCombineBatch];
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        const int sp = sp0 + u < Pe ? sp0 + u : Pe - 1;
        const float* b = rec(sp);
        const float ms = __ldcg(b + kHeadDim);
        w[u] = (sp0 + u < Pe && ms != -INFINITY) ? expf(ms - M) : 0.f;  // empty partials weigh nothing
        a[u] = __ldcg(reinterpret_cast<const float4*>(b + 4 * lane));
      }
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        if (w[u] == 0.f) continue;  // uniform over the warp; skips partials never written
        o0 += w[u] * a[u].x;
        o1 += w[u] * a[u].y;
        o2 += w[u] * a[u].z;
        o3 += w[u] * a[u].w;
      }
    }
    const float inv = 1.f / L;
    const __half2 r01 = __floats2half2_rn(o0 * inv, o1 * inv), r23 = __floats2half2_rn(o2 * inv, o3 * inv);
    __half2* op = reinterpret_cast<__half2*>(p.out + m * p.ldo + qh * kHeadDim + 4 * lane);
    op[0] = r01;
    op[1] = r23;
    if (p.out_il) {
      __half* il = p.out_il + 4 * (qh * kHeadDim + 4 * lane) + m;
      il[0] = __low2half(r01);
      il[4] = __high2half(r01);
      il[8] = __low2half(r23);
      il[12] = __high2half(r23);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) p.cnt[m * p.nkv + kvh] = 0;
}

struct SwigluParams {
  GatherWait wait;
  const __half* gu;  // [4][ldg]: gate (I values) then up (I values)
  int64_t ldg;
  __half* y;         // [4][ldy]
  int64_t ldy;
  __half* y_il;      // optional interleaved copy: y_il[4 * i + m] = y[m][i]
  int I;
};

__device__ __forceinline__ __half swiglu1(__half g_, __half u) {
  const float g = __half2float(g_);
  const __half sg = __float2half_rn(g / (1.f + expf(-g)));
  return __float2half_rn(__half2float(sg) * __half2float(u));
}

// A thread produces elements 2j, 2j + 1 of the four models: 4-byte loads and
// stores, and the interleaved copy of the pair as one 16-byte store (PAIRS:
// even I, ldg and ldy, 4-byte aligned rows, 16-byte aligned y_il); else one
// element of the four models per thread.
template <bool PAIRS>
__global__ void swiglu_kernel(const SwigluParams p) {
  pdl_launch_dependents();  // the next packed Linear may start its weight-only prologue
  pdl_wait();
  gather_wait_block(p.wait);
  const int n = PAIRS ? p.I / 2 : p.I;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
    if constexpr (PAIRS) {
      __half a[kModels], b[kModels];
#pragma unroll
      for (int m = 0; m < kModels; ++m) {
        const __half2 g = *reinterpret_cast<const __half2*>(p.gu + m * p.ldg + 2 * j);
        const __half2 u = *reinterpret_cast<const __half2*>(p.gu + m * p.ldg + p.I + 2 * j);
        a[m] = swiglu1(__low2half(g), __low2half(u));
        b[m] = swiglu1(__high2half(g), __high2half(u));
        *reinterpret_cast<__half2*>(p.y + m * p.ldy + 2 * j) = __halves2half2(a[m], b[m]);
      }
      if (p.y_il) {
        const uint2 lo = pack4(a), hi = pack4(b);
        *reinterpret_cast<uint4*>(p.y_il + 8 * j) = make_uint4(lo.x, lo.y, hi.x, hi.y);
      }
    } else {
      __half v[kModels];
#pragma unroll
      for (int m = 0; m < kModels; ++m) {
        v[m] = swiglu1(p.gu[m * p.ldg + j], p.gu[m * p.ldg + p.I + j]);
        p.y[m * p.ldy + j] = v[m];
      }
      if (p.y_il) *reinterpret_cast<uint2*>(p.y_il + 4 * j) = pack4(v);
    }
  }
}

bool g_attn_attr[2][64];
int g_attn_limit[2][64];

}  // namespace
}  // namespace pp

extern "C" {

int pp_embed_rows(const int* tokens, const void* const tables[4], int64_t vocab, int64_t H, void* h, int64_t ldh,
                  int* status, void* stream) {
  if (!tokens || !tables || !h || H <= 0 || vocab <= 0 || ldh < H || H > INT32_MAX || vocab > INT32_MAX) {
    pp::set_error("pp_embed_rows: invalid arguments");
    return PP_ERR_INVALID;
  }
  pp::EmbedParams p{};
  p.tokens = tokens;
  for (int k = 0; k < 4; ++k) {
    if (!tables[k]) {
      pp::set_error("pp_embed_rows: table %d is NULL", k);
      return PP_ERR_INVALID;
    }
    p.table[k] = reinterpret_cast<const __half*>(tables[k]);
  }
  p.h = reinterpret_cast<__half*>(h);
  p.ldh = ldh;
  p.H = (int)H;
  p.vocab = (int)vocab;
  p.status = status;
  return pp::launch_kernel("embed_kernel", pp::launch_overlap(), pp::embed_kernel, dim3(4), dim3(256), 0,
                           reinterpret_cast<cudaStream_t>(stream), p);
}

int pp_rmsnorm_rows(const void* x, int64_t ldx, const void* const w[4], int64_t H, float eps, void* y, int64_t ldy,
                    void* y_il, const uint32_t* wait_flags, int wait_world, const uint32_t* wait_epoch,
                    int* wait_status, void* stream) {
  if (wait_flags && (!wait_epoch || wait_world < 1 || wait_world > 8)) {
    pp::set_error("pp_rmsnorm_rows: a wait needs its epoch and 1..8 ranks");
    return PP_ERR_INVALID;
  }
  if (!x || !w || !y || H <= 0 || H > INT32_MAX / 4 || ldx < H || ldy < H || (y_il && !pp::aligned(y_il, 8))) {
    pp::set_error("pp_rmsnorm_rows: invalid arguments");
    return PP_ERR_INVALID;
  }
  pp::NormParams p{};
  p.x = reinterpret_cast<const __half*>(x);
  p.ldx = ldx;
  for (int k = 0; k < 4; ++k) {
    if (!w[k]) {
      pp::set_error("pp_rmsnorm_rows: weight %d is NULL", k);
      return PP_ERR_INVALID;
    }
    p.w[k] = reinterpret_cast<const __half*>(w[k]);
  }
  p.y = reinterpret_cast<__half*>(y);
  p.ldy = ldy;
  p.y_il = reinterpret_cast<__half*>(y_il);
  p.H = (int)H;
  p.eps = eps;
  p.wait = pp::make_wait(wait_flags, wait_world, wait_epoch, wait_status);
  return pp::launch_kernel("rmsnorm_kernel", pp::launch_overlap(), pp::rmsnorm_kernel, dim3(4),
                           dim3(pp::kNormThreads), 0, reinterpret_cast<cudaStream_t>(stream), p);
}

int pp_decode_attention_workspace_bytes(int64_t nq, int64_t nkv, int64_t splits, size_t* bytes) {
  if (!bytes || nq <= 0 || nkv <= 0 || splits <= 0) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  *bytes = pp::align_up((size_t)4 * nkv * sizeof(int), 256) +
           (size_t)4 * nq * splits * pp::kAttnWarps * pp::kPartStride * sizeof(float);
  return PP_OK;
}

int pp_decode_attention(void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t hd, const void* cos_t,
                        const void* sin_t, void* const k_cache[4], void* const v_cache[4], int64_t max_pos,
                        const int* pos, float scale, void* out, int64_t ldo, void* out_il, int64_t splits,
                        void* workspace,
                        size_t workspace_bytes, int* status, const uint32_t* wait_flags, int wait_world,
                        const uint32_t* wait_epoch, int* wait_status, void* stream) {
  if (wait_flags && (!wait_epoch || wait_world < 1 || wait_world > 8)) {
    pp::set_error("pp_decode_attention: a wait needs its epoch and 1..8 ranks");
    return PP_ERR_INVALID;
  }
  if (!qkv || !cos_t || !sin_t || !k_cache || !v_cache || !pos || !out || !status || hd != pp::kHeadDim ||
      nq <= 0 || nkv <= 0 || nq % nkv || nq / nkv > 16 || splits <= 0 || splits > 4096 || max_pos <= 0 ||
      max_pos > INT32_MAX || !pp::aligned(qkv, 8) || ldq % 4 || ldq < (nq + 2 * nkv) * hd || !pp::aligned(out, 4) ||
      ldo % 2 || nkv * 4 > 65535 || (out_il && !pp::aligned(out_il, 8))) {
    pp::set_error("pp_decode_attention: head_dim must be %d, nq a multiple of nkv (at most 16 q heads per kv "
                  "head), 1..4096 splits, 8-byte aligned qkv rows holding nq + 2 nkv heads, 4-byte aligned output "
                  "rows, a status word",
                  pp::kHeadDim);
    return PP_ERR_INVALID;
  }
  size_t need = 0;
  pp_decode_attention_workspace_bytes(nq, nkv, splits, &need);
  if (!workspace || workspace_bytes < need || !pp::aligned(workspace, 256)) {
    pp::set_error("pp_decode_attention: workspace of %zu bytes (256-byte aligned, zero-filled) required", need);
    return PP_ERR_WORKSPACE;
  }
  pp::AttnParams p{};
  p.qkv = reinterpret_cast<const __half*>(qkv);
  p.ldq = ldq;
  p.cos_t = reinterpret_cast<const __half*>(cos_t);
  p.sin_t = reinterpret_cast<const __half*>(sin_t);
  for (int k = 0; k < 4; ++k) {
    // the tiles arrive by 256-byte bulk copies of cache rows: 16-byte aligned caches
    if (!k_cache[k] || !v_cache[k] || !pp::aligned(k_cache[k], 16) || !pp::aligned(v_cache[k], 16)) {
      pp::set_error("pp_decode_attention: cache of model %d is NULL or not 16-byte aligned", k);
      return PP_ERR_INVALID;
    }
    p.kc[k] = reinterpret_cast<__half*>(k_cache[k]);
    p.vc[k] = reinterpret_cast<__half*>(v_cache[k]);
  }
  p.pos = pos;
  p.out = reinterpret_cast<__half*>(out);
  p.ldo = ldo;
  p.out_il = reinterpret_cast<__half*>(out_il);
  p.cnt = reinterpret_cast<int*>(workspace);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) +
                                    pp::align_up((size_t)4 * nkv * sizeof(int), 256));
  p.status = status;
  p.nq = (int)nq;
  p.nkv = (int)nkv;
  p.splits = (int)splits;
  p.max_pos = (int)max_pos;
  p.scale = scale;
  p.wait = pp::make_wait(wait_flags, wait_world, wait_epoch, wait_status);
  const bool two = nq / nkv > 8;
  auto kern = two ? pp::decode_attention_kernel<2> : pp::decode_attention_kernel<1>;
  const int smem = two ? pp::AttnSmem<2>::kBytes : pp::AttnSmem<1>::kBytes;
  int lim = 0;
  const int rc = two ? pp::ensure_smem_attr(kern, pp::g_attn_attr[1], pp::g_attn_limit[1], &lim)
                     : pp::ensure_smem_attr(kern, pp::g_attn_attr[0], pp::g_attn_limit[0], &lim);
  if (rc) return rc;
  if (lim < smem) {
    pp::set_error("pp_decode_attention: %d bytes of shared memory needed, %d available", smem, lim);
    return PP_ERR_CUDA;
  }
  return pp::launch_kernel("decode_attention_kernel", pp::launch_overlap(), kern,
                           dim3((unsigned)splits, (unsigned)nkv, 4), dim3(32 * pp::kAttnWarps), (size_t)smem,
                           reinterpret_cast<cudaStream_t>(stream), p);
}

int pp_swiglu_rows(const void* gate_up, int64_t ldg, int64_t I, void* y, int64_t ldy, void* y_il,
                   const uint32_t* wait_flags, int wait_world, const uint32_t* wait_epoch, int* wait_status,
                   void* stream) {
  if (wait_flags && (!wait_epoch || wait_world < 1 || wait_world > 8)) {
    pp::set_error("pp_swiglu_rows: a wait needs its epoch and 1..8 ranks");
    return PP_ERR_INVALID;
  }
  if (!gate_up || !y || I <= 0 || I > INT32_MAX / 4 || ldg < 2 * I || ldy < I || (y_il && !pp::aligned(y_il, 8))) {
    pp::set_error("pp_swiglu_rows: invalid arguments");
    return PP_ERR_INVALID;
  }
  pp::SwigluParams p{pp::make_wait(wait_flags, wait_world, wait_epoch, wait_status),
                     reinterpret_cast<const __half*>(gate_up), ldg, reinterpret_cast<__half*>(y), ldy,
                     reinterpret_cast<__half*>(y_il), (int)I};
  const bool pairs = I % 2 == 0 && ldg % 2 == 0 && ldy % 2 == 0 && pp::aligned(gate_up, 4) && pp::aligned(y, 4) &&
                     (!y_il || pp::aligned(y_il, 16));
  const int64_t n = pairs ? I / 2 : I;
  const unsigned gx = (unsigned)((n + 255) / 256 < 128 ? (n + 255) / 256 : 128);
  return pp::launch_kernel("swiglu_kernel", pp::launch_overlap(),
                           pairs ? pp::swiglu_kernel<true> : pp::swiglu_kernel<false>, dim3(gx), dim3(256), 0,
                           reinterpret_cast<cudaStream_t>(stream), p);
}

}  // extern "C"
