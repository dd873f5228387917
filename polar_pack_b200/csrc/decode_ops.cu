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
// graph of the step can be replayed for every position.  Each kernel lets
// the next launch of its stream start at once (griddepcontrol): a packed
// Linear launched with launch overlap then streams its tables and first
// codes while this kernel runs, and waits for it before reading activations.
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
  __syncthreads();
  return s;
}

__global__ void rmsnorm_kernel(const NormParams p) {
  __shared__ float red[32];
  pdl_launch_dependents();  // the next packed Linear may start its weight-only prologue
  gather_wait_block(p.wait);
  const int m = blockIdx.x;
  const __half* x = p.x + m * p.ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < p.H; i += blockDim.x) {
    const float v = __half2float(x[i]);
    ss = fmaf(v, v, ss);
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)p.H + p.eps);
  for (int i = threadIdx.x; i < p.H; i += blockDim.x) {
    const __half n = __float2half_rn(__half2float(x[i]) * r);
    p.y[m * p.ldy + i] = __float2half_rn(__half2float(p.w[m][i]) * __half2float(n));
  }
}

constexpr int kHeadDim = 128;  // 4 dimensions per lane
constexpr int kPartStride = kHeadDim + 4;  // floats per partial: acc, max, sum, 2 unused (16-byte rows)
constexpr int kUnroll = 4;                 // cache positions whose loads are in flight together
constexpr int kCombineBatch = 16;          // splits whose partials the combine loads together

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
  float* part;            // [4][nq][splits][kPartStride] partials (acc, max, sum)
  int* cnt;               // [4][nkv] split arrivals (zero between launches)
  int* status;            // position outside the cache: 5
  int nq, nkv, splits, max_pos;
  float scale;
};

// Rotary embedding of the four dimensions 4l..4l+3 a lane holds of a head
// (v: those dimensions, FP32 of FP16): the pair of dimension d < hd/2 is
// d + hd/2, held by lane l ^ 16.  q' = fp16(fp16(q cos) + fp16(rotate_half(q) sin)).
__device__ __forceinline__ void rope4(float (&v)[4], const __half* cs, const __half* sn, int lane) {
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = __shfl_xor_sync(0xffffffffu, v[j], 16);
  const bool lo = lane < 16;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int d = 4 * lane + j;
    const float c = __half2float(cs[d]), sn_ = __half2float(sn[d]);
    const float rot = lo ? -o[j] : o[j];  // rotate_half: (-x2, x1)
    v[j] = __half2float(__float2half_rn(__half2float(__float2half_rn(v[j] * c)) +
                                        __half2float(__float2half_rn(rot * sn_))));
  }
}

// Split-K decode attention with the rotary embedding and the KV-cache append
// of the token fused in.  CTA (split, kv head, model); warp w is query head
// kvh * group + w, rotates its query and walks keys [s0, s1) with an online
// softmax, kUnroll positions' loads at a time; lane l holds dimensions
// 4l..4l+3.  The CTA whose range holds the token's position first writes
// the token's rotated key and its value into the caches.  The CTA whose
// arrival completes its (model, kv head) combines the splits in order
// (deterministic).
__global__ void decode_attention_kernel(const AttnParams p) {
  __shared__ int last;
  pdl_launch_dependents();  // the next packed Linear may start its weight-only prologue
  gather_wait_block(p.wait);
  const int split = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
  const int group = p.nq / p.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = kvh * group + warp;
  const int pos = *p.pos;
  if (pos < 0 || pos >= p.max_pos) {
    if (threadIdx.x == 0 && split == 0 && kvh == 0 && m == 0 && p.status) atomicExch(p.status, 5);
    return;
  }
  const int len = pos + 1;
  const int chunk = (len + p.splits - 1) / p.splits;
  const int s0 = split * chunk, s1 = min(len, s0 + chunk);
  const __half* row = p.qkv + m * p.ldq;
  const __half* cs = p.cos_t + (int64_t)pos * kHeadDim;
  const __half* sn = p.sin_t + (int64_t)pos * kHeadDim;
  const int64_t stride = (int64_t)p.nkv * kHeadDim;
  if (s0 <= pos && pos < s1) {  // this CTA holds the token: append its key (rotated) and value first
    if (warp == 0) {
      const uint2 kr = *reinterpret_cast<const uint2*>(row + (p.nq + kvh) * kHeadDim + 4 * lane);
      const uint2 vr = *reinterpret_cast<const uint2*>(row + (p.nq + p.nkv + kvh) * kHeadDim + 4 * lane);
      const float2 k01 = __half22float2(u2h(kr.x)), k23 = __half22float2(u2h(kr.y));
      float kv[4] = {k01.x, k01.y, k23.x, k23.y};
      rope4(kv, cs, sn, lane);
      __half2* kd = reinterpret_cast<__half2*>(p.kc[m] + (int64_t)pos * stride + kvh * kHeadDim + 4 * lane);
      kd[0] = __floats2half2_rn(kv[0], kv[1]);
      kd[1] = __floats2half2_rn(kv[2], kv[3]);
      *reinterpret_cast<uint2*>(p.vc[m] + (int64_t)pos * stride + kvh * kHeadDim + 4 * lane) = vr;
    }
    __syncthreads();
  }
  const uint2 qr = *reinterpret_cast<const uint2*>(row + qh * kHeadDim + 4 * lane);
  const float2 q01 = __half22float2(u2h(qr.x)), q23 = __half22float2(u2h(qr.y));
  float q[4] = {q01.x, q01.y, q23.x, q23.y};
  rope4(q, cs, sn, lane);
  const __half* kb = p.kc[m] + (int64_t)kvh * kHeadDim + 4 * lane;
  const __half* vb = p.vc[m] + (int64_t)kvh * kHeadDim + 4 * lane;
  float mx = -INFINITY, sum = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int t0 = s0; t0 < s1; t0 += kUnroll) {
    uint2 kv[kUnroll], vv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int t = t0 + u < s1 ? t0 + u : s1 - 1;  // in range; duplicates are masked below
      kv[u] = *reinterpret_cast<const uint2*>(kb + t * stride);
      vv[u] = *reinterpret_cast<const uint2*>(vb + t * stride);
    }
    float sc[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const float2 k01 = __half22float2(u2h(kv[u].x)), k23 = __half22float2(u2h(kv[u].y));
      sc[u] = q[0] * k01.x + q[1] * k01.y + q[2] * k23.x + q[3] * k23.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (t0 + u >= s1) break;  // uniform over the warp
      const float s = sc[u] * p.scale;
      const float mn = fmaxf(mx, s);
      const float corr = expf(mx - mn), e = expf(s - mn);
      const float2 v01 = __half22float2(u2h(vv[u].x)), v23 = __half22float2(u2h(vv[u].y));
      sum = sum * corr + e;
      a0 = a0 * corr + e * v01.x;
      a1 = a1 * corr + e * v01.y;
      a2 = a2 * corr + e * v23.x;
      a3 = a3 * corr + e * v23.y;
      mx = mn;
    }
  }
  float* pp = p.part + (((int64_t)m * p.nq + qh) * p.splits + split) * kPartStride;
  *reinterpret_cast<float4*>(pp + 4 * lane) = make_float4(a0, a1, a2, a3);
  if (lane == 0) {
    pp[kHeadDim] = mx;
    pp[kHeadDim + 1] = sum;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(p.cnt + m * p.nkv + kvh, 1) == p.splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // combine: the maxima and sums with the lanes over the splits, then each
  // lane's four dimensions over the splits, kCombineBatch splits' loads at a
  // time (fixed order: deterministic)
  const float* base = p.part + ((int64_t)m * p.nq + qh) * p.splits * kPartStride;
  float M = -INFINITY;
  for (int sp = lane; sp < p.splits; sp += 32) M = fmaxf(M, __ldcg(base + sp * kPartStride + kHeadDim));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
  for (int sp = lane; sp < p.splits; sp += 32) {
    const float ms = __ldcg(base + sp * kPartStride + kHeadDim);
    if (ms != -INFINITY) L += expf(ms - M) * __ldcg(base + sp * kPartStride + kHeadDim + 1);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
  for (int sp0 = 0; sp0 < p.splits; sp0 += kCombineBatch) {
    float w[kCombineBatch];
    float4 a[kCombineBatch];
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      const int sp = sp0 + u < p.splits ? sp0 + u : p.splits - 1;
      const float* b = base + sp * kPartStride;
      const float ms = __ldcg(b + kHeadDim);
      w[u] = (sp0 + u < p.splits && ms != -INFINITY) ? expf(ms - M) : 0.f;  // empty splits weigh nothing
      a[u] = __ldcg(reinterpret_cast<const float4*>(b + 4 * lane));
    }
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      o0 += w[u] * a[u].x;
      o1 += w[u] * a[u].y;
      o2 += w[u] * a[u].z;
      o3 += w[u] * a[u].w;
    }
  }
  const float inv = 1.f / L;
  __half2* o = reinterpret_cast<__half2*>(p.out + m * p.ldo + qh * kHeadDim + 4 * lane);
  o[0] = __floats2half2_rn(o0 * inv, o1 * inv);
  o[1] = __floats2half2_rn(o2 * inv, o3 * inv);
  __syncthreads();
  if (threadIdx.x == 0) p.cnt[m * p.nkv + kvh] = 0;
}

struct SwigluParams {
  GatherWait wait;
  const __half* gu;  // [4][ldg]: gate (I values) then up (I values)
  int64_t ldg;
  __half* y;         // [4][ldy]
  int64_t ldy;
  int I;
};

__global__ void swiglu_kernel(const SwigluParams p) {
  pdl_launch_dependents();  // the next packed Linear may start its weight-only prologue
  gather_wait_block(p.wait);
  const int m = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.I; i += gridDim.x * blockDim.x) {
    const float g = __half2float(p.gu[m * p.ldg + i]);
    const __half sg = __float2half_rn(g / (1.f + expf(-g)));
    p.y[m * p.ldy + i] = __float2half_rn(__half2float(sg) * __half2float(p.gu[m * p.ldg + p.I + i]));
  }
}

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
  pp::embed_kernel<<<4, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return pp::check_launch("embed_kernel");
}

int pp_rmsnorm_rows(const void* x, int64_t ldx, const void* const w[4], int64_t H, float eps, void* y, int64_t ldy,
                    const uint32_t* wait_flags, int wait_world, const uint32_t* wait_epoch, int* wait_status,
                    void* stream) {
  if (wait_flags && (!wait_epoch || wait_world < 1 || wait_world > 8)) {
    pp::set_error("pp_rmsnorm_rows: a wait needs its epoch and 1..8 ranks");
    return PP_ERR_INVALID;
  }
  if (!x || !w || !y || H <= 0 || H > INT32_MAX || ldx < H || ldy < H) {
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
  p.H = (int)H;
  p.eps = eps;
  p.wait = pp::make_wait(wait_flags, wait_world, wait_epoch, wait_status);
  pp::rmsnorm_kernel<<<4, 512, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return pp::check_launch("rmsnorm_kernel");
}

int pp_decode_attention_workspace_bytes(int64_t nq, int64_t nkv, int64_t splits, size_t* bytes) {
  if (!bytes || nq <= 0 || nkv <= 0 || splits <= 0) {
    pp::set_error("invalid arguments");
    return PP_ERR_INVALID;
  }
  *bytes = pp::align_up((size_t)4 * nkv * sizeof(int), 256) +
           (size_t)4 * nq * splits * pp::kPartStride * sizeof(float);
  return PP_OK;
}

int pp_decode_attention(void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t hd, const void* cos_t,
                        const void* sin_t, void* const k_cache[4], void* const v_cache[4], int64_t max_pos,
                        const int* pos, float scale, void* out, int64_t ldo, int64_t splits, void* workspace,
                        size_t workspace_bytes, int* status, const uint32_t* wait_flags, int wait_world,
                        const uint32_t* wait_epoch, int* wait_status, void* stream) {
  if (wait_flags && (!wait_epoch || wait_world < 1 || wait_world > 8)) {
    pp::set_error("pp_decode_attention: a wait needs its epoch and 1..8 ranks");
    return PP_ERR_INVALID;
  }
  if (!qkv || !cos_t || !sin_t || !k_cache || !v_cache || !pos || !out || hd != pp::kHeadDim || nq <= 0 ||
      nkv <= 0 || nq % nkv || nq / nkv > 32 || splits <= 0 || splits > 65535 || max_pos <= 0 ||
      max_pos > INT32_MAX || !pp::aligned(qkv, 8) || ldq % 4 || ldq < (nq + 2 * nkv) * hd || !pp::aligned(out, 4) ||
      ldo % 2) {
    pp::set_error("pp_decode_attention: head_dim must be %d, nq a multiple of nkv (at most 32 q heads per kv "
                  "head), 8-byte aligned qkv rows holding nq + 2 nkv heads, 4-byte aligned output rows",
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
    if (!k_cache[k] || !v_cache[k] || !pp::aligned(k_cache[k], 8) || !pp::aligned(v_cache[k], 8)) {
      pp::set_error("pp_decode_attention: cache of model %d is NULL or not 8-byte aligned", k);
      return PP_ERR_INVALID;
    }
    p.kc[k] = reinterpret_cast<__half*>(k_cache[k]);
    p.vc[k] = reinterpret_cast<__half*>(v_cache[k]);
  }
  p.pos = pos;
  p.out = reinterpret_cast<__half*>(out);
  p.ldo = ldo;
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
  pp::decode_attention_kernel<<<dim3((unsigned)splits, (unsigned)nkv, 4), (unsigned)(32 * (nq / nkv)), 0,
                                reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return pp::check_launch("decode_attention_kernel");
}

int pp_swiglu_rows(const void* gate_up, int64_t ldg, int64_t I, void* y, int64_t ldy, const uint32_t* wait_flags,
                   int wait_world, const uint32_t* wait_epoch, int* wait_status, void* stream) {
  if (wait_flags && (!wait_epoch || wait_world < 1 || wait_world > 8)) {
    pp::set_error("pp_swiglu_rows: a wait needs its epoch and 1..8 ranks");
    return PP_ERR_INVALID;
  }
  if (!gate_up || !y || I <= 0 || I > INT32_MAX || ldg < 2 * I || ldy < I) {
    pp::set_error("pp_swiglu_rows: invalid arguments");
    return PP_ERR_INVALID;
  }
  pp::SwigluParams p{pp::make_wait(wait_flags, wait_world, wait_epoch, wait_status),
                     reinterpret_cast<const __half*>(gate_up), ldg, reinterpret_cast<__half*>(y), ldy, (int)I};
  const unsigned gx = (unsigned)((I + 255) / 256 < 64 ? (I + 255) / 256 : 64);
  pp::swiglu_kernel<<<dim3(gx, 4), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return pp::check_launch("swiglu_kernel");
}

}  // extern "C"
