// Batched quad GEMM on the tcgen05 tensor cores, file layout (codes [N][K],
// K contiguous), batch rows 17..128 per launch.
//
// At these batch sizes the GEMV kernel would stream the codes once per 16
// batch rows; here every code is decoded once for all rows.  A CTA owns a
// tile of 128 output rows and a range of K (split-K across CTAs when there
// are fewer tiles than SMs), and runs three roles:
//   producer warp  -- TMA: per stage a 16 x 128 box of codes (64-byte
//                     swizzle) and the activations' 16 x nmma box (32-byte
//                     swizzle: already the canonical K-major B operand);
//   8 decoder warps -- decode the stage's 2048 codes through the replicated
//                     shared-memory tables (the FP16 chain of the reference)
//                     into four 128 x 16 FP16 A tiles, one per model, in the
//                     canonical K-major 32-byte-swizzled layout;
//   MMA warp       -- one thread issues tcgen05.mma (kind::f16, M = 128,
//                     N = nmma, K = 16) per model into four FP32 accumulators
//                     in tensor memory, and tcgen05.commit releases the
//                     stage when the tensor core is done with it.
// Plug entries (the `.quadpack` plug table) are substituted into the A tiles:
// per 64-column window the producer bulk-copies the window's segments of the
// Linear's unit-major plug stream (one per 8-row tile), and each decoder
// thread writes the plug values of its row and 8 columns over its decoded
// weights -- the reference's own substitution, before the matmul.  (Without
// the stream, a separate kernel computes an FP32 correction instead.)
// Decoder warps 0-3 then read the accumulators (tcgen05.ld), add the plug
// correction if any, scale and store FP16 -- or, with split-K, write FP32
// partials that the last CTA of the tile sums in split order (deterministic).
// Every mbarrier wait is bounded; tensor memory is released on every path.
#include "pp_common.cuh"
#include "pp_engine.cuh"
#include "pp_host.h"

namespace pp {

constexpr int kTcRows = 128;                                // tile rows = MMA M
constexpr int kTcK = 16;                                    // K per stage = MMA K
constexpr int kTcGroupWarps = 8;                            // decoder warps of one stage
constexpr int kTcGroups = 2;                                // decoder groups, alternate stages
constexpr int kTcDecodeWarps = kTcGroupWarps * kTcGroups;
constexpr int kTcThreads = (kTcDecodeWarps + 2) * 32;       // + producer + MMA warp
constexpr uint32_t kTcCodeBytes = kTcRows * kTcK * 4;       // 8 KiB
constexpr uint32_t kTcXBytes = 128 * kTcK * 2;              // activations, nmma <= 128 rows
constexpr uint32_t kTcATileBytes = kTcRows * kTcK * 2;      // 4 KiB per model
constexpr uint32_t kTcCSlotBytes = kTcCodeBytes + kTcXBytes;  // 12 KiB: one stage's TMA data
constexpr uint32_t kTcASlotBytes = 4 * kTcATileBytes;       // 16 KiB: one stage's four A tiles
constexpr int kTcMaxStages = 8;                             // code slots
constexpr int kTcASlots = 2;                                // A-tile slots: one per decoder group
constexpr int kTcMaxRows = 128;                             // batch rows per launch
constexpr uint32_t kTcPlugSeg = 512;                        // staged bytes of one unit's plug segment
constexpr uint32_t kTcPlugSlot = (kTcRows / 8) * kTcPlugSeg;  // one 64-column window: 16 segments
constexpr int kTcPlugMaxStages = 4;                         // code slots with plugs (slot reuse, see below)

struct QuadTcParams {
  CUtensorMap tmap_codes;  // (K, N) uint32, box 16 x 128, 64-byte swizzle
  CUtensorMap tmap_x;      // (K, M) fp16, box 16 x nmma, 32-byte swizzle
  const uint8_t* tables;   // prepared 128 KiB table image
  float scale[4];
  __half* out[4];
  int64_t ldo_m, ldo_n;
  const float* corr;       // plug correction (NULL: none): corr[q * corr_q + m * N + n]
  int64_t corr_q;
  int M, N, K;
  int nmma;                // batch rows rounded up to 16
  int splits, kchunks;     // K splits per tile, K chunks of 16
  int stages;              // code slots (stages of codes and activations in flight)
  uint32_t tmem_cols;
  uint32_t smem_bytes;
  float* slots;            // split-K partials [tiles * splits][4][nmma][128]
  int* counters;           // [tiles] arrival counters (zero between launches); [kMaxGrid - 1] status
  // in-tile plug substitution (uplugs NULL: none): the Linear's unit-major
  // plug stream (units of 8 rows x 64 columns, tile-major, upt per 8-row
  // tile; segment: 8 header words start | end << 10 | n << 20, n FP16x4
  // values, n column bytes) and its unit byte offsets; nrt 8-row tiles
  const uint8_t* uplugs;
  const uint32_t* uplug_off;
  int upt, nrt;
};

// Shared memory: tables at the first 64 KiB boundary when they fit (direct
// gathers), else at the base; then, first-fit below and above the tables
// (1 KiB aligned), S code slots (a stage's codes and activations, filled by
// TMA), two A-tile slots (a stage's decoded weights, one per decoder
// group), with plugs two plug window slots, then the mbarriers and the
// tensor-memory address slot.  The code ring runs ahead of the decode by up
// to S stages, so more code slots hide more HBM latency; the A tiles only
// need to cover the MMA of the group's previous stage.  (A third A-tile slot
// measured no faster and, with plugs, costs a code slot: 2048 x 11008 at 64
// rows took 207 us with three A slots and two code slots, 153 us with two
// and three.)
// A ring of equal slots: slots [0, n0) from b0 (below the tables), the rest
// from b1 (above them), so a slot address is plain arithmetic (no indexed
// array, which would live in local memory).
struct TcRing {
  uint32_t b0, n0, b1;
  __host__ __device__ uint32_t at(int i, uint32_t bytes) const {
    return (uint32_t)i < n0 ? b0 + (uint32_t)i * bytes : b1 + ((uint32_t)i - n0) * bytes;
  }
};

struct TcLayout {
  uint32_t lut, bars, tslot;
  TcRing cr, ar;  // code slots (kTcCSlotBytes), A-tile slots (kTcASlotBytes)
  uint32_t plug;  // two plug window slots (plugs only)
  int direct, ok;
};

__host__ __device__ inline TcLayout tc_layout(uint32_t base, uint32_t size, int S, bool plugs) {
  TcLayout L{};
  const uint64_t end = (uint64_t)base + size;
  const uint32_t small = 256;  // (2 S + 2 kTcASlots + 4) mbarriers + tmem slot
  for (int direct = 1; direct >= 0; --direct) {
    L = TcLayout{};
    const uint32_t lut = direct ? ((base + 0xFFFFu) & ~0xFFFFu) : base;
    if ((uint64_t)lut + kQuadLutBytes > end) continue;
    // free ranges: [fa, lut) and [fb, end); a ring takes as many slots as
    // fit below the tables, then the rest above them
    uint64_t fa = ((uint64_t)base + 1023u) & ~1023ull;
    uint64_t fb = ((uint64_t)lut + kQuadLutBytes + 1023u) & ~1023ull;
    auto ring = [&](int n, uint32_t bytes, TcRing* r) {
      const uint64_t below = fa < lut ? (lut - fa) / bytes : 0;
      r->n0 = (uint32_t)(below < (uint64_t)n ? below : (uint64_t)n);
      r->b0 = (uint32_t)fa;
      fa += (uint64_t)r->n0 * bytes;
      r->b1 = (uint32_t)fb;
      fb += (uint64_t)(n - (int)r->n0) * bytes;
      return fb <= end;
    };
    if (!ring(kTcASlots, kTcASlotBytes, &L.ar) || !ring(S, kTcCSlotBytes, &L.cr)) continue;
    if (plugs) {
      TcRing pr{};
      if (!ring(1, 2 * kTcPlugSlot, &pr)) continue;
      L.plug = pr.at(0, 2 * kTcPlugSlot);
    }
    if (fa + small <= lut) L.bars = (uint32_t)fa;
    else if (fb + small <= end) L.bars = (uint32_t)fb;
    else continue;
    L.tslot = L.bars + 240u;
    L.lut = lut;
    L.direct = direct;
    L.ok = 1;
    return L;
  }
  L.ok = 0;
  return L;
}

// ------------------------------------------------------------ tcgen05 PTX --
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (one thread)
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when all tcgen05.mma issued so far by this thread complete.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 32-byte swizzle (8-row atoms of
// 32-byte rows, 256 bytes apart), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (16ull << 32) | (1ull << 46) | (6ull << 61);
}

// Instruction descriptor: D = F32, A = B = F16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t tc_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

template <bool DIRECT>
__device__ __forceinline__ void tc_decode_stage(uint32_t codes, uint32_t a_tiles, uint32_t lb0, uint32_t lb1,
                                                uint32_t add0, uint32_t add1) {
  const int i = threadIdx.x & 255;    // thread of the decoder group, 0..255
  const int row = i & 127, h = i >> 7;  // row of the tile, 8-code half of the stage
  // codes: row at row * 64, 16-byte chunk c at (c ^ ((row >> 1) & 3)) * 16 (64-byte swizzle)
  const uint32_t rbase = codes + (uint32_t)row * 64u;
  const uint32_t sw = (uint32_t)((row >> 1) & 3);
  const uint4 q0 = lds128(rbase + ((((uint32_t)(2 * h)) ^ sw) << 4));
  const uint4 q1 = lds128(rbase + ((((uint32_t)(2 * h + 1)) ^ sw) << 4));
  const uint32_t cw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  QuadDec d[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) d[j] = decode_quad<DIRECT>(cw[j], lb0, lb1, add0, add1);
  // A tile element (row, k) at (row >> 3) * 256 + (row & 7) * 32 + ((k >> 3) ^ ((row >> 2) & 1)) * 16
  const uint32_t aoff = (uint32_t)((row >> 3) * 256 + (row & 7) * 32 + ((h ^ ((row >> 2) & 1)) << 4));
  const uint4 m0 = make_uint4(lo_pair(d[0].p1, d[1].p1), lo_pair(d[2].p1, d[3].p1), lo_pair(d[4].p1, d[5].p1),
                              lo_pair(d[6].p1, d[7].p1));
  const uint4 m1 = make_uint4(lo_pair(d[0].p2, d[1].p2), lo_pair(d[2].p2, d[3].p2), lo_pair(d[4].p2, d[5].p2),
                              lo_pair(d[6].p2, d[7].p2));
  const uint4 m2 = make_uint4(lo_pair(d[0].p3, d[1].p3), lo_pair(d[2].p3, d[3].p3), lo_pair(d[4].p3, d[5].p3),
                              lo_pair(d[6].p3, d[7].p3));
  const uint4 m3 = make_uint4(hi_pair(d[0].p3, d[1].p3), hi_pair(d[2].p3, d[3].p3), hi_pair(d[4].p3, d[5].p3),
                              hi_pair(d[6].p3, d[7].p3));
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a_tiles + aoff), "r"(m0.x), "r"(m0.y), "r"(m0.z),
               "r"(m0.w) : "memory");
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a_tiles + kTcATileBytes + aoff), "r"(m1.x),
               "r"(m1.y), "r"(m1.z), "r"(m1.w) : "memory");
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a_tiles + 2 * kTcATileBytes + aoff), "r"(m2.x),
               "r"(m2.y), "r"(m2.z), "r"(m2.w) : "memory");
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a_tiles + 3 * kTcATileBytes + aoff), "r"(m3.x),
               "r"(m3.y), "r"(m3.z), "r"(m3.w) : "memory");
}

// Plug values of this decoder thread's row and 8 columns written over its
// decoded weights (after its own stores of the stage, so they win).  The
// row's entries of the window's unit are sorted by column: the scan stops
// at the first column past the thread's range.  A segment larger than its
// staged bytes is read from global memory.
__device__ __forceinline__ void tc_patch_plugs(const QuadTcParams& p, uint32_t pslot, uint32_t a_tiles, int tile,
                                               int kc, int kq) {
  const int i = threadIdx.x & 255;
  const int row = i & 127, h = i >> 7;
  const int rt = tile * (kTcRows / 8) + (row >> 3);  // 8-row tile of the Linear
  if (rt >= p.nrt) return;
  const uint32_t seg = pslot + (uint32_t)(row >> 3) * kTcPlugSeg;
  const uint32_t hdr = lds_u32(seg + 4u * (uint32_t)(row & 7));
  const uint32_t lo = hdr & 1023u, hi = (hdr >> 10) & 1023u, n = hdr >> 20;
  if (lo >= hi) return;
  const uint32_t c0 = (uint32_t)(kq * kTcK + 8 * h);  // first column of the thread in the unit
  const uint32_t aoff = (uint32_t)((row >> 3) * 256 + (row & 7) * 32 + ((h ^ ((row >> 2) & 1)) << 4));
  const bool staged = 32u + 9u * n <= kTcPlugSeg;
  const uint8_t* gs = staged ? nullptr : p.uplugs + __ldg(p.uplug_off + (int64_t)rt * p.upt + kc);
  for (uint32_t e = lo; e < hi; ++e) {
    const uint32_t col = staged ? lds_u8(seg + 32u + 8u * n + e) : (uint32_t)__ldg(gs + 32u + 8u * n + e);
    if (col >= c0 + 8u) break;  // sorted: the rest lie past this thread's columns
    if (col < c0) continue;
    const uint2 v = staged ? lds_u2(seg + 32u + 8u * e) : __ldg(reinterpret_cast<const uint2*>(gs + 32u + 8u * e));
    const uint32_t a = a_tiles + aoff + 2u * (col - c0);
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(a), "h"((uint16_t)(v.x & 0xFFFFu)) : "memory");
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(a + kTcATileBytes), "h"((uint16_t)(v.x >> 16)) : "memory");
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(a + 2 * kTcATileBytes), "h"((uint16_t)(v.y & 0xFFFFu)) : "memory");
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(a + 3 * kTcATileBytes), "h"((uint16_t)(v.y >> 16)) : "memory");
  }
}

// Producer (one lane): the plug segments of 64-column window kc of the
// tile's 16 row tiles into a window slot, up to kTcPlugSeg bytes each, on
// the slot's barrier.
__device__ __forceinline__ void tc_issue_plugs(const QuadTcParams& p, uint32_t pslot, uint32_t bar, int tile,
                                               int kc) {
  uint32_t off[kTcRows / 8], len[kTcRows / 8];
  uint32_t total = 0;
#pragma unroll
  for (int t = 0; t < kTcRows / 8; ++t) {
    const int rt = tile * (kTcRows / 8) + t;
    off[t] = len[t] = 0u;
    if (rt < p.nrt) {
      const int64_t u = (int64_t)rt * p.upt + kc;
      off[t] = __ldg(p.uplug_off + u);
      const uint32_t l = __ldg(p.uplug_off + u + 1) - off[t];
      len[t] = l < kTcPlugSeg ? l : kTcPlugSeg;
    }
    total += len[t];
  }
  mbar_expect_tx(bar, total);
#pragma unroll
  for (int t = 0; t < kTcRows / 8; ++t)
    if (len[t]) bulk_load(pslot + (uint32_t)t * kTcPlugSeg, p.uplugs + off[t], len[t], bar);
}

__global__ void __launch_bounds__(kTcThreads, 1) quad_tc_kernel(const __grid_constant__ QuadTcParams p) {
  pdl_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int* status = p.counters + (kMaxGrid - 1);
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(pp_smem);
  const bool plugs = p.uplugs != nullptr;
  const TcLayout L = tc_layout(base, p.smem_bytes, p.stages, plugs);
  if (!L.ok) {  // the host plans for this never to happen
    if (tid == 0) atomicExch(status, 2);
    return;
  }
  const int S = p.stages;
  const int tile = blockIdx.x / p.splits, split = blockIdx.x - tile * p.splits;
  const int c0 = (int)((int64_t)split * p.kchunks / p.splits);
  const int c1 = (int)((int64_t)(split + 1) * p.kchunks / p.splits);
  const int nst = c1 - c0;  // stages of this CTA (>= 1, checked on the host)
  const int n0 = tile * kTcRows;
  // mbarriers: full[S], empty[S] (code slots), afull[2], aempty[2] (A-tile
  // slots), done, tables
  const uint32_t full = L.bars, empty = L.bars + 8u * S;
  const uint32_t afull = L.bars + 16u * S, aempty = afull + 8u * kTcASlots;
  const uint32_t done = aempty + 8u * kTcASlots, tbar = done + 8u;
  // plug window slots: window w (64 columns, four stages) goes to slot
  // (w - w0) & 1 on barrier pfull + 8 * slot.  A slot is refilled two
  // windows later, when the producer issues the first stage of that window:
  // it has then waited for stage r - S (S <= 4) to be multiplied, and every
  // stage before it, including the last stage of the slot's previous
  // window (r - 5 or earlier), was decoded and patched before that.
  const uint32_t pfull = tbar + 8u;
  const int w0 = (c0 * kTcK) / 64;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + 8u * s, 1);
      mbar_init(empty + 8u * s, 1);
    }
    for (int a = 0; a < kTcASlots; ++a) {
      mbar_init(afull + 8u * a, kTcGroupWarps);
      mbar_init(aempty + 8u * a, 1);
    }
    mbar_init(done, 1);
    mbar_init(tbar, 1);
    mbar_init(pfull, 1);
    mbar_init(pfull + 8u, 1);
    fence_mbar_init();
    mbar_expect_tx(tbar, kQuadLutBytes);
    for (uint32_t off = 0; off < kQuadLutBytes; off += 16384u) bulk_load(L.lut + off, p.tables + off, 16384u, tbar);
  }
  if (warp == kTcDecodeWarps + 1) {  // the MMA warp owns the tensor memory
    tmem_alloc(L.tslot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(pp_smem + (L.tslot - base));

  if (warp == kTcDecodeWarps) {
    // ----------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&p.tmap_codes);
      prefetch_tmap(&p.tmap_x);
      const uint32_t xbytes = (uint32_t)p.nmma * kTcK * 2u;
      // codes (and plug segments) of the first stages are weights: issue them before the wait
      const int pre = nst < S ? nst : S;
      for (int r = 0; r < pre; ++r) {
        mbar_expect_tx(full + 8u * r, kTcCodeBytes + xbytes);
        tma_load_2d(L.cr.at(r, kTcCSlotBytes), &p.tmap_codes, (c0 + r) * kTcK, n0, full + 8u * r);
        const int kc = ((c0 + r) * kTcK) / 64;
        if (plugs && (r == 0 || ((c0 + r) * kTcK) % 64 == 0)) {
          const uint32_t ps = (uint32_t)((kc - w0) & 1);
          tc_issue_plugs(p, L.plug + ps * kTcPlugSlot, pfull + 8u * ps, tile, kc);
        }
      }
      pdl_wait();  // activations may come from the previous kernel
      for (int r = 0; r < pre; ++r) tma_load_2d(L.cr.at(r, kTcCSlotBytes) + kTcCodeBytes, &p.tmap_x, (c0 + r) * kTcK, 0, full + 8u * r);
      for (int r = S; r < nst; ++r) {
        const int s = r % S;
        // the slot's last stage has been decoded and multiplied
        if (!mbar_wait_bounded(empty + 8u * s, (uint32_t)((r / S) - 1) & 1u, status)) break;
        mbar_expect_tx(full + 8u * s, kTcCodeBytes + xbytes);
        tma_load_2d(L.cr.at(s, kTcCSlotBytes), &p.tmap_codes, (c0 + r) * kTcK, n0, full + 8u * s);
        tma_load_2d(L.cr.at(s, kTcCSlotBytes) + kTcCodeBytes, &p.tmap_x, (c0 + r) * kTcK, 0, full + 8u * s);
        if (plugs && ((c0 + r) * kTcK) % 64 == 0) {
          const int kc = ((c0 + r) * kTcK) / 64;
          const uint32_t ps = (uint32_t)((kc - w0) & 1);
          tc_issue_plugs(p, L.plug + ps * kTcPlugSlot, pfull + 8u * ps, tile, kc);
        }
      }
    }
  } else if (warp == kTcDecodeWarps + 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc_idesc(p.nmma);
      bool ok = true;
      for (int r = 0; r < nst && ok; ++r) {
        const int s = r % S, a = r % kTcASlots;
        ok = mbar_wait_bounded(full + 8u * s, (uint32_t)(r / S) & 1u, status) &&
             mbar_wait_bounded(afull + 8u * a, (uint32_t)(r / kTcASlots) & 1u, status);
        if (!ok) break;
        tc_fence_after();
        const uint64_t bdesc = sw32_desc(L.cr.at(s, kTcCSlotBytes) + kTcCodeBytes);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          tc_mma(tmem + (uint32_t)(q * p.nmma), sw32_desc(L.ar.at(a, kTcASlotBytes) + q * kTcATileBytes), bdesc, idesc,
                 r > 0 ? 1u : 0u);
        tc_commit(empty + 8u * s);   // code slot free (its activations were read)
        tc_commit(aempty + 8u * a);  // A-tile slot free
      }
      tc_commit(done);  // fires once every MMA issued above has completed
    }
  } else {
    // ------------------------------------------------------------ decoders
    if (mbar_wait_bounded(tbar, 0u, status)) {
      const uint32_t lb0 = (L.direct ? L.lut : 0u) | ((uint32_t)lane * 4u);
      const uint32_t lb1 = (L.direct ? L.lut + 65536u : 0u) | ((uint32_t)lane * 4u);
      const uint32_t add0 = L.direct ? 0u : L.lut, add1 = L.direct ? 0u : L.lut + 65536u;
      // group g decodes stages g, g + kTcGroups, ...
      for (int r = warp / kTcGroupWarps; r < nst; r += kTcGroups) {
        const int s = r % S, a = r % kTcASlots;
        if (!mbar_wait_bounded(full + 8u * s, (uint32_t)(r / S) & 1u, status)) break;
        // the A-tile slot's previous stage has been multiplied
        if (r >= kTcASlots &&
            !mbar_wait_bounded(aempty + 8u * a, (uint32_t)((r / kTcASlots) - 1) & 1u, status))
          break;
        if (L.direct) tc_decode_stage<true>(L.cr.at(s, kTcCSlotBytes), L.ar.at(a, kTcASlotBytes), lb0, lb1, 0u, 0u);
        else tc_decode_stage<false>(L.cr.at(s, kTcCSlotBytes), L.ar.at(a, kTcASlotBytes), lb0, lb1, add0, add1);
        if (plugs) {
          const int kc = ((c0 + r) * kTcK) / 64;
          const uint32_t ps = (uint32_t)((kc - w0) & 1);
          if (!mbar_wait_bounded(pfull + 8u * ps, (uint32_t)((kc - w0) >> 1) & 1u, status)) break;
          tc_patch_plugs(p, L.plug + ps * kTcPlugSlot, L.ar.at(a, kTcASlotBytes), tile, kc,
                         (((c0 + r) * kTcK) % 64) / kTcK);
        }
        fence_proxy_async();  // the A tiles are read by the tensor core (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive(afull + 8u * a);
      }
    }
    // ------------------------------------------------------------ epilogue
    if (warp < 4) {
      const bool fin = mbar_wait_bounded(done, 0u, status);
      tc_fence_after();
      const int rl = warp * 32 + lane;  // row of the tile = tensor-memory lane
      const int row = n0 + rl;
      pdl_wait();  // outputs, workspace and the plug correction belong to the stream's order
      const bool split_k = p.splits > 1;
      float* slot = p.slots + (int64_t)blockIdx.x * 4 * p.nmma * kTcRows;
      for (int q = 0; q < 4; ++q)
        for (int cb = 0; cb < p.nmma; cb += 16) {
          float v[16];
          tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(q * p.nmma + cb), v);
          if (!fin) continue;
          if (split_k) {
#pragma unroll
            for (int j = 0; j < 16; ++j) __stcg(slot + ((int64_t)q * p.nmma + cb + j) * kTcRows + rl, v[j]);
            continue;
          }
          // the chunk's plug corrections are loaded before any output is
          // stored: otherwise each load would wait for the store before it
          // (the compiler cannot rule out that they alias)
          float cv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            cv[j] = (p.corr && cb + j < p.M && row < p.N)
                        ? __ldcg(p.corr + (int64_t)q * p.corr_q + (int64_t)(cb + j) * p.N + row)
                        : 0.f;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = cb + j;
            if (m < p.M && row < p.N)
              p.out[q][(int64_t)m * p.ldo_m + (int64_t)row * p.ldo_n] = __float2half_rn((v[j] + cv[j]) * p.scale[q]);
          }
        }
    }
  }
  // split-K: the last of the tile's CTAs sums every split's partial in split
  // order, spread over all threads of the CTA (coalesced along the rows)
  if (p.splits > 1) {
    pdl_wait();
    __threadfence();
    __syncthreads();
    int* flag = reinterpret_cast<int*>(pp_smem + (L.tslot - base)) + 1;
    if (tid == 0) *flag = atomicAdd(p.counters + tile, 1) == p.splits - 1;
    __syncthreads();
    if (*reinterpret_cast<volatile int*>(flag)) {
      __threadfence();
      const float* tslots = p.slots + (int64_t)tile * p.splits * 4 * p.nmma * kTcRows;
      const int per_split = 4 * p.nmma * kTcRows;
      const int total = 4 * p.M * kTcRows;
      // eight elements per thread at a time: every split's partial and the
      // plug correction of all eight are loaded before any output is stored
      // (a load after a store would wait for it: they may alias), and each
      // element sums its splits in split order
      for (int e0 = tid; e0 < total; e0 += 8 * kTcThreads) {
        int off[8], qv[8], mv[8];
        float a[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int e = e0 + u * kTcThreads;
          const int rl = e & (kTcRows - 1), qm = e >> 7;
          qv[u] = qm / p.M;
          mv[u] = qm - qv[u] * p.M;
          off[u] = (e < total && n0 + rl < p.N) ? (qv[u] * p.nmma + mv[u]) * kTcRows + rl : -1;
          a[u] = 0.f;
        }
#pragma unroll 2
        for (int j = 0; j < p.splits; ++j) {
          const float* src = tslots + (int64_t)j * per_split;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (off[u] >= 0) a[u] += __ldcg(src + off[u]);
        }
        if (p.corr) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (off[u] >= 0)
              a[u] += __ldcg(p.corr + (int64_t)qv[u] * p.corr_q + (int64_t)mv[u] * p.N + n0 + (off[u] & (kTcRows - 1)));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (off[u] >= 0) {
            const int row = n0 + (off[u] & (kTcRows - 1));
            p.out[qv[u]][(int64_t)mv[u] * p.ldo_m + (int64_t)row * p.ldo_n] = __float2half_rn(a[u] * p.scale[qv[u]]);
          }
      }
      if (tid == 0) p.counters[tile] = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcDecodeWarps + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

// ------------------------------------------------------------------ host --
namespace {
bool g_tc_attr_done[64];
int g_tc_attr_limit[64];
}  // namespace

struct QuadTcPlan {
  int nmma = 0, tiles = 0, splits = 0, kchunks = 0;
  size_t slots_bytes = 0;
};

inline QuadTcPlan quad_tc_plan(int64_t Mc, int64_t N, int64_t K, int sms) {
  QuadTcPlan pl;
  pl.nmma = (int)((Mc + 15) / 16 * 16);
  pl.tiles = (int)cdiv(N, kTcRows);
  pl.kchunks = (int)(K / kTcK);
  // at most one wave of CTAs, at least 8 stages of K each (more splits in
  // several waves measured slower at 64 rows: the partials cost more than
  // the idle SMs of one wave)
  int sp = sms / pl.tiles;
  const int cap = pl.kchunks / 8 > 1 ? pl.kchunks / 8 : 1;
  pl.splits = sp < cap ? sp : cap;
  if (pl.splits < 1) pl.splits = 1;
  pl.slots_bytes = pl.splits > 1 ? (size_t)pl.tiles * pl.splits * 4 * pl.nmma * kTcRows * sizeof(float) : 0;
  return pl;
}

// Whether the tensor-core path takes a problem (file layout, prepared
// tables).  Besides the operand constraints it needs either enough 128-row
// tiles or a long enough K: with few tiles and a short K the split-K
// partials move about as many bytes as the codes, and the GEMV kernel in
// 16-row chunks is about as fast on B200 (2048 x 2048: 36 vs 42 us at 32
// rows, 68 vs 64 us at 64; 2048 x 256: 55 vs 82 us at 64 rows), while
// 2048 x 11008 and 11008 x 2048 go the other way (1.9-2.6x at 64 rows).
bool quad_tc_ok(int64_t M, int64_t N, int64_t K, const uint32_t* codes, int64_t ldw, const void* x, int64_t ldx_m,
                int64_t ldx_k) {
  return M > 16 && (N >= 4096 || K >= 4096) && K % kTcK == 0 && K >= kTcK && ldx_k == 1 && aligned(x, 16) &&
         (ldx_m * 2) % 16 == 0 && aligned(codes, 16) && (ldw * 4) % 16 == 0 && cdiv(N, kTcRows) < kMaxGrid - 1;
}

// Split-K partial slots of the launches of an M-row problem (rows in
// launches of at most 128).
size_t quad_tc_slots_bytes(int64_t M, int64_t N, int64_t K, int sms) {
  const int64_t Mc = M < kTcMaxRows ? M : kTcMaxRows;
  return quad_tc_plan(Mc, N, K, sms).slots_bytes;
}

// One launch over batch rows [0, Mc) of x / out (Mc <= 128).
int launch_quad_tc(const void* x, int64_t ldx_m, const uint32_t* codes, int64_t ldw, const void* tables,
                   const float scales[4], void* const out[4], int64_t ldo_m, int64_t ldo_n, const float* corr,
                   int64_t corr_q, int64_t Mc, int64_t N, int64_t K, int* counters, float* slots,
                   const void* uplugs, const uint32_t* uplug_off, cudaStream_t s) {
  const int dev = current_device();
  const int sms = device_sm_count(dev);
  int max_smem = 0;
  int rc = ensure_smem_attr(quad_tc_kernel, g_tc_attr_done, g_tc_attr_limit, &max_smem);
  if (rc) return rc;
  const QuadTcPlan pl = quad_tc_plan(Mc, N, K, sms);
  QuadTcParams prm{};
  if ((rc = encode_tmap_2d(&prm.tmap_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, codes, (uint64_t)K, (uint64_t)N,
                           (uint64_t)ldw * 4, kTcK, kTcRows, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  if ((rc = encode_tmap_2d(&prm.tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, (uint64_t)K, (uint64_t)Mc,
                           (uint64_t)ldx_m * 2, kTcK, (uint32_t)pl.nmma, CU_TENSOR_MAP_SWIZZLE_32B)))
    return rc;
  prm.tables = reinterpret_cast<const uint8_t*>(tables);
  for (int q = 0; q < 4; ++q) {
    prm.scale[q] = scales[q];
    prm.out[q] = reinterpret_cast<__half*>(out[q]);
  }
  prm.ldo_m = ldo_m;
  prm.ldo_n = ldo_n;
  prm.corr = corr;
  prm.corr_q = corr_q;
  prm.M = (int)Mc;
  prm.N = (int)N;
  prm.K = (int)K;
  prm.nmma = pl.nmma;
  prm.splits = pl.splits;
  prm.kchunks = pl.kchunks;
  uint32_t cols = 32;
  while (cols < (uint32_t)(4 * pl.nmma)) cols <<= 1;
  prm.tmem_cols = cols;
  prm.counters = counters;
  prm.slots = slots;
  const bool plugs = uplugs != nullptr;
  prm.uplugs = reinterpret_cast<const uint8_t*>(uplugs);
  prm.uplug_off = uplug_off;
  prm.upt = (int)cdiv(K, 64);
  prm.nrt = (int)cdiv(N, 8);
  const uint32_t reserved = (uint32_t)reserved_smem(dev);
  int S = plugs ? kTcPlugMaxStages : kTcMaxStages;
  while (S > 1 && !tc_layout(reserved, (uint32_t)max_smem, S, plugs).ok) --S;
  if (!tc_layout(reserved, (uint32_t)max_smem, S, plugs).ok) {
    set_error("no shared memory layout for the tensor-core kernel within %d bytes", max_smem);
    return PP_ERR_INVALID;
  }
  prm.stages = S;
  prm.smem_bytes = (uint32_t)max_smem;
  return launch_kernel("quad_tc_kernel", launch_overlap(), quad_tc_kernel, dim3(pl.tiles * pl.splits),
                       dim3(kTcThreads), (size_t)max_smem, s, prm);
}

}  // namespace pp
