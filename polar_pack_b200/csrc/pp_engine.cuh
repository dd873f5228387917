// Work partition and deterministic split-K reduction shared by the fused
// dequant GEMV kernels.
//
// A "tile" is the set of output features one warp accumulates (8 rows for
// the file layout, 32 or 64 features for the kernel layout); a "unit" is
// one K chunk of a tile.  Units are numbered tile-major.  The grid's CTAs
// take equal contiguous unit ranges, and each warp of a CTA an equal
// contiguous piece of its CTA's range, which it streams front to back: a
// warp's consecutive units are consecutive K chunks of the same rows.
//
// A tile that lies wholly inside one warp's range is stored by that warp.
// A tile cut by a warp boundary leaves FP32 partials in shared memory (at
// most two per warp); after the only barrier of the kernel the CTA sums
// them in warp order.  A tile cut by a CTA boundary goes one level further:
// each CTA writes its partial to the workspace, fences, bumps a counter, and
// the last CTA to arrive sums all partials in CTA order, stores the result
// and resets the counter.  No thread ever waits for another CTA, and the
// summation order is fixed, so results are deterministic.
//
// Two streaming engines share this partition: a register engine (each warp
// keeps one unit in flight in registers, prefetches ahead into L2 and
// reduces split tiles after a CTA barrier) and a TMA engine (each warp
// refills its own shared-memory ring and reduces split tiles at warp
// level, described below).
#pragma once

#include <stdint.h>

namespace pp {

// Workspace: a fixed 4 KiB counter block (one arrival counter per CTA,
// zero between launches) followed by the partial-sum slots.  A tile shared
// by CTAs c_first < ... < c_last uses counter c_last: c_last contains the
// tile's last unit and starts inside it, so no CTA is c_last of two shared
// tiles, and counters never overlap slot memory of any other plan.
constexpr int kMaxGrid = 1024;
constexpr size_t kCounterBytes = kMaxGrid * sizeof(int);

struct Partition {
  int units;      // total units (< 2^31, checked on the host)
  int upt;        // units per tile
  int* counters;  // [kMaxGrid] arrival counters (zero between launches)
  float* slots;   // [grid][2][nout * M * tile_w] cross-CTA partials
  // TMA engine only: unit start of every CTA (cta_start[G] = units), a
  // table the host fills; NULL for the register engine (equal split)
  const int* cta_start;
  // TMA engine only: this CTA's index among the CTAs that share the
  // partition, and their number (blockIdx.x and gridDim.x of a launch that
  // runs one problem; a grouped launch gives each problem a range of CTAs)
  int cta, ncta;
};

// CTA ranges of the TMA engine come from a host-filled table of at most
// kMaxCtaTable + 1 starts, passed in the kernel parameters.
constexpr int kMaxCtaTable = 256;

// largest c < G with start[c] <= x (binary search over the table)
__device__ __forceinline__ int cta_of_unit(const int* start, int G, int x) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= x) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ int range_start(int U, int parts, int i) {
  return (int)(((int64_t)U * i) / parts);
}

// largest c with range_start(U, G, c) <= x
__device__ __forceinline__ int part_of_unit(int x, int U, int G) {
  const int c = (int)((((int64_t)x + 1) * G + U - 1) / U) - 1;
  return c < G - 1 ? c : G - 1;
}

// The reduction of a CTA's tiles after its warps finished their ranges
// (shared by both engines): warp partials in warp order, then the
// cross-CTA protocol for the (at most two) tiles cut by a CTA boundary.
template <class Op>
__device__ __forceinline__ void reduce_partials(Op& op, const Partition& pt, const float* red, int* s_flag,
                                                int cu0, int cu1, int nval) {
  constexpr int NW = Op::kWarps;
  constexpr int TW = Op::kTileW;
  const int tid = threadIdx.x;
  const int U = pt.units, G = gridDim.x, upt = pt.upt, M = op.M();
  const int R = cu1 - cu0;
  const int ct0 = cu0 / upt, ct1 = (cu1 - 1) / upt;
  int pend[2];
  int npend = 0;
  for (int tt = ct0; tt <= ct1; ++tt) {
    const int a = tt * upt, b = a + upt;  // unit range of the tile
    const int w_first = part_of_unit((a > cu0 ? a : cu0) - cu0, R, NW);
    const int w_last = part_of_unit((b < cu1 ? b : cu1) - 1 - cu0, R, NW);
    const bool one_warp = w_first == w_last && a >= cu0 + range_start(R, NW, w_first) &&
                          b <= cu0 + range_start(R, NW, w_first + 1);
    const bool cta_whole = a >= cu0 && b <= cu1;
    if (one_warp && cta_whole) continue;  // stored by its warp
    float* slot = pt.slots + ((int64_t)blockIdx.x * 2 + (tt == ct0 ? 0 : 1)) * (int64_t)nval;
    for (int e = tid; e < nval; e += (int)blockDim.x) {
      float s = 0.f;
      for (int w = w_first; w <= w_last; ++w) {
        const int ws0 = cu0 + range_start(R, NW, w);
        if (ws0 == cu0 + range_start(R, NW, w + 1)) continue;  // empty range (fewer units than warps)
        const int which = (ws0 >= a) ? 0 : 1;  // the tile is w's first tile iff w starts in it
        s += red[(w * 2 + which) * nval + e];
      }
      if (cta_whole) {
        const int o = e / (M * TW);
        const int rem = e - o * M * TW;
        const int bat = rem / TW;
        const int f = tt * TW + (rem - bat * TW);
        if (f < op.N()) op.store(o, bat, f, s);
      } else {
        __stcg(slot + e, s);
      }
    }
    if (!cta_whole && npend < 2) pend[npend++] = tt;
  }
  for (int i = 0; i < npend; ++i) {
    const int tt = pend[i];
    const int c_first = part_of_unit(tt * upt, U, G);
    const int c_last = part_of_unit(tt * upt + upt - 1, U, G);
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int old = atomicAdd(pt.counters + c_last, 1);
      *s_flag = (old == c_last - c_first) ? 1 : 0;
    }
    __syncthreads();
    if (*s_flag) {
      __threadfence();
      for (int e = tid; e < nval; e += (int)blockDim.x) {
        float s = 0.f;
        for (int c = c_first; c <= c_last; ++c) {
          // only the first contributor can have started before the tile
          const int w = (c == c_first && range_start(U, G, c) < tt * upt) ? 1 : 0;
          s += __ldcg(pt.slots + ((int64_t)c * 2 + w) * (int64_t)nval + e);
        }
        const int o = e / (M * TW);
        const int rem = e - o * M * TW;
        const int bat = rem / TW;
        const int f = tt * TW + (rem - bat * TW);
        if (f < op.N()) op.store(o, bat, f, s);
      }
      if (tid == 0) pt.counters[c_last] = 0;
    }
    __syncthreads();
  }
}

// Op interface (device struct):
//   static constexpr int kWarps, kTileW, kNOut, kNBat
//   using Buf = ...;
//   void zero();                                accumulators := 0
//   void load(Buf&, int tile, int kc) const;    issue loads of one unit
//   void prefetch(int tile, int kc) const;      L2 prefetch of one unit
//   void compute(const Buf&, int tile, int kc);
//   void write_partial(float* slot, int M);     compact [out][bat < M][fi]
//   void begin(int tile, int kc); void preload(int tile, int kc);
//                                               side data of the first / next unit
//   int  M() const; int N() const;
//   void store_tile(int tile) const;            whole tile from registers
//   void store(int out, int bat, int f, float v) const;
//
// Shared memory `red` holds kWarps * 2 compact slots of nout * M * tile_w floats.
template <class Op>
__device__ __forceinline__ void run_partition(Op& op, const Partition& pt, float* red, int* s_flag) {
  constexpr int NW = Op::kWarps;
  constexpr int TW = Op::kTileW;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int U = pt.units;
  const int G = gridDim.x;
  const int cu0 = range_start(U, G, blockIdx.x), cu1 = range_start(U, G, blockIdx.x + 1);
  if (cu0 >= cu1) return;  // uniform over the CTA
  const int upt = pt.upt;
  const int M = op.M();
  const int nval = Op::kNOut * M * TW;
  const int R = cu1 - cu0;
  const int wu0 = cu0 + range_start(R, NW, warp), wu1 = cu0 + range_start(R, NW, warp + 1);

  if (wu0 < wu1) {
    constexpr int kPrefetch = 4;
    int t = wu0 / upt, kc = wu0 - t * upt;        // current unit
    const int t_first = t;
    int pt_t = t, pt_kc = kc;                      // prefetch cursor
    for (int i = 1; i <= kPrefetch; ++i) {         // units wu0+2 .. wu0+kPrefetch-1 now
      if (++pt_kc == upt) { pt_kc = 0; ++pt_t; }
      if (i >= 2 && i < kPrefetch && wu0 + i < wu1) op.prefetch(pt_t, pt_kc);
    }
    typename Op::Buf bufA, bufB;
    op.zero();
    op.load(bufA, t, kc);
    int u = wu0;
    auto step = [&](const typename Op::Buf& cur, typename Op::Buf& nxt) -> bool {
      // prefetch kPrefetch ahead, load the next unit, decode this one
      if (u + kPrefetch < wu1) op.prefetch(pt_t, pt_kc);
      if (++pt_kc == upt) { pt_kc = 0; ++pt_t; }
      int nt = t, nkc = kc + 1;
      if (nkc == upt) { nkc = 0; ++nt; }
      if (u + 1 < wu1) op.load(nxt, nt, nkc);
      op.compute(cur, t, kc);
      const bool tile_end = nkc == 0;
      const bool last = u + 1 == wu1;
      if (tile_end || last) {
        const bool whole = (t * upt >= wu0) && tile_end;
        if (whole) {
          op.store_tile(t);
        } else {
          const int which = t == t_first ? 0 : 1;
          op.write_partial(red + (warp * 2 + which) * nval, M);
        }
        op.zero();
      }
      t = nt;
      kc = nkc;
      return ++u < wu1;
    };
    while (step(bufA, bufB) && step(bufB, bufA)) {
    }
  }
  __syncthreads();
  reduce_partials(op, pt, red, s_flag, cu0, cu1, nval);
}

// ------------------------------------------------------------ TMA engine --
// Each warp streams its unit range through a private ring of S shared-memory
// slots filled by TMA, one mbarrier per slot (one arrival plus the
// transaction bytes of the copy).  Before the CTA builds its tables, lane 0
// initialises the ring and issues the first S units, so those copies are in
// flight during the build.  In the loop all lanes wait for the slot, copy
// the unit into registers and sync; lane 0 refills the slot with the unit S
// ahead before the unit is decoded.  Every wait is bounded
// (mbar_wait_bounded); after a timeout the status word is set and the warp
// stops streaming, so the kernel always ends.
//
// Split tiles are reduced at warp level, with no CTA barrier after the
// table build.  A warp's range is cut into up to three segments, processed
// in this order: the part of its last tile when that tile continues into
// the next warp (split tail), the part of its first tile when that tile is
// shared with a neighbour (split head), then whole tiles.  Split tiles thus
// finish early in every warp.  Ending a split tile, a warp writes its FP32
// partial to its shared-memory slot (slot 0: the tile holding its first
// unit, slot 1: the tile holding its last unit), fences and bumps the
// tile's arrival counter; the warp that arrives last sums the partials of
// all warps touching the tile, in warp order, and stores the tile if it
// lies inside the CTA.  A tile cut by a CTA boundary (at most two per CTA)
// then goes through the workspace: the same warp writes the CTA's sum to
// the CTA's workspace slot, fences and bumps the tile's counter, and the
// warp whose CTA arrives last sums all CTA slots in CTA order and stores
// the tile.  No warp ever waits for another, and every sum has a fixed
// order, so results are deterministic.
//
// Op additions: kUnitBytes; void read(Buf&, uint32_t slot, int s, int tile)
// const (the unit in ring slot s, before the slot is refilled);
// void side(int p, int u, int kc) (side data of unit u in side slot p; a
// warp has one side slot more than ring slots, so the slot of the unit
// being computed is not refilled before the next unit's wait); void
// end_chunk() (before the accumulators of a chunk are stored or reduced).
// The issue functor is called on lane 0 as issue(slot address, mbarrier,
// side slot index, tile, kc).

// Per-CTA tables in shared memory, filled before the table-build barrier.
struct CtaTables {
  int* wstart;  // [NW + 1] warp range starts, wstart[NW] = end of the CTA range
  int* wtile;   // [NW + 1] tile of wstart[w]
  int* cnt;     // [2 * NW] split-tile arrival counters, indexed 2 * (first warp) + slot;
                // cnt[2 * NW]: warps of the CTA done (the gather's completion signal)
};

// Warp w of the CTA range [cu0, cu1) starts at cu0 + (cu1 - cu0) * w / NW;
// the host keeps (cu1 - cu0) * NW below 2^31.
template <int NW>
__device__ __forceinline__ int warp_start(int cu0, int cu1, int w) {
  return cu0 + (int)((uint32_t)((cu1 - cu0) * w) / (uint32_t)NW);
}

template <int NW>
__device__ __forceinline__ void cta_tables_init(const CtaTables& tb, int cu0, int cu1, int upt) {
  const int i = threadIdx.x;
  if (i <= NW) {
    const int w0 = warp_start<NW>(cu0, cu1, i);
    tb.wstart[i] = w0;
    tb.wtile[i] = w0 / upt;
  }
  if (i <= 2 * NW) tb.cnt[i] = 0;
}

// The unit order of one warp: segments [a0,b0) split tail, [a1,b1) split
// head, [a2,b2) whole tiles (seg 3 = done).  `end` caches the end of the
// current segment.
struct UnitSeq {
  int a0, b0, a1, b1, a2, b2;
  int seg, u, t, kc, upt, end;

  __device__ __forceinline__ void enter(int sg) {
    seg = sg;
    while (seg < 3 && (seg == 0 ? a0 == b0 : seg == 1 ? a1 == b1 : a2 == b2)) ++seg;
    if (seg < 3) {
      u = seg == 0 ? a0 : seg == 1 ? a1 : a2;
      end = seg == 0 ? b0 : seg == 1 ? b1 : b2;
      t = u / upt;
      kc = u - t * upt;
    }
  }

  // non-empty range [wu0, wu1)
  __device__ __forceinline__ void init(int wu0, int wu1, int upt_) {
    upt = upt_;
    const int tf = wu0 / upt, tl = (wu1 - 1) / upt;
    const int hf = (tf + 1) * upt;
    const bool head_whole = wu0 == tf * upt && wu1 >= hf;
    const bool split_tail = tl > tf && wu1 < (tl + 1) * upt;
    a0 = split_tail ? tl * upt : wu1;
    b0 = wu1;
    a1 = wu0;
    b1 = head_whole ? wu0 : (wu1 < hf ? wu1 : hf);
    a2 = b1;
    b2 = split_tail ? tl * upt : wu1;
    enter(0);
  }

  // n units forward (n > 0, not past the segment end)
  __device__ __forceinline__ void skip(int n) {
    u += n;
    kc += n;
    while (kc >= upt) {
      kc -= upt;
      ++t;
    }
    if (u == end) enter(seg + 1);
  }

  __device__ __forceinline__ void advance() {
    ++u;
    if (++kc == upt) {
      kc = 0;
      ++t;
    }
    if (u == end) enter(seg + 1);
  }
};

struct TmaRing {
  uint32_t ring, bars;  // this warp's S slots and S mbarriers
  int S;
  int P = 1, pn = 0;    // side slots (S + 1) and the side slot of the next issue
  UnitSeq next;         // next unit to issue

  // every lane advances the cursors; only `leader` issues
  template <class Issue>
  __device__ __forceinline__ void issue_next(const Issue& issue, int s, uint32_t unit, bool leader) {
    if (leader) issue(ring + (uint32_t)s * unit, bars + 8u * (uint32_t)s, pn, next.t, next.kc);
    next.advance();
    if (++pn == P) pn = 0;
  }

  // lane 0: barriers and the first min(S, units) copies
  template <class Issue>
  __device__ __forceinline__ void prologue(const Issue& issue, uint32_t unit) {
    for (int i = 0; i < S; ++i) mbar_init(bars + 8u * (uint32_t)i, 1);
    fence_mbar_init();
    for (int i = 0; i < S && next.seg < 3; ++i) issue_next(issue, i, unit, true);
  }
};

// Stores U reduced elements e0, e0 + step, ... (< nval) of tile T.  The
// elements' plug corrections (Op::corr_at) are all loaded before the first
// store: a load after a store would otherwise wait for it, as the compiler
// cannot rule out that output and correction alias.
template <class Op, int U>
__device__ __forceinline__ void store_outputs(const Op& op, int e0, int step, int nval, int T, const float (&sv)[U]) {
  constexpr int TW = Op::kTileW;
  const int M = op.M();
  float cv[U];
  int ob[U], fb[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int e = e0 + step * u;
    const int o = e / (M * TW);
    const int rem = e - o * M * TW;
    const int bat = rem / TW;
    const int f = T * TW + (rem - bat * TW);
    ob[u] = o * 65536 + bat;
    fb[u] = (e < nval && f < op.N()) ? f : -1;
    cv[u] = fb[u] >= 0 ? op.corr_at(o, bat, f) : 0.f;
  }
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (fb[u] >= 0) op.store_raw(ob[u] >> 16, ob[u] & 0xFFFF, fb[u], sv[u] + cv[u]);
}

// Ends split tile T of warp `warp` (slot `which`), see above.  The warps
// that hold units of T are found in parallel (lane w checks warp w) and
// their partial-slot offsets broadcast once, so the closing warp's sums
// issue independent loads; the additions stay in warp order.
template <class Op>
__device__ __forceinline__ void close_split(Op& op, const Partition& pt, const CtaTables& tb, float* red,
                                            int warp, int T, int which, int cu0, int cu1) {
  constexpr int NW = Op::kWarps;
  static_assert(NW <= 31, "one lane per warp of the CTA, plus the range end");
  const int lane = threadIdx.x & 31;
  const int upt = pt.upt;
  const int M = op.M();
  const int nval = Op::kNOut * M * Op::kTileW;
  op.write_partial(red + (warp * 2 + which) * nval, M);
  const int x0 = T * upt > cu0 ? T * upt : cu0;                    // first unit of T in the CTA
  const int x1 = T * upt + upt < cu1 ? T * upt + upt : cu1;        // end of T in the CTA
  // lane w < NW: warp w's range [s0, s1) overlaps [x0, x1); the tile is
  // the warp's first (slot 0) iff the warp starts in it
  const int wl = lane < NW ? lane : NW;
  const int s0 = tb.wstart[wl], s1 = tb.wstart[lane < NW ? lane + 1 : NW];
  const bool holds = lane < NW && s1 > s0 && s0 < x1 && s1 > x0;
  const int myoff = holds ? (2 * lane + (tb.wtile[wl] == T ? 0 : 1)) * nval : -1;
  const uint32_t mask = __ballot_sync(0xffffffffu, holds);
  const int wf = __ffs((int)mask) - 1;  // holds x0, owns the tile's counter
  const int n = __popc(mask);
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    __threadfence_block();
    last = atomicAdd(tb.cnt + 2 * wf + (tb.wtile[wf] == T ? 0 : 1), 1) == n - 1;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  int so[NW];
#pragma unroll
  for (int w = 0; w < NW; ++w) so[w] = __shfl_sync(0xffffffffu, myoff, w);
  __syncwarp();
  __threadfence_block();
  const bool inside = T * upt >= cu0 && T * upt + upt <= cu1;
  float* gslot = pt.slots + ((int64_t)pt.cta * 2 + (T == tb.wtile[0] ? 0 : 1)) * (int64_t)nval;
  // one element per lane (batch 1): plain stores; larger tiles take eight
  // elements per lane at a time, whose plug corrections are loaded before
  // any of them is stored (store_outputs)
  if (nval <= 32) {
    float sum = 0.f;
    if (lane < nval) {
#pragma unroll
      for (int w = 0; w < NW; ++w)
        if (so[w] >= 0) sum += red[so[w] + lane];
    }
    if constexpr (Op::kGather16) {  // batch-1 gather: 16-byte stores (all lanes)
      if (inside && nval == 32 && op.gather16(T)) {
        op.gather_store16(T, sum);
        return;
      }
    }
    if (lane < nval) {
      if (inside) {
        const float sv[1] = {sum};
        store_outputs<Op, 1>(op, lane, 32, nval, T, sv);
      } else {
        __stcg(gslot + lane, sum);
      }
    }
  } else
  for (int e0 = lane; e0 < nval; e0 += 32 * 8) {
    float sv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) sv[u] = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if (so[w] < 0) continue;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (e0 + 32 * u < nval) sv[u] += red[so[w] + e0 + 32 * u];
    }
    if (inside) {
      store_outputs<Op, 8>(op, e0, 32, nval, T, sv);
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (e0 + 32 * u < nval) __stcg(gslot + e0 + 32 * u, sv[u]);
    }
  }
  if (inside) return;
  // tile cut by a CTA boundary
  const int G = pt.ncta;
  const int c_first = cta_of_unit(pt.cta_start, G, T * upt);
  const int c_last = cta_of_unit(pt.cta_start, G, T * upt + upt - 1);
  // the warp's slot stores are ordered before lane 0 (__syncwarp) and its
  // acquire-release arrival at GPU scope; the last CTA's lanes read the
  // slots after that arrival (shuffle)
  __syncwarp();
  int lastc = 0;
  if (lane == 0) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(old) : "l"(pt.counters + c_last) : "memory");
    lastc = old == c_last - c_first;
  }
  lastc = __shfl_sync(0xffffffffu, lastc, 0);
  if (!lastc) return;
  if (nval <= 32) {
    float sum = 0.f;
    if (lane < nval)
      for (int c = c_first; c <= c_last; ++c) {
        const int w = (c == c_first && pt.cta_start[c] < T * upt) ? 1 : 0;
        sum += __ldcg(pt.slots + ((int64_t)c * 2 + w) * (int64_t)nval + lane);
      }
    bool done16 = false;
    if constexpr (Op::kGather16) {  // batch-1 gather: 16-byte stores (all lanes)
      if (nval == 32 && op.gather16(T)) {
        op.gather_store16(T, sum);
        done16 = true;
      }
    }
    if (!done16 && lane < nval) {
      const float sv[1] = {sum};
      store_outputs<Op, 1>(op, lane, 32, nval, T, sv);
    }
  } else
  for (int e0 = lane; e0 < nval; e0 += 32 * 8) {
    float sv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) sv[u] = 0.f;
    for (int c = c_first; c <= c_last; ++c) {
      // only the first contributor can have started before the tile
      const int w = (c == c_first && pt.cta_start[c] < T * upt) ? 1 : 0;
      const float* src = pt.slots + ((int64_t)c * 2 + w) * (int64_t)nval;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (e0 + 32 * u < nval) sv[u] += __ldcg(src + e0 + 32 * u);
    }
    store_outputs<Op, 8>(op, e0, 32, nval, T, sv);
  }
  if (lane == 0) pt.counters[c_last] = 0;
}

// Streams the range [wu0, wu1) of warp `warp` (non-empty; the prologue ran
// on lane 0, so the other lanes first replay its cursor advances).  The
// loop runs chunk by chunk -- the units of one tile inside one segment --
// so the per-unit body carries no tile or segment bookkeeping.
template <class Op, class Issue>
__device__ __forceinline__ void tma_stream(Op& op, const Issue& issue, TmaRing& rg, const Partition& pt,
                                           const CtaTables& tb, float* red, int warp, int wu0, int wu1,
                                           int cu0, int cu1, int* status) {
  const bool leader = (threadIdx.x & 31) == 0;
  if (!leader)
    for (int i = 0; i < rg.S && rg.next.seg < 3; ++i) rg.issue_next(issue, i, Op::kUnitBytes, false);
  const int upt = pt.upt;
  UnitSeq sq;
  sq.init(wu0, wu1, upt);
  int s = 0, sp = 0;
  uint32_t ph = 0;
  typename Op::Buf buf;
  // L2 prefetch: unit kc + S + D of a chunk is prefetched when unit kc + S
  // is copied into the ring (D = Op::kPrefetch), the chunk's units S .. S +
  // D - 1 when the chunk starts
  constexpr int D = Op::kPrefetch;
  while (sq.seg < 3) {
    const int t = sq.t, kc0 = sq.kc;
    const int n = (upt - kc0) < (sq.end - sq.u) ? (upt - kc0) : (sq.end - sq.u);
    if (D > 0 && leader)
      for (int i = 0; i < D && rg.S + i < n; ++i) op.prefetch(t, kc0 + rg.S + i);
    op.zero();
    for (int kc = kc0; kc < kc0 + n; ++kc) {
      if (!mbar_wait_bounded(rg.bars + 8u * (uint32_t)s, ph, status)) return;
      op.read(buf, rg.ring + (uint32_t)s * Op::kUnitBytes, s, t);
      __syncwarp();
      if (D > 0 && leader && kc + rg.S + D < kc0 + n) op.prefetch(t, kc + rg.S + D);
      if (rg.next.seg < 3) rg.issue_next(issue, s, Op::kUnitBytes, leader);  // warp-uniform test
      op.side(sp, t * upt + kc, kc);
      if (++sp == rg.P) sp = 0;
      if (++s == rg.S) {
        s = 0;
        ph ^= 1u;
      }
      op.compute(buf, t, kc);
    }
    op.end_chunk();
    if (sq.seg == 2) op.store_tile(t);
    else close_split(op, pt, tb, red, warp, t, sq.seg == 0 ? 1 : 0, cu0, cu1);
    sq.skip(n);
  }
}

// Host-side partition sizing shared by the launchers.
struct PartitionPlan {
  int64_t tiles = 0, upt = 0, units = 0;
  int grid = 0;
  bool tile_aligned = false;  // CTA ranges start on tile boundaries (no cross-CTA tiles)
  size_t counters_bytes = 0, slots_bytes = 0;
  size_t total() const { return counters_bytes + slots_bytes; }
};

// Unit start of every CTA of a TMA-engine launch (start[grid] = units).
// Tile-aligned ranges save the cross-CTA reduction at the end of the
// launch (no tile is split across CTAs), so they are taken when cheap:
// whole tiles on min(grid, tiles)
// CTAs when the busiest of them holds at most `slack` units more than the
// busiest CTA of the equal split over all pl.grid CTAs, else the equal
// split.  (Fewer tiles than CTAs must not shrink the grid: a tall, narrow
// matrix would then leave most SMs idle.)
inline void plan_cta_starts(PartitionPlan& pl, int* start, int64_t slack) {
  const int64_t split_max = (pl.units + pl.grid - 1) / pl.grid;
  const int G2 = pl.grid < pl.tiles ? pl.grid : (int)pl.tiles;
  const int64_t aligned_max = (pl.tiles + G2 - 1) / G2 * pl.upt;
  if (aligned_max <= split_max + slack) {
    pl.grid = G2;
    pl.tile_aligned = true;
    for (int c = 0; c <= G2; ++c) start[c] = (int)(pl.tiles * c / G2 * pl.upt);
  } else {
    pl.tile_aligned = false;
    for (int c = 0; c <= pl.grid; ++c) start[c] = (int)(pl.units * c / pl.grid);
  }
}

inline PartitionPlan plan_partition(int64_t tiles, int64_t upt, int warps, int sms, int nout, int64_t M,
                                    int tile_w) {
  PartitionPlan pl;
  pl.tiles = tiles;
  pl.upt = upt;
  pl.units = tiles * upt;
  if (pl.units == 0) return pl;
  // at least ~2 units per warp before another CTA is worth its table set-up
  const int64_t want = (pl.units + 2 * warps - 1) / (2 * warps);
  const int cap = sms < kMaxGrid ? sms : kMaxGrid;
  pl.grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
  pl.counters_bytes = kCounterBytes;
  pl.slots_bytes = (size_t)pl.grid * 2 * (size_t)(nout * M * tile_w) * sizeof(float);
  return pl;
}

// Shared memory for the warps' partial slots of one launch.
__host__ __device__ inline size_t red_bytes(int warps, int nout, int64_t M, int tile_w) {
  return (size_t)warps * 2 * (size_t)(nout * M * tile_w) * sizeof(float);
}

}  // namespace pp
