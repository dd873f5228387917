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
// Each warp keeps one unit in flight in registers (loaded before the
// current unit is decoded) and bulk-prefetches the unit kPrefetch steps
// ahead into L2.
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
};

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
    for (int e = tid; e < nval; e += NW * 32) {
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
      for (int e = tid; e < nval; e += NW * 32) {
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

// TMA engine: same partition and reduction, but each warp streams its range
// through a private ring of S shared-memory slots filled by TMA.  Lane 0
// keeps the next S units of the warp's range in flight (one mbarrier per
// slot, phase = fill count & 1); all lanes wait for the slot, copy the unit
// into registers, sync, and lane 0 refills the slot with the unit S ahead
// before the unit is decoded.  Waits are bounded (mbar_wait_bounded).
//
// Op additions: kUnitBytes; void issue(uint32_t slot, uint32_t bar, int tile,
// int kc) const (lane 0 only); void read(Buf&, uint32_t slot) const.
template <class Op>
__device__ __forceinline__ void run_partition_tma(Op& op, const Partition& pt, float* red, int* s_flag,
                                                  uint32_t ring, uint32_t bars, int S, int* status) {
  constexpr int NW = Op::kWarps;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int U = pt.units;
  const int G = gridDim.x;
  const int cu0 = range_start(U, G, blockIdx.x), cu1 = range_start(U, G, blockIdx.x + 1);
  if (cu0 >= cu1) return;  // uniform over the CTA
  const int upt = pt.upt;
  const int M = op.M();
  const int nval = Op::kNOut * M * Op::kTileW;
  const int R = cu1 - cu0;
  const int wu0 = cu0 + range_start(R, NW, warp), wu1 = cu0 + range_start(R, NW, warp + 1);
  const uint32_t my_ring = ring + (uint32_t)(warp * S * Op::kUnitBytes);
  const uint32_t my_bar = bars + (uint32_t)(warp * S * 8);

  if (wu0 < wu1) {
    if (lane == 0) {
      for (int i = 0; i < S; ++i) mbar_init(my_bar + 8u * i, 1);
      fence_mbar_init();
    }
    __syncwarp();
    int t = wu0 / upt, kc = wu0 - t * upt;  // current unit
    const int t_first = t;
    int it = t, ikc = kc;                   // next unit to issue
    for (int i = 0; i < S && wu0 + i < wu1; ++i) {
      if (lane == 0) op.issue(my_ring + (uint32_t)(i * Op::kUnitBytes), my_bar + 8u * i, it, ikc);
      if (++ikc == upt) { ikc = 0; ++it; }
    }
    int slot = 0;
    uint32_t parity = 0;
    op.zero();
    op.begin(t, kc);
    typename Op::Buf buf;
    for (int u = wu0; u < wu1; ++u) {
      const uint32_t sl = my_ring + (uint32_t)(slot * Op::kUnitBytes);
      mbar_wait_bounded(my_bar + 8u * slot, parity, status);
      op.read(buf, sl);
      __syncwarp();
      if (u + S < wu1) {
        if (lane == 0) op.issue(sl, my_bar + 8u * slot, it, ikc);
        if (++ikc == upt) { ikc = 0; ++it; }
      }
      if (++slot == S) { slot = 0; parity ^= 1u; }
      int nt = t, nkc = kc + 1;
      if (nkc == upt) { nkc = 0; ++nt; }
      if (u + 1 < wu1) op.preload(nt, nkc);
      op.compute(buf, t, kc);
      if (nkc == 0 || u + 1 == wu1) {
        if ((t * upt >= wu0) && nkc == 0) {
          op.store_tile(t);
        } else {
          op.write_partial(red + (warp * 2 + (t == t_first ? 0 : 1)) * nval, M);
        }
        op.zero();
      }
      t = nt;
      kc = nkc;
    }
  }
  __syncthreads();
  reduce_partials(op, pt, red, s_flag, cu0, cu1, nval);
}

// Host-side partition sizing shared by the launchers.
struct PartitionPlan {
  int64_t tiles = 0, upt = 0, units = 0;
  int grid = 0;
  size_t counters_bytes = 0, slots_bytes = 0;
  size_t total() const { return counters_bytes + slots_bytes; }
};

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
