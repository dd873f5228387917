// Work partition and deterministic split-K reduction shared by the fused
// dequant GEMV kernels.
//
// A "tile" is the set of output features one warp accumulates (8 rows for
// the file layout, 32 or 64 features for the kernel layout); a "unit" is
// one K chunk of a tile.  Units are numbered tile-major and the grid's CTAs
// take equal contiguous ranges.  Inside a CTA all warps work on the same
// tile at a time: warp w takes units seg0 + w, seg0 + w + NW, ... of the
// CTA's segment of that tile, then the warps' FP32 partials are summed in
// warp order through shared memory.  A tile that lies wholly inside the
// CTA's range is stored directly; a tile shared with neighbouring CTAs (at
// most the first and the last tile of a range) is reduced through the
// workspace: each CTA writes its partial, fences, bumps the tile counter,
// and the last CTA to arrive sums all partials in CTA order, stores the
// result and resets the counter to zero.  No CTA ever waits for another.
// Loads for a warp's next unit are issued before the current unit is
// decoded, across tile boundaries too, so the barrier at the end of a tile
// overlaps the next tile's loads; a second cursor runs kPrefetch units
// further ahead and pulls those units into L2 with bulk prefetches, which
// keeps enough bytes in flight per SM without spending registers.
#pragma once

#include <stdint.h>

namespace pp {

// Workspace: a fixed 4 KiB counter block (one arrival counter per CTA,
// zero between launches) followed by the partial-sum slots.  A tile shared
// by CTAs c_first < ... < c_last uses counter c_last: c_last contains the
// tile's last unit and starts inside it, so no CTA is c_last of two shared
// tiles.  Counters therefore never overlap slot memory of any other plan.
constexpr int kMaxGrid = 1024;
constexpr size_t kCounterBytes = kMaxGrid * sizeof(int);

struct Partition {
  int64_t units;  // total units
  int upt;        // units per tile
  int* counters;  // [kMaxGrid] arrival counters (zero between launches)
  float* slots;   // [grid][2][nout * M * tile_w] cross-CTA partials
};

__device__ __forceinline__ int64_t cta_of_unit(int64_t x, int64_t U, int64_t G) {
  // largest c with floor(U*c/G) <= x
  const int64_t c = ((x + 1) * G + U - 1) / U - 1;
  return c < G - 1 ? c : G - 1;
}

// Op interface (device struct):
//   static constexpr int kWarps, kTileW, kNOut, kNBat, kSlot (= kNOut*kNBat*kTileW)
//   using Buf = ...;
//   void zero();                                   accumulators := 0
//   void load(Buf&, int64_t tile, int kc) const;   issue loads of one unit
//   void prefetch(int64_t tile, int kc) const;     L2 prefetch of one unit
//   void compute(const Buf&, int64_t tile, int kc);
//   void write_partial(float* red) const;          this warp's kSlot floats
//   int  M() const; int64_t N() const;
//   void store(int out, int bat, int64_t f, float v) const;  final FP16 store
template <class Op>
__device__ __forceinline__ void run_partition(Op& op, const Partition& pt, float* red, int* s_flag) {
  constexpr int NW = Op::kWarps;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int64_t U = pt.units;
  const int64_t G = gridDim.x;
  const int64_t cu0 = U * blockIdx.x / G, cu1 = U * (blockIdx.x + 1) / G;
  if (cu0 >= cu1) return;  // uniform over the CTA
  const int upt = pt.upt;
  const int64_t t_first = cu0 / upt;
  const int64_t t_last = (cu1 - 1) / upt;

  // this warp's unit cursor: (tile, unit); valid == false at the end
  int64_t cur_t = 0, cur_u = 0, nxt_t = 0, nxt_u = 0;
  bool cur_ok = false, nxt_ok = false;
  auto first_from = [&](int64_t tt, int64_t& ot, int64_t& ou) -> bool {
    for (; tt <= t_last; ++tt) {
      const int64_t s0 = tt * upt > cu0 ? tt * upt : cu0;
      const int64_t s1 = (tt + 1) * upt < cu1 ? (tt + 1) * upt : cu1;
      if (s0 + warp < s1) {
        ot = tt;
        ou = s0 + warp;
        return true;
      }
    }
    return false;
  };
  auto advance = [&](int64_t t, int64_t u, int64_t& ot, int64_t& ou) -> bool {
    const int64_t s1 = (t + 1) * upt < cu1 ? (t + 1) * upt : cu1;
    if (u + NW < s1) {
      ot = t;
      ou = u + NW;
      return true;
    }
    return first_from(t + 1, ot, ou);
  };

  typename Op::Buf bufA, bufB;
  cur_ok = first_from(t_first, cur_t, cur_u);
  // prefetch cursor: kPrefetch units of this warp ahead of the current one
  constexpr int kPrefetch = 4;
  int64_t pf_t = cur_t, pf_u = cur_u;
  bool pf_ok = cur_ok;
  if (cur_ok) {
    op.load(bufA, cur_t, (int)(cur_u - cur_t * upt));
    nxt_ok = advance(cur_t, cur_u, nxt_t, nxt_u);
    // units cur+2 .. cur+kPrefetch now; cur+1 is loaded into registers
    pf_ok = nxt_ok && advance(nxt_t, nxt_u, pf_t, pf_u);
#pragma unroll 1
    for (int i = 2; i <= kPrefetch && pf_ok; ++i) {
      op.prefetch(pf_t, (int)(pf_u - pf_t * upt));
      pf_ok = advance(pf_t, pf_u, pf_t, pf_u);
    }
  }

  int64_t pend[2];
  int npend = 0;
  const int M = op.M();
  constexpr int TW = Op::kTileW;
  const int nval = Op::kNOut * M * TW;  // compact partial: [out][bat < M][fi]

  for (int64_t tt = t_first; tt <= t_last; ++tt) {
    op.zero();
    while (cur_ok && cur_t == tt) {
      if (pf_ok) {
        op.prefetch(pf_t, (int)(pf_u - pf_t * upt));
        pf_ok = advance(pf_t, pf_u, pf_t, pf_u);
      }
      if (nxt_ok) op.load(bufB, nxt_t, (int)(nxt_u - nxt_t * upt));
      op.compute(bufA, cur_t, (int)(cur_u - cur_t * upt));
      bufA = bufB;
      cur_ok = nxt_ok;
      cur_t = nxt_t;
      cur_u = nxt_u;
      if (cur_ok) nxt_ok = advance(cur_t, cur_u, nxt_t, nxt_u);
    }
    op.write_partial(red + warp * Op::kSlot);
    __syncthreads();
    const bool whole = (tt * upt >= cu0) && ((tt + 1) * upt <= cu1);
    const int which = tt == t_first ? 0 : 1;
    float* slot = pt.slots + ((int64_t)blockIdx.x * 2 + which) * (int64_t)nval;
    for (int e = tid; e < nval; e += NW * 32) {
      const int o = e / (M * TW);
      const int rem = e - o * M * TW;
      const int bat = rem / TW;
      const int fi = rem - bat * TW;
      const int ri = (o * Op::kNBat + bat) * TW + fi;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += red[w * Op::kSlot + ri];
      if (whole) {
        const int64_t f = tt * TW + fi;
        if (f < op.N()) op.store(o, bat, f, s);
      } else {
        __stcg(slot + e, s);
      }
    }
    if (!whole && npend < 2) pend[npend++] = tt;
    __syncthreads();
  }

  // tiles shared with other CTAs: last arrival reduces in CTA order
  for (int i = 0; i < npend; ++i) {
    const int64_t tt = pend[i];
    const int64_t c_first = cta_of_unit(tt * upt, U, G);
    const int64_t c_last = cta_of_unit(tt * upt + upt - 1, U, G);
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int old = atomicAdd(pt.counters + c_last, 1);
      *s_flag = (old == (int)(c_last - c_first)) ? 1 : 0;
    }
    __syncthreads();
    if (*s_flag) {
      __threadfence();
      for (int e = tid; e < nval; e += NW * 32) {
        const int o = e / (M * TW);
        const int rem = e - o * M * TW;
        const int bat = rem / TW;
        const int fi = rem - bat * TW;
        float s = 0.f;
        for (int64_t c = c_first; c <= c_last; ++c) {
          // only the first contributor can have started before the tile
          const int w = (c == c_first && U * c / G < tt * upt) ? 1 : 0;
          s += __ldcg(pt.slots + (c * 2 + w) * (int64_t)nval + e);
        }
        const int64_t f = tt * TW + fi;
        if (f < op.N()) op.store(o, bat, f, s);
      }
      if (tid == 0) pt.counters[c_last] = 0;
    }
    __syncthreads();
  }
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

}  // namespace pp
