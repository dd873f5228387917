// Shared-memory layout of one quad GEMV CTA: plain C++ shared by the host
// planner, the kernel and a CPU test (compiled there with g++).
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define PP_HD __host__ __device__
#else
#define PP_HD
#endif

namespace pp {

constexpr uint32_t kQuadTableBytes = 2u * 65536u;  // the four replicated tables
constexpr uint32_t kQuadUnitBytes = 2048u;         // one TMA ring slot
// fused plug correction: unit offsets each warp keeps in shared memory (its
// unit range [wu0, wu1] inclusive, so at most kPlugTabEntries - 1 units)
constexpr uint32_t kPlugTabEntries = 64u;

// Shared-memory layout of one CTA, computed identically on the host (for
// the expected dynamic base) and in the kernel (for the actual one).  The
// tables go to the first 64 KiB boundary when everything else fits around
// them (DIRECT gathers); the consumer rings fill the gap below the tables
// (region A), then the space above (region B); the ring mbarriers, a flag
// word, the per-CTA int tables, the scratch block and (with a fused plug
// correction) the plug region go where room is left.  The scratch block
// stages the table build and afterwards holds the consumers' partial slots
// (written while other rings are still streaming, so it never overlaps a
// ring).  The plug region holds, per warp, S + 1 plug slots of pcap bytes
// (one more than ring slots, so the unit being computed keeps its slot
// while the next ones arrive), then the warps' unit-offset tables.  Without room for the aligned placement the tables start
// at the base.
struct QuadLayout {
  uint32_t lut, ringA, ringB, bars, flag, tables, scratch, plug, ptab;
  int splitw, direct, ok;
};

// bytes of the plug region for nw warps of S + 1 slots of pcap bytes (0: none)
PP_HD inline uint32_t quad_plug_region_bytes(int nw, int S, uint32_t pcap) {
  return pcap ? (uint32_t)nw * ((uint32_t)(S + 1) * pcap + kPlugTabEntries * 4u) : 0u;
}

// bytes of the per-CTA int tables (warp range starts, their tiles, split
// tile counters: 4 * warps + 2 ints, at most 16 warps)
constexpr uint32_t kQuadTablesBytes = 512u;

PP_HD inline QuadLayout quad_layout(uint32_t base, uint32_t size, int nw, int S, uint32_t redb,
                                    bool allow_direct, uint32_t pcap = 0u) {
  QuadLayout L{};
  const uint32_t plugb = quad_plug_region_bytes(nw, S, pcap);
  const uint32_t rw = (uint32_t)S * kQuadUnitBytes;
  const uint32_t barb = ((uint32_t)(nw * S * 8) + 15u) & ~15u;
  const uint32_t smallb = barb + 16u + kQuadTablesBytes;  // bars, flag, tables
  const uint32_t scr = ((redb + 15u) & ~15u) > 4096u ? ((redb + 15u) & ~15u) : 4096u;
  const uint64_t end = (uint64_t)base + size;
  const uint32_t lut = (base + 0xFFFFu) & ~0xFFFFu;
  if (allow_direct && (uint64_t)lut + kQuadTableBytes <= end) {
    const uint32_t a = (base + 1023u) & ~1023u;
    const int inA = lut > a ? ((lut - a) / rw < (uint32_t)nw ? (int)((lut - a) / rw) : nw) : 0;
    uint64_t fa = (uint64_t)a + (uint64_t)inA * rw;  // free space [fa, lut)
    uint64_t fb = (uint64_t)lut + kQuadTableBytes;     // free space [fb, end)
    L.lut = lut;
    L.ringA = a;
    L.splitw = inA;
    L.ringB = (uint32_t)fb;
    fb += (uint64_t)(nw - inA) * rw;
    uint64_t* at = (fa + smallb <= lut) ? &fa : &fb;
    L.bars = (uint32_t)*at;
    L.flag = L.bars + barb;
    L.tables = L.flag + 16u;
    *at += smallb;
    at = (fa + scr <= lut) ? &fa : &fb;
    L.scratch = (uint32_t)*at;
    *at += scr;
    if (plugb) {
      at = (fa + plugb <= lut) ? &fa : &fb;
      L.plug = (uint32_t)*at;
      L.ptab = L.plug + (uint32_t)nw * (uint32_t)(S + 1) * pcap;
      *at += plugb;
    }
    if (fb <= end) {
      L.direct = 1;
      L.ok = 1;
      return L;
    }
  }
  L = QuadLayout{};
  L.lut = base;
  uint64_t p = ((uint64_t)base + kQuadTableBytes + 1023u) & ~(uint64_t)1023u;
  L.ringA = (uint32_t)p;
  L.splitw = nw;
  L.ringB = (uint32_t)p;
  p += (uint64_t)nw * rw;
  L.bars = (uint32_t)p;
  L.flag = L.bars + barb;
  L.tables = L.flag + 16u;
  p += smallb;
  L.scratch = (uint32_t)p;
  p += scr;
  if (plugb) {
    L.plug = (uint32_t)p;
    L.ptab = L.plug + (uint32_t)nw * (uint32_t)(S + 1) * pcap;
    p += plugb;
  }
  L.ok = p <= end;
  return L;
}

}  // namespace pp
