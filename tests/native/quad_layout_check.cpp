// CPU check of the quad GEMV shared-memory layout (polar_pack_b200/csrc/
// quad_layout.h): for every kernel variant, batch size, ring depth and a
// range of dynamic-base addresses, each block lies inside the window, no two
// blocks overlap, alignments hold, and DIRECT implies 64 KiB-aligned tables.
// Prints one line per variant with the depth the host planner would pick.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../polar_pack_b200/csrc/quad_layout.h"

using namespace pp;

struct Blk {
  uint64_t a, b;
  const char* what;
};

static int check(uint32_t base, uint32_t size, int nw, int S, uint32_t redb, bool direct_ok, uint32_t pcap) {
  const QuadLayout L = quad_layout(base, size, nw, S, redb, direct_ok, pcap);
  if (!L.ok) return 0;
  const uint64_t end = (uint64_t)base + size;
  const uint32_t rw = (uint32_t)S * kQuadUnitBytes;
  std::vector<Blk> b;
  b.push_back({L.lut, (uint64_t)L.lut + kQuadTableBytes, "tables"});
  for (int w = 0; w < nw; ++w) {
    const uint64_t r = w < L.splitw ? L.ringA + (uint64_t)w * rw : L.ringB + (uint64_t)(w - L.splitw) * rw;
    if (r % 1024) {
      printf("FAIL ring %d not 1 KiB aligned\n", w);
      return -1;
    }
    b.push_back({r, r + rw, "ring"});
  }
  b.push_back({L.bars, (uint64_t)L.bars + (uint64_t)nw * S * 8u, "bars"});
  if (L.bars % 8) {
    printf("FAIL bars misaligned\n");
    return -1;
  }
  b.push_back({L.flag, (uint64_t)L.flag + 4u, "flag"});
  b.push_back({L.tables, (uint64_t)L.tables + kQuadTablesBytes, "tables"});
  if (L.tables % 16 || (uint32_t)(4 * nw + 2) * 4u > kQuadTablesBytes) {
    printf("FAIL int tables\n");
    return -1;
  }
  const uint32_t scr = ((redb + 15u) & ~15u) > 4096u ? ((redb + 15u) & ~15u) : 4096u;
  if (L.scratch % 16) {
    printf("FAIL scratch misaligned\n");
    return -1;
  }
  b.push_back({L.scratch, (uint64_t)L.scratch + scr, "scratch"});
  if (pcap) {
    if (L.plug % 16 || L.ptab % 16 || L.ptab != L.plug + (uint32_t)nw * (S + 1) * pcap) {
      printf("FAIL plug region misaligned or misplaced\n");
      return -1;
    }
    b.push_back({L.plug, (uint64_t)L.plug + (uint64_t)nw * (S + 1) * pcap, "plug slots"});
    b.push_back({L.ptab, (uint64_t)L.ptab + (uint64_t)nw * kPlugTabEntries * 4u, "plug tables"});
  }
  if (L.direct && (L.lut % 65536u)) {
    printf("FAIL direct tables not 64 KiB aligned\n");
    return -1;
  }
  if (L.lut % 16) {
    printf("FAIL tables misaligned\n");
    return -1;
  }
  for (size_t i = 0; i < b.size(); ++i) {
    if (b[i].a < base || b[i].b > end) {
      printf("FAIL %s [%llu,%llu) outside [%u,%llu) nw=%d S=%d redb=%u\n", b[i].what, (unsigned long long)b[i].a,
             (unsigned long long)b[i].b, base, (unsigned long long)end, nw, S, redb);
      return -1;
    }
    for (size_t j = i + 1; j < b.size(); ++j)
      if (b[i].a < b[j].b && b[j].a < b[i].b) {
        printf("FAIL %s overlaps %s (nw=%d S=%d redb=%u base=%u)\n", b[i].what, b[j].what, nw, S, redb, base);
        return -1;
      }
  }
  return L.direct ? 2 : 1;
}

int main() {
  const struct {
    const char* name;
    int nw, tile_w, mmax;
    uint32_t pcap;
  } variants[] = {{"nk1", 16, 8, 8, 0u},  {"nk2", 8, 8, 16, 0u}, {"kn1", 8, 32, 8, 0u},
                  {"kn2", 4, 32, 16, 0u}, {"nk1plug", 16, 8, 1, 512u}};
  const uint32_t bases[] = {0u, 16u, 1024u, 2048u, 4096u, 40000u, 65536u - 1024u, 65536u};
  const uint32_t sizes[] = {232448u, 200000u, 166912u};
  long n = 0;
  for (auto& v : variants)
    for (int M = 1; M <= v.mmax; ++M) {
      const uint32_t redb = (uint32_t)v.nw * 2u * 4u * (uint32_t)M * (uint32_t)v.tile_w * 4u;
      for (uint32_t base : bases)
        for (uint32_t size : sizes)
          for (int S = 1; S <= 4; ++S)
            for (int d = 0; d < 2; ++d) {
              if (check(base, size, v.nw, S, redb, d != 0, v.pcap) < 0) return 1;
              ++n;
            }
      // what the host planner picks for the usual window (1 KiB reserved, 227 KiB)
      int plain = 0, pick = 0, direct = 0;
      for (int S = 4; S >= 1 && !pick; --S) {
        if (!quad_layout(1024u, 232448u, v.nw, S, redb, false, v.pcap).ok) continue;
        if (!plain) plain = S;
        if (S >= 2 && quad_layout(1024u, 232448u, v.nw, S, redb, true, v.pcap).direct) pick = S, direct = 1;
      }
      if (!pick) pick = plain;
      if (M == 1 || M == v.mmax) printf("%s M=%d stages=%d direct=%d\n", v.name, M, pick, direct);
      if (pick == 0) {
        printf("FAIL no layout for %s M=%d\n", v.name, M);
        return 1;
      }
    }
  printf("OK %ld layouts\n", n);
  return 0;
}
