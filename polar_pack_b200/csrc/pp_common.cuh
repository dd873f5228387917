// Shared device helpers for the polar_pack B200 kernels (sm_100a).
//
// Lookup tables live in shared memory, replicated once per warp lane so
// that a warp-wide gather with 32 random indices is one conflict-free
// shared-memory wavefront: lane l always reads bank l.  A table entry is
// a 256-byte row; copy l of entry i sits at byte  i*256 + slot*128 + 4*l.
// That makes the gather address for code byte b equal to
// __byte_perm(code, 4*lane, 0x76b4) -- one PRMT per table read.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

// The dynamic shared memory of every kernel in this library.  Addressing
// the tables through the symbol (not a pointer) lets the table offset fold
// into the shared-load instruction.
extern __shared__ __align__(1024) uint8_t pp_smem[];

namespace pp {

constexpr int kWarpSize = 32;

// ----------------------------------------------------------------- PTX --
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Streaming 128-bit load of packed codes: read once, keep out of L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Activation / table loads: small, reused by many warps -> cache in L1.
__device__ __forceinline__ uint2 ldg_u2(const void* p) {
  return __ldg(reinterpret_cast<const uint2*>(p));
}
__device__ __forceinline__ uint32_t ldg_u32(const void* p) {
  return __ldg(reinterpret_cast<const unsigned int*>(p));
}
__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
  return __ldg(reinterpret_cast<const unsigned short*>(p));
}

// Coherent loads for data that the previous kernel of the stream may have
// written while this one was already running (launch overlap): activations
// and the plug correction.  The read-only path above is for weights only.
__device__ __forceinline__ uint2 ld_u2(const void* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t ld_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint16_t ld_u16(const void* p) { return *reinterpret_cast<const uint16_t*>(p); }

// Per-thread prefetch of the cache line holding `p` into L2 (one
// instruction for a whole warp's worth of different rows).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

// ------------------------------------------- programmatic dependent launch --
// A kernel launched with programmatic stream serialisation may start while
// the previous kernel of its stream is still running.  pdl_wait() blocks
// until that kernel has completed and its memory is visible; everything a
// kernel does before it must not depend on the previous kernel's output.
// pdl_launch_dependents() lets the next such kernel start launching.  Both
// are no-ops for an ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------ TMA + mbarrier --
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Prefetch of one tensor-map box into L2 (no shared-memory destination, no
// barrier); the same alignment rule for x as tma_load_2d.
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Raises the transaction count of the current phase without arriving: the
// phase cannot complete before a later arrive, whatever copies finish first.
__device__ __forceinline__ void mbar_expect_tx_only(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of the barrier, giving up after a bounded number
// of polls (each try_wait already suspends for a while): on timeout the
// status word is set and false is returned, so the kernel always ends.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int* status) {
  for (int i = 0; i < (1 << 21); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(status, 1);
  return false;
}

// 2D tiled TMA load into this CTA's shared memory, completing on `bar`.  x is the innermost
// coordinate; x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Bulk copy (no tensor map, one destination CTA) of `bytes` from global memory to
// this CTA's shared memory, completing on `bar`.  Both addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t saddr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
  return v;
}

// Small shared-memory loads by 32-bit shared address.  Like lds128 they
// are volatile (kept in order with the mbarrier waits, which are volatile
// too) but carry no memory clobber, so ordinary loads may move across them.
__device__ __forceinline__ uint2 lds_u2(uint32_t saddr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(saddr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t saddr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(saddr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t saddr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(saddr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t saddr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(saddr));
  return v;
}
__device__ __forceinline__ void sts_u32(uint32_t saddr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(saddr), "r"(v) : "memory");
}

// D += A(16x16, row) * B(16x8, col), FP16 inputs, FP32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lo_pair(uint32_t x, uint32_t y) { return __byte_perm(x, y, 0x5410); }
__device__ __forceinline__ uint32_t hi_pair(uint32_t x, uint32_t y) { return __byte_perm(x, y, 0x7632); }

// ------------------------------------------------------ quad LUT region --
// Four tables of half2 words: T0 = (norm, norm), T1 = (cos1, sin1),
// T2 = (cos2, sin2), T3 = (cos3, sin3).  Table t is at region (t>>1)
// (64 KiB each) and slot (t&1).
constexpr uint32_t kQuadLutBytes = 2u * 65536u;

__device__ __forceinline__ uint32_t lut_off(int table) {
  return (uint32_t)(table >> 1) * 65536u + (uint32_t)(table & 1) * 128u;
}

// Fill the replicated quad tables from the seven FP16[256] tables in three
// steps: every thread loads its share of the 1024 table words into
// registers (all global loads of a thread in flight at once; blockDim.x >=
// 128), stores them to `stage` (4 KiB of shared memory), and after a CTA
// barrier the words fan out to the 32 lane copies with 16-byte stores,
// eight consecutive threads per 128-byte entry row.
constexpr int kLutWordsPerThread = 8;

__device__ __forceinline__ void quad_lut_load(uint32_t (&v)[kLutWordsPerThread], const __half* const* luts) {
#pragma unroll
  for (int j = 0; j < kLutWordsPerThread; ++j) {
    const int i = threadIdx.x + j * (int)blockDim.x;
    v[j] = 0u;
    if (i < 1024) {
      const int t = i >> 8, e = i & 255;
      const uint16_t* lo = reinterpret_cast<const uint16_t*>(luts[t == 0 ? 0 : 2 * t - 1]);
      const uint16_t* hi = reinterpret_cast<const uint16_t*>(luts[t == 0 ? 0 : 2 * t]);
      v[j] = (uint32_t)ldg_u16(lo + e) | ((uint32_t)ldg_u16(hi + e) << 16);
    }
  }
}

__device__ __forceinline__ void quad_lut_stage(uint32_t* stage, const uint32_t (&v)[kLutWordsPerThread]) {
#pragma unroll
  for (int j = 0; j < kLutWordsPerThread; ++j) {
    const int i = threadIdx.x + j * (int)blockDim.x;
    if (i < 1024) stage[i] = v[j];
  }
}

// after a barrier that follows quad_lut_stage
__device__ __forceinline__ void quad_lut_fanout(uint8_t* lut, const uint32_t* stage) {
  for (int idx = threadIdx.x; idx < 4 * 256 * 8; idx += blockDim.x) {
    const int t = idx >> 11, e = (idx >> 3) & 255, part = idx & 7;
    const uint32_t w = stage[idx >> 3];
    *reinterpret_cast<uint4*>(lut + lut_off(t) + (uint32_t)e * 256u + (uint32_t)part * 16u) =
        make_uint4(w, w, w, w);
  }
}

// Prepared tables: the same 128 KiB image, written once to global memory
// (pp_quad_prepare_tables) and copied into shared memory as is.  Thread
// `i` of the preparing grid writes 16-byte chunk i.
__device__ __forceinline__ uint32_t quad_table_word(const __half* const* luts, int t, int e) {
  const uint16_t* lo = reinterpret_cast<const uint16_t*>(luts[t == 0 ? 0 : 2 * t - 1]);
  const uint16_t* hi = reinterpret_cast<const uint16_t*>(luts[t == 0 ? 0 : 2 * t]);
  return (uint32_t)ldg_u16(lo + e) | ((uint32_t)ldg_u16(hi + e) << 16);
}

// All three steps; called by every thread of the CTA, caller syncs after.
__device__ __forceinline__ void build_quad_lut(uint8_t* lut, uint32_t* stage, const __half* const* luts) {
  uint32_t v[kLutWordsPerThread];
  quad_lut_load(v, luts);
  quad_lut_stage(stage, v);
  __syncthreads();
  quad_lut_fanout(lut, stage);
}

// Decoded tuple as three half2 words:
//   p1 = (w1, rs), p2 = (w2, rss), p3 = (w3, w4)
// following the FP16 product chain of the reference kernel: every product
// rounds to FP16 (round to nearest even) exactly once.
struct QuadDec {
  uint32_t p1, p2, p3;
};

// Shared-memory placement of the quad tables.  DIRECT: the tables start at
// a 64 KiB boundary.  Then __byte_perm(code, lb, 0x7634) -- code byte 3 in
// bits 8..15, the lane offset in bits 0..7, the 64 KiB-aligned region
// address in bits 16..31 -- is the complete shared address of a gather,
// and the second table of a region (+128) is a load immediate: no add per
// gather.  Otherwise each gather adds the table base.

template <int OFF>
__device__ __forceinline__ uint32_t lds_off(uint32_t saddr) {
  uint32_t v;
  asm("ld.shared.b32 %0, [%1+%2];" : "=r"(v) : "r"(saddr), "n"(OFF));
  return v;
}

// DIRECT: lb0 = lut_saddr | (4 * lane) and lb1 = (lut_saddr + 65536) |
// (4 * lane) address the two 64 KiB table regions, add0 = add1 = 0.
// Otherwise lb0 = lb1 = 4 * lane, add0 = lut_saddr, add1 = lut_saddr + 65536.
template <bool DIRECT>
__device__ __forceinline__ QuadDec decode_quad(uint32_t code, uint32_t lb0, uint32_t lb1, uint32_t add0,
                                               uint32_t add1) {
  const uint32_t a0 = __byte_perm(code, lb0, 0x7634) + (DIRECT ? 0u : add0);  // norm (byte 3)
  const uint32_t a1 = __byte_perm(code, lb0, 0x7624) + (DIRECT ? 0u : add0);  // t1   (byte 2)
  const uint32_t a2 = __byte_perm(code, lb1, 0x7614) + (DIRECT ? 0u : add1);  // t2   (byte 1)
  const uint32_t a3 = __byte_perm(code, lb1, 0x7604) + (DIRECT ? 0u : add1);  // t3   (byte 0)
  const uint32_t rr = lds_off<0>(a0);
  const uint32_t cs1 = lds_off<128>(a1);
  const uint32_t cs2 = lds_off<0>(a2);
  const uint32_t cs3 = lds_off<128>(a3);
  const __half2 p1 = __hmul2_rn(u2h(rr), u2h(cs1));                // (r*c1, r*s1)
  const __half2 p2 = __hmul2_rn(__high2half2(p1), u2h(cs2));       // (rs*c2, rs*s2)
  const __half2 p3 = __hmul2_rn(__high2half2(p2), u2h(cs3));       // (rss*c3, rss*s3)
  return QuadDec{h2u(p1), h2u(p2), h2u(p3)};
}

// ------------------------------------------------------ dual LUT region --
// Amplitude table: 64 FP32 entries, indexed by the raw code bits 15..10
// (the +32768 bias of the stored int16 flips bit 15, folded into the
// table order).  Phase table: 1024 half2 (cos, sin) entries.  Entry
// stride 128 bytes (32 lanes x 4 bytes) in both.
constexpr uint32_t kDualAmpBytes = 64u * 128u;
constexpr uint32_t kDualPhaseBytes = 1024u * 128u;
constexpr uint32_t kDualLutBytes = kDualAmpBytes + kDualPhaseBytes;

// Dual tables in two steps, like the quad ones: the 64 + 1024 table words
// are staged (4352 bytes), then after a CTA barrier fanned out to the 32
// lane copies.
__device__ __forceinline__ void dual_lut_stage(uint32_t* stage, const __half* amp_lut, const __half* cos_lut,
                                               const __half* sin_lut) {
  const uint16_t* a = reinterpret_cast<const uint16_t*>(amp_lut);
  const uint16_t* c = reinterpret_cast<const uint16_t*>(cos_lut);
  const uint16_t* s = reinterpret_cast<const uint16_t*>(sin_lut);
  for (int e = threadIdx.x; e < 64 + 1024; e += blockDim.x) {
    uint32_t v;
    if (e < 64) {
      // stored bits b = ((u >> 10) & 63) ^ 32 where u = p + 32768
      v = __float_as_uint(__half2float(__ushort_as_half(ldg_u16(a + (e ^ 32)))));
    } else {
      v = (uint32_t)ldg_u16(c + (e - 64)) | ((uint32_t)ldg_u16(s + (e - 64)) << 16);
    }
    stage[e] = v;
  }
}

// after a barrier that follows dual_lut_stage
__device__ __forceinline__ void dual_lut_fanout(uint8_t* smem, const uint32_t* stage) {
  for (int idx = threadIdx.x; idx < (64 + 1024) * 8; idx += blockDim.x) {
    const int e = idx >> 3, part = idx & 7;
    const uint32_t v = stage[e];
    const uint32_t off = e < 64 ? (uint32_t)e * 128u : kDualAmpBytes + (uint32_t)(e - 64) * 128u;
    *reinterpret_cast<uint4*>(smem + off + (uint32_t)part * 16u) = make_uint4(v, v, v, v);
  }
}

__device__ __forceinline__ void build_dual_lut(uint8_t* smem, uint32_t* stage, const __half* amp_lut,
                                               const __half* cos_lut, const __half* sin_lut) {
  dual_lut_stage(stage, amp_lut, cos_lut, sin_lut);
  __syncthreads();
  dual_lut_fanout(smem, stage);
}

}  // namespace pp
