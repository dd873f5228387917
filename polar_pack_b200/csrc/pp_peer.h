// Outputs gathered over the GPUs of one node through peer memory.
//
// A row-sharded Linear on `world` GPUs needs every rank's output rows on
// every rank.  Instead of a separate all-gather, the GEMV's epilogue stores
// each output element into the gather buffer of every rank (mapped into
// this process with CUDA IPC; plain point-to-point stores over NVLink).  The
// last warp of the launch to finish then bumps this launch's epoch and
// writes it, with release semantics at system scope, into this rank's flag
// word on every rank.  A reader waits (gather_wait_kernel, bounded) until
// every rank's flag has reached its own epoch count, which is the number of
// launches it made into the buffer, identical on all ranks.  Epochs live in
// device memory and advance on the device, so CUDA-graph replays stay in
// step.  Reuse of a buffer while a peer may still read it is the caller's
// concern: alternating two buffers is enough when every use is followed by
// a wait on every rank.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace pp {

constexpr int kMaxPeers = 8;

struct PeerGather {
  __half* out[kMaxPeers];     // rank q's gather buffer, model-major: element model * ld + row
  uint32_t* flag[kMaxPeers];  // this rank's flag word in rank q's flag array
  int64_t ld;                 // elements between the model blocks
  int64_t row0;               // the launch's first output row in the buffer
  uint32_t* epoch;            // launches made into this buffer by this rank (device)
  uint32_t* done;             // warps of the launch that finished (zero between launches)
  int world;                  // 0: no gather (outputs go to `out` as usual)
  int ctas;                   // CTAs in the grid
  int vec;                    // ld, row0 and every out[] allow 16-byte stores of 8 rows
};

#ifdef __CUDACC__
// Called by every warp of the launch at its end.  `cta_arrivals` is the
// CTA's shared arrival counter (zeroed before the CTA's first barrier), or
// NULL in a CTA that left before setting it up (uniform over the CTA; its
// warp 0 then stands for the CTA).  A warp's stores are ordered before its
// lane 0 (__syncwarp) and lane 0's release on the CTA counter; the CTA's
// last warp acquires them and releases the CTA on the grid counter (GPU
// scope), whose last arrival acquires every CTA, advances the epoch and
// publishes it with a system-scope fence and release stores, which carry
// every store that happens before them to the peers (cumulativity).  Two
// levels keep the grid counter at one atomic per CTA, and one system-scope
// fence per launch: a fence in every warp would wait for each warp's
// stores to reach the peers.
__device__ __forceinline__ void gather_signal(const PeerGather& g, int* cta_arrivals, int cta_warps) {
  __syncwarp();
  if ((threadIdx.x & 31) != 0) return;
  if (cta_arrivals) {
    uint32_t old_cta;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                 : "=r"(old_cta)
                 : "r"((uint32_t)__cvta_generic_to_shared(cta_arrivals))
                 : "memory");
    if (old_cta != (uint32_t)cta_warps - 1u) return;
  } else if (threadIdx.x != 0) {
    return;
  }
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(g.done) : "memory");
  if (old != (uint32_t)g.ctas - 1u) return;
  *g.done = 0u;  // the next launch on the stream starts its epilogue after this one has completed
  const uint32_t e = *g.epoch + 1u;
  *g.epoch = e;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll
  for (int q = 0; q < kMaxPeers; ++q)
    if (q < g.world) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(g.flag[q]), "r"(e) : "memory");
}
#endif

}  // namespace pp
