/*
 * polar_pack_b200 -- C ABI of the B200 (sm_100a) fused dequant-matmul path
 * for polar_pack's packed multi-model weight streams.
 *
 * Conventions
 *  - Every pointer argument named a tensor is DEVICE memory owned by the
 *    caller; the library allocates nothing per call.  Scalars and the
 *    `scales` arrays are host values.
 *  - FP16 data is passed as `void*` (IEEE binary16, little endian).
 *  - Strides are in ELEMENTS, like torch's Tensor.stride().
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call
 *    only enqueues work on that stream and returns; nothing synchronises.
 *  - Return value: PP_OK (0) or an error code; pp_last_error() gives a
 *    message for the calling thread.  Shape and argument errors are
 *    detected on the host before anything is enqueued.  No function traps
 *    or asserts on the device.
 *  - Workspace: entry points that split the reduction over K across warps
 *    and thread blocks need scratch memory of the size that the matching
 *    *_workspace_bytes() function returns.  It must be zero-filled ONCE
 *    when it is allocated; every call leaves it zero-filled again.  Two
 *    calls that may run concurrently must not share a workspace.
 */
#ifndef POLAR_PACK_B200_H
#define POLAR_PACK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PP_API __attribute__((visibility("default")))
#else
#define PP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PP_VERSION 1

#define PP_OK 0
#define PP_ERR_INVALID 1     /* bad shape, stride, alignment or argument */
#define PP_ERR_WORKSPACE 2   /* workspace missing or too small */
#define PP_ERR_CUDA 3        /* CUDA runtime / launch error */

/* Message describing the last error returned on this thread. */
PP_API const char* pp_last_error(void);

/* Version of this ABI (PP_VERSION). */
PP_API int pp_version(void);

/* Number of SMs of `device` (what the work partition is sized for). */
PP_API int pp_device_sm_count(int device);

/* Launch overlap (programmatic dependent launch), process-wide, off by
 * default; returns the previous setting.  No counterpart in the reference.
 * When on, pp_quad_gemm / pp_quad_linear kernels are launched so that they
 * may start while the previous kernel of their stream is still running:
 * they build their tables and start streaming codes, then wait for that
 * kernel to complete before reading activations or writing anything.
 * Contract while on: the codes, tables and plug arrays passed to those
 * calls must not be written by the kernel launched immediately before them
 * on the same stream (weights loaded earlier, as usual, are fine).
 */
PP_API int pp_set_launch_overlap(int enable);

/* ------------------------------------------------------------------ quad --
 * Kernel-layout fused dequant GEMM, the drop-in for `quad_bitpacked`
 * (reference quad_kernels.py:146-159) and its Triton kernel
 * `quad_bitpacked_kernel` (quad_kernels.py:68-143):
 *
 *   W_k = FP16 decode of codes[k][n] through the seven FP16[256] tables
 *         luts = {norm, cos1, sin1, cos2, sin2, cos3, sin3}
 *   out_k[m][n] = fp16( scales[k] * sum_k' a[m][k'] * W_k[k'][n] )   (FP32 acc)
 *
 * a: (M, K) FP16, element strides (lda_m, lda_k).
 * codes: (K, N) uint32, element strides (ldc_k, ldc_n).  Either dimension may
 *   be the contiguous one; other layouts run on a slower generic kernel.
 * out[4]: four (M, N) FP16 outputs sharing strides (ldo_m, ldo_n).
 * scales: 4 host floats (the per-model RMS `s_k`).
 * Any M >= 0, N >= 0, K >= 0 (K == 0 writes zeros, as the reference does).
 */
PP_API int pp_quad_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t ldc_k, int64_t ldc_n,
                                 size_t* bytes);

PP_API int pp_quad_gemm(const void* a, int64_t lda_m, int64_t lda_k,
                 const uint32_t* codes, int64_t ldc_k, int64_t ldc_n,
                 const void* const luts[7], const float scales[4],
                 void* const out[4], int64_t ldo_m, int64_t ldo_n,
                 int64_t M, int64_t N, int64_t K,
                 void* workspace, size_t workspace_bytes, void* stream);

/* pp_quad_gemm with its split-K scratch in a file-scope device array of the
 * library instead of a caller-provided workspace.  No counterpart in the
 * reference (its Triton launch needs no scratch); it exists for callers that
 * cannot call cudaMalloc: plugin hosts that pass only tensor pointers while
 * their own pool owns all device memory, and code that must not allocate
 * because cudaMalloc can synchronise the device.  It allocates nothing.
 * Limit: 1 MiB of scratch per device (the file layout at any batch size; the
 * kernel layout up to at least M = 6 on a 148-SM device); larger plans fail
 * with PP_ERR_WORKSPACE before anything is enqueued.  All calls on a device
 * share the one array: calls that can overlap (different streams or host
 * threads) race on it and must be serialised by the caller.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress,
 * with that device current) and keeps it; make that first call before any
 * stream capture on the device.  Each call clears the counters at the front
 * of the array on its stream before the kernel runs.
 */
PP_API int pp_quad_gemm_static_scratch(const void* a, int64_t lda_m, int64_t lda_k,
                                       const uint32_t* codes, int64_t ldc_k, int64_t ldc_n,
                                       const void* const luts[7], const float scales[4],
                                       void* const out[4], int64_t ldo_m, int64_t ldo_n,
                                       int64_t M, int64_t N, int64_t K, void* stream);

/* Prepared tables: the replicated shared-memory image of the seven FP16
 * tables (128 KiB, pp_quad_tables_bytes), written once by
 * pp_quad_prepare_tables into a caller-allocated, 16-byte aligned device
 * buffer.  The *_prepared entry points take it instead of `luts`: their
 * kernels copy it into shared memory with bulk copies instead of building
 * the replicas, which shortens every launch.  No counterpart in the
 * reference (its kernel reads the seven tables directly).  The image must
 * be prepared again whenever the tables change.
 */
PP_API int pp_quad_tables_bytes(size_t* bytes);

PP_API int pp_quad_prepare_tables(const void* const luts[7], void* tables, void* stream);

/* pp_quad_gemm with prepared tables. */
PP_API int pp_quad_gemm_prepared(const void* a, int64_t lda_m, int64_t lda_k,
                                 const uint32_t* codes, int64_t ldc_k, int64_t ldc_n,
                                 const void* tables, const float scales[4],
                                 void* const out[4], int64_t ldo_m, int64_t ldo_n,
                                 int64_t M, int64_t N, int64_t K,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* File-layout fused Linear with plug-table merge, the per-Linear decode of a
 * `.quadpack` stream (reference quaternion_packer.py:141-214: the codes of one
 * nn.Linear are (out=N, in=K) row-major at a flat stream offset; plug entries
 * replace the decoded normalised 4-tuple, quaternion_packer.py:187-193):
 *
 *   y_k[m][n] = fp16( scales[k] * sum_i x[m][i] * Wp_k[n][i] )
 *   Wp_k[n][i] = plug value if (n*K + i) is plugged, else the FP16 decode.
 *
 * x: (M, K) FP16 with strides (ldx_m, ldx_k).  codes: row n at codes + n*ldw,
 *   prepared once by pp_quad_prepare_plugs() when the Linear has plugs.
 * plug_idx / plug_vals: this Linear's slice [p_lo, p_hi) of the stream's plug
 *   table (uint32 positions, (P, 4) FP16 values), base_lo32 the low 32 bits
 *   of the Linear's stream offset.  plug_window_base: as built by
 *   pp_quad_prepare_plugs().  All three pointers may be NULL when P == 0.
 * out[4]: (M, N) FP16 with strides (ldo_m, ldo_n).
 * The plug values enter as an FP32 sparse correction added to the same
 * accumulators, so the result equals the substituted-weight product within
 * the FP32 accumulation tolerance.
 */
PP_API int pp_quad_linear_workspace_bytes(int64_t M, int64_t N, int64_t K, size_t* bytes);

PP_API int pp_quad_linear(const void* x, int64_t ldx_m, int64_t ldx_k,
                          const uint32_t* codes, int64_t ldw,
                          const uint32_t* plug_idx, const void* plug_vals,
                          const uint32_t* plug_window_base, uint32_t base_lo32,
                          const void* const luts[7], const float scales[4],
                          void* const out[4], int64_t ldo_m, int64_t ldo_n,
                          int64_t M, int64_t N, int64_t K,
                          void* workspace, size_t workspace_bytes, void* stream);

/* pp_quad_linear with prepared tables. */
PP_API int pp_quad_linear_prepared(const void* x, int64_t ldx_m, int64_t ldx_k,
                                   const uint32_t* codes, int64_t ldw,
                                   const uint32_t* plug_idx, const void* plug_vals,
                                   const uint32_t* plug_window_base, uint32_t base_lo32,
                                   const void* tables, const float scales[4],
                                   void* const out[4], int64_t ldo_m, int64_t ldo_n,
                                   int64_t M, int64_t N, int64_t K,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* Load-time preparation of one Linear's plug entries for pp_quad_linear:
 *  - plug_window_base[w] (uint32, N * ceil(K/64) + 1 entries) := number of
 *    entries of the slice [p_lo, p_hi) whose position lies before window
 *    w = (row, col/64), i.e. the index of its first plug; the last entry is P;
 *  - the norm byte of every plugged code in `codes` (row stride ldw) is set
 *    to zero, so the main kernel decodes it to exact zeros (the tables built
 *    from a stream header have norm[0] == 0, quad_kernels.py:40).
 * Positions are the stream's uint32 plug index (ascending; reference
 * quaternion_packer.py:97-116) minus base_lo32 modulo 2^32, so tables whose
 * positions wrapped past 2^32 still index correctly.  Entries outside the
 * Linear or out of order are skipped and counted into *bad_count (device
 * int, may be NULL).  Idempotent.
 */
PP_API int pp_quad_prepare_plugs(uint32_t* codes, int64_t ldw, const uint32_t* plug_idx,
                                 int64_t p_lo, int64_t p_hi, uint32_t base_lo32, int64_t N, int64_t K,
                                 uint32_t* plug_window_base, int* bad_count, void* stream);

/* Unit-major copy of one Linear's plug entries, streamed by the GEMV beside
 * the codes so that the plug correction needs no kernel of its own (no
 * reference counterpart: a load-time layout of the plug table that
 * quaternion_packer.py:187-193 merges on the host).  Work unit
 * u = t * ceil(K/64) + kc covers rows 8t..8t+7 and columns 64kc..64kc+63;
 * its segment starts at byte unit_plug_off[u] (a multiple of 16):
 *   32-byte header of eight uint32, one per tile row r:
 *     start_r | end_r << 10 | n << 20 (row 8t + r owns entries [start_r, end_r));
 *   the n entries' FP16x4 values (row-major, column ascending);
 *   their n column bytes (column - 64kc); zeros to a multiple of 16.
 * unit_plug_off has ceil(N/8) * ceil(K/64) + 1 entries; the last is the
 * stream's length.  pp_quad_unit_plugs_bytes gives a size that always
 * suffices and the number of offsets.  Inputs: the Linear's plug slice and
 * plug_window_base as for pp_quad_linear (run pp_quad_prepare_plugs first).
 */
PP_API int pp_quad_unit_plugs_bytes(int64_t N, int64_t K, int64_t n_plugs, size_t* stream_bytes,
                                    int64_t* n_offsets);

PP_API int pp_quad_prepare_unit_plugs(const uint32_t* plug_idx, const void* plug_vals, int64_t n_plugs,
                                      uint32_t base_lo32, const uint32_t* plug_window_base, int64_t N,
                                      int64_t K, void* unit_plugs, size_t unit_plugs_bytes,
                                      uint32_t* unit_plug_off, void* stream);

/* pp_quad_linear_prepared with the plug correction inside the GEMV when
 * the batch is one row (M == 1): one launch when every warp's share of the
 * work units fits its offset table (at most 63 units, i.e. about
 * 148 * 16 * 63 units per launch), else one launch per chunk of rows that
 * fits.  Other batch sizes run as pp_quad_linear_prepared, which is why the
 * CSR arguments are required as well.  unit_plugs / unit_plug_off: as
 * built by pp_quad_prepare_unit_plugs (both NULL for a Linear without
 * plugs).  Same result within the FP32
 * accumulation tolerance; the summation order of the plug terms differs.
 */
PP_API int pp_quad_linear_fused(const void* x, int64_t ldx_m, int64_t ldx_k,
                                const uint32_t* codes, int64_t ldw,
                                const uint32_t* plug_idx, const void* plug_vals,
                                const uint32_t* plug_window_base, uint32_t base_lo32,
                                const void* unit_plugs, const uint32_t* unit_plug_off,
                                const void* tables, const float scales[4],
                                void* const out[4], int64_t ldo_m, int64_t ldo_n,
                                int64_t M, int64_t N, int64_t K,
                                void* workspace, size_t workspace_bytes, void* stream);

/* Several independent file-layout Linears in ONE launch (no counterpart in
 * the reference, whose callers launch one Triton kernel per matrix; each
 * member computes what pp_quad_linear_fused computes for it).  Member j gets
 * a share of the SMs in proportion to its codes and runs there as a launch
 * of its own would, so the members' fixed per-launch costs (launch, table
 * copy, first code copies, tail of the partition) overlap instead of adding
 * up.  The members must be independent: no member reads what another writes.
 * One launch when every member has batch 1 (M == 1), unit plugs, prepared
 * tables, 16-byte aligned codes with K % 4 == 0, contiguous 8-byte aligned
 * activation rows, the same flags, at most 8 members, and fits its SM share
 * (at most 63 work units of 8 rows x 64 codes per warp;
 * pp_quad_linear_group_single_launch says whether it does); otherwise the
 * members run one after another through pp_quad_linear_fused, which neither
 * flags nor an epilogue allow (PP_ERR_INVALID).  Workspace as for the other
 * entry points (pp_quad_linear_group_workspace_bytes).
 */
typedef struct pp_quad_linear_desc {
  const void* x;                    /* (M, K) FP16, strides (ldx_m, ldx_k) */
  int64_t ldx_m, ldx_k;
  const uint32_t* codes;            /* row n at codes + n * ldw */
  int64_t ldw;
  const uint32_t* plug_idx;         /* as for pp_quad_linear_fused */
  const void* plug_vals;
  const uint32_t* plug_window_base;
  uint32_t base_lo32;
  const void* unit_plugs;
  const uint32_t* unit_plug_off;
  const void* tables;               /* prepared tables */
  float scales[4];
  void* out[4];                     /* (M, N) FP16, strides (ldo_m, ldo_n) */
  int64_t ldo_m, ldo_n;
  int64_t M, N, K;
  /* PP_QUAD_PER_MODEL_X: x holds one activation row per model (4 rows, row
   * stride ldx_m); model k multiplies row k and writes row 0 of out[k]
   * (M == 1).  The four models of a decode step each carry their own
   * hidden state, which this serves in the same single pass over the codes. */
  uint32_t flags;
  /* optional epilogue, per model (NULL: none): y = fp16(s_k * acc + bias[k][n]),
   * then y = fp16(y + resid[k][m * ldo_m + n * ldo_n]); resid may equal out */
  const void* bias[4];
  const void* resid[4];
  /* PP_QUAD_PER_MODEL_X, optional (NULL: none): the same four activation
   * rows interleaved, x_il[4 * k + q] = x[q][k] (FP16, 8-byte aligned).  The
   * fused plug correction then reads the four models' activations of a
   * plugged column with one load instead of four. */
  const void* x_il;
} pp_quad_linear_desc;

#define PP_QUAD_PER_MODEL_X 1u

PP_API int pp_quad_linear_group_workspace_bytes(int count, const pp_quad_linear_desc* descs, size_t* bytes);

/* 1 if the group runs as one launch on the current device, else 0. */
PP_API int pp_quad_linear_group_single_launch(int count, const pp_quad_linear_desc* descs);

PP_API int pp_quad_linear_group(int count, const pp_quad_linear_desc* descs, void* workspace,
                                size_t workspace_bytes, void* stream);

/* FP16 decode of a (R, C) code matrix into four (R, C) FP16 matrices,
 * bit-exact with the reference kernel's chain (quad_kernels.py:103-121).
 * scales == NULL keeps the normalised weights; otherwise each is multiplied
 * by scales[k] in FP32 and rounded to FP16 once.
 */
PP_API int pp_quad_decode(const uint32_t* codes, int64_t ldc_r, int64_t ldc_c, int64_t R, int64_t C,
                   const void* const luts[7], const float* scales,
                   void* const out[4], int64_t ldo_r, int64_t ldo_c, void* stream);

/* Restore n flat positions of a `.quadpack` stream on the GPU: FP16 decode
 * (as pp_quad_decode) with plug entries [p_lo, p_hi) of the file's plug
 * table substituted (positions relative to `base_lo32`, as above), then
 * optional per-model scale.  Counterpart of unpack_quad
 * (quaternion_packer.py:170-196) on the FP16 tables.
 */
PP_API int pp_quad_unpack(const uint32_t* codes, int64_t n, const uint32_t* plug_idx, const void* plug_vals,
                   int64_t p_lo, int64_t p_hi, uint32_t base_lo32,
                   const void* const luts[7], const float* scales,
                   void* const out[4], void* stream);

/* Plain FP16 Linear for the rows of a `.quadpack` Linear past the coded
 * range: the per-model FP16 tails, which the reference writes raw for every
 * model longer than n_min (quaternion_packer.py:118-126) and restores as is
 * (quaternion_packer.py:201-210).  For every model k with w[k] != NULL:
 *
 *   out_k[m][r] = fp16( sum_i x_k[m][i] * w_k[r][i] )   (FP32 accumulate)
 *
 * x_k = x + k * ldx_model (ldx_model = 0: all models read the same (M, K)
 * activations, row stride ldx_m, contiguous rows).  w[k]: R rows of K FP16
 * weights, row stride ldw >= K, any alignment (tail rows start wherever the
 * Linear crosses n_min).  out[k]: (M, R) FP16 with strides (ldo_m, ldo_n);
 * models with w[k] == NULL are not written.
 */
PP_API int pp_f16_linear(const void* x, int64_t ldx_m, int64_t ldx_model, int64_t M, int64_t K,
                         const void* const w[4], int64_t ldw, int64_t R, void* const out[4], int64_t ldo_m,
                         int64_t ldo_n, void* stream);

/* ------------------------------------------------------- decoder step --
 * The operations of a decoder step between the packed Linears, for the four
 * models of a `.quadpack` decoding one token each (row m of every buffer
 * belongs to model m).  No counterpart in the reference's code: its models
 * run these steps inside Hugging Face Qwen2 modules during generate
 * (polar_inference.py:224-229); the arithmetic follows those modules' FP16
 * steps (see decode_ops.cu).  Positions are read from device memory so that a
 * captured step can be replayed for every token.  A status word (device
 * int, may be NULL) receives 4 for a token id outside the vocabulary (its
 * row is zeroed) and 5 for a position outside the cache (nothing written).
 * RMSNorm, attention and SwiGLU can first wait for a gathered input buffer
 * (wait_flags != NULL: this rank's flag array of the buffer, wait_world
 * ranks, wait_epoch this rank's launches into it; the same bounded wait as
 * pp_gather_wait, run by every block before it reads), which saves the
 * separate pp_gather_wait launch after a gathered Linear.
 */
/* h[m][:] = tables[m][tokens[m]][:] (FP16 rows of H). */
PP_API int pp_embed_rows(const int* tokens, const void* const tables[4], int64_t vocab, int64_t H, void* h,
                         int64_t ldh, int* status, void* stream);

/* y[m] = fp16(w[m] * fp16(x[m] * rsqrt(mean(x[m]^2) + eps))), FP32 statistics.
 * y_il (optional, NULL: none; 8-byte aligned): the same values interleaved,
 * y_il[4 * i + m] = y[m][i], as pp_quad_linear_desc.x_il takes them. */
PP_API int pp_rmsnorm_rows(const void* x, int64_t ldx, const void* const w[4], int64_t H, float eps, void* y,
                           int64_t ldy, void* y_il, const uint32_t* wait_flags, int wait_world,
                           const uint32_t* wait_epoch, int* wait_status, void* stream);

/* Grouped-query decode attention of one token per model, with the token's
 * rotary embedding and KV-cache append fused in.  Row m of qkv holds the
 * token's nq query, nkv key and nkv value heads of hd = 128 FP16 values, not
 * rotated; cos_t / sin_t are FP16 [max_pos][hd] rotation tables (both
 * halves).  The token's key is rotated and stored with its value into
 * k_cache[m] / v_cache[m] ([max_pos][nkv][hd]) at *pos, then
 *   out[m][h] = softmax(rope(q[m][h]) k^T * scale) v   over positions 0..*pos
 * with kv head h / (nq / nkv), at most 16 query heads per kv head.  Scores
 * and the softmax run in FP32 on the tensor cores (all query heads of a kv
 * head share each 32-position tile of keys and values); the softmax weights
 * are rounded to FP16 for the value product.  Split over `splits` (1..4096)
 * position ranges of eight 32-position warp tiles each; the last arriving
 * block combines the partial results in order (deterministic).  Caches
 * 16-byte aligned (rows arrive by bulk copies); status must not be NULL
 * here (a tile copy that never lands sets it to 1).  out_il (optional,
 * 8-byte aligned): the output also interleaved, out_il[4 * i + m] = out[m][i].
 * Workspace: pp_decode_attention_workspace_bytes, zero-filled once. */
PP_API int pp_decode_attention_workspace_bytes(int64_t nq, int64_t nkv, int64_t splits, size_t* bytes);

PP_API int pp_decode_attention(void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t hd, const void* cos_t,
                               const void* sin_t, void* const k_cache[4], void* const v_cache[4], int64_t max_pos,
                               const int* pos, float scale, void* out, int64_t ldo, void* out_il, int64_t splits,
                               void* workspace, size_t workspace_bytes, int* status, const uint32_t* wait_flags,
                               int wait_world, const uint32_t* wait_epoch, int* wait_status, void* stream);

/* y[m][i] = fp16(fp16(silu(gate_up[m][i])) * gate_up[m][I + i]); y_il as for
 * pp_rmsnorm_rows. */
PP_API int pp_swiglu_rows(const void* gate_up, int64_t ldg, int64_t I, void* y, int64_t ldy, void* y_il,
                          const uint32_t* wait_flags, int wait_world, const uint32_t* wait_epoch, int* wait_status,
                          void* stream);

/* ------------------------------------------------------------------ dual --
 * Kernel-layout fused dequant GEMM, the drop-in for `polar_dual_bitpacked`
 * (reference polar_kernels.py:98-115, kernel 30-95):
 *   u = packed + 32768, amp = (u >> 10) & 63, ph = u & 1023
 *   A = fp32(amp_lut[amp]) * fp32(bmax[(k*N + n) / group_size])
 *   B1 = fp16(A * fp32(cos_lut[ph])), B2 = fp16(A * fp32(sin_lut[ph]))
 *   out_j[m][n] = fp16( sum_k a[m][k] * B_j[k][n] )                  (FP32 acc)
 * packed: (K, N) int16 with strides (ldp_k, ldp_n); the group index always
 * uses the logical row-major position k*N + n, as the reference does.
 */
PP_API int pp_dual_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t ldp_k, int64_t ldp_n,
                                 size_t* bytes);

PP_API int pp_dual_gemm(const void* a, int64_t lda_m, int64_t lda_k,
                 const int16_t* packed, int64_t ldp_k, int64_t ldp_n,
                 const void* bmax, int64_t group_size,
                 const void* amp_lut, const void* cos_lut, const void* sin_lut,
                 void* out1, void* out2, int64_t ldo_m, int64_t ldo_n,
                 int64_t M, int64_t N, int64_t K,
                 void* workspace, size_t workspace_bytes, void* stream);

/* `.dualpack` file streams (reference polar_bitpack.py:26-29, 79-91,
 * 160-172): 2-byte big-endian codes amp << phase_bits | phase per pair of
 * weights, FP16 group maxima (groups of group_size pairs restarting at every
 * chunk of chunk_size pairs), ascending uint32 plug positions with exact FP16
 * amplitudes.
 *
 * Restore of pairs [start, start + n), the counterpart of unpack_dual_models
 * (polar_bitpack.py:194-260), bit-exact: amp = float32(amp_norm[aq] * scale[g])
 * (or float32(plug value) at plugged positions), w1 = float32(amp * cos_t[ph]),
 * w2 = float32(amp * sin_t[ph]), all products in float64.  amp_norm / cos_t /
 * sin_t: the float64 tables of the restore ([2^amp_bits], [2^phase_bits]).
 * plug_idx / plug_vals: the plug entries of the range (positions relative to
 * base_lo32, the low 32 bits of `start`, modulo 2^32).  Outputs: float32 w1/w2
 * and/or their FP16 roundings h1/h2 (any may be NULL). */
PP_API int pp_dual_unpack(const uint8_t* codes, const void* scales, int64_t chunk_size, int64_t group_size,
                          int phase_bits, const double* amp_norm, const double* cos_t, const double* sin_t,
                          const uint32_t* plug_idx, const void* plug_vals, int64_t n_plugs, uint32_t base_lo32,
                          int64_t start, int64_t n, float* w1, float* w2, void* h1, void* h2, void* stream);

/* One nn.Linear (out N, in K) of the two models straight from the file layout:
 * pairs [offset + n K, offset + n K + K) are row n;
 *   y_j[m][n] = fp16( sum_k x[m][k] * fp16(w_j[n][k]) )   (FP32 accumulation)
 * with w_j decoded in FP32 from amp_norm (FP32 [2^amp_bits]) and cos_sin
 * (FP32 (cos, sin) pairs [2^phase_bits]).  Plugged pairs must have their
 * amplitude field cleared in `codes` (they decode to zero) and come as a
 * per-row list: entries [row_ptr[n], row_ptr[n + 1]) of plug_col (int) and
 * plug_w (FP16 (W1, W2) pairs).  codes 16-byte aligned and readable up to
 * the next 16-byte boundary; chunk and group sizes multiples of 8;
 * M <= 4; x (M, K) FP16 with row stride ldx; y1 / y2 (M, N) with row stride ldy. */
PP_API int pp_dual_file_linear(const uint8_t* codes, const void* scales, int64_t chunk_size, int64_t group_size,
                               int phase_bits, const float* amp_norm, const void* cos_sin, int64_t offset,
                               const int* row_ptr, const int* plug_col, const void* plug_w, const void* x,
                               int64_t ldx, int64_t M, int64_t N, int64_t K, void* y1, void* y2, int64_t ldy,
                               void* stream);

/* FP16 decode of a (K, N) int16 matrix into two FP16 matrices, bit-exact with
 * the reference kernel (polar_kernels.py:64-79). */
PP_API int pp_dual_decode(const int16_t* packed, int64_t ldp_k, int64_t ldp_n, int64_t K, int64_t N,
                   const void* bmax, int64_t group_size,
                   const void* amp_lut, const void* cos_lut, const void* sin_lut,
                   void* out1, void* out2, int64_t ldo_k, int64_t ldo_n, void* stream);

/* ------------------------------------------------------- peer gather --
 * Row-sharded Linears on the GPUs of one node without a separate
 * all-gather (no counterpart in the reference, which runs one model per
 * process on one GPU; replaces the NCCL all-gather of the outputs).  Each
 * rank's GEMV stores its output rows straight into every rank's gather
 * buffer over NVLink, then publishes a per-buffer epoch to every rank;
 * pp_gather_wait makes a stream wait until every rank has published.
 *
 * Buffers are ordinary device allocations shared between the processes with
 * CUDA IPC: pp_ipc_handle gives the 64-byte handle of the allocation that
 * holds `ptr` and ptr's offset in it; a peer maps it with pp_ipc_open (add
 * the offset) and unmaps with pp_ipc_close.
 */
#define PP_IPC_HANDLE_BYTES 64

PP_API int pp_ipc_handle(const void* ptr, void* handle, size_t* offset);
PP_API int pp_ipc_open(const void* handle, void** base);
PP_API int pp_ipc_close(void* base);

/* pp_quad_linear_fused at batch 1 (x is (1, K) with element stride ldx_k)
 * whose four outputs are gathered: for every rank q < world, model k's
 * output row n goes to element k * gather_ld + gather_row0 + n of
 * gather_out[q] (FP16; rank q's buffer as mapped in this process).  After
 * the launch's last store the kernel advances *gather_epoch (this rank's
 * count of launches into the buffer, device memory, initially 0) and writes
 * it to *gather_flag[q] (this rank's flag word in rank q's flag array) with
 * release semantics at system scope.  Readers call pp_gather_wait first.
 * The buffer must not be rewritten while a peer may still read it: with a
 * wait after every use, alternating two buffers suffices.
 */
PP_API int pp_quad_linear_gather(const void* x, int64_t ldx_k, const uint32_t* codes, int64_t ldw,
                                 const uint32_t* plug_idx, const void* plug_vals,
                                 const uint32_t* plug_window_base, uint32_t base_lo32,
                                 const void* unit_plugs, const uint32_t* unit_plug_off,
                                 const void* tables, const float scales[4], int world,
                                 void* const gather_out[], int64_t gather_ld, int64_t gather_row0,
                                 uint32_t* const gather_flag[], uint32_t* gather_epoch,
                                 int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* pp_quad_linear_group whose members' outputs are gathered as in
 * pp_quad_linear_gather: member j's model-k row n goes to element
 * k * gather_ld + gather_row0[j] + n of every rank's buffer, and the launch
 * publishes ONE epoch for the whole group (one pp_gather_wait per group
 * instead of one per Linear).  The members' out[] are not written.  Needs the
 * one-launch conditions of pp_quad_linear_group (PP_ERR_INVALID otherwise):
 * every rank must make the same number of launches into a buffer, so there
 * is no member-by-member fallback.
 */
PP_API int pp_quad_linear_group_gather(int count, const pp_quad_linear_desc* descs, int world,
                                       void* const gather_out[], int64_t gather_ld, const int64_t* gather_row0,
                                       uint32_t* const gather_flag[], uint32_t* gather_epoch, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* Makes `stream` wait until flags[q] (rank q's flag word in this rank's
 * flag array, q < world) has reached *epoch.  The wait is bounded (about a
 * second); a rank that never publishes sets *status to 3 (device int) and
 * the stream continues.  world <= 8.
 */
PP_API int pp_gather_wait(const uint32_t* flags, int world, const uint32_t* epoch, int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* POLAR_PACK_B200_H */
