/* C ABI of libcfk_b200.so: the B200 (sm_100a) kernels behind colabfold-kernels' Evoformer hot path.
 *
 * Conventions (modelled on the reference's own native FFI, src/colabfold_kernels/volta.py:100-461 and
 * contract.py:48-53): every pointer is DEVICE memory owned by the caller; entry points take their scratch
 * from the caller (a buffer sized by the matching *_workspace_bytes query, as the reference requests
 * scratch as an extra output, contract.py:16-17); work is enqueued on `stream` (a cudaStream_t) without host
 * synchronisation; absent optional tensors are NULL.  Every function returns CFK_OK or a negative status
 * and never throws or aborts.  dtype tags: CFK_F32, CFK_BF16, CFK_E4M3.
 *
 * One process may drive several devices: every entry works on the current device.  The one allocation the
 * library makes is a 16-byte status word (with a 4-byte pinned host mirror) per device, on the first call of
 * any tensor-core entry on that device: make that call before any stream capture is begun there.
 *
 * Timeouts: every device-side wait is bounded.  A kernel whose wait runs out records an id in the status
 * word and returns; from then on kernels of this library return at once WITHOUT writing their outputs, and
 * every entry point answers CFK_ERR_DEVICE_WAIT, until cfk_last_device_status(1) has read and cleared the
 * word.  The call during which the wait ran out may itself have returned CFK_OK (the work is asynchronous):
 * outputs produced since the last clean read of the status word are valid only if the next read is 0.
 *
 * Citations name the reference interface each entry replaces (paths inside mirditalab/colabfold-kernels).
 */
#ifndef CFK_B200_H_
#define CFK_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CFK_API __attribute__((visibility("default")))
#else
#define CFK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  CFK_OK = 0,
  CFK_ERR_SHAPE = -1,       /* a size is zero/negative or outside what the kernel takes */
  CFK_ERR_DTYPE = -2,       /* dtype tag not supported by this entry */
  CFK_ERR_ALIGN = -3,       /* a pointer or stride is not 16-byte aligned where TMA / vector loads need it */
  CFK_ERR_NULL = -4,        /* a required pointer is NULL */
  CFK_ERR_WORKSPACE = -5,   /* workspace too small */
  CFK_ERR_LAUNCH = -6,      /* the CUDA runtime refused the launch */
  CFK_ERR_TMA = -7,         /* tensor-map encoding failed */
  CFK_ERR_UNSUPPORTED = -8, /* valid request this build has no kernel for (caller runs its own path) */
  CFK_ERR_DEVICE_WAIT = -9  /* a bounded device-side wait ran out (cfk_last_device_status) */
};

enum { CFK_F32 = 0, CFK_BF16 = 1, CFK_E4M3 = 2 };

/* Library identification string. */
CFK_API const char* cfk_version(void);

/* Reads (and optionally clears) the per-device status word that kernels set when one of their bounded
 * waits ran out: 0 = clean.  Synchronises the device.  No reference counterpart (the reference's
 * handlers report through XLA's FFI error object). */
CFK_API int cfk_last_device_status(int reset);

/* Self-test of the bounded waits: one thread block waits `limit_clocks` (at most 2^24) GPU clocks on a
 * barrier that nothing arrives on, records `code` (> 0) in the status word and returns; nothing spins past
 * the limit and nothing traps.  cfk_last_device_status then reports `code`.  No reference counterpart. */
CFK_API int cfk_debug_wait_timeout(int64_t limit_clocks, int code, void* stream);

/* Number of kernels this library has launched in this process (optionally reset to zero): lets a caller
 * check that its work ran here and not in a fallback.  No reference counterpart. */
CFK_API long long cfk_launch_count(int reset);

/* ---- LayerNorm ------------------------------------------------------------------------------------
 * y = (x - mean) * rsqrt(var + eps) * scale + offset over the last axis, fp32 statistics.
 * x, y [m, c] in `dtype` (CFK_BF16 or CFK_F32); scale, offset [c] fp32.
 * Replaces pallas_layer_norm, tri_mul.py:492-512 (FFI shape: volta.py:223-229). */
CFK_API int cfk_layer_norm(const void* x, const float* scale, const float* offset, void* y, int64_t m, int c, int dtype,
                   float eps, void* stream);

/* LayerNorm backward, grads.py:25-39: dx [m,c] in `dtype`; dscale, doffset [c] fp32 (overwritten).
 * workspace: cfk_layer_norm_bwd_workspace_bytes(m, c) bytes. */
CFK_API size_t cfk_layer_norm_bwd_workspace_bytes(int64_t m, int c);
CFK_API int cfk_layer_norm_bwd(const void* x, const float* scale, const void* dy, void* dx, float* dscale, float* doffset,
                       int64_t m, int c, int dtype, float eps, void* workspace, size_t workspace_bytes, void* stream);

/* cfk_layer_norm_bwd without a workspace argument and without any allocation: the per-block partial sums
 * live in a fixed 1 MiB array inside the library's device image.  It has no counterpart in the reference
 * (whose handlers get all scratch from XLA).  For callers that hold no allocator at the call site and may
 * not call one: a handler running inside a pre-planned buffer assignment, or a replay-only serving loop
 * whose memory pool is frozen after start-up.
 *   - Limits: c <= 256 and at most 512 launch blocks (two per SM); beyond either the call does nothing
 *     and returns CFK_ERR_WORKSPACE.
 *   - The first call on each device performs set-up (it asks the runtime for the array's device address,
 *     which also loads the module there): make it once, with that device current, before any stream
 *     capture is begun.  Later calls only launch.
 *   - Nothing needs clearing between calls: the kernels overwrite every partial sum they later read.
 *   - The array is shared by all callers of this entry on a device: two calls that overlap in time
 *     (different streams or threads) race on it.  Issue them on one stream, or order them.
 * Results are bit-identical to cfk_layer_norm_bwd. */
CFK_API int cfk_layer_norm_bwd_static(const void* x, const float* scale, const void* dy, void* dx, float* dscale,
                              float* doffset, int64_t m, int c, int dtype, float eps, void* stream);

/* ---- Bias-fused attention ---------------------------------------------------------------------------
 * out = softmax_k(scale * q.k + bias[h,q,k], masked keys -> finite floor) . v, per (batch n, head h).
 * q [n,h,sq,d] ('heads') or [n,sq,h,d] (seq_major); k, v likewise with sk; bias [h,sq,sk] in `dtype` or NULL;
 * kmask [n,sk] uint8 (0 = masked); out in q's layout and dtype; lse [n,h,sq] fp32 (log2 domain) or NULL.
 * dtype CFK_BF16 (tcgen05 path when d == 32 and sk % 8 == 0, else the fp32-math path) or CFK_F32.
 * Replaces tri_flash / pallas_attention's kernel call, tri_flash.py:242-290,452-478 (FFI: volta.py:100-115). */
CFK_API int cfk_attention_fwd(const void* q, const void* k, const void* v, const void* bias, const uint8_t* kmask, void* out,
                      float* lse, int n, int h, int sq, int sk, int d, int dtype, int seq_major, float scale,
                      void* stream);

/* Backward of the above: tri_flash_bwd, tri_flash.py:365-413,434-446 (FFI: volta.py:118-130).
 * dq, dk, dv in `dtype` and q/k/v's layout; dbias [h,sq,sk] fp32 or NULL (not wanted).
 * workspace: cfk_attention_bwd_workspace_bytes(...) bytes, contents undefined on return. */
CFK_API size_t cfk_attention_bwd_workspace_bytes(int n, int h, int sq, int sk, int d, int dtype);
CFK_API int cfk_attention_bwd(const void* q, const void* k, const void* v, const void* bias, const uint8_t* kmask,
                      const void* out, const void* dout, const float* lse, void* dq, void* dk, void* dv, float* dbias,
                      int n, int h, int sq, int sk, int d, int dtype, int seq_major, float scale, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Attention reading q/k/v/gate in place from the packed projection p [X,Y,G,H,D] (slots q,k,v[,gate]):
 * rows attend along Y (batch X), columns along X (batch Y); out [X,Y,H,D] = o * sigmoid(gate + gate_bias[h,:])
 * when G == 4.  bias [H,S,S] or NULL; kmask [batch,S] uint8; gate_bias [H,D] in `dtype` (G == 4) or NULL.
 * trim_limits (NULL = off): int32 [batch + 1] from cfk_trim_limits; rows with no live key and queries past
 * the last live key of any row then give zeros (packed_attn.py:123-137).  lse [batch,H,S] fp32 or NULL.
 * Replaces packed_attention, packed_attn.py:26-120 (FFI: volta.py:200-220, where the limits are likewise
 * one extra int32 input). */
CFK_API int cfk_packed_attention_fwd(const void* p, const void* bias, const uint8_t* kmask, const void* gate_bias, void* out,
                             float* lse, const int32_t* trim_limits, int x, int y, int g, int h, int d, int dtype,
                             int column, float scale, void* stream);

/* The opt-in FP8 form of the packed attention: q and k come in e4m3 from qk8 [X,Y,2,H,D] (q already multiplied by its
 * static scale before rounding, as ln_projection's f8_slots / f8_scales write it, packed_attn.py:214-216), and the
 * scores run on the 8-bit tensor-core path; p [X,Y,G,H,D] in bf16 keeps the other slots: v (G == 1) or v, gate
 * (G == 2).  `scale` multiplies the raw q8.k8 products (sm_scale divided by q's static scale: ln 2 for the
 * sm_scale * log2(e) the reference uses).  P.V, the softmax and the output stay as in cfk_packed_attention_fwd.
 * Head dim 32 only; CFK_ERR_UNSUPPORTED otherwise (the selector then returns no FP8 slots).
 * Replaces the e4m3 q.k form of packed_attention (fused_ops.py:83-97,122-136; Mosaic kernel mgpu_attn.py:57). */
CFK_API int cfk_packed_attention_fwd_qk8(const void* p, const void* qk8, const void* bias, const uint8_t* kmask,
                                         const void* gate_bias, void* out, float* lse, const int32_t* trim_limits,
                                         int x, int y, int g, int h, int d, int column, float scale, void* stream);

/* limits[b] = 1 + index of the last live key of batch row b (0 when none), limits[batch] = their maximum:
 * trim_limits(kmask, 1) of packed_attn.py:123-129, concatenated as volta.py:212-213 passes them. */
CFK_API int cfk_trim_limits(const uint8_t* kmask, int32_t* limits, int batch, int s, void* stream);

/* ---- Triangle-multiplication contraction ---------------------------------------------------------------
 * out[c,i,j] = alpha * sum_k a[c,i,k] * b[c,j,k]; a [C,I,K], b [C,J,K] in `dtype` (CFK_BF16, or CFK_E4M3 with
 * alpha = scale_a * scale_b, 1.0 for the reference's unscaled saturating cast); out [C,I,J] bf16; fp32
 * accumulation.  K * itemsize must be a multiple of 16 and J of 8 (the reference's own rule, contract.py:43-45).
 * Replaces CckFp8Contract (contract.py:48-53; no workspace output is needed here) and the XLA batched GEMM the
 * bf16 path is left to (tri_mul.py:6-7). */
CFK_API int cfk_contract(const void* a, const void* b, void* out, int c, int i, int j, int k, int dtype, float alpha,
                         void* stream);

/* The same contraction with b given as [parts, C, J/parts, K]: what an all-gather over `parts` ranks of per-rank
 * [C, J/parts, K] right operands leaves in memory, read in place (no re-layout copy).  J/parts must be a multiple
 * of 128.  The reference runs on one device and has no counterpart; this serves the row-sharded block. */
CFK_API int cfk_contract_gathered(const void* a, const void* b, void* out, int c, int i, int j, int k, int dtype,
                                  float alpha, int parts, void* stream);

/* The same contraction between two all-to-alls over the channel axis (the row-sharded block's triangle
 * multiplication: each rank contracts C = channels / parts whole channels instead of gathering the right operand).
 * split_k == 0: a is [parts, C, I/parts, K] and b [parts, C, J/parts, K], what the all-to-all leaves when every rank
 * sent its rows of all channels; split_k != 0: a is [parts, C, I, K/parts] and b [parts, C, J, K/parts], every rank
 * having sent its slice of the contracted axis (incoming edges).  The product is stored as [parts, C, I/parts, J]:
 * the send buffer of the all-to-all back to row shards, no re-layout copy on either side.  I/parts and J/parts
 * (split_k == 0) must be multiples of 128, K/parts (split_k != 0) a multiple of 64 (bf16) or 128 (e4m3) elements.
 * No reference counterpart (the reference runs on one device). */
CFK_API int cfk_contract_exchanged(const void* a, const void* b, void* out, int c, int i, int j, int k, int dtype,
                                   float alpha, int parts, int split_k, void* stream);

/* cfk_contract_exchanged with the all-to-all of the product back to row shards done by its stores: out_ptrs is a HOST
 * array of `parts` device pointers, entry q = rank q's receive buffer [parts, c, i / parts, j] bf16 (this rank's own for
 * q == rank, NVLink peer mappings otherwise); rows [q i/parts, (q+1) i/parts) of this rank's product land at index
 * `rank` of buffer q (TMA stores, no multicast).  parts <= 8.  The caller orders the exchange as for
 * cfk_ln_gated_dual_proj_peer: a barrier across the ranks after this call and before any rank reads its buffer. */
CFK_API int cfk_contract_exchanged_peer(const void* a, const void* b, void* const* out_ptrs, int rank, int c, int i, int j,
                                        int k, int dtype, float alpha, int parts, int split_k, void* stream);

/* All-to-all over NVLink peer memory for the row-sharded block (one process per GPU): part p of `send` is written into
 * rank p's receive buffer by plain 16-byte stores of a kernel of this library (no TMA, no multicast), followed by a flag
 * barrier after which every rank's receive buffer holds all parts.  A part is `rows` runs of run_bytes: run i of part p
 * is read at src_part_bytes * p + src_row_bytes * i and written at dst_part_bytes * rank + dst_row_bytes * i of rank p's
 * buffer, so a switch between row and column sharding needs no packing or re-layout copy (rows = 1 is the plain
 * [parts][chunk] exchange); all byte counts multiples of 16.  recv_ptrs: device array of `parts` pointers, entry p =
 * rank p's receive buffer; flag_ptrs: device array of `parts` pointers, entry p = rank p's array of `parts` int32 flags
 * (zero-initialised); counter: two int32 on this device (zero-initialised): the barrier number, so that a replayed CUDA
 * graph keeps counting, and the count of finished blocks (the last block of the copy kernel runs the barrier).  Buffers and flags are symmetric memory the caller set up (peer access enabled).  The
 * wait for the peers is bounded (about a second): a missing peer leaves code 1901 in the device status word instead of
 * a hang.  The reference has no multi-GPU code; this replaces an NCCL all-to-all between kernels. */
CFK_API int cfk_peer_alltoall(const void* send, const void* recv_ptrs, const void* flag_ptrs, void* counter, int rank,
                              int parts, int64_t rows, int64_t run_bytes, int64_t src_part_bytes, int64_t src_row_bytes,
                              int64_t dst_part_bytes, int64_t dst_row_bytes, void* stream);

/* The outer product of the outer-product-mean over the MSA depth, for 32-channel projections:
 * out[i, j, c, e] = sum_s a[i*32 + c, s] * b[j*32 + e, s]; a [ri*32, s], b [rj*32, s] in `dtype` (CFK_BF16 or CFK_E4M3),
 * out [ri, rj, 32, 32] bf16 - the layout the output linear of the module contracts over (c, e) without a transposed
 * copy.  s * itemsize must be a multiple of 16.  The reference has the shallow forms only (opm_outer, opm.py:122-168:
 * the same sum for 16 MSA rows); the deep form is left to XLA inside ColabFold. */
CFK_API int cfk_opm_outer_product(const void* a, const void* b, void* out, int ri, int rj, int s, int dtype, void* stream);

/* ---- Projection family (bf16; K, the contracted width, must be 64, 128 or 256; unsupported widths return
 * CFK_ERR_UNSUPPORTED and the caller runs its own path, as the reference's selectors return None) -----------
 *
 * Gated dual projection: y = mask[m] * (x wp + bp) * act(x wg + bg); x [m,k]; wp, wg [k,p]; bp, bg [p]; mask [m];
 * activation 0 = sigmoid, 1 = swish.  split = 0: out0 [m,p].  split = 1: out0, out1 = columns [0,p/2), [p/2,p) as
 * two arrays, each [m,p/2] or, with channel_major, [p/2,m].
 * Replaces gated_dual_proj, tri_mul.py:163-219 (FFI: volta.py:244-250). */
CFK_API int cfk_gated_dual_proj(const void* x, const void* wp, const void* bp, const void* wg, const void* bg,
                                const void* mask, void* out0, void* out1, int64_t m, int k, int p, int split,
                                int channel_major, int activation, void* stream);

/* LayerNorm fused in front of the split channel-major gated dual projection.  b == 0: x [a,k], mask [a] ->
 * left, right [p/2, a'].  b > 0: the pair x [a,b,k], mask [a,b] -> [p/2, a, b'] or, with transpose (the pair read
 * transposed, for incoming edges), [p/2, b, a'].  The primed axis is zero-padded to a multiple of `pad`;
 * negative mask values count as zero; fp8 stores saturating e4m3 of value * fp8_scale (a per-tensor scale chosen by
 * the caller, > 0; 1.0 is the reference's unscaled cast, tri_mul.py:228; the contraction undoes two scaled operands
 * with alpha = 1 / (scale_left * scale_right) on cfk_contract).  ln_scale, ln_offset fp32 [k].
 * The mask also filters 128-row tiles: a tile whose mask is all zero gets zeros without its rows being read, a tile
 * whose mask is below zero everywhere is not written (transition.py:29-38).
 * Replaces ln_gated_dual_proj, tri_mul.py:222-283 (FFI: volta.py:328-334). */
CFK_API int cfk_ln_gated_dual_proj(const void* x, const float* ln_scale, const float* ln_offset, const void* wp,
                                   const void* bp, const void* wg, const void* bg, const void* mask, void* left,
                                   void* right, int64_t a, int64_t b, int k, int p, int transpose, int pad, int fp8,
                                   float fp8_scale, float eps, void* stream);

/* The same projection (bf16, k = 128, p = 256, pair x [a,b,k]) with the all-to-all over channels of the row-sharded
 * triangle multiplication done by its stores: left_ptrs / right_ptrs are HOST arrays of `parts` device pointers,
 * entry q = rank q's receive buffer [parts, 128 / parts, outer, inner'] (this rank's own buffer for q == rank, NVLink
 * peer mappings otherwise); channel part q of this rank's result lands at index `rank` of buffer q (TMA stores, no
 * multicast).  parts divides 16, parts <= 8.  The caller orders the exchange: a barrier across the ranks
 * (cfk_peer_alltoall with rows == 0) after this call and before any rank reads its buffer, and one between the last
 * read of a buffer and the next call that writes it.  parts == 1 is cfk_ln_gated_dual_proj with left_ptrs[0],
 * right_ptrs[0].  CFK_ERR_UNSUPPORTED for other shapes.
 * Replaces ln_gated_dual_proj, tri_mul.py:222-283, followed by the exchange the reference (one device) does not need. */
CFK_API int cfk_ln_gated_dual_proj_peer(const void* x, const float* ln_scale, const float* ln_offset, const void* wp,
                                        const void* bp, const void* wg, const void* bg, const void* mask,
                                        void* const* left_ptrs, void* const* right_ptrs, int rank, int parts, int64_t a,
                                        int64_t b, int k, int p, int transpose, int pad, float eps, void* stream);

/* Triangle-multiplication output: out = (LN(x_cm^T) wo + bo) * sigmoid(g wg + bg) (+ residual | + act).
 * x_cm [c,m] channel-major product (x_cm_dtype CFK_BF16 or CFK_F32); act [m,ca] is the gate input: already normed
 * when in_scale == NULL, else the raw module input normed here with in_scale/in_offset; add_input adds act itself
 * (needs ca == o; out may alias act).  residual [m,o] bf16 or NULL.  c is 64 or 128.
 * keep [m] (keep_dtype CFK_BF16 or CFK_F32) or NULL marks the rows that matter (transition.py:29-38): a 128-row tile
 * whose largest keep is > 0 is computed in full, one of zeros (padding) gets zeros - or the residual / act rows where
 * those are added - without the work, one below zero everywhere is not written.  The same holds for every entry
 * below that takes `keep`.
 * Replaces trimul_epilogue / trimul_epilogue_ln, tri_mul.py:371-438 (FFI: volta.py:345-352). */
CFK_API int cfk_trimul_epilogue(const void* x_cm, int x_cm_dtype, const void* act, const float* in_scale,
                                const float* in_offset, const float* ln_scale, const float* ln_offset, const void* wo,
                                const void* bo, const void* wg, const void* bg, const void* residual, const void* keep,
                                int keep_dtype, void* out, int64_t m, int c, int ca, int o, float eps, int add_input,
                                void* stream);

/* LayerNorm then the packed attention projection: p[m, g*n + j] = (LN(x) w[g])[m,j]; x [m,a]; w [g,a,n]; no biases.
 * f8 != 0 writes saturating e4m3 of (value * f8_scale) instead of bf16.
 * Replaces ln_projection's slot outputs, packed_attn.py:234-305 (FFI: volta.py:368-383). */
CFK_API int cfk_ln_projection(const void* x, const float* ln_scale, const float* ln_offset, const void* w,
                              const void* keep, int keep_dtype, void* p_out, int64_t m, int a, int g, int n, int f8,
                              float f8_scale, float eps, void* stream);

/* The per-head bias of the same op, channel-major: bias_out[h, m] = (LN(x) wb)[m, h]; wb [a, h_padded] with
 * h_padded a multiple of 8 (columns past h are ignored).  packed_attn.py:225-229. */
CFK_API int cfk_ln_head_bias(const void* x, const float* ln_scale, const float* ln_offset, const void* wb,
                             const void* keep, int keep_dtype, void* bias_out, int64_t m, int a, int h, int h_padded,
                             float eps, void* stream);

/* out = o w + b (+ residual); o [m,k]; w [k,c]; b [c]; residual, out [m,c] (out may alias residual).
 * Replaces output_projection, packed_attn.py:352-384 (FFI: volta.py:400-408). */
CFK_API int cfk_output_projection(const void* o, const void* w, const void* b, const void* residual, const void* keep,
                                  int keep_dtype, void* out, int64_t m, int k, int c, void* stream);

/* First half of the LN-MLP transition: h[m, hdim] = relu(LN(x) w1 + b1) in bf16; x [m,c], w1 [c,hdim], b1 [hdim];
 * c in {64,128,256}, hdim a multiple of 64.  keep [m] or NULL: a 128-row block it marks nowhere is written as zeros
 * (its h contributes nothing to the second GEMM; the caller restores x + b2 there as transition.py:88-92 asks).
 * Together with a GEMM h w2 + b2 (+ x) it replaces fused_transition, transition.py:100-138 (FFI: volta.py:418-428);
 * the hidden activation makes one round trip through HBM where the reference keeps it on chip. */
CFK_API int cfk_transition_hidden(const void* x, const float* ln_scale, const float* ln_offset, const void* w1,
                                  const void* b1, const void* keep, int keep_dtype, void* h_out, int64_t m, int c,
                                  int hdim, float eps, void* stream);

/* The whole LN-MLP transition in one kernel: out = relu(LN(x) w1 + b1) w2 + b2 (+ x); x, out [m,c] bf16 (out may
 * alias x: a 128-row block is read only by the CTA that writes it), w1 [c,hdim], b1 [hdim], w2 [hdim,c], b2 [c] bf16;
 * c in {128, 256}, hdim a multiple of 64.  keep [m] (CFK_F32 or CFK_BF16) or NULL: a 128-row block whose keep is
 * nowhere positive is not computed - its rows come out as x (zeros without add_input), and a block whose keep is
 * negative throughout is left unwritten (transition.py:29-38).  Both GEMMs run on the tensor cores and the hidden
 * activation never leaves the chip, as in the reference's kernel.  Replaces fused_transition, transition.py:100-138
 * (FFI: volta.py:418-428). */
CFK_API int cfk_transition(const void* x, const float* ln_scale, const float* ln_offset, const void* w1, const void* b1,
                           const void* w2, const void* b2, const void* keep, int keep_dtype, void* out, int64_t m, int c,
                           int hdim, float eps, int add_input, void* stream);

/* left, right = mask[m] * (LN(x) lw + lb), mask[m] * (LN(x) rw + rb); x [m,c]; lw, rw [c,k]; k <= 128.
 * Replaces opm_projection, opm.py:36-59. */
CFK_API int cfk_opm_projection(const void* x, const float* ln_scale, const float* ln_offset, const void* lw,
                               const void* lb, const void* rw, const void* rb, const void* mask, void* left,
                               void* right, int64_t m, int c, int k, float eps, void* stream);

/* The same two projections written channel-major with the MSA depth contiguous: x [s,r,c], mask [s,r] ->
 * left, right [k, r, pitch] (pitch >= s, a multiple of 8; columns s..pitch-1 are zeros); k <= 32.  This is the operand
 * layout of cfk_opm_fused.  The reference's opm_projection (opm.py:36-59) writes [s,r,k]; the layout is internal to
 * the deep outer product mean. */
CFK_API int cfk_opm_projection_cm(const void* x, const float* ln_scale, const float* ln_offset, const void* lw,
                                  const void* lb, const void* rw, const void* rb, const void* mask, void* left,
                                  void* right, int64_t s, int64_t r, int c, int k, int64_t pitch, float eps,
                                  void* stream);

/* norm[i,j] = sum_s mask_left[s,i] * mask_right[s,j] in fp32: the overlap count the outer product mean divides by
 * (ColabFold computes it with an XLA einsum; no kernel of the reference).  Masks [depth, ri], [depth, rj] in
 * mask_dtype (CFK_BF16 or CFK_F32). */
CFK_API int cfk_opm_norm(const void* mask_left, const void* mask_right, int mask_dtype, float* norm, int depth, int ri,
                         int rj, void* stream);

/* Deep outer product mean in one kernel:
 * out[i,j,:] = ((sum_s left[:,i,s] (x) right[:,j,s]) rounded to bf16 . w + bias) / (eps + norm[i,j]) (+ residual[i,j,:]).
 * left_cm [c, ri, pitch], right_cm [c, rj, pitch] bf16 (cfk_opm_projection_cm), w [c*c, f] bf16 with row index
 * a*c + b, bias [f] bf16, norm [ri,rj] fp32, residual (or NULL) and out [ri,rj,f] bf16 (out may alias residual).
 * c == 32 and f == 128, else CFK_ERR_UNSUPPORTED (the caller composes cfk_opm_outer_product, cfk_contract and
 * cfk_opm_finish).  The outer product never reaches memory, as in the reference's opm_outer (opm.py:122-162: per left
 * channel the product is rounded to the input type, then multiplied by its rows of w), here at any MSA depth. */
CFK_API int cfk_opm_fused(const void* left_cm, const void* right_cm, const void* w, const void* bias, const float* norm,
                          const void* residual, void* out, int ri, int rj, int depth, int64_t pitch, int c, int f,
                          float eps, void* stream);

/* Outer-product-mean tail: out[m,f] = (x[m,f] + bias[f]) / (eps + norm[m]) + residual[m,f] (residual may be NULL,
 * out may alias it); x, bias, residual, out bf16, norm fp32.  The pair update of opm_update, opm.py:69-88,116-119,
 * applied after the two GEMMs of the deep-MSA outer product (cfk_contract). */
CFK_API int cfk_opm_finish(const void* x, const void* bias, const float* norm, const void* residual, void* out,
                           int64_t m, int f, float eps, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CFK_B200_H_ */
