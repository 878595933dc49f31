/*
 * b200q -- C ABI of the B200 (sm_100a) quantised dequant-GEMM library.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t passed
 * as void*, launches asynchronously on that stream, never allocates or frees
 * device memory, never synchronises, and returns B200Q_OK (0) or a negative
 * status.  b200q_last_error() gives the message of the last failure on the
 * calling host thread.  Scratch memory ("workspace") is always caller-owned:
 * query its size, allocate it once, zero it once; the kernels leave it in the
 * zeroed state again when they finish (a split-K counter that the last CTA of
 * each output strip resets).  One workspace must not be used by two launches
 * that can overlap on the GPU.
 *
 * Matrix layouts are the reference's (lilian-muyaoli/kernelbench-harbor),
 * row-major and contiguous:
 *   x        [M, K]      activations, fp16 or bf16 (dtype argument)
 *   qweight  [K, N/8]    int32, 8 unsigned 4-bit codes per word packed along N:
 *                        nibble i (bits 4i..4i+3) of word [k, j] is column 8j+i
 *   scales   [K/group, N] activation dtype
 *   zeros    [K/group, N] activation dtype, integer-valued
 *   y        [M, N]      activation dtype
 *   w[k, n] = (nibble(k, n) - zeros[k/group, n]) * scales[k/group, n]
 */
#ifndef B200Q_H_
#define B200Q_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200Q_OK 0
#define B200Q_ERR_SHAPE (-1)       /* a size is out of the supported range        */
#define B200Q_ERR_ALIGN (-2)       /* pointer or row pitch violates TMA alignment */
#define B200Q_ERR_UNSUPPORTED (-3) /* dtype / group / mode not implemented        */
#define B200Q_ERR_CUDA (-4)        /* a CUDA runtime call or launch failed        */
#define B200Q_ERR_WORKSPACE (-5)   /* workspace missing or too small              */
#define B200Q_ERR_DEVICE (-6)      /* a kernel reported a device-side error       */

#define B200Q_DTYPE_FP16 0
#define B200Q_DTYPE_BF16 1

/* Library version, (major << 16) | minor. */
int b200q_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* b200q_last_error(void);

/* Reads and clears the device status word at the start of a workspace: waits
 * for `stream`, returns 0 when no kernel reported an error, otherwise the
 * or-ed device error bits (1 = a bounded wait timed out). Returns a negative
 * status if the copy itself fails.  After a device error the workspace may
 * hold a kernel's unfinished split-K counters: zero the whole workspace again
 * before reusing it. */
int b200q_workspace_status(void* workspace, void* stream);

/* Weight prefetch across kernel boundaries (off by default; process-wide).
 * When on, the small-M W4A16 kernel (M <= 16, single GPU) is launched with
 * programmatic dependent launch: it starts while the previous kernel in the
 * stream is still running and streams its first qweight / scales / zeros
 * tiles before waiting for that kernel to finish; x is read and y written
 * only after the wait.  The caller promises that the kernel launched just
 * before each such call on the same stream does not write that call's
 * qweight, scales or zeros (true whenever weights are loaded once and reused,
 * as in inference).  Returns the previous setting.  No counterpart in the
 * reference, whose operator is a single stand-alone call. */
int b200q_set_weight_prefetch(int enable);

/* Bytes of zero-initialised workspace b200q_w4a16_gemm needs for this shape on
 * `device` (the split-K decomposition depends on the SM count). */
size_t b200q_w4a16_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t group, int device);

/* y = x . dequant(qweight, scales, zeros).
 * Replaces the reference operator Model.forward(x, qweight, scales, zeros) of
 * QUANT_REF (generate_tasks.py:54-61) and its Triton oracle ModelNew.forward
 * (common/oracles/quant_w4a16_pa.py:69-98), with y in x's dtype.
 * Requirements: M >= 0; N % 32 == 0; K % group == 0; group in {32, 64, 128,
 * 256}; 16-byte aligned pointers.  M == 0 is a no-op. */
int b200q_w4a16_gemm(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                     void* y, int64_t M, int64_t N, int64_t K, int64_t group, int dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of zero-initialised workspace b200q_w8a8_gemm needs for this shape. */
size_t b200q_w8a8_workspace_bytes(int64_t M, int64_t N, int64_t K, int device);

/* y[M, N] = fp16((x_int8 . w_int8) * x_scale[m] * w_scale[n]), int32 accumulation.
 * Replaces W8A8_REF.forward(x_int8, w_int8, x_scale, w_scale)
 * (generate_tasks.py:204-206): x_int8 [M, K] int8, w_int8 [K, N] int8 (N
 * contiguous), x_scale [M] fp16 (the reference's [M, 1]), w_scale [N] fp16
 * (its [1, N]), y [M, N] fp16.  Requirements: K % 16 == 0, N % 32 == 0,
 * 16-byte aligned pointers.  The product is exact (int32); the reference's
 * fp32 matmul rounds it. */
int b200q_w8a8_gemm(const void* x_int8, const void* w_int8, const void* x_scale, const void* w_scale, void* y,
                    int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* Top-2 routing of a mixture of experts (MOE_REF / FUSED_QMOE_REF routing,
 * generate_tasks.py:171-173, 368-371): softmax of the fp32-upcast logits
 * [T, E], the two largest (equal logits: lower expert index first), gates =
 * renormalised pair in the logits' dtype.  Also builds the permutation: per
 * expert e the routed tokens in ascending order in slots [offsets[e],
 * offsets[e+1]) (slot_token [2T]), and each token's two slots (token_slot
 * [T, 2]).  topi [T, 2] int32, gates [T, 2], offsets [E + 1].  2 <= E <= 256. */
int b200q_moe_route(const void* logits, int64_t T, int64_t E, int dtype, int32_t* topi, void* gates,
                    int32_t* offsets, int32_t* slot_token, int32_t* token_slot, void* stream);

/* xg[s, :] = x[slot_token[s], :] for s < nslots (rows of D fp16/bf16, D % 8 == 0). */
int b200q_moe_gather(const void* x, const int32_t* slot_token, int64_t nslots, int64_t D, void* xg, void* stream);

/* h = (silu(gate.float()) * up.float()).to(dtype), elementwise over n values
 * (the SiLU.mul of FUSED_SILU_REF, generate_tasks.py:336-337). */
int b200q_silu_mul(const void* gate, const void* up, void* h, int64_t n, int dtype, void* stream);

/* y[t] = ye[token_slot[t,0]] * gates[t,0] + ye[token_slot[t,1]] * gates[t,1],
 * products and sum rounded to dtype as the reference's (sel * topv).sum(1)
 * (generate_tasks.py:377-378).  ye [2T, D], y [T, D], D % 8 == 0, 16-byte
 * aligned ye and y. */
int b200q_moe_combine(const void* ye, const int32_t* token_slot, const void* gates, void* y, int64_t T, int64_t D,
                      int dtype, void* stream);

/* Expert-parallel exchange helpers for a rank of P holding E/P experts, with C
 * row slots per (source, destination) rank pair (the benchmark's
 * expert-parallel MoE; the reference MoE is single-GPU, generate_tasks.py:
 * 368-378, so these have no counterpart there).  Rows are fp16/bf16 with
 * D % 8 == 0; exchanged rows carry D + 8 values, value D being the local
 * expert index of the row as a small integer (-1: empty slot).
 * ep_pack: from b200q_moe_route's offsets / slot_token / token_slot over this
 * rank's T tokens, send [P * C, D + 8] gets in slot d * C + j the j-th row
 * routed to rank d, and pair_slot [T, 2] each token's two slots (to pass as
 * b200q_moe_combine's token_slot on the returned rows).  C >= 2 T. */
int b200q_ep_pack(const void* x, int64_t T, int64_t D, int dtype, const int32_t* offsets, const int32_t* slot_token,
                  const int32_t* token_slot, int64_t E, int64_t P, int64_t C, void* send, int32_t* pair_slot,
                  void* stream);

/* ep_regroup: the R received rows [R, D + 8] ordered stably by local expert:
 * loc_offsets [n_local + 1], src [R] (received row at grouped position j, -1
 * past the last), row_pos [R] (grouped position of received row r, -1 for an
 * empty slot).  One CTA; no host synchronisation. */
int b200q_ep_regroup(const void* recv, int64_t R, int64_t D, int dtype, int64_t n_local, int32_t* loc_offsets,
                     int32_t* src, int32_t* row_pos, void* stream);

/* ep_gather: dst[j, :D] = src[idx[j], :D] for j < n with idx[j] >= 0 (other
 * rows untouched); row pitches in elements, multiples of 8. */
int b200q_ep_gather(const void* src, int64_t src_pitch, const int32_t* idx, int64_t n, int64_t D, void* dst,
                    int64_t dst_pitch, void* stream);

/* Bytes of zero-initialised workspace b200q_mxfp8_gemm needs (the status
 * word: split-K is reduced over DSMEM inside a thread-block cluster). */
size_t b200q_mxfp8_workspace_bytes(int64_t M, int64_t N, int64_t K, int device);

/* MXFP8 block-scaled GEMM: y[M, N] = fp16(A_deq . B_deq^T), A [M, K] and B
 * [N, K] e4m3 codes (K-major), scales_a [M, K/32] and scales_b [N, K/32] E8M0
 * (OCP MX v1.0, bias 127), fp32 accumulation.  The reference has no MX module;
 * its nearest operator is FP8_REF.forward (generate_tasks.py:226-229, a
 * weight-only fp8 GEMM with fp16 block scales).  Requirements: K % 128 == 0,
 * N % 32 == 0, 16-byte aligned A/B/y, 4-byte aligned scales. */
int b200q_mxfp8_gemm(const void* a, const void* scales_a, const void* b, const void* scales_b, void* y, int64_t M,
                     int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* y = x . dequant(qweight, scales, zeros) for 1 <= M <= 32, with no workspace
 * argument and no allocation: for callers that cannot call cudaMalloc (a
 * plugin inside a host program that owns all device memory, a fixed memory
 * budget).  No counterpart in the reference; it is an addition of this
 * library.  Its split-K scratch is a fixed 8 MiB device array inside the
 * library, held on every GPU that loads it until exit; shapes needing more are
 * rejected with B200Q_ERR_SHAPE.  The first call on a device looks up that
 * array's address and should come before any stream capture.  All calls share
 * the array, so calls that can overlap on the GPU race: serialise them.  Same
 * layouts, requirements and results as b200q_w4a16_gemm. */
int b200q_w4a16_gemm_noalloc(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                             void* y, int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* stream);

/* Device status of the last b200q_w4a16_gemm_noalloc call on the current
 * device, read from the fixed array's header and cleared, like
 * b200q_workspace_status (waits for `stream`; 0 = no error, else the device
 * error bits).  Each noalloc call clears the header first, so read it before
 * the next call.  No counterpart in the reference. */
int b200q_w4a16_noalloc_status(void* stream);

/* GPU weight packer: 4-bit codes [K, N] (int8, one code per byte, row-major)
 * -> qweight [K, N/8] int32 packed along N, nibble i of word j = column 8j+i:
 * the packing loop of QUANT_REF.get_inputs (generate_tasks.py:65-69).
 * offset 0: codes are unsigned nibbles in [0, 15] (the reference format);
 * offset 8: codes are signed symmetric int4 in [-8, 7] (FUSED_QMOE_REF and
 * LORA_REF weights, generate_tasks.py:385, 414), stored as q + 8 so that the
 * W4A16 kernels with zero point 8 reproduce q * s exactly.  N % 8 == 0,
 * codes 8-byte aligned.  A code out of range sets B200Q_DEV_ERR_BOUNDS in the
 * workspace status word (when workspace is non-NULL) and is masked to 4 bits. */
int b200q_pack_int4(const void* codes, int64_t K, int64_t N, int offset, int32_t* qweight, void* workspace,
                    void* stream);

/* Fused SiLU * mul + per-group dynamic fp8 quantisation (FUSED_SILU_REF,
 * generate_tasks.py:321-348).  y [T, 2H] = concat(gate, up) in fp16/bf16
 * (dtype 0/1), H % 128 == 0.  For each row and group of 128 columns:
 * act = SiLU(gate) * up in fp32, scale = max(amax|act| / 448, 1e-12),
 * q = e4m3(clamp(act / scale, +-448)) (round to nearest even).  Outputs, any
 * of which may be NULL (not all): out_dequant [T, H] fp32 = q * scale (the
 * reference module's result), q_out [T, H] e4m3 codes, scales_out
 * [T, H/128] fp32. */
int b200q_silu_mul_fp8(const void* y, int64_t T, int64_t H, int dtype, float* out_dequant, uint8_t* q_out,
                       float* scales_out, void* stream);

/* Multi-LoRA (LORA_REF, generate_tasks.py:397-424), the adapter part of
 * y[t] = x[t] . dequant(W) + (x[t] . A[id_t]) . B[id_t].
 * shrink: lo [T, r] = x [T, D] . A[id_t] [D, r] per token (A [L, D, r]),
 * fp32 accumulation, rounded to the activation type.  expand_add:
 * y [T, N] = base [T, N] + round(lo . B[id_t]) (B [L, r, N]), rounded once;
 * y may be base.  lora_ids [T] int64; r <= 64.  An id outside [0, L) sets
 * B200Q_DEV_ERR_BOUNDS (shrink, when workspace is non-NULL) and contributes
 * zero. */
int b200q_lora_shrink(const void* x, const void* A, const int64_t* lora_ids, int64_t T, int64_t D, int64_t r,
                      int64_t L, int dtype, void* lo, void* workspace, void* stream);
int b200q_lora_expand_add(const void* base, const void* lo, const void* B, const int64_t* lora_ids, int64_t T,
                          int64_t r, int64_t N, int64_t L, int dtype, void* y, void* stream);

/* Grouped W4A16 GEMM over the experts of a MoE layer, one launch for all
 * experts.  x [rows, K] holds every expert's rows contiguously, expert e's at
 * [offsets[e], offsets[e+1]) (offsets [E+1] int32 on the device, as written
 * by b200q_moe_route; read by the kernel, so no host synchronisation).
 * Expert weights are stacked: qweight [E, K, N/8] int32, scales / zeros
 * [E, K/group, N] in x's dtype.  Without the *_up arrays (NULL):
 * y [rows, N] = x . W_e row by row.  With them (the gate and up projections,
 * same shapes): y [rows, N] = SiLU(x . Wg_e) * (x . Wu_e), the products
 * rounded to the activation type before SiLU and the result rounded once, as
 * b200q_w4a16_gemm + b200q_silu_mul compute it.  K a multiple of 64,
 * 1 <= E <= 64, workspace >= 256 bytes (status word).  Replaces the
 * per-expert loop of FUSED_QMOE_REF.forward (generate_tasks.py:372-378) and
 * the SiLU.mul of FUSED_SILU_REF (:336-337). */
int b200q_moe_grouped_gemm(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                           const int32_t* qweight_up, const void* scales_up, const void* zeros_up,
                           const int32_t* offsets, int64_t E, void* y, int64_t rows, int64_t N, int64_t K,
                           int64_t group, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Column-sharded W4A16 GEMM with the all-gather fused into its epilogue.
 * Computes columns [col0, col0 + N) of y = x . W from this rank's shard
 * (qweight [K, N/8], scales/zeros [K/group, N]) and stores every finished
 * tile into each of the n_peers buffers y_peers[i] ([M, ldy] row-major, the
 * same dtype as x): normally y_peers[i] is rank i's full output mapped into
 * this process (CUDA IPC / symmetric memory; NVLink peer stores, no
 * multicast).  Needs col0 and ldy multiples of 32, col0 + N <= ldy,
 * 1 <= n_peers <= 8; workspace as for b200q_w4a16_gemm with the shard's
 * (M, N, K).
 * pads: NULL, or rank i's signal pad for every i < n_peers (64 zeroed uint32
 * words each, mapped into this process; this process's rank is `rank`).
 * With pads the call orders itself against the peers, which must make the
 * same sequence of calls: no rank stores into a peer's output before that
 * peer has reached the same call, and the call completes on the stream only
 * once every rank's columns have landed in every output.  A peer that does
 * not arrive within 10 s sets B200Q_DEV_ERR_TIMEOUT in the status word.
 * Without pads the ordering is the caller's (b200q_peer_barrier before and
 * after).  No counterpart in the reference, which is single-GPU
 * (generate_tasks.py:149); it replaces b200q_w4a16_gemm + an all-gather. */
int b200q_w4a16_gemm_peers(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                           void* const* y_peers, int n_peers, int64_t ldy, int64_t col0, void* const* pads,
                           int rank, int64_t M, int64_t N, int64_t K, int64_t group, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Column-sharded MXFP8 GEMM with the all-gather fused into its epilogue: the
 * same contract as b200q_w4a16_gemm_peers (destinations, pads, ordering,
 * timeouts) for b200q_mxfp8_gemm's operands, where B and scales_b hold this
 * rank's N output columns.  No counterpart in the reference (single-GPU,
 * generate_tasks.py:149); it replaces b200q_mxfp8_gemm + an all-gather. */
int b200q_mxfp8_gemm_peers(const void* a, const void* scales_a, const void* b, const void* scales_b,
                           void* const* y_peers, int n_peers, int64_t ldy, int64_t col0, void* const* pads, int rank,
                           int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* Barrier across the world ranks of one node, enqueued on `stream`.
 * pads[i] is rank i's signal pad (as above; the barrier uses words disjoint
 * from the GEMM's).  Orders this stream's earlier writes (peer stores
 * included) before the peers' later work.  A rank that does not arrive within
 * 10 s makes the wait give up and sets B200Q_DEV_ERR_TIMEOUT in the workspace
 * status word. */
int b200q_peer_barrier(void* const* pads, int world, int rank, void* workspace, void* stream);

/* Wait limit of b200q_peer_barrier in milliseconds (process-wide; <= 0
 * restores the default 10 s).  Returns the previous limit.  Lets a test or a
 * health check give up on a missing peer sooner.  No counterpart in the
 * reference. */
int64_t b200q_set_peer_barrier_timeout_ms(int64_t ms);

#ifdef __cplusplus
}
#endif

#endif /* B200Q_H_ */
