/*
 * yanchor_b200 — C ABI of the B200 (sm_100a) kernels for YANchor's
 * data-parallel hot path: the gated delta rule (GDN) recurrence (chunked
 * prefill and per-token decode), the fixed-capacity anchor memory read/write,
 * and final-logit sampling.
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise; the caller
 *     owns all memory.  Sizes and strides are int64 element counts.
 *   - `stream` is a cudaStream_t passed as void*.  Nothing here synchronises
 *     the stream or allocates device memory, so every call may be captured in
 *     a CUDA graph.
 *   - Every entry point returns YB_OK (0) or an error code; argument errors
 *     are detected on the host before any launch.  yb_last_error() gives a
 *     message for the calling thread's last failure.
 *   - dtype codes: YB_F32, YB_F16, YB_BF16 (values), YB_I32, YB_I64 (positions).
 *
 * The reference binds these operations as Python callables; the comment above
 * each entry point names the reference interface it replaces (paths inside
 * the reference project; "fla:" is flash-linear-attention 0.5.1, the
 * third-party package the reference pins in requirements.txt:20).
 */
#ifndef YANCHOR_B200_H
#define YANCHOR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum yb_dtype { YB_F32 = 0, YB_F16 = 1, YB_BF16 = 2, YB_I32 = 3, YB_I64 = 4 };

enum yb_status {
  YB_OK = 0,
  YB_ERR_ARGUMENT = 1,     /* bad shape, stride, dtype or pointer */
  YB_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement */
  YB_ERR_CUDA = 3,         /* a CUDA launch failed */
  YB_ERR_WORKSPACE = 4     /* workspace missing or too small */
};

/* GDN flags */
#define YB_GDN_QK_L2NORM 1u        /* use_qk_l2norm_in_kernel */
#define YB_GDN_GATE_IN_KERNEL 2u   /* g holds raw `a`; decay = -exp(A_log) * softplus(a + dt_bias) */
#define YB_GDN_BETA_SIGMOID 4u     /* beta holds logits; beta = sigmoid(beta) */
#define YB_GDN_TRANSPOSE_STATE 8u  /* state layout [N, HV, V, K] instead of [N, HV, K, V] */
#define YB_GDN_STATE_F16 16u       /* yb_gdn_recurrent_fwd: h0 / ht are float16 (else float32) */
#define YB_GDN_STATE_BF16 32u      /* yb_gdn_recurrent_fwd: h0 / ht are bfloat16 */

/* Message of the calling thread's last failed call ("" if none). */
const char *yb_last_error(void);
/* ABI version of this library. */
int yb_abi_version(void);
/*
 * Error word of the kernels that synchronise through time-bounded waits (the
 * tensor-core kernels, the one-launch decode layer's state prefetch, the
 * single-token fp32 decode's state copy, 0x601) or skip a store whose index
 * leaves its table (the decode bookkeeping, 0x401): 0 when every wait
 * completed and every index
 * was in range, else the first code recorded (that launch's outputs are then
 * invalid).
 * Synchronises the current device; `clear` resets the word.  No reference
 * counterpart: the reference's Triton kernels have no such waits.
 */
int yb_device_error(int clear);

/*
 * Per-token gated delta rule over T steps (T = 1 is batched decode).
 * Replaces fla: ops/gated_delta_rule/fused_recurrent.py:291
 * `fused_recurrent_gated_delta_rule`, as bound by modeling_yanchor.py:398-406
 * and by the in-place decode override runtime/model/inference_kernels.py:147-173
 * (h0 == ht: the state is updated in place).
 *
 *   q, k  [B, T, H, K]    v, o  [B, T, HV, V]    g, beta  [B, T, HV]
 *   h0, ht [N, HV, K, V] fp32 (or [N, HV, V, K] with YB_GDN_TRANSPOSE_STATE);
 *   either may be NULL; they may alias.  With YB_GDN_STATE_F16 or
 *   YB_GDN_STATE_BF16 (K = V = 128) both are float16 / bfloat16: the
 *   reference's reduced-precision state storage for decode
 *   (runtime/model/inference_kernels.py:437-457, modeling_yanchor.py:733-750);
 *   the state is widened to fp32 for the step and rounded to nearest when
 *   stored.
 *   *_tok_stride: elements between consecutive tokens of the flattened
 *   (B*T) token axis; heads and features are contiguous inside a token.
 *   cu_seqlens: NULL, or [N+1] int64 with B == 1 (varlen packing).
 *   A_log, dt_bias: [HV] fp32, used with YB_GDN_GATE_IN_KERNEL.
 *   z, norm_weight: optional fused gated RMSNorm epilogue
 *   (transformers qwen3_5 Qwen3_5RMSNormGated, modeling_qwen3_5.py:175-190):
 *   o = norm_weight * rmsnorm(o) * silu(z); z [B, T, HV, V] contiguous,
 *   norm_weight [V], both in io_dtype.  Pass NULL to skip.
 */
int yb_gdn_recurrent_fwd(const void *q, const void *k, const void *v, int64_t q_tok_stride,
                         int64_t k_tok_stride, int64_t v_tok_stride, const void *g, const void *beta,
                         int64_t g_tok_stride, int64_t beta_tok_stride, const float *A_log,
                         const float *dt_bias, const void *h0, void *ht, void *o, const void *z,
                         const void *norm_weight, float norm_eps, const int64_t *cu_seqlens, int64_t B,
                         int64_t T, int64_t H, int64_t HV, int64_t K, int64_t V, int64_t N, float scale,
                         int io_dtype, int g_dtype, int beta_dtype, uint32_t flags, void *stream);

/*
 * One GDN layer's decode core in one launch: the short conv update over the
 * fused q/k/v projection (kernel width 4, SiLU), the gates
 * (decay = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b)), the
 * q/k L2 norm, the gated delta rule with the state updated in place, and
 * the gated RMSNorm of the output with z and norm_weight.  Replaces the
 * sequence of runtime/model/inference_kernels.py:693-721
 * `_fused_gdn_gate_native_decode_forward` between in_proj and out_proj
 * (fused gates :668-691, causal_conv1d_update :339-376, the in-place
 * recurrence :147-173, Qwen3_5RMSNormGated), with the same roundings.
 *
 *   mixed [N*T, 2*H*K + HV*V] (channels q | k | v), z [N*T, HV, V],
 *   a, b [N*T, HV] (logits) — bf16 or fp16 (io_dtype), token strides in
 *   elements; conv_state [N, 2*H*K + HV*V, 4] in io_dtype, updated in place;
 *   conv_weight [C, 4], conv_bias [C] (or NULL) fp32; state [N, HV, K, V]
 *   (or [N, HV, V, K] with YB_GDN_TRANSPOSE_STATE) in state_dtype (YB_F32,
 *   YB_BF16 or YB_F16), updated in place; A_log, dt_bias [HV] fp32;
 *   norm_weight [V] io_dtype; o [N*T, HV, V] io_dtype.  K = V = 128.
 */
int yb_gdn_decode_fused(const void *mixed, int64_t mixed_tok_stride, const void *z, int64_t z_tok_stride,
                        const void *a, const void *b, int64_t ab_tok_stride, void *conv_state,
                        int64_t conv_batch_stride, int64_t conv_width, const float *conv_weight,
                        const float *conv_bias, int64_t conv_ks, void *state, int state_dtype,
                        const float *A_log, const float *dt_bias, const void *norm_weight, float norm_eps,
                        void *o, int64_t N, int64_t T, int64_t H, int64_t HV, int64_t K, int64_t V, float scale,
                        int io_dtype, uint32_t flags, void *stream);

/*
 * Sliding-window attention decode over the physical ring cache.  Ring key /
 * value [B, KVH, W, D] (each head's W positions are contiguous rows of D;
 * batch / head strides in elements), ring valid [B, W] (bool bytes), one
 * device write index for the whole batch (index_dtype YB_I32, as the
 * reference's cache keeps it, or YB_I64).
 *
 * yb_swa_ring_write: the new token's key / value [B, KVH, 1, D] (strides in
 * elements, D contiguous) and valid [B] go to ring position *ring_index,
 * then *ring_index advances modulo W.  Replaces
 * runtime/model/inference_kernels.py:1828-1879
 * `triton_fixed_memory_swa_physical_ring_update`.
 *
 * yb_swa_decode_attention: query [B, 1, QH, D] -> out [B, 1, QH, D]; each
 * query head h attends to the valid positions of KV head h / (QH / KVH),
 * scale D^-1/2 (a row with no valid position gives zeros).  D in
 * {32, 64, 128, 256}, QH / KVH in {1, 2, 4, 8}.  Workspace:
 * yb_swa_decode_workspace_bytes(B, KVH, QH, W, D).  Replaces
 * runtime/model/inference_kernels.py:1881-1897
 * `fixed_memory_physical_ring_decode_attention`.
 */
int yb_swa_ring_write(const void *key, const void *value, int64_t kv_batch_stride, int64_t kv_head_stride,
                      const uint8_t *valid, void *ring_key, void *ring_value, int64_t ring_batch_stride,
                      int64_t ring_head_stride, uint8_t *ring_valid, int64_t ring_valid_batch_stride,
                      void *ring_index, int index_dtype, int64_t B, int64_t KVH, int64_t W, int64_t D, int dtype,
                      void *stream);
int64_t yb_swa_decode_workspace_bytes(int64_t B, int64_t KVH, int64_t QH, int64_t W, int64_t D);
int yb_swa_decode_attention(const void *query, const void *ring_key, const void *ring_value,
                            int64_t ring_batch_stride, int64_t ring_head_stride, const uint8_t *valid,
                            int64_t valid_batch_stride, void *out, int64_t B, int64_t QH, int64_t KVH, int64_t W,
                            int64_t D, int dtype, void *workspace, int64_t workspace_bytes, void *stream);

/*
 * Causal depthwise conv1d in front of the recurrence (the GDN layer's short
 * convolution over the fused q/k/v projection):
 *   y[t, c] = act(sum_{j < KS} weight[c, j] * x[t - (KS - 1) + j, c] + bias[c]),
 * act = SiLU when silu != 0, fp32 arithmetic, one rounding to dtype.
 * Activations are token-major with channels contiguous: x, out [B, T, C]
 * (the memory of the reference's [B, C, T] transposed view), given by batch
 * and token strides in elements.  State [B, C, W], W = KS (the cache's
 * convention) or KS - 1 (`initial_states` of the causal-conv1d package),
 * given by batch, channel and tap strides in elements: packed rows (W, 1),
 * or channels contiguous with taps C apart (1, C), which is how the
 * reference's cache holds it after padding the transposed projection
 * (transformers qwen3_5 modeling_qwen3_5.py:466-467); any layout whose
 * (channel, tap) elements do not overlap is accepted;
 * its last KS - 1 entries are the inputs before t = 0.  weight [C, KS] and
 * bias [C] (or NULL) are fp32.  KS in {2, 3, 4}.
 *
 * yb_conv1d_update: one token (T = 1); the state is shifted left and the
 * input appended, in place.  Replaces runtime/model/inference_kernels.py:
 * 339-376 `triton_graph_safe_causal_conv1d_update` and modeling_yanchor.py:
 * 349-353 `torch_causal_conv1d_update`.
 *
 * yb_conv1d_fwd: a segment of T tokens; inputs before it come from
 * initial_state (NULL: zeros); final_state (NULL: not written, may alias
 * initial_state) receives the last W inputs of [initial_state | x], zeros
 * where there are none.  Replaces the prefill convolution of transformers
 * qwen3_5 modeling_qwen3_5.py:462-480 (`causal_conv1d_fn` / `conv1d`).
 */
int yb_conv1d_update(const void *x, int64_t x_batch_stride, void *conv_state, int64_t state_batch_stride,
                     int64_t state_channel_stride, int64_t state_tap_stride, int64_t state_width,
                     const float *weight, const float *bias, void *out, int64_t out_batch_stride, int64_t B,
                     int64_t C, int64_t KS, int silu, int dtype, void *stream);
int yb_conv1d_fwd(const void *x, int64_t x_batch_stride, int64_t x_token_stride, const void *initial_state,
                  void *final_state, int64_t state_batch_stride, int64_t state_channel_stride,
                  int64_t state_tap_stride, int64_t state_width, const float *weight, const float *bias, void *out,
                  int64_t out_batch_stride, int64_t out_token_stride, int64_t B, int64_t T, int64_t C, int64_t KS,
                  int silu, int dtype, void *stream);

/*
 * Chunked (64-token WY/UT transform) gated delta rule for prefill.
 * Replaces fla: ops/gated_delta_rule/chunk.py:365 `chunk_gated_delta_rule`
 * (bound at modeling_yanchor.py:397-405; the torch restatement is
 * transformers qwen3_5 modeling_qwen3_5.py:234-311).
 * Same tensor conventions as yb_gdn_recurrent_fwd (no fused norm epilogue).
 * workspace: device scratch of at least yb_gdn_chunk_workspace_bytes(...)
 * bytes (may be NULL when that is 0).
 */
int64_t yb_gdn_chunk_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t HV, int64_t K, int64_t V,
                                     int64_t N, int io_dtype);
int yb_gdn_chunk_fwd(const void *q, const void *k, const void *v, int64_t q_tok_stride,
                     int64_t k_tok_stride, int64_t v_tok_stride, const void *g, const void *beta,
                     int64_t g_tok_stride, int64_t beta_tok_stride, const float *A_log, const float *dt_bias,
                     const float *h0, float *ht, void *o, const int64_t *cu_seqlens, int64_t B, int64_t T,
                     int64_t H, int64_t HV, int64_t K, int64_t V, int64_t N, float scale, int io_dtype,
                     int g_dtype, int beta_dtype, uint32_t flags, void *workspace, int64_t workspace_bytes,
                     void *stream);

/*
 * GDN gates: beta = sigmoid(b) (io_dtype) and g = -exp(A_log) * softplus(a + dt_bias)
 * (fp32, linear above 20).  b, a: [rows, heads] with row strides; A_log, dt_bias [heads] fp32.
 * Replaces runtime/model/inference_kernels.py:683-691 `triton_qwen35_fused_gdn_gates`
 * (the expression of transformers qwen3_5 modeling_qwen3_5.py:500-502).
 */
int yb_gdn_gates(const void *b, const void *a, int64_t b_row_stride, int64_t a_row_stride,
                 const float *A_log, const float *dt_bias, void *beta_out, float *g_out, int64_t rows,
                 int64_t heads, int io_dtype, void *stream);

/*
 * Anchor memory, decode read: softmax over the CAP committed slots plus a
 * null slot (logit 0, value 0); empty slots have position < 0.
 * Replaces runtime/model/independent_memory.py:177 `committed_gqa`
 * (torch: modeling_yanchor.py:283-290).
 *   query, out [B, 1, H, D] contiguous; keys, values [*, G, CAP, D] with batch
 *   stride kv_stride0; positions [*, G, CAP] int32 with batch stride
 *   pos_stride0; indices NULL or [B] int64 (state row per request, -1 = skip,
 *   output zeros).
 */
int yb_mem_decode_read(const void *query, const void *keys, const void *values, const int32_t *positions,
                       const int64_t *indices, void *out, int64_t B, int64_t H, int64_t G, int64_t CAP,
                       int64_t D, int64_t kv_stride0, int64_t pos_stride0, int dtype, void *stream);

/*
 * Anchor memory, decode write/commit (state mutated in place).
 * Replaces runtime/model/independent_memory.py:190 `commit_decode`
 * (torch: modeling_yanchor.py:291-312).
 *   key, value [B, 1, G, D] contiguous; scores [B, 1, G] fp32; active [B] bool.
 *   Bank: keys/values [*, G, CAP, D] (batch stride kv_stride0), scores fp32 and
 *   positions int32 [*, G, CAP] (batch stride meta_stride0).  Pending:
 *   pending_keys/values [*, G, PC, D] (pkv_stride0), pending_scores [*, G, PC]
 *   (pmeta_stride0).  count/total int64 [*] (count_stride0).  chunk <= PC.
 */
int yb_mem_decode_commit(const void *key, const void *value, const float *scores, const uint8_t *active,
                         int64_t chunk, void *keys, void *values, float *bank_scores, int32_t *positions,
                         void *pending_keys, void *pending_values, float *pending_scores, int64_t *count,
                         int64_t *total, const int64_t *indices, int64_t B, int64_t G, int64_t CAP,
                         int64_t PC, int64_t D, int64_t kv_stride0, int64_t meta_stride0,
                         int64_t pkv_stride0, int64_t pmeta_stride0, int64_t count_stride0, int dtype,
                         void *stream);

/*
 * Anchor memory, one decode step of a memory layer: yb_mem_decode_read, then
 * yb_mem_decode_commit on the same state, in one launch where the read takes
 * its tensor-core path (16-bit, CAP <= 64, CAP + chunk <= 128): each
 * (row, group) CTA reads its group in four warps and commits that same group
 * (push, and the merge when the chunk fills) in four more beside them.  Only
 * that CTA reads the group's bank, and the commit writes it only after the
 * read holds its rows, so every read still sees the bank from before this
 * step's commit, as with the two calls in that order.  The last of the row's
 * G CTAs to finish its commit updates count / total and sets the row's
 * arrival counter back to 0.  Otherwise it makes those two calls.
 * Results are identical to the two calls.
 * The sequence of runtime/model/independent_memory.py:177 `committed_gqa`
 * then :190 `commit_decode` in the reference's decode layer
 * (modeling_yanchor.py:283-312).
 *   Arguments as in the two calls (one indices array serves both), plus
 *   arrive: B int32 counters, zero before the first call, left zero by every
 *   call.  Calls that overlap on the GPU must not share them.
 */
int yb_mem_decode_step(const void *query, void *out, const void *key, const void *value, const float *scores,
                       const uint8_t *active, int64_t chunk, void *keys, void *values, float *bank_scores,
                       int32_t *positions, void *pending_keys, void *pending_values, float *pending_scores,
                       int64_t *count, int64_t *total, const int64_t *indices, int32_t *arrive, int64_t B,
                       int64_t H, int64_t G, int64_t CAP, int64_t PC, int64_t D, int64_t kv_stride0,
                       int64_t meta_stride0, int64_t pkv_stride0, int64_t pmeta_stride0, int64_t count_stride0,
                       int dtype, void *stream);

/*
 * Anchor memory, prefill read: each block's queries attend to their group's
 * referenced rows plus the null slot.
 * Replaces runtime/model/independent_memory.py:38 `indexed_gqa`
 * (torch: modeling_yanchor.py:22-42 `indexed_gqa_torch`).
 *   query, out [B, blocks, chunk, H, D]; key, value [KB, S, G, D] (KB = 1 or B);
 *   references [B, blocks, G, CAP] int64, -1 = empty.  All contiguous.
 */
int yb_mem_indexed_read(const void *query, const void *key, const void *value, const int64_t *references,
                        void *out, int64_t B, int64_t blocks, int64_t chunk, int64_t H, int64_t G,
                        int64_t D, int64_t S, int64_t KB, int64_t CAP, int dtype, void *stream);
/*
 * yb_mem_indexed_read_timeline: the same read for the prefill orchestration,
 * addressing the prompt's own tensors: query / out [B, T, H, D]; block slot
 * s (0 <= s < blocks * chunk) of row b is token s + token_shift[b]; only
 * slots in [write_lo[b], write_hi[b]) whose token lies in [0, T) are
 * computed and written — every other output row is left untouched.
 * token_shift / write_lo / write_hi: device int64 [B].  Replaces the
 * reference's gather of the query onto the timeline and of the read back
 * (modeling_yanchor.py:196-198, 260-265) around `indexed_gqa`.
 *   key_new, value_new (may be null, then S_new = 0): a second source of
 *   rows [S_new, G, D], contiguous, for key batch KB = 1: reference S + i
 *   reads row i there.  The prefill passes the state's old rows as key /
 *   value and the writer's new rows here, instead of the reference's
 *   concatenation of both (modeling_yanchor.py:238-241).
 */
int yb_mem_indexed_read_timeline(const void *query, const void *key, const void *value, const void *key_new,
                                 const void *value_new, const int64_t *references, void *out, int64_t B, int64_t T,
                                 int64_t blocks, int64_t chunk, int64_t H, int64_t G, int64_t D, int64_t S,
                                 int64_t S_new, int64_t KB, int64_t CAP, const int64_t *token_shift,
                                 const int64_t *write_lo, const int64_t *write_hi, int dtype, void *stream);

/*
 * Top-CAP selection of anchor candidates.  Order: score descending (NaN
 * first, -0.0 equal to 0.0), then position ascending with invalid entries
 * (reference < 0) last, then candidate index.  Outputs: scores float32,
 * positions int64 (-1 where the reference is < 0), references int64; rows
 * with fewer candidates than `capacity` are padded with (-inf, -1, -1).
 * positions_dtype is YB_I32 or YB_I64.  All arrays contiguous.
 *
 * yb_mem_select_topk: per row of `n` candidates (n <= 4096).
 * Replaces modeling_yanchor.py:51-60 `select_topk` (and `merge_topk`,
 * :62-63, which is select_topk of the concatenation).
 *
 * yb_mem_exclusive_prefix_topk: inputs [B, blocks, G, chunk] (chunk <= 4096);
 * outputs [B, blocks + 1, G, capacity] (capacity <= 512): entry i is the
 * top-capacity over blocks 0 .. i-1, entry `blocks` over all of them.  With
 * initial_scores non-NULL, a bank [B, G, capacity] (scores, positions and
 * references; initial_references NULL means "slot index where the position
 * is >= 0, else -1") joins every entry, as the reference's merge of each
 * prefix with the state's bank.  Equal to the reference when valid
 * positions are distinct within a (row, group) and invalid references are
 * -1, which holds for the prefill orchestration.  Replaces
 * modeling_yanchor.py:65-78 `exclusive_prefix_topk` and :206-208.
 */
int yb_mem_select_topk(const float *scores, const void *positions, int positions_dtype, const int64_t *references,
                       int64_t rows, int64_t n, int64_t capacity, float *out_scores, int64_t *out_positions,
                       int64_t *out_references, void *stream);
int yb_mem_exclusive_prefix_topk(const float *scores, const void *positions, int positions_dtype,
                                 const int64_t *references, int64_t B, int64_t blocks, int64_t G, int64_t chunk,
                                 int64_t capacity, const float *initial_scores, const void *initial_positions,
                                 int initial_positions_dtype, const int64_t *initial_references,
                                 float *out_scores, int64_t *out_positions, int64_t *out_references,
                                 void *stream);

/*
 * The prefill orchestration of one memory layer on the device, the index work
 * of IndependentGQAMemory._sequence (modeling_yanchor.py:178-275) between the
 * selection and the read, in four calls (every tensor contiguous unless a
 * stride is given; shift = capacity with a state, 0 without).
 *
 * yb_mem_prefill_timeline (modeling_yanchor.py:186-205): each row's slots
 *   [the state's pending tokens | new tokens, valid first], padded to extent
 *   (a multiple of chunk).  scores [B, T, G] f32; order [B, T] int64 (the
 *   stable valid-first order) or NULL; n_new [B] (valid tokens) or NULL (T);
 *   count / total [B] at count_stride0 and pending_scores [B, G, PC] at
 *   pmeta_stride0 (the state; ignored when shift = 0).  Writes snapshot
 *   [3, B] (count, total, n_new before the call), slot scores / positions /
 *   references [B, extent / chunk, G, chunk] (the selection's input) and the
 *   token of every slot [B, extent].
 */
int yb_mem_prefill_timeline(const float *scores, const int64_t *order, const int64_t *n_new, const int64_t *count,
                            const int64_t *total, int64_t count_stride0, const float *pending_scores,
                            int64_t pmeta_stride0, int64_t B, int64_t T, int64_t G, int64_t chunk, int64_t extent,
                            int64_t shift, int64_t PC, int64_t *snapshot, float *slot_scores,
                            int64_t *slot_positions, int64_t *slot_references, int64_t *slot_tokens, void *stream);
/*
 * yb_mem_prefill_table (modeling_yanchor.py:206-244): from the prefix top-CAP
 * references [B, blocks + 1, G, capacity], which new slots need a writer row
 * (needed [B, extent] bytes) and the slot -> source-row table
 * [B, shift + extent] (old rows b * (capacity + chunk) + s; -1 elsewhere).
 * With capture_safe the writer ran on every slot (row b * extent + slot after
 * the old rows), so the needed slots are filled in and read_references
 * [B, blocks, G, capacity] is written too; otherwise the caller fills in the
 * needed slots and calls yb_mem_prefill_read_references.
 */
int yb_mem_prefill_table(const int64_t *prefix_references, const int64_t *snapshot, int64_t B, int64_t G,
                         int64_t chunk, int64_t extent, int64_t capacity, int has_state, int capture_safe,
                         uint8_t *needed, int64_t *table, int64_t *read_references, void *stream);
/* yb_mem_prefill_read_references: each block's prefix top-CAP as source rows (-1 = empty). */
int yb_mem_prefill_read_references(const int64_t *prefix_references, const int64_t *table, int64_t B, int64_t G,
                                   int64_t chunk, int64_t extent, int64_t capacity, int has_state,
                                   int64_t *read_references, void *stream);
/*
 * yb_mem_prefill_state (modeling_yanchor.py:266-275): the new bank (the prefix
 * entry after the last complete block) and pending chunk (the incomplete
 * tail), their rows from old_keys / old_values [B * (capacity + chunk), G, D]
 * (a copy of the bank and pending rows taken before the call) or new_keys /
 * new_values [N, G, D] (the writer's rows), and count / total.  The state's
 * fields at their batch strides (inner dimensions contiguous).
 */
int yb_mem_prefill_state(const float *prefix_scores, const int64_t *prefix_positions,
                         const int64_t *prefix_references, const int64_t *table, const int64_t *snapshot,
                         const float *slot_scores, const void *old_keys, const void *old_values, const void *new_keys,
                         const void *new_values, void *keys, void *values, int64_t kv_stride0, float *bank_scores,
                         int32_t *positions, int64_t meta_stride0, void *pending_keys, void *pending_values,
                         int64_t pkv_stride0, float *pending_scores, int64_t pmeta_stride0, int64_t *count,
                         int64_t *total, int64_t count_stride0, int64_t B, int64_t G, int64_t chunk, int64_t extent,
                         int64_t capacity, int64_t PC, int64_t D, int dtype, void *stream);

/*
 * Sampling.  scores [B, vocab] (row stride in elements) in dtype; out [B] int64.
 * Workspace: device scratch of at least yb_sample_workspace_bytes(B, vocab, top_k).
 *
 * yb_sample_greedy: index of the first maximum per row (argmax).
 * Replaces the top_k == 1 branch of runtime/model/inference_kernels.py:73-88
 * `sample_top_k_top_p_counter` (scores.argmax(-1)).
 *
 * yb_sample_top_k_top_p_counter: top-k (k <= 256; top_k <= 0 means the whole
 * vocabulary, allowed only with top_p == 1) → softmax(values / temperature) →
 * top-p truncation → inverse-CDF pick with the stateless counter uniform of
 * (attempt id, step, seed, stream).  steps NULL means every row uses
 * scalar_step.  Replaces inference_kernels.py:73-88 and the fused top-20
 * sampler inference_kernels.py:1119-1167.
 */
int64_t yb_sample_workspace_bytes(int64_t B, int64_t vocab, int64_t top_k);
int yb_sample_greedy(const void *scores, int64_t row_stride, int64_t B, int64_t vocab, int dtype, int64_t *out,
                     void *workspace, int64_t workspace_bytes, void *stream);
/*
 * yb_sample_greedy_noalloc: the same argmax as yb_sample_greedy, for callers
 * that cannot allocate device memory where they sample — a host runtime
 * binding this ABI without a device allocator of its own, or a decode loop
 * that must not allocate while its stream is being captured.  It takes no
 * workspace: its partial results go to a fixed 64 KiB device array inside
 * this library, which covers at most 4096 rows (larger batches get
 * YB_ERR_UNSUPPORTED).  It allocates nothing and frees nothing.  The first
 * call in a CUDA context looks the array's device address up once for that
 * context (a context made after cudaDeviceReset looks it up again), so make
 * that first call before any stream capture.  All calls on a device
 * share the array: calls that may run at the same time on the GPU (different
 * streams with no ordering between them) race on it.  No counterpart in the
 * reference, which always lets torch allocate.
 */
int yb_sample_greedy_noalloc(const void *scores, int64_t row_stride, int64_t B, int64_t vocab, int dtype,
                             int64_t *out, void *stream);
int yb_sample_top_k_top_p_counter(const void *scores, int64_t row_stride, int64_t B, int64_t vocab, int dtype,
                                  const int64_t *attempt_ids, const int64_t *steps, int64_t scalar_step,
                                  int64_t seed, int64_t stream_id, float temperature, int64_t top_k,
                                  float top_p, int64_t *out, void *workspace, int64_t workspace_bytes,
                                  void *stream);

/*
 * scores[i] -= penalty * seen[i] over n elements (seen: bool bytes).
 * Replaces runtime/model/inference_kernels.py:1104-1114 `_apply_dense_presence_penalty_`.
 */
int yb_presence_penalty(void *scores, const uint8_t *seen, int64_t n, float penalty, int dtype, void *stream);

/*
 * Sliding-window attention over a prompt (prefill), on the tcgen05 tensor
 * cores.  Replaces modeling_yanchor.py:412-427 `reference_swa` (and the
 * FlashAttention call of `flash_swa`, :429-449, on rows whose valid tokens
 * form one run).  q / out [B, Tq, QH, D], k / v [B, Tk, KVH, D], contiguous
 * bf16, D = 256, QH / KVH in {1, 2, 4, 8}.  Query i sits at absolute
 * position query_start + i and key j at j; query i admits key j when
 * i_abs - window < j <= i_abs and key_valid[b, j] (key_valid [B, Tk] bool
 * bytes at valid_batch_stride, or NULL); scale D^-1/2.  A query whose own
 * key_valid entry (at i_abs) is false, or that admits no key, gives zeros.
 * Other shapes return YB_ERR_UNSUPPORTED.
 */
int yb_swa_prefill_attention(const void *q, const void *k, const void *v, const uint8_t *key_valid,
                             int64_t valid_batch_stride, void *out, int64_t B, int64_t Tq, int64_t Tk, int64_t QH,
                             int64_t KVH, int64_t D, int64_t window, int64_t query_start, int dtype, void *stream);

/*
 * Decode-loop bookkeeping after one sampled token per slot, in one launch.
 * Replaces runtime/model/inference_kernels.py:1206-1208
 * `_update_fixed_decode_state_` (Triton kernel :1169-1204) and the torch
 * statements it stands for (:1701-1717).  Per slot r:
 *   active = !finished[r] && slot_rows[r] >= 0; token = active ? sampled : pad
 *   write row = active ? slot_rows[r] : sink_rows[r];
 *   write column = active ? row_steps[r] : maximum_new_tokens
 *   storage[row, column] = token; dense_seen[r, token] = 1
 *   next = row_steps[r] + active; generated_lengths[row] = next (if active)
 *   finished_by_eos[row] |= active && token in eos_tokens
 *   finished[r] |= active && (eos || next >= slot_caps[r])
 *   row_steps[r] = next; row_positions[r] += active
 *   decode_ids[r] = finished[r] ? pad : token; *useful_events += #active
 * storage: [storage_rows, storage_stride] of storage_dtype (YB_I32 as the
 * reference allocates it, or YB_I64), storage_cols = maximum_new_tokens + 1
 * usable columns; dense_seen: [slots, seen_stride] bool with vocab columns;
 * generated_lengths / finished_by_eos: [storage_rows]; the slot vectors
 * [slots] (sampled_token and decode_ids at their row strides);
 * useful_events a device int64 scalar.  eos_tokens: host array of
 * eos_count (<= 8) ids.  Row indices must be distinct across active slots
 * and sink rows (the reference's slot table guarantees it).  A token outside
 * [0, vocab) or a write outside storage skips that store and is reported by
 * yb_device_error() (0x401).  Capture-safe; one kernel launch.
 */
int yb_decode_state_update(const int64_t *sampled_token, int64_t sampled_stride, void *storage, int storage_dtype,
                           int64_t storage_rows, int64_t storage_cols, int64_t storage_stride, uint8_t *dense_seen,
                           int64_t seen_stride, int64_t vocab, int64_t *generated_lengths, uint8_t *finished_by_eos,
                           uint8_t *finished, const int64_t *slot_rows, const int64_t *sink_rows,
                           const int64_t *slot_caps, int64_t *row_steps, int64_t *row_positions, int64_t *decode_ids,
                           int64_t decode_ids_stride, int64_t *useful_events, int64_t slots,
                           int64_t maximum_new_tokens, int64_t pad_token, const int64_t *eos_tokens, int eos_count,
                           void *stream);

#ifdef __cplusplus
}
#endif

#endif /* YANCHOR_B200_H */
