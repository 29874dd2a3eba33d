// Internal launcher interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace yb {

struct GdnArgs {
  const void *q, *k, *v;
  int64_t q_ts, k_ts, v_ts;  // token strides (elements)
  const void *g, *beta;
  int64_t g_ts, beta_ts;
  const float *A_log, *dt_bias;
  const float *h0;
  float *ht;
  void *o;
  const void *z, *norm_w;
  float norm_eps;
  const int64_t *cu_seqlens;
  int64_t B, T, H, HV, K, V, N;
  float scale;
  int io_dtype, g_dtype, beta_dtype;
  uint32_t flags;
  void *workspace;
  int64_t workspace_bytes;
  cudaStream_t stream;
};

int launch_gdn_recurrent(const GdnArgs &a);
int launch_gdn_chunk(const GdnArgs &a);
int launch_gdn_chunk_simt(const GdnArgs &a);
bool gdn_chunk_tc_supported(const GdnArgs &a);
int launch_gdn_chunk_tc(const GdnArgs &a);
int read_device_error(int clear);
int64_t gdn_chunk_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t HV, int64_t K, int64_t V,
                                  int64_t N, int io_dtype);

int launch_gdn_gates(const void *b, const void *a, int64_t b_rs, int64_t a_rs, const float *A_log,
                     const float *dt_bias, void *beta_out, float *g_out, int64_t rows, int64_t heads,
                     int io_dtype, cudaStream_t stream);

struct MemReadArgs {
  const void *query, *keys, *values;
  const int32_t *positions;
  const int64_t *indices;
  void *out;
  int64_t B, H, G, CAP, D, kv_s0, pos_s0;
  int dtype;
  cudaStream_t stream;
};
int launch_mem_decode_read(const MemReadArgs &a);

struct MemCommitArgs {
  const void *key, *value;
  const float *scores;
  const uint8_t *active;
  int64_t chunk;
  void *keys, *values;
  float *bank_scores;
  int32_t *positions;
  void *pkeys, *pvalues;
  float *pscores;
  int64_t *count, *total;
  const int64_t *indices;
  int64_t B, G, CAP, PC, D, kv_s0, meta_s0, pkv_s0, pmeta_s0, count_s0;
  int dtype;
  cudaStream_t stream;
};
int launch_mem_decode_commit(const MemCommitArgs &a);
// read then commit of one memory layer: one launch on the tensor-core read path, else two
int launch_mem_decode_step(const MemReadArgs &r, const MemCommitArgs &c, int32_t *arrive);

struct MemIndexedArgs {
  const void *query, *key, *value;
  const int64_t *refs;
  void *out;
  int64_t B, blocks, chunk, H, G, D, S, KB, CAP;
  int dtype;
  cudaStream_t stream;
  // timeline mode: query / out are [B, T, H, D]; slot s of row b is token
  // s + tok_shift[b]; only slots in [w_lo[b], w_hi[b]) are written
  const int64_t *tok_shift = nullptr, *w_lo = nullptr, *w_hi = nullptr;
  int64_t T = 0;
  // optional second source (KB == 1): references S .. S + S2 - 1 are rows 0 .. S2 - 1 of key2 / value2
  const void *key2 = nullptr, *value2 = nullptr;
  int64_t S2 = 0;
};
int launch_mem_indexed_read(const MemIndexedArgs &a);
bool mem_indexed_tc_supported(const MemIndexedArgs &a);
int launch_mem_indexed_tc(const MemIndexedArgs &a);
int read_device_error_idx(int clear);

// Anchor-memory prefill orchestration (the index work around the selection and read kernels).
struct PrefillGlueArgs {
  int64_t B = 0, T = 0, G = 0, chunk = 0, extent = 0, blocks = 0, cap = 0, PC = 0, shift = 0, D = 0;
  int has_state = 0, capture_safe = 0, dtype = 0;
  const int64_t *count = nullptr, *total = nullptr;   // the state's counters (read by the timeline phase)
  int64_t count_s0 = 0;
  const float *pend_scores = nullptr;                  // [B, G, PC] at pmeta_s0
  int64_t pmeta_s0 = 0;
  const int64_t *order = nullptr, *n_new = nullptr;    // [B, T] / [B] or null
  const float *scores = nullptr;                       // [B, T, G]
  int64_t *snap = nullptr;                             // [3, B]: count, total, new tokens before the prefill
  float *s_blk = nullptr;                              // [B, blocks, G, chunk]
  int64_t *pos_blk = nullptr, *ref_blk = nullptr;
  int64_t *tok = nullptr;                              // [B, extent]
  const int64_t *pre_r = nullptr;                      // [B, blocks + 1, G, cap]
  const float *pre_s = nullptr;
  const int64_t *pre_p = nullptr;
  uint8_t *needed = nullptr;                           // [B, extent]
  int64_t *table = nullptr;                            // [B, shift + extent]
  int64_t *read_refs = nullptr;                        // [B, blocks, G, cap]
  const void *old_k = nullptr, *old_v = nullptr;       // [B * (cap + chunk), G, D]
  const void *new_k = nullptr, *new_v = nullptr;       // [N, G, D]
  void *keys = nullptr, *values = nullptr;             // the state, written by the state phase
  int64_t kv_s0 = 0;
  float *bank_scores = nullptr;
  int32_t *positions = nullptr;
  int64_t meta_s0 = 0;
  void *pkeys = nullptr, *pvalues = nullptr;
  int64_t pkv_s0 = 0;
  float *pscores = nullptr;
  int64_t *count_out = nullptr, *total_out = nullptr;
  cudaStream_t stream = nullptr;
};
// phase 0: timeline; 1: needed + table; 2: read references; 3: the new state
int launch_prefill_glue(const PrefillGlueArgs &a, int phase);

struct TopkArgs {
  const float *scores;
  const void *positions;
  const int64_t *refs;
  int pos_dtype;
  int64_t rows, n, cap;
  float *out_s;
  int64_t *out_p, *out_r;
  cudaStream_t stream;
};
int launch_select_topk(const TopkArgs &a);

struct PrefixTopkArgs {
  const float *scores;
  const void *positions;
  const int64_t *refs;
  int pos_dtype;
  int64_t B, blocks, G, chunk, cap;
  const float *init_s;
  const void *init_p;
  const int64_t *init_r;
  int init_pos_dtype;
  float *out_s;
  int64_t *out_p, *out_r;
  cudaStream_t stream;
};
int launch_exclusive_prefix_topk(const PrefixTopkArgs &a);

struct FusedArgs {
  const void *mixed;
  int64_t mixed_ts;
  const void *z;
  int64_t z_ts;
  const void *a, *b;
  int64_t ab_ts;
  void *conv_state;
  int64_t conv_bs, conv_width, conv_ks;
  const float *conv_w, *conv_b;
  void *state;
  int state_dtype;
  bool trans;
  const float *A_log, *dt_bias;
  const void *norm_w;
  float norm_eps, scale;
  void *o;
  int64_t N, T, H, HV, K, V;
  int io_dtype;
  cudaStream_t stream;
};
int launch_gdn_decode_fused(const FusedArgs &a);
int read_device_error_fused(int clear);
int read_device_error_rec(int clear);

struct SwaArgs {
  const void *new_k, *new_v;      // ring write: the new token [B, KVH, 1, D]
  int64_t new_bs, new_hs;
  const uint8_t *new_valid;       // [B]
  void *ring_k, *ring_v;          // [B, KVH, W, D]
  int64_t ring_bs, ring_hs;
  uint8_t *ring_valid;            // [B, W]
  int64_t valid_bs;
  void *ring_index;               // device scalar, int32 (as the reference keeps it) or int64
  int index_i64;
  const void *query;              // attention: [B, 1, QH, D]
  void *out;                      // [B, 1, QH, D]
  int64_t B, QH, KVH, W, D;
  int dtype;
  cudaStream_t stream;
};
// Grouped-query decode attention on mma.sync: R = QH / G query heads of one
// KV group attend to up to 64 stored positions per CTA.  Direct mode (the
// anchor-memory read) writes normalised output with an optional null slot;
// partial mode (the sliding-window ring) writes per-slice sums for
// swa_combine_kernel.
struct GqaDecodeArgs {
  const void *query;              // [B, QH, D] contiguous
  const void *keys, *values;      // row s, group g, position p at s*kv_bs + g*kv_gs + p*D
  int64_t kv_bs, kv_gs;
  const int32_t *positions;       // mask by position >= 0 (s*pos_bs + g*pos_gs + p), or
  int64_t pos_bs, pos_gs;
  const uint8_t *valid;           // mask by valid[b*valid_bs + p]
  int64_t valid_bs;
  const int64_t *indices;         // optional stored row per request (-1 skips it)
  void *out;                      // direct mode: [B, QH, D]
  float *partial;                 // partial mode: [B*G, slices, R, D + 2]
  int null_slot;                  // add the null logit 0 (value 0) to the softmax
  int64_t B, G, QH, D, P;
  int dtype;
  cudaStream_t stream;
};
bool gqa_decode_mma_supported(int dtype, int64_t QH, int64_t G, int64_t D);
int launch_gqa_decode_mma(const GqaDecodeArgs &a);
// A direct memory read followed, in the same launch, by the commit of each row (done by the last
// of the row's G CTAs; `arrive` holds B zeroed counters, left zeroed).
struct MemCommitTail {
  MemCommitArgs c;
  int32_t *arrive;
};
bool gqa_decode_commit_fits(const GqaDecodeArgs &a, const MemCommitArgs &c);
int launch_gqa_decode_commit(const GqaDecodeArgs &a, const MemCommitArgs &c, int32_t *arrive);

// Decode-loop bookkeeping after a sampled token (one launch per step).
constexpr int kMaxEos = 8;
struct DecodeStateArgs {
  const int64_t *sampled;         // [slots] at sampled_stride
  int64_t sampled_stride;
  void *storage;                  // [storage_rows, storage_stride] int32 (or int64)
  int storage_i64;
  int64_t storage_rows, storage_cols, storage_stride;
  uint8_t *dense_seen;            // [slots, seen_stride] bool
  int64_t seen_stride, vocab;
  int64_t *generated_lengths;     // [storage_rows]
  uint8_t *finished_by_eos;       // [storage_rows]
  uint8_t *finished;              // [slots]
  const int64_t *slot_rows, *sink_rows, *slot_caps;
  int64_t *row_steps, *row_positions;
  int64_t *decode_ids;            // [slots] at decode_ids_stride
  int64_t decode_ids_stride;
  int64_t *useful_events;         // device scalar
  int64_t slots, max_new, pad;
  int64_t eos[kMaxEos];
  int eos_count;
  cudaStream_t stream;
};
int launch_decode_state_update(const DecodeStateArgs &a);
int read_device_error_loop(int clear);

// Sliding-window prefill attention (tcgen05): q / out [B, Tq, QH, D], k / v
// [B, Tk, KVH, D], contiguous; key_valid [B, Tk] bytes or null.
struct SwaPrefillArgs {
  const void *q, *k, *v;
  const uint8_t *key_valid;
  int64_t valid_bs;
  void *out;
  int64_t B, Tq, Tk, QH, KVH, D, window, query_start;
  int dtype;
  cudaStream_t stream;
};
bool swa_prefill_tc_supported(const SwaPrefillArgs &a);
int launch_swa_prefill_tc(const SwaPrefillArgs &a);
int read_device_error_swa(int clear);

int launch_swa_ring_write(const SwaArgs &a);
int launch_swa_decode_attention(const SwaArgs &a, void *workspace);
int64_t swa_workspace_bytes(int64_t B, int64_t KVH, int64_t QH, int64_t W, int64_t D);

struct ConvArgs {
  const void *x;
  int64_t x_bs, x_ts;             // batch / token strides (elements); channels contiguous
  void *state;                    // update: [B, C, W], in place
  const void *state_in;           // prefill: optional initial state
  void *state_out;                // prefill: optional final state (may alias state_in)
  int64_t state_bs, W;            // state batch stride (elements), width (KS or KS - 1)
  int64_t state_cs, state_ts;     // state channel / tap strides (elements): W and 1 when packed
  const float *weight, *bias;     // [C, KS] fp32, [C] fp32 or null
  void *out;
  int64_t out_bs, out_ts;
  int64_t B, T, C, KS;
  bool silu;
  int dtype;
  cudaStream_t stream;
};
int launch_conv1d(const ConvArgs &a, bool update);

struct SampleArgs {
  const void *scores;
  int64_t row_stride, B, vocab;
  int dtype;
  const int64_t *attempt_ids, *steps;
  int64_t scalar_step, seed, stream_id;
  float temperature;
  int64_t top_k;
  float top_p;
  int64_t *out;
  void *workspace;
  int64_t workspace_bytes;
  cudaStream_t stream;
};
int64_t sample_workspace_bytes(int64_t B, int64_t vocab, int64_t top_k);
int launch_sample_greedy(const SampleArgs &a);
int launch_sample_greedy_noalloc(const SampleArgs &a);
int64_t greedy_builtin_scratch_bytes();
int launch_sample_topk_topp(const SampleArgs &a);
int launch_sample_nucleus(const SampleArgs &a);
int launch_sample_cdf(const SampleArgs &a);
int launch_presence_penalty(void *scores, const uint8_t *seen, int64_t n, float penalty, int dtype,
                            cudaStream_t stream);

}  // namespace yb
