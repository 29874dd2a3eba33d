// extern "C" entry points: validate arguments on the host, then dispatch to
// the kernel launchers.  Errors never reach the device: a bad call returns a
// status code and a message (yb_last_error) before any launch.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace yb {

static thread_local char g_err[512] = "";

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return YB_OK;
}

static bool dtype_ok(int d) { return d == YB_F32 || d == YB_F16 || d == YB_BF16; }
static int dtype_size(int d) { return d == YB_F32 ? 4 : 2; }
static bool aligned(const void *p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

#define YB_REQUIRE(cond, ...)                                 \
  do {                                                        \
    if (!(cond)) return set_error(YB_ERR_ARGUMENT, __VA_ARGS__); \
  } while (0)

static int check_gdn(const GdnArgs &a, const char *op) {
  YB_REQUIRE(dtype_ok(a.io_dtype) && dtype_ok(a.g_dtype) && dtype_ok(a.beta_dtype), "%s: bad dtype code", op);
  YB_REQUIRE(a.B >= 0 && a.T >= 0 && a.H > 0 && a.HV > 0 && a.K > 0 && a.V > 0, "%s: bad sizes", op);
  YB_REQUIRE(a.HV % a.H == 0, "%s: HV=%lld must be a multiple of H=%lld", op, (long long)a.HV, (long long)a.H);
  YB_REQUIRE(a.B * a.T == 0 || (a.q && a.k && a.v && a.g && a.beta && a.o), "%s: null tensor", op);
  if (a.cu_seqlens) {
    YB_REQUIRE(a.B == 1, "%s: cu_seqlens requires B == 1 (got %lld)", op, (long long)a.B);
    YB_REQUIRE(a.N >= 0, "%s: bad N", op);
  } else {
    YB_REQUIRE(a.N == a.B, "%s: N (%lld) must equal B (%lld) without cu_seqlens", op, (long long)a.N,
               (long long)a.B);
  }
  const int es = dtype_size(a.io_dtype);
  YB_REQUIRE(a.q_ts >= a.H * a.K && a.k_ts >= a.H * a.K && a.v_ts >= a.HV * a.V, "%s: token stride too small", op);
  YB_REQUIRE((a.q_ts * es) % 16 == 0 && (a.k_ts * es) % 16 == 0 && (a.v_ts * es) % 16 == 0,
             "%s: token strides must be multiples of 16 bytes", op);
  YB_REQUIRE(aligned(a.q, 16) && aligned(a.k, 16) && aligned(a.v, 16) && aligned(a.o, 16),
             "%s: q, k, v, o must be 16-byte aligned", op);
  YB_REQUIRE(!a.h0 || aligned(a.h0, 16), "%s: h0 must be 16-byte aligned", op);
  YB_REQUIRE(!a.ht || aligned(a.ht, 16), "%s: ht must be 16-byte aligned", op);
  if (a.flags & YB_GDN_GATE_IN_KERNEL) YB_REQUIRE(a.A_log != nullptr, "%s: A_log required with gate-in-kernel", op);
  YB_REQUIRE(!(a.flags & ~63u), "%s: unknown flag bits 0x%x", op, a.flags);
  YB_REQUIRE((a.flags & (YB_GDN_STATE_F16 | YB_GDN_STATE_BF16)) != (YB_GDN_STATE_F16 | YB_GDN_STATE_BF16),
             "%s: at most one state storage flag", op);
  return YB_OK;
}

}  // namespace yb

using namespace yb;

extern "C" {

const char *yb_last_error(void) { return g_err; }
int yb_abi_version(void) { return 1; }
int yb_device_error(int clear) {
  const int a = read_device_error(clear), b = read_device_error_idx(clear), c = read_device_error_fused(clear),
            d = read_device_error_loop(clear), e = read_device_error_swa(clear), f = read_device_error_rec(clear);
  return a ? a : (b ? b : (c ? c : (d ? d : (e ? e : f))));
}

int yb_gdn_recurrent_fwd(const void *q, const void *k, const void *v, int64_t q_tok_stride, int64_t k_tok_stride,
                         int64_t v_tok_stride, const void *g, const void *beta, int64_t g_tok_stride,
                         int64_t beta_tok_stride, const float *A_log, const float *dt_bias, const void *h0,
                         void *ht, void *o, const void *z, const void *norm_weight, float norm_eps,
                         const int64_t *cu_seqlens, int64_t B, int64_t T, int64_t H, int64_t HV, int64_t K,
                         int64_t V, int64_t N, float scale, int io_dtype, int g_dtype, int beta_dtype, uint32_t flags,
                         void *stream) {
  GdnArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_ts = q_tok_stride; a.k_ts = k_tok_stride; a.v_ts = v_tok_stride;
  a.g = g; a.beta = beta; a.g_ts = g_tok_stride; a.beta_ts = beta_tok_stride;
  // a 16-bit state (YB_GDN_STATE_F16 / _BF16) travels through the float-typed
  // fields untouched; the decode kernel reads them with the flagged type
  a.A_log = A_log; a.dt_bias = dt_bias; a.h0 = static_cast<const float *>(h0); a.ht = static_cast<float *>(ht);
  a.o = o;
  a.z = z; a.norm_w = norm_weight; a.norm_eps = norm_eps; a.cu_seqlens = cu_seqlens;
  a.B = B; a.T = T; a.H = H; a.HV = HV; a.K = K; a.V = V; a.N = N; a.scale = scale;
  a.io_dtype = io_dtype; a.g_dtype = g_dtype; a.beta_dtype = beta_dtype; a.flags = flags;
  a.stream = static_cast<cudaStream_t>(stream);
  int rc = check_gdn(a, "gdn_recurrent");
  if (rc) return rc;
  if ((z == nullptr) != (norm_weight == nullptr))
    return set_error(YB_ERR_ARGUMENT, "gdn_recurrent: z and norm_weight go together");
  if (z && !(aligned(z, 16) && aligned(norm_weight, 16)))
    return set_error(YB_ERR_ARGUMENT, "gdn_recurrent: z and norm_weight must be 16-byte aligned");
  return launch_gdn_recurrent(a);
}

int64_t yb_gdn_chunk_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t HV, int64_t K, int64_t V, int64_t N,
                                     int io_dtype) {
  return gdn_chunk_workspace_bytes(B, T, H, HV, K, V, N, io_dtype);
}

int yb_gdn_chunk_fwd(const void *q, const void *k, const void *v, int64_t q_tok_stride, int64_t k_tok_stride,
                     int64_t v_tok_stride, const void *g, const void *beta, int64_t g_tok_stride,
                     int64_t beta_tok_stride, const float *A_log, const float *dt_bias, const float *h0, float *ht,
                     void *o, const int64_t *cu_seqlens, int64_t B, int64_t T, int64_t H, int64_t HV, int64_t K,
                     int64_t V, int64_t N, float scale, int io_dtype, int g_dtype, int beta_dtype, uint32_t flags,
                     void *workspace, int64_t workspace_bytes, void *stream) {
  GdnArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_ts = q_tok_stride; a.k_ts = k_tok_stride; a.v_ts = v_tok_stride;
  a.g = g; a.beta = beta; a.g_ts = g_tok_stride; a.beta_ts = beta_tok_stride;
  a.A_log = A_log; a.dt_bias = dt_bias; a.h0 = h0; a.ht = ht; a.o = o; a.cu_seqlens = cu_seqlens;
  a.B = B; a.T = T; a.H = H; a.HV = HV; a.K = K; a.V = V; a.N = N; a.scale = scale;
  a.io_dtype = io_dtype; a.g_dtype = g_dtype; a.beta_dtype = beta_dtype; a.flags = flags;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes;
  a.stream = static_cast<cudaStream_t>(stream);
  int rc = check_gdn(a, "gdn_chunk");
  if (rc) return rc;
  if (flags & (YB_GDN_STATE_F16 | YB_GDN_STATE_BF16))
    return set_error(YB_ERR_UNSUPPORTED, "gdn_chunk: 16-bit state storage is a decode feature (prefill keeps fp32)");
  const int64_t need = gdn_chunk_workspace_bytes(B, T, H, HV, K, V, N, io_dtype);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return set_error(YB_ERR_WORKSPACE, "gdn_chunk: workspace of %lld bytes required", (long long)need);
  return launch_gdn_chunk(a);
}

int yb_gdn_gates(const void *b, const void *a, int64_t b_row_stride, int64_t a_row_stride, const float *A_log,
                 const float *dt_bias, void *beta_out, float *g_out, int64_t rows, int64_t heads, int io_dtype,
                 void *stream) {
  YB_REQUIRE(dtype_ok(io_dtype), "gdn_gates: bad dtype");
  YB_REQUIRE(rows >= 0 && heads > 0, "gdn_gates: bad sizes");
  YB_REQUIRE(b && a && A_log && beta_out && g_out, "gdn_gates: null tensor");
  YB_REQUIRE(b_row_stride >= heads && a_row_stride >= heads, "gdn_gates: row stride too small");
  return launch_gdn_gates(b, a, b_row_stride, a_row_stride, A_log, dt_bias, beta_out, g_out, rows, heads, io_dtype,
                          static_cast<cudaStream_t>(stream));
}

int yb_mem_decode_read(const void *query, const void *keys, const void *values, const int32_t *positions,
                       const int64_t *indices, void *out, int64_t B, int64_t H, int64_t G, int64_t CAP, int64_t D,
                       int64_t kv_stride0, int64_t pos_stride0, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "mem_decode_read: bad dtype");
  YB_REQUIRE(B >= 0 && H > 0 && G > 0 && CAP > 0 && D > 0 && H % G == 0, "mem_decode_read: bad sizes");
  YB_REQUIRE(query && keys && values && positions && out, "mem_decode_read: null tensor");
  YB_REQUIRE(kv_stride0 >= G * CAP * D && pos_stride0 >= G * CAP, "mem_decode_read: batch stride too small");
  YB_REQUIRE((kv_stride0 * dtype_size(dtype)) % 16 == 0, "mem_decode_read: key batch stride must be 16-byte multiple");
  YB_REQUIRE(aligned(query, 16) && aligned(keys, 16) && aligned(values, 16) && aligned(out, 16),
             "mem_decode_read: tensors must be 16-byte aligned");
  MemReadArgs a{query, keys, values, positions, indices, out, B, H, G, CAP, D, kv_stride0, pos_stride0, dtype,
                static_cast<cudaStream_t>(stream)};
  return launch_mem_decode_read(a);
}

int yb_mem_decode_commit(const void *key, const void *value, const float *scores, const uint8_t *active, int64_t chunk,
                         void *keys, void *values, float *bank_scores, int32_t *positions, void *pending_keys,
                         void *pending_values, float *pending_scores, int64_t *count, int64_t *total,
                         const int64_t *indices, int64_t B, int64_t G, int64_t CAP, int64_t PC, int64_t D,
                         int64_t kv_stride0, int64_t meta_stride0, int64_t pkv_stride0, int64_t pmeta_stride0,
                         int64_t count_stride0, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "mem_decode_commit: bad dtype");
  YB_REQUIRE(B >= 0 && G > 0 && CAP > 0 && PC > 0 && D > 0, "mem_decode_commit: bad sizes");
  YB_REQUIRE(chunk >= 1 && chunk <= PC, "mem_decode_commit: chunk=%lld must be in [1, PC=%lld]", (long long)chunk,
             (long long)PC);
  YB_REQUIRE(key && value && scores && active && keys && values && bank_scores && positions && pending_keys &&
                 pending_values && pending_scores && count && total,
             "mem_decode_commit: null tensor");
  YB_REQUIRE(kv_stride0 >= G * CAP * D && meta_stride0 >= G * CAP && pkv_stride0 >= G * PC * D &&
                 pmeta_stride0 >= G * PC && count_stride0 >= 1,
             "mem_decode_commit: batch stride too small");
  MemCommitArgs a{key, value, scores, active, chunk, keys, values, bank_scores, positions, pending_keys,
                  pending_values, pending_scores, count, total, indices, B, G, CAP, PC, D, kv_stride0,
                  meta_stride0, pkv_stride0, pmeta_stride0, count_stride0, dtype, static_cast<cudaStream_t>(stream)};
  return launch_mem_decode_commit(a);
}

int yb_mem_decode_step(const void *query, void *out, const void *key, const void *value, const float *scores,
                       const uint8_t *active, int64_t chunk, void *keys, void *values, float *bank_scores,
                       int32_t *positions, void *pending_keys, void *pending_values, float *pending_scores,
                       int64_t *count, int64_t *total, const int64_t *indices, int32_t *arrive, int64_t B,
                       int64_t H, int64_t G, int64_t CAP, int64_t PC, int64_t D, int64_t kv_stride0,
                       int64_t meta_stride0, int64_t pkv_stride0, int64_t pmeta_stride0, int64_t count_stride0,
                       int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "mem_decode_step: bad dtype");
  YB_REQUIRE(B >= 0 && H > 0 && G > 0 && CAP > 0 && PC > 0 && D > 0 && H % G == 0, "mem_decode_step: bad sizes");
  YB_REQUIRE(chunk >= 1 && chunk <= PC, "mem_decode_step: chunk=%lld must be in [1, PC=%lld]", (long long)chunk,
             (long long)PC);
  YB_REQUIRE(query && out && key && value && scores && active && keys && values && bank_scores && positions &&
                 pending_keys && pending_values && pending_scores && count && total && arrive,
             "mem_decode_step: null tensor");
  YB_REQUIRE(kv_stride0 >= G * CAP * D && meta_stride0 >= G * CAP && pkv_stride0 >= G * PC * D &&
                 pmeta_stride0 >= G * PC && count_stride0 >= 1,
             "mem_decode_step: batch stride too small");
  YB_REQUIRE((kv_stride0 * dtype_size(dtype)) % 16 == 0, "mem_decode_step: key batch stride must be 16-byte multiple");
  YB_REQUIRE(aligned(query, 16) && aligned(keys, 16) && aligned(values, 16) && aligned(out, 16),
             "mem_decode_step: tensors must be 16-byte aligned");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  MemReadArgs r{query, keys, values, positions, indices, out, B, H, G, CAP, D, kv_stride0, meta_stride0, dtype, st};
  MemCommitArgs c{key, value, scores, active, chunk, keys, values, bank_scores, positions, pending_keys,
                  pending_values, pending_scores, count, total, indices, B, G, CAP, PC, D, kv_stride0,
                  meta_stride0, pkv_stride0, pmeta_stride0, count_stride0, dtype, st};
  return launch_mem_decode_step(r, c, arrive);
}

int yb_mem_indexed_read(const void *query, const void *key, const void *value, const int64_t *references, void *out,
                        int64_t B, int64_t blocks, int64_t chunk, int64_t H, int64_t G, int64_t D, int64_t S,
                        int64_t KB, int64_t CAP, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "mem_indexed_read: bad dtype");
  YB_REQUIRE(B >= 0 && blocks >= 0 && chunk > 0 && H > 0 && G > 0 && D > 0 && S >= 0 && CAP > 0 && H % G == 0,
             "mem_indexed_read: bad sizes");
  YB_REQUIRE(KB == 1 || KB == B, "mem_indexed_read: key batch must be 1 or B");
  YB_REQUIRE(query && key && value && references && out, "mem_indexed_read: null tensor");
  YB_REQUIRE(aligned(query, 16) && aligned(key, 16) && aligned(value, 16) && aligned(out, 16),
             "mem_indexed_read: tensors must be 16-byte aligned");
  MemIndexedArgs a{query, key, value, references, out, B, blocks, chunk, H, G, D, S, KB, CAP, dtype,
                   static_cast<cudaStream_t>(stream)};
  return launch_mem_indexed_read(a);
}

int yb_mem_indexed_read_timeline(const void *query, const void *key, const void *value, const void *key_new,
                                 const void *value_new, const int64_t *references, void *out, int64_t B, int64_t T,
                                 int64_t blocks, int64_t chunk, int64_t H, int64_t G, int64_t D, int64_t S,
                                 int64_t S_new, int64_t KB, int64_t CAP, const int64_t *token_shift,
                                 const int64_t *write_lo, const int64_t *write_hi, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "mem_indexed_read_timeline: bad dtype");
  YB_REQUIRE(B >= 0 && T >= 0 && blocks >= 0 && chunk > 0 && H > 0 && G > 0 && D > 0 && S >= 0 && S_new >= 0 &&
                 CAP > 0 && H % G == 0 && blocks * chunk < 0x7fffffffLL && T < 0x7fffffffLL,
             "mem_indexed_read_timeline: bad sizes");
  YB_REQUIRE(KB == 1 || KB == B, "mem_indexed_read_timeline: key batch must be 1 or B");
  YB_REQUIRE(query && key && value && references && out && token_shift && write_lo && write_hi,
             "mem_indexed_read_timeline: null tensor");
  YB_REQUIRE(S_new == 0 || (key_new && value_new && KB == 1),
             "mem_indexed_read_timeline: a second source needs both tensors and key batch 1");
  YB_REQUIRE(aligned(query, 16) && aligned(key, 16) && aligned(value, 16) && aligned(out, 16) &&
                 (S_new == 0 || (aligned(key_new, 16) && aligned(value_new, 16))),
             "mem_indexed_read_timeline: tensors must be 16-byte aligned");
  MemIndexedArgs a{query, key, value, references, out, B, blocks, chunk, H, G, D, S, KB, CAP, dtype,
                   static_cast<cudaStream_t>(stream)};
  a.tok_shift = token_shift;
  a.w_lo = write_lo;
  a.w_hi = write_hi;
  a.T = T;
  if (S_new > 0) {
    a.key2 = key_new;
    a.value2 = value_new;
    a.S2 = S_new;
  }
  return launch_mem_indexed_read(a);
}

int yb_gdn_decode_fused(const void *mixed, int64_t mixed_tok_stride, const void *z, int64_t z_tok_stride,
                        const void *a, const void *b, int64_t ab_tok_stride, void *conv_state,
                        int64_t conv_batch_stride, int64_t conv_width, const float *conv_weight,
                        const float *conv_bias, int64_t conv_ks, void *state, int state_dtype,
                        const float *A_log, const float *dt_bias, const void *norm_weight, float norm_eps,
                        void *o, int64_t N, int64_t T, int64_t H, int64_t HV, int64_t K, int64_t V, float scale,
                        int io_dtype, uint32_t flags, void *stream) {
  YB_REQUIRE(io_dtype == YB_BF16 || io_dtype == YB_F16, "gdn_decode_fused: activations must be bf16 or fp16");
  YB_REQUIRE(state_dtype == YB_F32 || state_dtype == YB_BF16 || state_dtype == YB_F16,
             "gdn_decode_fused: bad state dtype");
  YB_REQUIRE(N >= 0 && T >= 0 && H > 0 && HV > 0 && HV % H == 0 && K > 0 && V > 0, "gdn_decode_fused: bad sizes");
  YB_REQUIRE(!(flags & ~uint32_t(YB_GDN_TRANSPOSE_STATE)), "gdn_decode_fused: only YB_GDN_TRANSPOSE_STATE may be set");
  const int64_t C = 2 * H * K + HV * V;
  YB_REQUIRE(mixed_tok_stride >= C && z_tok_stride >= HV * V && ab_tok_stride >= HV,
             "gdn_decode_fused: token strides too small");
  YB_REQUIRE(N == 0 || conv_batch_stride >= C * conv_width, "gdn_decode_fused: conv state batch stride too small");
  YB_REQUIRE(N * T == 0 || (mixed && z && a && b && conv_state && conv_weight && state && A_log && norm_weight && o),
             "gdn_decode_fused: null tensor");
  YB_REQUIRE(aligned(mixed, 16) && aligned(z, 16) && aligned(conv_state, 16) && aligned(conv_weight, 16) &&
                 aligned(state, 16) && aligned(o, 16) && aligned(norm_weight, 16),
             "gdn_decode_fused: tensors must be 16-byte aligned");
  YB_REQUIRE((mixed_tok_stride * dtype_size(io_dtype)) % 16 == 0 && (z_tok_stride * dtype_size(io_dtype)) % 16 == 0,
             "gdn_decode_fused: token strides must be multiples of 16 bytes");
  FusedArgs f{};
  f.mixed = mixed; f.mixed_ts = mixed_tok_stride; f.z = z; f.z_ts = z_tok_stride; f.a = a; f.b = b;
  f.ab_ts = ab_tok_stride; f.conv_state = conv_state; f.conv_bs = conv_batch_stride; f.conv_width = conv_width;
  f.conv_ks = conv_ks; f.conv_w = conv_weight; f.conv_b = conv_bias; f.state = state; f.state_dtype = state_dtype;
  f.trans = flags & YB_GDN_TRANSPOSE_STATE; f.A_log = A_log; f.dt_bias = dt_bias; f.norm_w = norm_weight;
  f.norm_eps = norm_eps; f.scale = scale; f.o = o; f.N = N; f.T = T; f.H = H; f.HV = HV; f.K = K; f.V = V;
  f.io_dtype = io_dtype; f.stream = static_cast<cudaStream_t>(stream);
  return launch_gdn_decode_fused(f);
}

int yb_swa_ring_write(const void *key, const void *value, int64_t kv_batch_stride, int64_t kv_head_stride,
                      const uint8_t *valid, void *ring_key, void *ring_value, int64_t ring_batch_stride,
                      int64_t ring_head_stride, uint8_t *ring_valid, int64_t ring_valid_batch_stride,
                      void *ring_index, int index_dtype, int64_t B, int64_t KVH, int64_t W, int64_t D, int dtype,
                      void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "swa_ring_write: bad dtype");
  YB_REQUIRE(index_dtype == YB_I32 || index_dtype == YB_I64, "swa_ring_write: the index must be int32 or int64");
  YB_REQUIRE(B >= 0 && KVH > 0 && W > 0 && (D == 32 || D == 64 || D == 128 || D == 256),
             "swa_ring_write: bad sizes (D in 32/64/128/256)");
  YB_REQUIRE(B == 0 || (key && value && valid && ring_key && ring_value && ring_valid && ring_index),
             "swa_ring_write: null tensor");
  YB_REQUIRE(ring_head_stride >= W * D && (B <= 1 || ring_batch_stride >= KVH * ring_head_stride) &&
                 kv_head_stride >= D && (B <= 1 || kv_batch_stride >= KVH * kv_head_stride) &&
                 (B <= 1 || ring_valid_batch_stride >= W),
             "swa_ring_write: strides too small");
  YB_REQUIRE(aligned(key, 16) && aligned(value, 16) && aligned(ring_key, 16) && aligned(ring_value, 16) &&
                 ((kv_batch_stride | kv_head_stride | ring_batch_stride | ring_head_stride) * dtype_size(dtype)) % 16 == 0,
             "swa_ring_write: tensors and strides must be 16-byte aligned");
  SwaArgs a{};
  a.new_k = key; a.new_v = value; a.new_bs = kv_batch_stride; a.new_hs = kv_head_stride; a.new_valid = valid;
  a.ring_k = ring_key; a.ring_v = ring_value; a.ring_bs = ring_batch_stride; a.ring_hs = ring_head_stride;
  a.ring_valid = ring_valid; a.valid_bs = ring_valid_batch_stride; a.ring_index = ring_index;
  a.index_i64 = index_dtype == YB_I64;
  a.B = B; a.KVH = KVH; a.W = W; a.D = D; a.dtype = dtype; a.stream = static_cast<cudaStream_t>(stream);
  return launch_swa_ring_write(a);
}

int64_t yb_swa_decode_workspace_bytes(int64_t B, int64_t KVH, int64_t QH, int64_t W, int64_t D) {
  return swa_workspace_bytes(B, KVH, QH, W, D);
}

int yb_swa_decode_attention(const void *query, const void *ring_key, const void *ring_value,
                            int64_t ring_batch_stride, int64_t ring_head_stride, const uint8_t *valid,
                            int64_t valid_batch_stride, void *out, int64_t B, int64_t QH, int64_t KVH, int64_t W,
                            int64_t D, int dtype, void *workspace, int64_t workspace_bytes, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "swa_decode_attention: bad dtype");
  YB_REQUIRE(B >= 0 && KVH > 0 && QH % KVH == 0 && W > 0 && D > 0, "swa_decode_attention: bad sizes");
  YB_REQUIRE(B == 0 || (query && ring_key && ring_value && valid && out), "swa_decode_attention: null tensor");
  YB_REQUIRE(ring_head_stride >= W * D && (B <= 1 || ring_batch_stride >= KVH * ring_head_stride) &&
                 (B <= 1 || valid_batch_stride >= W),
             "swa_decode_attention: strides too small");
  YB_REQUIRE(aligned(query, 16) && aligned(ring_key, 16) && aligned(ring_value, 16) && aligned(out, 16) &&
                 ((ring_batch_stride | ring_head_stride) * dtype_size(dtype)) % 16 == 0,
             "swa_decode_attention: tensors and strides must be 16-byte aligned");
  const int64_t need = swa_workspace_bytes(B, KVH, QH, W, D);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(YB_ERR_WORKSPACE, "swa_decode_attention: workspace of %lld bytes required", (long long)need);
  SwaArgs a{};
  a.query = query; a.ring_k = const_cast<void *>(ring_key); a.ring_v = const_cast<void *>(ring_value);
  a.ring_bs = ring_batch_stride; a.ring_hs = ring_head_stride; a.ring_valid = const_cast<uint8_t *>(valid);
  a.valid_bs = valid_batch_stride; a.out = out; a.B = B; a.QH = QH; a.KVH = KVH; a.W = W; a.D = D;
  a.dtype = dtype; a.stream = static_cast<cudaStream_t>(stream);
  return launch_swa_decode_attention(a, workspace);
}

int yb_conv1d_update(const void *x, int64_t x_batch_stride, void *conv_state, int64_t state_batch_stride,
                     int64_t state_channel_stride, int64_t state_tap_stride, int64_t state_width,
                     const float *weight, const float *bias, void *out, int64_t out_batch_stride, int64_t B,
                     int64_t C, int64_t KS, int silu, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "conv1d_update: bad dtype");
  YB_REQUIRE(B >= 0 && C >= 0 && KS >= 2 && KS <= 8 && (state_width == KS || state_width == KS - 1),
             "conv1d_update: bad sizes (state width must be KS or KS - 1)");
  YB_REQUIRE(state_channel_stride >= 1 && state_tap_stride >= 1 &&
             (state_channel_stride >= state_width * state_tap_stride || state_tap_stride >= C * state_channel_stride),
             "conv1d_update: state channel / tap strides overlap");
  YB_REQUIRE(B <= 1 || (x_batch_stride >= C && out_batch_stride >= C && state_batch_stride >= C * state_width),
             "conv1d_update: batch strides too small");   // (a size-1 axis may carry any stride)
  YB_REQUIRE(B * C == 0 || (x && conv_state && weight && out), "conv1d_update: null tensor");
  ConvArgs a{};
  a.x = x; a.x_bs = x_batch_stride; a.x_ts = 0;
  a.state = conv_state; a.state_bs = state_batch_stride; a.W = state_width;
  a.state_cs = state_channel_stride; a.state_ts = state_tap_stride;
  a.weight = weight; a.bias = bias; a.out = out; a.out_bs = out_batch_stride; a.out_ts = 0;
  a.B = B; a.T = 1; a.C = C; a.KS = KS; a.silu = silu != 0; a.dtype = dtype;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_conv1d(a, true);
}

int yb_conv1d_fwd(const void *x, int64_t x_batch_stride, int64_t x_token_stride, const void *initial_state,
                  void *final_state, int64_t state_batch_stride, int64_t state_channel_stride,
                  int64_t state_tap_stride, int64_t state_width, const float *weight, const float *bias, void *out,
                  int64_t out_batch_stride, int64_t out_token_stride, int64_t B, int64_t T, int64_t C, int64_t KS,
                  int silu, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "conv1d_fwd: bad dtype");
  YB_REQUIRE(B >= 0 && T >= 0 && C >= 0 && KS >= 2 && KS <= 8 && (state_width == KS || state_width == KS - 1),
             "conv1d_fwd: bad sizes (state width must be KS or KS - 1)");
  YB_REQUIRE(state_channel_stride >= 1 && state_tap_stride >= 1 &&
             (state_channel_stride >= state_width * state_tap_stride || state_tap_stride >= C * state_channel_stride),
             "conv1d_fwd: state channel / tap strides overlap");
  YB_REQUIRE(T <= 1 || (x_token_stride >= C && out_token_stride >= C), "conv1d_fwd: token strides too small");
  YB_REQUIRE(B <= 1 || (!initial_state && !final_state) || state_batch_stride >= C * state_width,
             "conv1d_fwd: state batch stride too small");
  YB_REQUIRE(B * C * T == 0 || (x && weight && out), "conv1d_fwd: null tensor");
  ConvArgs a{};
  a.x = x; a.x_bs = x_batch_stride; a.x_ts = x_token_stride;
  a.state_in = initial_state; a.state_out = final_state; a.state_bs = state_batch_stride; a.W = state_width;
  a.state_cs = state_channel_stride; a.state_ts = state_tap_stride;
  a.weight = weight; a.bias = bias; a.out = out; a.out_bs = out_batch_stride; a.out_ts = out_token_stride;
  a.B = B; a.T = T; a.C = C; a.KS = KS; a.silu = silu != 0; a.dtype = dtype;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_conv1d(a, false);
}

static bool pos_dtype_ok(int d) { return d == YB_I32 || d == YB_I64; }

int yb_mem_select_topk(const float *scores, const void *positions, int positions_dtype, const int64_t *references,
                       int64_t rows, int64_t n, int64_t capacity, float *out_scores, int64_t *out_positions,
                       int64_t *out_references, void *stream) {
  YB_REQUIRE(pos_dtype_ok(positions_dtype), "select_topk: positions must be YB_I32 or YB_I64");
  YB_REQUIRE(rows >= 0 && n >= 0 && capacity >= 0 && rows <= 0x7fffffffLL, "select_topk: bad sizes");
  YB_REQUIRE(rows * n == 0 || (scores && positions && references), "select_topk: null input");
  YB_REQUIRE(rows * capacity == 0 || (out_scores && out_positions && out_references), "select_topk: null output");
  TopkArgs a{scores, positions, references, positions_dtype, rows, n, capacity, out_scores, out_positions,
             out_references, static_cast<cudaStream_t>(stream)};
  return launch_select_topk(a);
}

int yb_mem_exclusive_prefix_topk(const float *scores, const void *positions, int positions_dtype,
                                 const int64_t *references, int64_t B, int64_t blocks, int64_t G, int64_t chunk,
                                 int64_t capacity, const float *initial_scores, const void *initial_positions,
                                 int initial_positions_dtype, const int64_t *initial_references,
                                 float *out_scores, int64_t *out_positions, int64_t *out_references,
                                 void *stream) {
  YB_REQUIRE(pos_dtype_ok(positions_dtype), "exclusive_prefix_topk: positions must be YB_I32 or YB_I64");
  YB_REQUIRE(B >= 0 && blocks >= 0 && G > 0 && chunk >= 0 && capacity >= 0 && B * G <= 0x7fffffffLL &&
                 B * blocks * G <= 0x7fffffffLL,
             "exclusive_prefix_topk: bad sizes");
  YB_REQUIRE(B * blocks * chunk == 0 || (scores && positions && references), "exclusive_prefix_topk: null input");
  YB_REQUIRE(B * capacity == 0 || (out_scores && out_positions && out_references),
             "exclusive_prefix_topk: null output");
  YB_REQUIRE(!initial_scores || (initial_positions && pos_dtype_ok(initial_positions_dtype)),
             "exclusive_prefix_topk: initial bank needs positions (YB_I32 or YB_I64)");
  PrefixTopkArgs a{scores, positions, references, positions_dtype, B, blocks, G, chunk, capacity,
                   initial_scores, initial_positions, initial_references, initial_positions_dtype,
                   out_scores, out_positions, out_references, static_cast<cudaStream_t>(stream)};
  return launch_exclusive_prefix_topk(a);
}

static bool glue_sizes_ok(int64_t B, int64_t G, int64_t chunk, int64_t extent, int64_t cap) {
  return B >= 0 && G > 0 && chunk > 0 && extent >= 0 && extent % chunk == 0 && cap > 0 && B * extent < (1LL << 40);
}

int yb_mem_prefill_timeline(const float *scores, const int64_t *order, const int64_t *n_new, const int64_t *count,
                            const int64_t *total, int64_t count_stride0, const float *pending_scores,
                            int64_t pmeta_stride0, int64_t B, int64_t T, int64_t G, int64_t chunk, int64_t extent,
                            int64_t shift, int64_t PC, int64_t *snapshot, float *slot_scores,
                            int64_t *slot_positions, int64_t *slot_references, int64_t *slot_tokens, void *stream) {
  YB_REQUIRE(glue_sizes_ok(B, G, chunk, extent, 1) && T > 0 && shift >= 0 && PC >= 0,
             "mem_prefill_timeline: bad sizes");
  YB_REQUIRE(scores && snapshot && slot_scores && slot_positions && slot_references && slot_tokens,
             "mem_prefill_timeline: null tensor");
  YB_REQUIRE(shift == 0 || (count && total && pending_scores && PC >= chunk),
             "mem_prefill_timeline: a state needs its counters and pending scores");
  PrefillGlueArgs a;
  a.B = B; a.T = T; a.G = G; a.chunk = chunk; a.extent = extent; a.blocks = extent / chunk; a.shift = shift;
  a.PC = PC; a.has_state = shift > 0;
  a.count = count; a.total = total; a.count_s0 = count_stride0;
  a.pend_scores = pending_scores; a.pmeta_s0 = pmeta_stride0;
  a.order = order; a.n_new = n_new; a.scores = scores; a.snap = snapshot;
  a.s_blk = slot_scores; a.pos_blk = slot_positions; a.ref_blk = slot_references; a.tok = slot_tokens;
  a.stream = static_cast<cudaStream_t>(stream);
  if (B * extent == 0) return YB_OK;
  return launch_prefill_glue(a, 0);
}

int yb_mem_prefill_table(const int64_t *prefix_references, const int64_t *snapshot, int64_t B, int64_t G,
                         int64_t chunk, int64_t extent, int64_t capacity, int has_state, int capture_safe,
                         uint8_t *needed, int64_t *table, int64_t *read_references, void *stream) {
  YB_REQUIRE(glue_sizes_ok(B, G, chunk, extent, capacity), "mem_prefill_table: bad sizes");
  YB_REQUIRE(prefix_references && snapshot && needed && table, "mem_prefill_table: null tensor");
  YB_REQUIRE(!capture_safe || read_references, "mem_prefill_table: capture_safe computes the read references");
  PrefillGlueArgs a;
  a.B = B; a.G = G; a.chunk = chunk; a.extent = extent; a.blocks = extent / chunk; a.cap = capacity;
  a.has_state = has_state != 0; a.shift = has_state ? capacity : 0; a.capture_safe = capture_safe != 0;
  a.pre_r = prefix_references; a.snap = const_cast<int64_t *>(snapshot); a.needed = needed; a.table = table;
  a.read_refs = read_references;
  a.stream = static_cast<cudaStream_t>(stream);
  if (B * extent == 0) return YB_OK;
  int rc = launch_prefill_glue(a, 1);
  if (!rc && capture_safe) rc = launch_prefill_glue(a, 2);
  return rc;
}

int yb_mem_prefill_read_references(const int64_t *prefix_references, const int64_t *table, int64_t B, int64_t G,
                                   int64_t chunk, int64_t extent, int64_t capacity, int has_state,
                                   int64_t *read_references, void *stream) {
  YB_REQUIRE(glue_sizes_ok(B, G, chunk, extent, capacity), "mem_prefill_read_references: bad sizes");
  YB_REQUIRE(prefix_references && table && read_references, "mem_prefill_read_references: null tensor");
  PrefillGlueArgs a;
  a.B = B; a.G = G; a.chunk = chunk; a.extent = extent; a.blocks = extent / chunk; a.cap = capacity;
  a.has_state = has_state != 0; a.shift = has_state ? capacity : 0;
  a.pre_r = prefix_references; a.table = const_cast<int64_t *>(table); a.read_refs = read_references;
  a.stream = static_cast<cudaStream_t>(stream);
  if (B * extent == 0) return YB_OK;
  return launch_prefill_glue(a, 2);
}

int yb_mem_prefill_state(const float *prefix_scores, const int64_t *prefix_positions,
                         const int64_t *prefix_references, const int64_t *table, const int64_t *snapshot,
                         const float *slot_scores, const void *old_keys, const void *old_values, const void *new_keys,
                         const void *new_values, void *keys, void *values, int64_t kv_stride0, float *bank_scores,
                         int32_t *positions, int64_t meta_stride0, void *pending_keys, void *pending_values,
                         int64_t pkv_stride0, float *pending_scores, int64_t pmeta_stride0, int64_t *count,
                         int64_t *total, int64_t count_stride0, int64_t B, int64_t G, int64_t chunk, int64_t extent,
                         int64_t capacity, int64_t PC, int64_t D, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "mem_prefill_state: bad dtype");
  const int64_t vec = 16 / (dtype == YB_F32 ? 4 : 2);
  YB_REQUIRE(glue_sizes_ok(B, G, chunk, extent, capacity) && PC >= chunk && D > 0 && D % vec == 0,
             "mem_prefill_state: bad sizes");
  YB_REQUIRE(prefix_scores && prefix_positions && prefix_references && table && snapshot && slot_scores &&
                 old_keys && old_values && keys && values && bank_scores && positions && pending_keys &&
                 pending_values && pending_scores && count && total,
             "mem_prefill_state: null tensor");
  YB_REQUIRE(aligned(old_keys, 16) && aligned(old_values, 16) && aligned(keys, 16) && aligned(values, 16) &&
                 aligned(pending_keys, 16) && aligned(pending_values, 16) &&
                 (!new_keys || (aligned(new_keys, 16) && aligned(new_values, 16))) && kv_stride0 % vec == 0 &&
                 pkv_stride0 % vec == 0,
             "mem_prefill_state: rows must be 16-byte aligned");
  PrefillGlueArgs a;
  a.B = B; a.G = G; a.chunk = chunk; a.extent = extent; a.blocks = extent / chunk; a.cap = capacity; a.PC = PC;
  a.D = D; a.dtype = dtype; a.has_state = 1; a.shift = capacity;
  a.pre_s = prefix_scores; a.pre_p = prefix_positions; a.pre_r = prefix_references;
  a.table = const_cast<int64_t *>(table); a.snap = const_cast<int64_t *>(snapshot);
  a.s_blk = const_cast<float *>(slot_scores);
  a.old_k = old_keys; a.old_v = old_values; a.new_k = new_keys; a.new_v = new_values;
  a.keys = keys; a.values = values; a.kv_s0 = kv_stride0;
  a.bank_scores = bank_scores; a.positions = positions; a.meta_s0 = meta_stride0;
  a.pkeys = pending_keys; a.pvalues = pending_values; a.pkv_s0 = pkv_stride0;
  a.pscores = pending_scores; a.pmeta_s0 = pmeta_stride0;
  a.count_out = count; a.total_out = total; a.count_s0 = count_stride0;
  a.stream = static_cast<cudaStream_t>(stream);
  if (B == 0) return YB_OK;
  return launch_prefill_glue(a, 3);
}

int64_t yb_sample_workspace_bytes(int64_t B, int64_t vocab, int64_t top_k) {
  return sample_workspace_bytes(B, vocab, top_k);
}

int yb_sample_greedy_noalloc(const void *scores, int64_t row_stride, int64_t B, int64_t vocab, int dtype,
                             int64_t *out, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "sample_greedy_noalloc: bad dtype");
  YB_REQUIRE(B >= 0 && vocab > 0 && row_stride >= vocab, "sample_greedy_noalloc: bad sizes");
  YB_REQUIRE(B == 0 || (scores && out), "sample_greedy_noalloc: null tensor");
  SampleArgs a{};
  a.scores = scores; a.row_stride = row_stride; a.B = B; a.vocab = vocab; a.dtype = dtype; a.out = out;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_sample_greedy_noalloc(a);
}

int yb_sample_greedy(const void *scores, int64_t row_stride, int64_t B, int64_t vocab, int dtype, int64_t *out,
                     void *workspace, int64_t workspace_bytes, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "sample_greedy: bad dtype");
  YB_REQUIRE(B >= 0 && vocab > 0 && row_stride >= vocab, "sample_greedy: bad sizes");
  YB_REQUIRE(scores && out, "sample_greedy: null tensor");
  const int64_t need = sample_workspace_bytes(B, vocab, 1);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(YB_ERR_WORKSPACE, "sample_greedy: workspace of %lld bytes required", (long long)need);
  SampleArgs a{};
  a.scores = scores; a.row_stride = row_stride; a.B = B; a.vocab = vocab; a.dtype = dtype; a.out = out;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.stream = static_cast<cudaStream_t>(stream);
  return launch_sample_greedy(a);
}

int yb_sample_top_k_top_p_counter(const void *scores, int64_t row_stride, int64_t B, int64_t vocab, int dtype,
                                  const int64_t *attempt_ids, const int64_t *steps, int64_t scalar_step, int64_t seed,
                                  int64_t stream_id, float temperature, int64_t top_k, float top_p, int64_t *out,
                                  void *workspace, int64_t workspace_bytes, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "sample_top_k_top_p_counter: bad dtype");
  YB_REQUIRE(B >= 0 && vocab > 0 && row_stride >= vocab, "sample_top_k_top_p_counter: bad sizes");
  YB_REQUIRE(scores && out && attempt_ids, "sample_top_k_top_p_counter: null tensor");
  YB_REQUIRE(temperature > 0.f && top_p > 0.f && top_p <= 1.f, "invalid top-k/top-p sampling parameters");
  YB_REQUIRE(top_k <= vocab, "top-k exceeds the vocabulary");
  SampleArgs a{};
  a.scores = scores; a.row_stride = row_stride; a.B = B; a.vocab = vocab; a.dtype = dtype;
  a.attempt_ids = attempt_ids; a.steps = steps; a.scalar_step = scalar_step; a.seed = seed; a.stream_id = stream_id;
  a.temperature = temperature; a.top_k = top_k; a.top_p = top_p; a.out = out;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.stream = static_cast<cudaStream_t>(stream);
  if (top_k == 1) {
    const int64_t need = sample_workspace_bytes(B, vocab, 1);
    if (workspace == nullptr || workspace_bytes < need)
      return set_error(YB_ERR_WORKSPACE, "sample: workspace of %lld bytes required", (long long)need);
    return launch_sample_greedy(a);
  }
  if (top_k <= 0) {
    const int64_t need = sample_workspace_bytes(B, vocab, top_k);
    if (workspace == nullptr || workspace_bytes < need)
      return set_error(YB_ERR_WORKSPACE, "sample: workspace of %lld bytes required", (long long)need);
    // the whole vocabulary in index order (top_p = 1), or its sorted nucleus
    return top_p == 1.0f ? launch_sample_cdf(a) : launch_sample_nucleus(a);
  }
  const int64_t need = sample_workspace_bytes(B, vocab, top_k);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(YB_ERR_WORKSPACE, "sample: workspace of %lld bytes required", (long long)need);
  return launch_sample_topk_topp(a);
}

int yb_presence_penalty(void *scores, const uint8_t *seen, int64_t n, float penalty, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "presence_penalty: bad dtype");
  YB_REQUIRE(n >= 0 && (n == 0 || (scores && seen)), "presence_penalty: bad arguments");
  return launch_presence_penalty(scores, seen, n, penalty, dtype, static_cast<cudaStream_t>(stream));
}

int yb_decode_state_update(const int64_t *sampled_token, int64_t sampled_stride, void *storage, int storage_dtype,
                           int64_t storage_rows, int64_t storage_cols, int64_t storage_stride, uint8_t *dense_seen,
                           int64_t seen_stride, int64_t vocab, int64_t *generated_lengths, uint8_t *finished_by_eos,
                           uint8_t *finished, const int64_t *slot_rows, const int64_t *sink_rows,
                           const int64_t *slot_caps, int64_t *row_steps, int64_t *row_positions, int64_t *decode_ids,
                           int64_t decode_ids_stride, int64_t *useful_events, int64_t slots,
                           int64_t maximum_new_tokens, int64_t pad_token, const int64_t *eos_tokens, int eos_count,
                           void *stream) {
  YB_REQUIRE(slots >= 0 && storage_rows >= 0 && storage_cols >= 0 && vocab >= 0, "decode state: negative size");
  YB_REQUIRE(storage_dtype == YB_I32 || storage_dtype == YB_I64, "decode state: storage must be int32 or int64");
  YB_REQUIRE(storage_stride >= storage_cols && seen_stride >= vocab, "decode state: row strides too small");
  YB_REQUIRE(eos_count >= 0 && (eos_count == 0 || eos_tokens), "decode state: bad EOS list");
  YB_REQUIRE(slots == 0 || (sampled_token && storage && dense_seen && generated_lengths && finished_by_eos &&
                            finished && slot_rows && sink_rows && slot_caps && row_steps && row_positions &&
                            decode_ids && useful_events),
             "decode state: null pointer");
  if (eos_count > kMaxEos)
    return set_error(YB_ERR_UNSUPPORTED, "decode state: %d EOS ids (at most %d)", eos_count, kMaxEos);
  DecodeStateArgs a{};
  a.sampled = sampled_token; a.sampled_stride = sampled_stride;
  a.storage = storage; a.storage_i64 = storage_dtype == YB_I64;
  a.storage_rows = storage_rows; a.storage_cols = storage_cols; a.storage_stride = storage_stride;
  a.dense_seen = dense_seen; a.seen_stride = seen_stride; a.vocab = vocab;
  a.generated_lengths = generated_lengths; a.finished_by_eos = finished_by_eos; a.finished = finished;
  a.slot_rows = slot_rows; a.sink_rows = sink_rows; a.slot_caps = slot_caps;
  a.row_steps = row_steps; a.row_positions = row_positions;
  a.decode_ids = decode_ids; a.decode_ids_stride = decode_ids_stride; a.useful_events = useful_events;
  a.slots = slots; a.max_new = maximum_new_tokens; a.pad = pad_token;
  for (int e = 0; e < eos_count; ++e) a.eos[e] = eos_tokens[e];
  a.eos_count = eos_count;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_decode_state_update(a);
}

int yb_swa_prefill_attention(const void *q, const void *k, const void *v, const uint8_t *key_valid,
                             int64_t valid_batch_stride, void *out, int64_t B, int64_t Tq, int64_t Tk, int64_t QH,
                             int64_t KVH, int64_t D, int64_t window, int64_t query_start, int dtype, void *stream) {
  YB_REQUIRE(dtype_ok(dtype), "swa_prefill: bad dtype");
  YB_REQUIRE(B >= 0 && Tq >= 0 && Tk >= 0 && QH > 0 && KVH > 0 && QH % KVH == 0 && window >= 1 && query_start >= 0,
             "swa_prefill: bad sizes");
  YB_REQUIRE(B * Tq == 0 || (q && k && v && out), "swa_prefill: null tensor");
  YB_REQUIRE(key_valid == nullptr || B <= 1 || valid_batch_stride >= Tk, "swa_prefill: key_valid stride too small");
  SwaPrefillArgs a{};
  a.q = q; a.k = k; a.v = v; a.key_valid = key_valid; a.valid_bs = valid_batch_stride; a.out = out;
  a.B = B; a.Tq = Tq; a.Tk = Tk; a.QH = QH; a.KVH = KVH; a.D = D; a.window = window; a.query_start = query_start;
  a.dtype = dtype; a.stream = static_cast<cudaStream_t>(stream);
  return launch_swa_prefill_tc(a);
}

}  // extern "C"
