// Fused per-token gated delta rule (decode).  One CTA owns one (sequence,
// value head) pair and keeps that head's fp32 state in registers for all of
// the sequence's tokens, so the state crosses HBM exactly once in and once
// out.  Per token it fuses: q/k L2 norm, the GDN gates (optional), the state
// decay, the delta-rule update, the output read and (optionally) the gated
// RMSNorm epilogue.
//
// Algorithm (transformers qwen3_5 modeling_qwen3_5.py:314-353, fla
// fused_recurrent.py:28-170):
//   S <- exp(g) S;  d = beta (v - S^T k);  S <- S + k d^T;  o = scale S^T q
// Both reductions over the key axis are taken from the decayed state before
// the update: o = scale (S_dec^T q + d (k . q)), so the state is read once.
//
// Thread layout: the state tile is ROWS x COLS with COLS the contiguous axis
// of the stored layout (V for [K,V], K for [V,K]).  Each thread owns 4
// contiguous columns (one 16- or 8-byte vector) of RPT consecutive rows; a
// warp covers whole rows, so every state access is fully coalesced.
//
// State storage: fp32, or bf16 / fp16 (the reference's reduced-precision
// recurrent-state storage for decode, runtime/model/inference_kernels.py:
// 437-457 and modeling_yanchor.py:733-750).  A 16-bit state is widened to
// fp32 on load, all arithmetic is fp32, and it is rounded to nearest on the
// final store — as fla's fused recurrent kernel does with a 16-bit h0 / ht.
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace yb {
namespace {

constexpr int kThreads = 256;

struct RecParams {
  const void *q, *k, *v;
  int64_t q_ts, k_ts, v_ts;
  const void *g, *beta;
  int64_t g_ts, beta_ts;
  int g_dtype, beta_dtype;
  const float *A_log, *dt_bias;
  const void *h0;
  void *ht;
  void *o;
  const void *z, *norm_w;
  float norm_eps;
  const int64_t *cu;
  int64_t T;
  int H, HV;
  float scale;
  uint32_t flags;
};

__device__ __forceinline__ float load_scalar(const void *p, int64_t idx, int dtype) {
  if (dtype == YB_F32) return static_cast<const float *>(p)[idx];
  if (dtype == YB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[idx]);
  return __half2float(static_cast<const __half *>(p)[idx]);
}

// four consecutive state values: streaming load / store in the storage type
__device__ __forceinline__ void ld_state4(const float *src, float *x) {
  const float4 v = __ldcs(reinterpret_cast<const float4 *>(src));
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <typename T16>
__device__ __forceinline__ void ld_state4(const T16 *src, float *x) {
  const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(src));
  const T16 *h = reinterpret_cast<const T16 *>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = to_f(h[j]);
}
__device__ __forceinline__ void st_state4(float *dst, const float *x) {
  __stcs(reinterpret_cast<float4 *>(dst), make_float4(x[0], x[1], x[2], x[3]));
}
template <typename T16>
__device__ __forceinline__ void st_state4(T16 *dst, const float *x) {
  uint2 v;
  T16 *h = reinterpret_cast<T16 *>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = from_f<T16>(x[j]);
  __stcs(reinterpret_cast<uint2 *>(dst), v);
}

template <typename TIO, typename TS, int K, int V, bool TRANS, bool NORM>
__global__ void __launch_bounds__(kThreads) gdn_recurrent_kernel(const RecParams p) {
  constexpr int ROWS = TRANS ? V : K;
  constexpr int COLS = TRANS ? K : V;
  constexpr int NCG = COLS / 4;       // column groups (threads per row)
  constexpr int RG = kThreads / NCG;  // row groups
  constexpr int RPT = ROWS / RG;      // rows per thread
  static_assert(NCG <= 32 && 32 % NCG == 0, "a row must fit in one warp");
  static_assert(ROWS % RG == 0, "rows must split evenly");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = tid % NCG, rg = tid / NCG, c0 = cg * 4;
  const int n = blockIdx.x / p.HV, hv = blockIdx.x % p.HV;
  const int h = hv / (p.HV / p.H);
  int64_t bos, len;
  if (p.cu) {
    bos = p.cu[n];
    len = p.cu[n + 1] - bos;
  } else {
    bos = int64_t(n) * p.T;
    len = p.T;
  }

  __shared__ __align__(16) float sq[K];
  __shared__ __align__(16) float sk[K];
  __shared__ __align__(16) float sv[V];
  __shared__ __align__(16) float so[V];
  __shared__ __align__(16) float red_k[TRANS ? 1 : RG][TRANS ? 4 : V];
  __shared__ __align__(16) float red_q[TRANS ? 1 : RG][TRANS ? 4 : V];
  __shared__ float s_decay, s_beta, s_kq;

  // State tile into registers (issued first: it is the long-latency stream).
  // Under a dependent launch it is only prefetched into L2 before the wait:
  // the previous kernel may be the one that wrote it.
  const int64_t head = (int64_t(n) * p.HV + hv) * K * V;
  if (p.h0) {
    const TS *src = static_cast<const TS *>(p.h0) + head;
#pragma unroll
    for (int i = 0; i < RPT; i += (sizeof(TS) == 4 ? 1 : 2)) prefetch_l2(src + (rg * RPT + i) * COLS + c0);
  }
  pdl_wait();
  pdl_release();
  float s[RPT][4];
  if (p.h0) {
    const TS *src = static_cast<const TS *>(p.h0) + head;
#pragma unroll
    for (int i = 0; i < RPT; ++i) ld_state4(src + (rg * RPT + i) * COLS + c0, s[i]);
  } else {
#pragma unroll
    for (int i = 0; i < RPT; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
  }

  const bool l2 = p.flags & YB_GDN_QK_L2NORM;
  const bool gate_in = p.flags & YB_GDN_GATE_IN_KERNEL;
  const bool beta_sig = p.flags & YB_GDN_BETA_SIGMOID;
  const TIO *qp = static_cast<const TIO *>(p.q);
  const TIO *kp = static_cast<const TIO *>(p.k);
  const TIO *vp = static_cast<const TIO *>(p.v);
  TIO *op = static_cast<TIO *>(p.o);

  for (int64_t t = 0; t < len; ++t) {
    const int64_t tok = bos + t;
    // ---- stage q, k (normalised, q scaled), v, decay, beta ----
    if (warp == 0) {
      float qv[4] = {0.f, 0.f, 0.f, 0.f}, kv[4] = {0.f, 0.f, 0.f, 0.f};
      if (lane < K / 4) {
        load4(qp + tok * p.q_ts + int64_t(h) * K + lane * 4, qv);
        load4(kp + tok * p.k_ts + int64_t(h) * K + lane * 4, kv);
      }
      float qn = 1.f, kn = 1.f;
      if (l2) {
        float qs2 = qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3];
        float ks2 = kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3];
        qn = rsqrtf(warp_sum(qs2) + 1e-6f);
        kn = rsqrtf(warp_sum(ks2) + 1e-6f);
      }
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qv[j] *= qn * p.scale;
        kv[j] *= kn;
        dot += qv[j] * kv[j];
      }
      dot = warp_sum(dot);
      if (lane < K / 4) {
        *reinterpret_cast<float4 *>(sq + lane * 4) = make_float4(qv[0], qv[1], qv[2], qv[3]);
        *reinterpret_cast<float4 *>(sk + lane * 4) = make_float4(kv[0], kv[1], kv[2], kv[3]);
      }
      if (lane == 0) s_kq = dot;
    } else if (warp == 1) {
      if (lane < V / 4) {
        float vv[4];
        load4(vp + tok * p.v_ts + int64_t(hv) * V + lane * 4, vv);
        *reinterpret_cast<float4 *>(sv + lane * 4) = make_float4(vv[0], vv[1], vv[2], vv[3]);
      }
      if (lane == 0) {
        float gl = load_scalar(p.g, tok * p.g_ts + hv, p.g_dtype);
        if (gate_in) gl = -expf(p.A_log[hv]) * softplus20(gl + (p.dt_bias ? p.dt_bias[hv] : 0.f));
        float b = load_scalar(p.beta, tok * p.beta_ts + hv, p.beta_dtype);
        s_decay = expf(gl);
        s_beta = beta_sig ? round_to<TIO>(sigmoidf_(b)) : b;   // sigmoid(b) in the input dtype, as the reference stores beta
      }
    }
    __syncthreads();
    const float dec = s_decay, bet = s_beta, kq = s_kq;

    if constexpr (!TRANS) {
      // rows = key index, cols = value index
      float ak[4] = {0.f, 0.f, 0.f, 0.f}, aq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float kr = sk[rg * RPT + i], qr = sq[rg * RPT + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] *= dec;
          ak[j] = fmaf(s[i][j], kr, ak[j]);
          aq[j] = fmaf(s[i][j], qr, aq[j]);
        }
      }
      *reinterpret_cast<float4 *>(&red_k[rg][c0]) = make_float4(ak[0], ak[1], ak[2], ak[3]);
      *reinterpret_cast<float4 *>(&red_q[rg][c0]) = make_float4(aq[0], aq[1], aq[2], aq[3]);
      __syncthreads();
      float kvs[4] = {0.f, 0.f, 0.f, 0.f}, qss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        float4 a = *reinterpret_cast<const float4 *>(&red_k[r][c0]);
        float4 b = *reinterpret_cast<const float4 *>(&red_q[r][c0]);
        kvs[0] += a.x; kvs[1] += a.y; kvs[2] += a.z; kvs[3] += a.w;
        qss[0] += b.x; qss[1] += b.y; qss[2] += b.z; qss[3] += b.w;
      }
      float delta[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) delta[j] = bet * (sv[c0 + j] - kvs[j]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float kr = sk[rg * RPT + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(kr, delta[j], s[i][j]);
      }
      if (rg == 0) {
        float ov[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) ov[j] = fmaf(delta[j], kq, qss[j]);
        *reinterpret_cast<float4 *>(so + c0) = make_float4(ov[0], ov[1], ov[2], ov[3]);
      }
    } else {
      // rows = value index, cols = key index (contiguous)
      float kc[4], qc[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kc[j] = sk[c0 + j];
        qc[j] = sq[c0 + j];
      }
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        float pk = 0.f, pq = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] *= dec;
          pk = fmaf(s[i][j], kc[j], pk);
          pq = fmaf(s[i][j], qc[j], pq);
        }
        pk = group_sum<NCG>(pk);
        pq = group_sum<NCG>(pq);
        const int r = rg * RPT + i;
        const float delta = bet * (sv[r] - pk);
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(kc[j], delta, s[i][j]);
        if (cg == 0) so[r] = fmaf(delta, kq, pq);
      }
    }
    __syncthreads();

    // ---- output (and the fused gated RMSNorm) by warp 0 ----
    if (warp == 0) {
      float ov[4] = {0.f, 0.f, 0.f, 0.f};
      if (lane < V / 4) {
        float4 x = *reinterpret_cast<const float4 *>(so + lane * 4);
        ov[0] = x.x; ov[1] = x.y; ov[2] = x.z; ov[3] = x.w;
      }
      TIO *dst = op + tok * int64_t(p.HV) * V + int64_t(hv) * V + lane * 4;
      if constexpr (NORM) {
        // Qwen3_5RMSNormGated on the io-dtype output, with its roundings.
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ov[j] = round_to<TIO>(ov[j]);
          ss += ov[j] * ov[j];
        }
        const float inv = rsqrtf(warp_sum(ss) / float(V) + p.norm_eps);
        if (lane < V / 4) {
          float zz[4], w[4];
          load4(static_cast<const TIO *>(p.z) + tok * int64_t(p.HV) * V + int64_t(hv) * V + lane * 4, zz);
          load4(static_cast<const TIO *>(p.norm_w) + lane * 4, w);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float y = round_to<TIO>(w[j] * round_to<TIO>(ov[j] * inv));
            ov[j] = y * (zz[j] * sigmoidf_(zz[j]));
          }
          store4(dst, ov);
        }
      } else {
        if (lane < V / 4) store4(dst, ov);
      }
    }
  }

  if (p.ht) {
    TS *dst = static_cast<TS *>(p.ht) + head;
#pragma unroll
    for (int i = 0; i < RPT; ++i) st_state4(dst + (rg * RPT + i) * COLS + c0, s[i]);
  }
}

// One token per sequence, row-major state: the state is staged in shared
// memory by four bulk copies (16 KB each for fp32, 8 KB for a 16-bit state)
// rather than held in registers, so three (fp32) or five (16-bit) CTAs share
// an SM and more bytes are in flight per SM than with register-resident
// CTAs; four copies instead of sixteen vector loads per thread.  The copies'
// wait is bounded: on timeout the CTA records ERR_REC_STATE, skips the
// update, and waits (bounded) for the copies before it exits.  The arithmetic
// is the generic kernel's, so the results are identical.
constexpr int ERR_REC_STATE = 0x601;
template <typename TS> __host__ __device__ constexpr uint32_t staged_bytes() { return 128u * 128u * uint32_t(sizeof(TS)); }
// 4 consecutive state values of the staged tile, widened to fp32
__device__ __forceinline__ void lds4(const float *p, float *x) {
  const float4 v = *reinterpret_cast<const float4 *>(p);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <typename T16>
__device__ __forceinline__ void lds4(const T16 *p, float *x) {
  const uint2 v = *reinterpret_cast<const uint2 *>(p);
  const T16 *e = reinterpret_cast<const T16 *>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = to_f(e[j]);
}

__device__ __forceinline__ void bulk_load_state(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(tc::smem_u32(dst)), "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
               : "memory");
}

template <typename TIO, typename TS, bool NORM>
__global__ void __launch_bounds__(kThreads, sizeof(TS) == 4 ? 3 : 5) gdn_recurrent_sst_kernel(const RecParams p) {
  constexpr int K = 128, V = 128, COLS = V, NCG = COLS / 4, RG = kThreads / NCG, RPT = K / RG;
  constexpr uint32_t kS32Bytes = staged_bytes<TS>();
  extern __shared__ __align__(128) unsigned char s32_dyn[];
  TS *st = reinterpret_cast<TS *>(s32_dyn);                          // [K][V]
  uint64_t *bar = reinterpret_cast<uint64_t *>(s32_dyn + kS32Bytes);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bar + 1);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = tid % NCG, rg = tid / NCG, c0 = cg * 4;
  const int n = blockIdx.x / p.HV, hv = blockIdx.x % p.HV;
  const int h = hv / (p.HV / p.H);
  const int64_t tok = int64_t(n) * p.T;   // the sequence's only token

  __shared__ __align__(16) float sq[K];
  __shared__ __align__(16) float sk[K];
  __shared__ __align__(16) float sv[V];
  __shared__ __align__(16) float so[V];
  __shared__ __align__(16) float red_k[RG][V];
  __shared__ __align__(16) float red_q[RG][V];
  __shared__ float s_decay, s_beta, s_kq;

  const int64_t head = (int64_t(n) * p.HV + hv) * K * V;
  const TS *src = static_cast<const TS *>(p.h0) + head;
  if (tid == 0) {
    *abort_flag = 0;
    tc::mbar_init(bar, 1);
    tc::mbar_fence_init();
    // warm L2 with the state before the wait (an L2 prefetch is safe even if the previous kernel writes it)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(kS32Bytes) : "memory");
  }
  __syncthreads();
  pdl_wait();
  pdl_release();
  if (warp == 0) {
    // four 16 KB copies (32 rows each) on one barrier, so the copy engine works on them in parallel
    if (lane == 0) tc::mbar_arrive_expect_tx(bar, kS32Bytes);
    __syncwarp();
    if (lane < 4) bulk_load_state(st + lane * (K / 4) * COLS, src + lane * (K / 4) * COLS, kS32Bytes / 4, bar);
  }

  const bool l2 = p.flags & YB_GDN_QK_L2NORM;
  const bool gate_in = p.flags & YB_GDN_GATE_IN_KERNEL;
  const bool beta_sig = p.flags & YB_GDN_BETA_SIGMOID;
  const TIO *qp = static_cast<const TIO *>(p.q);
  const TIO *kp = static_cast<const TIO *>(p.k);
  const TIO *vp = static_cast<const TIO *>(p.v);
  TIO *op = static_cast<TIO *>(p.o);
  bool ok = true;
  {
    // ---- stage q, k (normalised, q scaled), v, decay, beta ----
    if (warp == 0) {
      float qv[4] = {0.f, 0.f, 0.f, 0.f}, kv[4] = {0.f, 0.f, 0.f, 0.f};
      if (lane < K / 4) {
        load4(qp + tok * p.q_ts + int64_t(h) * K + lane * 4, qv);
        load4(kp + tok * p.k_ts + int64_t(h) * K + lane * 4, kv);
      }
      float qn = 1.f, kn = 1.f;
      if (l2) {
        float qs2 = qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3];
        float ks2 = kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3];
        qn = rsqrtf(warp_sum(qs2) + 1e-6f);
        kn = rsqrtf(warp_sum(ks2) + 1e-6f);
      }
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qv[j] *= qn * p.scale;
        kv[j] *= kn;
        dot += qv[j] * kv[j];
      }
      dot = warp_sum(dot);
      if (lane < K / 4) {
        *reinterpret_cast<float4 *>(sq + lane * 4) = make_float4(qv[0], qv[1], qv[2], qv[3]);
        *reinterpret_cast<float4 *>(sk + lane * 4) = make_float4(kv[0], kv[1], kv[2], kv[3]);
      }
      if (lane == 0) s_kq = dot;
    } else if (warp == 1) {
      if (lane < V / 4) {
        float vv[4];
        load4(vp + tok * p.v_ts + int64_t(hv) * V + lane * 4, vv);
        *reinterpret_cast<float4 *>(sv + lane * 4) = make_float4(vv[0], vv[1], vv[2], vv[3]);
      }
      if (lane == 0) {
        float gl = load_scalar(p.g, tok * p.g_ts + hv, p.g_dtype);
        if (gate_in) gl = -expf(p.A_log[hv]) * softplus20(gl + (p.dt_bias ? p.dt_bias[hv] : 0.f));
        float b = load_scalar(p.beta, tok * p.beta_ts + hv, p.beta_dtype);
        s_decay = expf(gl);
        s_beta = beta_sig ? round_to<TIO>(sigmoidf_(b)) : b;   // sigmoid(b) in the input dtype, as the reference stores beta
      }
    }
    __syncthreads();
    ok = tc::mbar_wait(bar, 0, abort_flag, ERR_REC_STATE);
    ok = !__syncthreads_or(!ok);
    const float dec = s_decay, bet = s_beta, kq = s_kq;
    if (ok) {
      float ak[4] = {0.f, 0.f, 0.f, 0.f}, aq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        float x[4];
        lds4(st + (rg * RPT + i) * COLS + c0, x);
        const float kr = sk[rg * RPT + i], qr = sq[rg * RPT + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          x[j] *= dec;
          ak[j] = fmaf(x[j], kr, ak[j]);
          aq[j] = fmaf(x[j], qr, aq[j]);
        }
      }
      *reinterpret_cast<float4 *>(&red_k[rg][c0]) = make_float4(ak[0], ak[1], ak[2], ak[3]);
      *reinterpret_cast<float4 *>(&red_q[rg][c0]) = make_float4(aq[0], aq[1], aq[2], aq[3]);
    }
    __syncthreads();
    if (ok) {
      float kvs[4] = {0.f, 0.f, 0.f, 0.f}, qss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        float4 a = *reinterpret_cast<const float4 *>(&red_k[r][c0]);
        float4 b = *reinterpret_cast<const float4 *>(&red_q[r][c0]);
        kvs[0] += a.x; kvs[1] += a.y; kvs[2] += a.z; kvs[3] += a.w;
        qss[0] += b.x; qss[1] += b.y; qss[2] += b.z; qss[3] += b.w;
      }
      float delta[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) delta[j] = bet * (sv[c0 + j] - kvs[j]);
      TS *dst = static_cast<TS *>(p.ht) + head;
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        float x[4];
        lds4(st + (rg * RPT + i) * COLS + c0, x);
        const float kr = sk[rg * RPT + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          x[j] *= dec;
          x[j] = fmaf(kr, delta[j], x[j]);
        }
        st_state4(dst + (rg * RPT + i) * COLS + c0, x);
      }
      if (rg == 0) {
        float ov[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) ov[j] = fmaf(delta[j], kq, qss[j]);
        *reinterpret_cast<float4 *>(so + c0) = make_float4(ov[0], ov[1], ov[2], ov[3]);
      }
    }
    __syncthreads();
    if (ok) {
    // ---- output (and the fused gated RMSNorm) by warp 0 ----
    if (warp == 0) {
      float ov[4] = {0.f, 0.f, 0.f, 0.f};
      if (lane < V / 4) {
        float4 x = *reinterpret_cast<const float4 *>(so + lane * 4);
        ov[0] = x.x; ov[1] = x.y; ov[2] = x.z; ov[3] = x.w;
      }
      TIO *dst = op + tok * int64_t(p.HV) * V + int64_t(hv) * V + lane * 4;
      if constexpr (NORM) {
        // Qwen3_5RMSNormGated on the io-dtype output, with its roundings.
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ov[j] = round_to<TIO>(ov[j]);
          ss += ov[j] * ov[j];
        }
        const float inv = rsqrtf(warp_sum(ss) / float(V) + p.norm_eps);
        if (lane < V / 4) {
          float zz[4], w[4];
          load4(static_cast<const TIO *>(p.z) + tok * int64_t(p.HV) * V + int64_t(hv) * V + lane * 4, zz);
          load4(static_cast<const TIO *>(p.norm_w) + lane * 4, w);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float y = round_to<TIO>(w[j] * round_to<TIO>(ov[j] * inv));
            ov[j] = y * (zz[j] * sigmoidf_(zz[j]));
          }
          store4(dst, ov);
        }
      } else {
        if (lane < V / 4) store4(dst, ov);
      }
    }
    }
  }
  if (!ok && tid == 0) {
    // the copy may still land: wait for it (bounded, not cut short) before the CTA exits
    volatile int keep_waiting = 0;
    tc::mbar_wait(bar, 0, &keep_waiting, ERR_REC_STATE);
  }
}

template <typename TIO, int K, int V, typename TS = float>
int launch_kv(const GdnArgs &a, const RecParams &p) {
  const bool trans = a.flags & YB_GDN_TRANSPOSE_STATE;
  const bool norm = a.z != nullptr;
  dim3 grid(unsigned(a.N * a.HV));
  if constexpr (K == 128 && V == 128) {
    // one token per sequence: the state staged in shared memory, three (fp32) or five (16-bit)
    // CTAs per SM
    if (!trans && a.T == 1 && !a.cu_seqlens && a.h0 && a.ht && (reinterpret_cast<uintptr_t>(a.h0) & 15u) == 0) {
      auto ks = norm ? gdn_recurrent_sst_kernel<TIO, TS, true> : gdn_recurrent_sst_kernel<TIO, TS, false>;
      const int smem = int(staged_bytes<TS>()) + 16;
      cudaError_t e = cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e == cudaSuccess) e = launch_pdl(ks, grid, dim3(kThreads), size_t(smem), a.stream, p);
      if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gdn_recurrent_sst_kernel: %s", cudaGetErrorString(e));
      return check_launch("gdn_recurrent_sst_kernel");
    }
  }
  auto kern = trans ? (norm ? gdn_recurrent_kernel<TIO, TS, K, V, true, true> : gdn_recurrent_kernel<TIO, TS, K, V, true, false>)
                    : (norm ? gdn_recurrent_kernel<TIO, TS, K, V, false, true> : gdn_recurrent_kernel<TIO, TS, K, V, false, false>);
  const cudaError_t e = launch_pdl(kern, grid, dim3(kThreads), 0, a.stream, p);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gdn_recurrent_kernel: %s", cudaGetErrorString(e));
  return check_launch("gdn_recurrent_kernel");
}

template <typename TIO>
int launch_io(const GdnArgs &a, const RecParams &p) {
  if (a.flags & (YB_GDN_STATE_F16 | YB_GDN_STATE_BF16)) {   // 16-bit state storage: the YANchor head shape
    if (a.K != 128 || a.V != 128)
      return set_error(YB_ERR_UNSUPPORTED, "gdn recurrent: 16-bit state storage is built for K = V = 128");
    if (a.flags & YB_GDN_STATE_F16) return launch_kv<TIO, 128, 128, __half>(a, p);
    return launch_kv<TIO, 128, 128, __nv_bfloat16>(a, p);
  }
  if (a.K == 128 && a.V == 128) return launch_kv<TIO, 128, 128>(a, p);
  if (a.K == 64 && a.V == 64) return launch_kv<TIO, 64, 64>(a, p);
  if (a.K == 128 && a.V == 64) return launch_kv<TIO, 128, 64>(a, p);
  if (a.K == 64 && a.V == 128) return launch_kv<TIO, 64, 128>(a, p);
  if (a.K == 32 && a.V == 32) return launch_kv<TIO, 32, 32>(a, p);
  return set_error(YB_ERR_UNSUPPORTED, "gdn recurrent: (K, V) = (%lld, %lld) not built; supported 32/64/128",
                   (long long)a.K, (long long)a.V);
}

}  // namespace

int read_device_error_rec(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(tc::g_device_error, &z, sizeof(int));
  }
  return v;
}

int launch_gdn_recurrent(const GdnArgs &a) {
  RecParams p;
  p.q = a.q; p.k = a.k; p.v = a.v;
  p.q_ts = a.q_ts; p.k_ts = a.k_ts; p.v_ts = a.v_ts;
  p.g = a.g; p.beta = a.beta; p.g_ts = a.g_ts; p.beta_ts = a.beta_ts;
  p.g_dtype = a.g_dtype; p.beta_dtype = a.beta_dtype;
  p.A_log = a.A_log; p.dt_bias = a.dt_bias;
  p.h0 = a.h0; p.ht = a.ht; p.o = a.o;
  p.z = a.z; p.norm_w = a.norm_w; p.norm_eps = a.norm_eps;
  p.cu = a.cu_seqlens; p.T = a.T;
  p.H = int(a.H); p.HV = int(a.HV);
  p.scale = a.scale; p.flags = a.flags;
  if (a.N * a.HV == 0) return YB_OK;
  switch (a.io_dtype) {
    case YB_F32: return launch_io<float>(a, p);
    case YB_BF16: return launch_io<__nv_bfloat16>(a, p);
    case YB_F16: return launch_io<__half>(a, p);
  }
  return set_error(YB_ERR_ARGUMENT, "gdn recurrent: bad io dtype %d", a.io_dtype);
}

}  // namespace yb
