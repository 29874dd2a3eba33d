// One GDN layer's decode core in one launch: the short conv update over the
// fused q/k/v projection, the gates, the q/k L2 norm, the gated delta rule
// with the state updated in place, and the gated RMSNorm of the output —
// everything between the layer's input and output projections
// (runtime/model/inference_kernels.py:693-721 `_fused_gdn_gate_native_decode_
// forward`: fused gates :668-691, `causal_conv1d_update` :339-376, the
// recurrence, `Qwen3_5RMSNormGated`).
//
// Work item = (sequence, k-head) with one 256-thread group per value head of
// that k-head (R = HV / H groups): the q/k conv channels of a k-head are
// convolved, and their conv state shifted, by exactly one CTA, and the
// normalised q/k are staged once for all R value heads.  Inside a group the
// state layout and update are those of the recurrence kernel: each thread
// owns 4 contiguous columns of RPT rows, the state crosses HBM once each way.
//
// The CTA is persistent (one per SM) and walks items; the next item's state
// (R heads, up to 128 KB) is prefetched into shared memory by bulk copies
// while the current item computes, and the updated state streams back to HBM
// from registers — so loads, stores and the per-token work of successive
// items overlap without a second CTA on the SM (at 512 threads x 128
// registers only one fits).  The prefetch wait is bounded; on timeout the
// CTA records an error code, waits (bounded) for the copy in flight, exits.
//
// That persistent form serves HV = H; for HV = 2H the paired forms further
// down (two CTAs per k-head in a cluster) are faster and are used instead:
// one token with the row-major state stages the state in shared memory
// (three CTAs per SM for fp32, four for 16-bit); more tokens or the
// transposed layout keep it in registers (two CTAs per SM).
//
// Roundings follow the reference chain: conv outputs are rounded to the
// activation dtype (the conv update writes a bf16 tensor), beta = sigmoid(b)
// likewise (the fused gates kernel stores it in b's dtype), the decay stays
// fp32; the RMSNorm epilogue keeps Qwen3_5RMSNormGated's roundings.
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

#include <cooperative_groups.h>

namespace yb {
namespace {

using namespace tc;

constexpr int KD = 128, VD = 128, CONV_KS = 4;
constexpr int ERR_WAIT_STATE = 0x301;

// one bulk copy (non-multicast) global -> shared, completing on `bar`
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

struct FusedParams {
  const void *mixed;              // [tokens, 2*H*K + HV*V]
  int64_t mixed_ts;
  const void *z;                  // [tokens, HV, V]
  int64_t z_ts;
  const void *a, *b;              // [tokens, HV]
  int64_t ab_ts;
  void *conv_state;               // [N, C, 4]
  int64_t conv_bs;
  const float *conv_w, *conv_b;   // [C, 4], [C] or null
  void *state;                    // [N, HV, K, V] (or [N, HV, V, K])
  const float *A_log, *dt_bias;
  const void *norm_w;
  float norm_eps, scale;
  void *o;                        // [tokens, HV, V]
  int64_t T, N;
  int H, HV;
};

__device__ __forceinline__ void ld4s(const float *src, float *x) {
  const float4 v = __ldcs(reinterpret_cast<const float4 *>(src));
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <typename T16>
__device__ __forceinline__ void ld4s(const T16 *src, float *x) {
  const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(src));
  const T16 *h = reinterpret_cast<const T16 *>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = to_f(h[j]);
}
__device__ __forceinline__ void st4s(float *dst, const float *x) {
  __stcs(reinterpret_cast<float4 *>(dst), make_float4(x[0], x[1], x[2], x[3]));
}
template <typename T16>
__device__ __forceinline__ void st4s(T16 *dst, const float *x) {
  uint2 v;
  T16 *h = reinterpret_cast<T16 *>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = from_f<T16>(x[j]);
  __stcs(reinterpret_cast<uint2 *>(dst), v);
}

// conv update of NG groups of 4 consecutive channels (starting at cs[g]) of
// token `tok`: y[4 g + j] gets the (dtype-rounded) SiLU outputs and the conv
// state is shifted in place.  Every load is issued before any store (the
// stores would otherwise order the next group's loads behind them).
template <typename TIO, int NG, bool STORE = true>
__device__ __forceinline__ void conv_groups(const FusedParams &p, int64_t n, int64_t tok, const int64_t *cs,
                                            float *y, uint2 (*kept)[4] = nullptr) {
  const TIO *xrow = static_cast<const TIO *>(p.mixed) + tok * p.mixed_ts;
  TIO *srow = static_cast<TIO *>(p.conv_state) + n * p.conv_bs;
  uint2 xv[NG], sv[NG][4];
  float4 w[NG][4];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    xv[g] = *reinterpret_cast<const uint2 *>(xrow + cs[g]);                       // 4 inputs
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sv[g][j] = *reinterpret_cast<const uint2 *>(srow + (cs[g] + j) * CONV_KS);  // 4 taps of channel j
      w[g][j] = __ldg(reinterpret_cast<const float4 *>(p.conv_w + (cs[g] + j) * CONV_KS));
    }
  }
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const TIO *xin = reinterpret_cast<const TIO *>(&xv[g]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      TIO *s4 = reinterpret_cast<TIO *>(&sv[g][j]);
      float acc = p.conv_b ? p.conv_b[cs[g] + j] : 0.f;
      acc = fmaf(w[g][j].x, to_f(s4[1]), acc);
      acc = fmaf(w[g][j].y, to_f(s4[2]), acc);
      acc = fmaf(w[g][j].z, to_f(s4[3]), acc);
      acc = fmaf(w[g][j].w, to_f(xin[j]), acc);
      s4[0] = s4[1];
      s4[1] = s4[2];
      s4[2] = s4[3];
      s4[3] = xin[j];
      y[4 * g + j] = round_to<TIO>(acc * sigmoidf_(acc));
    }
  }
  if constexpr (STORE) {
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) *reinterpret_cast<uint2 *>(srow + (cs[g] + j) * CONV_KS) = sv[g][j];
  } else {
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) kept[g][j] = sv[g][j];
  }
}
// the shifted conv state kept by conv_groups<.., false>, stored for one group of 4 channels
template <typename TIO>
__device__ __forceinline__ void conv_state_store(const FusedParams &p, int64_t n, int64_t c, const uint2 *sv) {
  TIO *srow = static_cast<TIO *>(p.conv_state) + n * p.conv_bs;
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<uint2 *>(srow + (c + j) * CONV_KS) = sv[j];
}

template <typename TIO, typename TS, int R, bool TRANS>
__global__ void __launch_bounds__(256 * R, 1) gdn_decode_fused_kernel(const FusedParams p) {
  constexpr int ROWS = TRANS ? VD : KD;
  constexpr int COLS = TRANS ? KD : VD;
  constexpr int NCG = COLS / 4, RG = 256 / NCG, RPT = ROWS / RG;
  constexpr uint32_t HEAD_BYTES = uint32_t(KD) * VD * sizeof(TS);
  const int tid = threadIdx.x, grp = tid >> 8, gt = tid & 255, lane = tid & 31, gwarp = gt >> 5;
  const int cg = gt % NCG, rg = gt / NCG, c0 = cg * 4;
  extern __shared__ __align__(128) unsigned char dsm[];
  TS *sbuf = reinterpret_cast<TS *>(dsm);                                           // [R][K*V]
  uint64_t *bar = reinterpret_cast<uint64_t *>(dsm + size_t(R) * HEAD_BYTES);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bar + 1);

  __shared__ __align__(16) float sq[KD];
  __shared__ __align__(16) float sk[KD];
  __shared__ __align__(16) float sv[R][VD];
  __shared__ __align__(16) float so[R][VD];
  __shared__ __align__(16) float red_k[R][TRANS ? 1 : RG][TRANS ? 4 : VD];
  __shared__ __align__(16) float red_q[R][TRANS ? 1 : RG][TRANS ? 4 : VD];
  __shared__ float s_decay[R], s_beta[R], s_kq;

  const int64_t items = p.N * p.H;
  TS *state = static_cast<TS *>(p.state);
  if (tid == 0) {
    *abort_flag = 0;
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  auto prefetch = [&](int64_t it) {   // thread 0: the R value heads of item `it`
    const int64_t nn = it / p.H, hh = it % p.H;
    mbar_arrive_expect_tx(bar, R * HEAD_BYTES);
#pragma unroll
    for (int g = 0; g < R; ++g)
      bulk_load(sbuf + size_t(g) * KD * VD, state + ((nn * p.HV + hh * R + g) * KD * VD), HEAD_BYTES, bar);
  };
  if (tid == 0 && blockIdx.x < items) prefetch(blockIdx.x);
  uint32_t phase = 0;
  bool ok = true;
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
  const int64_t n = item / p.H;
  const int h = int(item % p.H);
  const int hv = h * R + grp;
  const int64_t qch = int64_t(h) * KD, kch = int64_t(p.H) * KD + int64_t(h) * KD;
  const int64_t vch = 2 * int64_t(p.H) * KD + int64_t(hv) * VD;
  ok = ok && mbar_wait(bar, phase, abort_flag, ERR_WAIT_STATE);
  ok = !__syncthreads_or(!ok);
  if (!ok) break;
  phase ^= 1u;
  float s[RPT][4];
  {
    const TS *src = sbuf + size_t(grp) * KD * VD;
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const TS *e = src + (rg * RPT + i) * COLS + c0;
      if constexpr (sizeof(TS) == 4) {
        const float4 v = *reinterpret_cast<const float4 *>(e);
        s[i][0] = v.x; s[i][1] = v.y; s[i][2] = v.z; s[i][3] = v.w;
      } else {
        const uint2 v = *reinterpret_cast<const uint2 *>(e);
        const TS *hh = reinterpret_cast<const TS *>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = to_f(hh[j]);
      }
    }
  }
  fence_async_smem();   // these reads come before the next prefetch's writes
  __syncthreads();
  if (tid == 0 && item + gridDim.x < items) prefetch(item + gridDim.x);
  TS *stp = state + (n * p.HV + hv) * KD * VD;

  for (int64_t t = 0; t < p.T; ++t) {
    const int64_t tok = n * p.T + t;
    if (grp == 0 && gwarp == 0) {
      // q and k of k-head h: conv, L2 norm, q scale, and q.k
      float qk[8];
      const int64_t cs[2] = {qch + lane * 4, kch + lane * 4};
      conv_groups<TIO, 2>(p, n, tok, cs, qk);
      float *qv = qk, *kv = qk + 4;
      float qs2 = qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3];
      float ks2 = kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3];
      const float qn = rsqrtf(warp_sum(qs2) + 1e-6f), kn = rsqrtf(warp_sum(ks2) + 1e-6f);
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qv[j] *= qn * p.scale;
        kv[j] *= kn;
        dot += qv[j] * kv[j];
      }
      dot = warp_sum(dot);
      *reinterpret_cast<float4 *>(sq + lane * 4) = make_float4(qv[0], qv[1], qv[2], qv[3]);
      *reinterpret_cast<float4 *>(sk + lane * 4) = make_float4(kv[0], kv[1], kv[2], kv[3]);
      if (lane == 0) s_kq = dot;
    } else if (gwarp == 1) {
      // v of value head hv, and its gates
      float vv[4];
      const int64_t cs[1] = {vch + lane * 4};
      conv_groups<TIO, 1>(p, n, tok, cs, vv);
      *reinterpret_cast<float4 *>(&sv[grp][lane * 4]) = make_float4(vv[0], vv[1], vv[2], vv[3]);
      if (lane == 0) {
        const float av = to_f(static_cast<const TIO *>(p.a)[tok * p.ab_ts + hv]);
        const float bv = to_f(static_cast<const TIO *>(p.b)[tok * p.ab_ts + hv]);
        const float gl = -expf(p.A_log[hv]) * softplus20(av + (p.dt_bias ? p.dt_bias[hv] : 0.f));
        s_decay[grp] = expf(gl);
        s_beta[grp] = round_to<TIO>(sigmoidf_(bv));
      }
    }
    __syncthreads();
    const float dec = s_decay[grp], bet = s_beta[grp], kq = s_kq;

    if constexpr (!TRANS) {
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
      *reinterpret_cast<float4 *>(&red_k[grp][rg][c0]) = make_float4(ak[0], ak[1], ak[2], ak[3]);
      *reinterpret_cast<float4 *>(&red_q[grp][rg][c0]) = make_float4(aq[0], aq[1], aq[2], aq[3]);
      __syncthreads();
      float kvs[4] = {0.f, 0.f, 0.f, 0.f}, qss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const float4 x = *reinterpret_cast<const float4 *>(&red_k[grp][r][c0]);
        const float4 y = *reinterpret_cast<const float4 *>(&red_q[grp][r][c0]);
        kvs[0] += x.x; kvs[1] += x.y; kvs[2] += x.z; kvs[3] += x.w;
        qss[0] += y.x; qss[1] += y.y; qss[2] += y.z; qss[3] += y.w;
      }
      float delta[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) delta[j] = bet * (sv[grp][c0 + j] - kvs[j]);
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
        *reinterpret_cast<float4 *>(&so[grp][c0]) = make_float4(ov[0], ov[1], ov[2], ov[3]);
      }
    } else {
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
        const float delta = bet * (sv[grp][r] - pk);
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(kc[j], delta, s[i][j]);
        if (cg == 0) so[grp][r] = fmaf(delta, kq, pq);
      }
    }
    __syncthreads();

    // ---- gated RMSNorm of the output (Qwen3_5RMSNormGated, io-dtype roundings) ----
    if (gwarp == 0) {
      float ov[4];
      const float4 x = *reinterpret_cast<const float4 *>(&so[grp][lane * 4]);
      ov[0] = x.x; ov[1] = x.y; ov[2] = x.z; ov[3] = x.w;
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ov[j] = round_to<TIO>(ov[j]);
        ss += ov[j] * ov[j];
      }
      const float inv = rsqrtf(warp_sum(ss) / float(VD) + p.norm_eps);
      float zz[4], w[4];
      load4(static_cast<const TIO *>(p.z) + tok * p.z_ts + int64_t(hv) * VD + lane * 4, zz);
      load4(static_cast<const TIO *>(p.norm_w) + lane * 4, w);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float yv = round_to<TIO>(w[j] * round_to<TIO>(ov[j] * inv));
        ov[j] = yv * (zz[j] * sigmoidf_(zz[j]));
      }
      store4(static_cast<TIO *>(p.o) + (tok * p.HV + hv) * int64_t(VD) + lane * 4, ov);
    }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) st4s(stp + (rg * RPT + i) * COLS + c0, s[i]);
  }   // items
  if (!ok && tid == 0) {
    // the copy this CTA waited for may still land: wait for it (bounded) before exiting
    volatile int keep_waiting = 0;
    mbar_wait(bar, phase, &keep_waiting, ERR_WAIT_STATE);
  }
}

// ---- the paired form (HV = 2 H): one CTA per (sequence, value head), launched as clusters of
// the two value heads of a k-head.  Rank 0 convolves the k-head's q channels and rank 1 its k
// channels (each shifting those channels' conv state once); after a cluster barrier each reads
// the other's half through distributed shared memory.  Each CTA convolves its own v channels.
// The state goes straight into registers as in the recurrence kernel, so two CTAs fit on an SM
// and every load of a CTA is issued at its start.  The exchange buffer is double-buffered by
// token parity: the barrier of token t + 1 orders the peer's reads of token t before its
// overwrite at token t + 2, and a last relaxed arrive (after the last read) with its wait at
// exit keeps this CTA's shared memory alive until the peer has read it. ----
template <typename TIO, typename TS, bool TRANS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 2) gdn_decode_pair_kernel(const FusedParams p) {
  constexpr int ROWS = TRANS ? VD : KD;
  constexpr int COLS = TRANS ? KD : VD;
  constexpr int NCG = COLS / 4, RG = 256 / NCG, RPT = ROWS / RG;
  namespace cgr = cooperative_groups;
  cgr::cluster_group cluster = cgr::this_cluster();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = tid % NCG, rg = tid / NCG, c0 = cg * 4;
  const int64_t n = blockIdx.x / p.HV;
  const int hv = int(blockIdx.x % p.HV), h = hv >> 1;
  const unsigned rank = cluster.block_rank();   // hv & 1

  __shared__ __align__(16) float sx[2][KD];     // this CTA's conv output: q (rank 0) or k (rank 1)
  __shared__ __align__(16) float sq[KD];
  __shared__ __align__(16) float sk[KD];
  __shared__ __align__(16) float sv[VD];
  __shared__ __align__(16) float so[VD];
  __shared__ __align__(16) float red_k[TRANS ? 1 : RG][TRANS ? 4 : VD];
  __shared__ __align__(16) float red_q[TRANS ? 1 : RG][TRANS ? 4 : VD];
  __shared__ float s_decay, s_beta, s_kq;

  TS *stp = static_cast<TS *>(p.state) + (n * p.HV + hv) * int64_t(KD) * VD;
  // the state into L2 before the wait (the previous kernel may be the one that wrote it), then
  // into registers
#pragma unroll
  for (int i = 0; i < RPT; i += (sizeof(TS) == 4 ? 1 : 2)) prefetch_l2(stp + (rg * RPT + i) * COLS + c0);
  pdl_wait();
  pdl_release();
  float s[RPT][4];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const TS *e = stp + (rg * RPT + i) * COLS + c0;
    if constexpr (sizeof(TS) == 4) {
      const float4 v = __ldcs(reinterpret_cast<const float4 *>(e));
      s[i][0] = v.x; s[i][1] = v.y; s[i][2] = v.z; s[i][3] = v.w;
    } else {
      const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(e));
      const TS *hh = reinterpret_cast<const TS *>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = to_f(hh[j]);
    }
  }
  const int64_t xch = rank == 0 ? int64_t(h) * KD : int64_t(p.H) * KD + int64_t(h) * KD;
  const int64_t vch = 2 * int64_t(p.H) * KD + int64_t(hv) * VD;

  for (int64_t t = 0; t < p.T; ++t) {
    const int64_t tok = n * p.T + t;
    const int buf = int(t & 1);
    // the shifted conv state of warp 0's or warp 1's channels, stored after the exchange barrier
    // (a release barrier would otherwise wait for those global stores)
    uint2 cst[1][4];
    if (warp == 0) {
      float y[4];
      const int64_t cs[1] = {xch + lane * 4};
      conv_groups<TIO, 1, false>(p, n, tok, cs, y, cst);
      *reinterpret_cast<float4 *>(&sx[buf][lane * 4]) = make_float4(y[0], y[1], y[2], y[3]);
    } else if (warp == 1) {
      // v of value head hv, and its gates
      float vv[4];
      const int64_t cs[1] = {vch + lane * 4};
      conv_groups<TIO, 1, false>(p, n, tok, cs, vv, cst);
      *reinterpret_cast<float4 *>(sv + lane * 4) = make_float4(vv[0], vv[1], vv[2], vv[3]);
      if (lane == 0) {
        const float av = to_f(static_cast<const TIO *>(p.a)[tok * p.ab_ts + hv]);
        const float bv = to_f(static_cast<const TIO *>(p.b)[tok * p.ab_ts + hv]);
        const float gl = -expf(p.A_log[hv]) * softplus20(av + (p.dt_bias ? p.dt_bias[hv] : 0.f));
        s_decay = expf(gl);
        s_beta = round_to<TIO>(sigmoidf_(bv));
      }
    }
    cluster.sync();   // q and k of the k-head written by the two CTAs
    if (warp < 2) conv_state_store<TIO>(p, n, (warp == 0 ? xch : vch) + lane * 4, cst[0]);
    if (warp == 0) {
      // q and k: L2 norm, q scale, and q.k
      const float *xq = rank == 0 ? &sx[buf][0] : cluster.map_shared_rank(&sx[buf][0], 0);
      const float *xk = rank == 1 ? &sx[buf][0] : cluster.map_shared_rank(&sx[buf][0], 1);
      const float4 q4 = *reinterpret_cast<const float4 *>(xq + lane * 4);
      const float4 k4 = *reinterpret_cast<const float4 *>(xk + lane * 4);
      float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
      float qs2 = qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3];
      float ks2 = kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3];
      const float qn = rsqrtf(warp_sum(qs2) + 1e-6f), kn = rsqrtf(warp_sum(ks2) + 1e-6f);
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qv[j] *= qn * p.scale;
        kv[j] *= kn;
        dot += qv[j] * kv[j];
      }
      dot = warp_sum(dot);
      *reinterpret_cast<float4 *>(sq + lane * 4) = make_float4(qv[0], qv[1], qv[2], qv[3]);
      *reinterpret_cast<float4 *>(sk + lane * 4) = make_float4(kv[0], kv[1], kv[2], kv[3]);
      if (lane == 0) s_kq = dot;
    }
    __syncthreads();
    // after the last token's exchange: this CTA is done reading the peer's buffer (the matching
    // wait comes at exit, so neither CTA's shared memory goes away while the other reads it)
    if (t == p.T - 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    const float dec = s_decay, bet = s_beta, kq = s_kq;

    if constexpr (!TRANS) {
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
        const float4 x = *reinterpret_cast<const float4 *>(&red_k[r][c0]);
        const float4 y = *reinterpret_cast<const float4 *>(&red_q[r][c0]);
        kvs[0] += x.x; kvs[1] += x.y; kvs[2] += x.z; kvs[3] += x.w;
        qss[0] += y.x; qss[1] += y.y; qss[2] += y.z; qss[3] += y.w;
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
        *reinterpret_cast<float4 *>(&so[c0]) = make_float4(ov[0], ov[1], ov[2], ov[3]);
      }
    } else {
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

    // ---- gated RMSNorm of the output (Qwen3_5RMSNormGated, io-dtype roundings) ----
    if (warp == 0) {
      float ov[4];
      const float4 x = *reinterpret_cast<const float4 *>(&so[lane * 4]);
      ov[0] = x.x; ov[1] = x.y; ov[2] = x.z; ov[3] = x.w;
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ov[j] = round_to<TIO>(ov[j]);
        ss += ov[j] * ov[j];
      }
      const float inv = rsqrtf(warp_sum(ss) / float(VD) + p.norm_eps);
      float zz[4], w[4];
      load4(static_cast<const TIO *>(p.z) + tok * p.z_ts + int64_t(hv) * VD + lane * 4, zz);
      load4(static_cast<const TIO *>(p.norm_w) + lane * 4, w);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float yv = round_to<TIO>(w[j] * round_to<TIO>(ov[j] * inv));
        ov[j] = yv * (zz[j] * sigmoidf_(zz[j]));
      }
      store4(static_cast<TIO *>(p.o) + (tok * p.HV + hv) * int64_t(VD) + lane * 4, ov);
    }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) st4s(stp + (rg * RPT + i) * COLS + c0, s[i]);
  if (p.T > 0) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");   // the peer has read this CTA's buffer
}

// ---- the staged paired form (HV = 2 H, one token, row-major state): the pair kernel's conv and
// q/k exchange, with the state staged in shared memory by four bulk copies (warmed into L2 before
// the dependent-launch wait, issued once the conv is done, in flight during the q/k norms), so
// three (fp32) or four (16-bit) CTAs share an SM.  The recurrence is the staged
// recurrence kernel's: same arithmetic, same order, identical results.  The copies' wait is
// bounded: on timeout the CTA records ERR_WAIT_STATE, skips the update, and waits (bounded) for
// the copies before it exits. ----
template <typename T16>
__device__ __forceinline__ void lds_state4(const T16 *p, float *x) {
  const uint2 v = *reinterpret_cast<const uint2 *>(p);
  const T16 *e = reinterpret_cast<const T16 *>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = to_f(e[j]);
}
__device__ __forceinline__ void lds_state4(const float *p, float *x) {
  const float4 v = *reinterpret_cast<const float4 *>(p);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <typename TS> __host__ __device__ constexpr uint32_t pair_staged_bytes() {
  return uint32_t(KD) * VD * uint32_t(sizeof(TS));
}

template <typename TIO, typename TS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, sizeof(TS) == 4 ? 3 : 4)
    gdn_decode_pair_sst_kernel(const FusedParams p) {
  constexpr int COLS = VD, NCG = COLS / 4, RG = 256 / NCG, RPT = KD / RG;
  constexpr uint32_t SB = pair_staged_bytes<TS>();
  namespace cgr = cooperative_groups;
  cgr::cluster_group cluster = cgr::this_cluster();
  extern __shared__ __align__(128) unsigned char pair_dyn[];
  TS *st = reinterpret_cast<TS *>(pair_dyn);                           // [K][V]
  uint64_t *bar = reinterpret_cast<uint64_t *>(pair_dyn + SB);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bar + 1);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = tid % NCG, rg = tid / NCG, c0 = cg * 4;
  const int64_t n = blockIdx.x / p.HV;
  const int hv = int(blockIdx.x % p.HV), h = hv >> 1;
  const unsigned rank = cluster.block_rank();   // hv & 1
  const int64_t tok = n;                        // the sequence's only token

  __shared__ __align__(16) float sx[KD];        // this CTA's conv output: q (rank 0) or k (rank 1)
  __shared__ __align__(16) float sq[KD];
  __shared__ __align__(16) float sk[KD];
  __shared__ __align__(16) float sv[VD];
  __shared__ __align__(16) float so[VD];
  __shared__ __align__(16) float red_k[RG][VD];
  __shared__ __align__(16) float red_q[RG][VD];
  __shared__ float s_decay, s_beta, s_kq;

  TS *stp = static_cast<TS *>(p.state) + (n * p.HV + hv) * int64_t(KD) * VD;
  if (tid == 0) {
    *abort_flag = 0;
    mbar_init(bar, 1);
    mbar_fence_init();
    // warm L2 with the state before the wait (an L2 prefetch is safe even if the previous kernel writes it)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(stp), "r"(SB) : "memory");
  }
  __syncthreads();
  pdl_wait();
  pdl_release();
  const int64_t xch = rank == 0 ? int64_t(h) * KD : int64_t(p.H) * KD + int64_t(h) * KD;
  const int64_t vch = 2 * int64_t(p.H) * KD + int64_t(hv) * VD;
  // the shifted conv state of warp 0's or warp 1's channels, stored after the exchange barrier
  uint2 cst[1][4];
  if (warp == 0) {
    float y[4];
    const int64_t cs[1] = {xch + lane * 4};
    conv_groups<TIO, 1, false>(p, n, tok, cs, y, cst);
    *reinterpret_cast<float4 *>(&sx[lane * 4]) = make_float4(y[0], y[1], y[2], y[3]);
  } else if (warp == 1) {
    // v of value head hv, and its gates
    float vv[4];
    const int64_t cs[1] = {vch + lane * 4};
    conv_groups<TIO, 1, false>(p, n, tok, cs, vv, cst);
    *reinterpret_cast<float4 *>(sv + lane * 4) = make_float4(vv[0], vv[1], vv[2], vv[3]);
    if (lane == 0) {
      const float av = to_f(static_cast<const TIO *>(p.a)[tok * p.ab_ts + hv]);
      const float bv = to_f(static_cast<const TIO *>(p.b)[tok * p.ab_ts + hv]);
      const float gl = -expf(p.A_log[hv]) * softplus20(av + (p.dt_bias ? p.dt_bias[hv] : 0.f));
      s_decay = expf(gl);
      s_beta = round_to<TIO>(sigmoidf_(bv));
    }
  }
  cluster.sync();   // q and k of the k-head written by the two CTAs
  if (warp == 2) {
    // four copies (32 rows each) on one barrier, so the copy engine works on them in parallel.
    // They go out once the conv is done: issued first, they queue the conv's small loads behind
    // 64 KB of state per CTA (24 layers at B=64: 1,415 us against 1,291 us this way).
    if (lane == 0) mbar_arrive_expect_tx(bar, SB);
    __syncwarp();
    if (lane < 4) bulk_load(st + lane * (KD / 4) * COLS, stp + lane * (KD / 4) * COLS, SB / 4, bar);
  }
  if (warp < 2) conv_state_store<TIO>(p, n, (warp == 0 ? xch : vch) + lane * 4, cst[0]);
  if (warp == 0) {
    // q and k: L2 norm, q scale, and q.k
    const float *xq = rank == 0 ? sx : cluster.map_shared_rank(sx, 0);
    const float *xk = rank == 1 ? sx : cluster.map_shared_rank(sx, 1);
    const float4 q4 = *reinterpret_cast<const float4 *>(xq + lane * 4);
    const float4 k4 = *reinterpret_cast<const float4 *>(xk + lane * 4);
    float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
    float qs2 = qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3];
    float ks2 = kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3];
    const float qn = rsqrtf(warp_sum(qs2) + 1e-6f), kn = rsqrtf(warp_sum(ks2) + 1e-6f);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      qv[j] *= qn * p.scale;
      kv[j] *= kn;
      dot += qv[j] * kv[j];
    }
    dot = warp_sum(dot);
    *reinterpret_cast<float4 *>(sq + lane * 4) = make_float4(qv[0], qv[1], qv[2], qv[3]);
    *reinterpret_cast<float4 *>(sk + lane * 4) = make_float4(kv[0], kv[1], kv[2], kv[3]);
    if (lane == 0) s_kq = dot;
  }
  __syncthreads();
  // this CTA is done reading the peer's buffer (the matching wait comes at exit, so neither CTA's
  // shared memory goes away while the other reads it)
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  bool ok = mbar_wait(bar, 0, abort_flag, ERR_WAIT_STATE);
  ok = !__syncthreads_or(!ok);
  const float dec = s_decay, bet = s_beta, kq = s_kq;
  if (ok) {
    float ak[4] = {0.f, 0.f, 0.f, 0.f}, aq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      float x[4];
      lds_state4(st + (rg * RPT + i) * COLS + c0, x);
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
      const float4 x = *reinterpret_cast<const float4 *>(&red_k[r][c0]);
      const float4 y = *reinterpret_cast<const float4 *>(&red_q[r][c0]);
      kvs[0] += x.x; kvs[1] += x.y; kvs[2] += x.z; kvs[3] += x.w;
      qss[0] += y.x; qss[1] += y.y; qss[2] += y.z; qss[3] += y.w;
    }
    float delta[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) delta[j] = bet * (sv[c0 + j] - kvs[j]);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      float x[4];
      lds_state4(st + (rg * RPT + i) * COLS + c0, x);
      const float kr = sk[rg * RPT + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[j] *= dec;
        x[j] = fmaf(kr, delta[j], x[j]);
      }
      st4s(stp + (rg * RPT + i) * COLS + c0, x);
    }
    if (rg == 0) {
      float ov[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) ov[j] = fmaf(delta[j], kq, qss[j]);
      *reinterpret_cast<float4 *>(&so[c0]) = make_float4(ov[0], ov[1], ov[2], ov[3]);
    }
  }
  __syncthreads();
  // ---- gated RMSNorm of the output (Qwen3_5RMSNormGated, io-dtype roundings) ----
  if (ok && warp == 0) {
    float ov[4];
    const float4 x = *reinterpret_cast<const float4 *>(&so[lane * 4]);
    ov[0] = x.x; ov[1] = x.y; ov[2] = x.z; ov[3] = x.w;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ov[j] = round_to<TIO>(ov[j]);
      ss += ov[j] * ov[j];
    }
    const float inv = rsqrtf(warp_sum(ss) / float(VD) + p.norm_eps);
    float zz[4], w[4];
    load4(static_cast<const TIO *>(p.z) + tok * p.z_ts + int64_t(hv) * VD + lane * 4, zz);
    load4(static_cast<const TIO *>(p.norm_w) + lane * 4, w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float yv = round_to<TIO>(w[j] * round_to<TIO>(ov[j] * inv));
      ov[j] = yv * (zz[j] * sigmoidf_(zz[j]));
    }
    store4(static_cast<TIO *>(p.o) + (tok * p.HV + hv) * int64_t(VD) + lane * 4, ov);
  }
  if (!ok && tid == 0) {
    // the copies this CTA waited for may still land: wait for them (bounded) before exiting
    volatile int keep_waiting = 0;
    mbar_wait(bar, 0, &keep_waiting, ERR_WAIT_STATE);
  }
  __syncwarp();   // the aligned barrier below wants every lane of the warp together
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");   // the peer has read this CTA's buffer
}

int sm_count() {
  static int count[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!count[dev] && cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    count[dev] = 148;
  return count[dev];
}

template <typename TIO, typename TS, int R>
int launch_r(const FusedArgs &a, const FusedParams &p) {
  const int64_t items = a.N * a.H;
  const unsigned grid = unsigned(items < sm_count() ? items : sm_count());
  const size_t smem = size_t(R) * KD * VD * sizeof(TS) + 16;
  auto kern = a.trans ? gdn_decode_fused_kernel<TIO, TS, R, true> : gdn_decode_fused_kernel<TIO, TS, R, false>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gdn decode fused: smem attribute: %s", cudaGetErrorString(e));
  kern<<<grid, 256 * R, smem, a.stream>>>(p);
  return check_launch("gdn_decode_fused_kernel");
}

template <typename TIO, typename TS>
int launch_pair(const FusedArgs &a, const FusedParams &p) {
  auto kern = a.trans ? gdn_decode_pair_kernel<TIO, TS, true> : gdn_decode_pair_kernel<TIO, TS, false>;
  const cudaError_t e = launch_pdl(kern, dim3(unsigned(a.N * a.HV)), dim3(256), 0, a.stream, p);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gdn_decode_pair_kernel: %s", cudaGetErrorString(e));
  return check_launch("gdn_decode_pair_kernel");
}

template <typename TIO, typename TS>
int launch_pair_sst(const FusedArgs &a, const FusedParams &p) {
  auto kern = gdn_decode_pair_sst_kernel<TIO, TS>;
  const int smem = int(pair_staged_bytes<TS>()) + 16;   // the staged state, its mbarrier and the abort flag
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = launch_pdl(kern, dim3(unsigned(a.N * a.HV)), dim3(256), size_t(smem), a.stream, p);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gdn_decode_pair_sst_kernel: %s", cudaGetErrorString(e));
  return check_launch("gdn_decode_pair_sst_kernel");
}

template <typename TIO, typename TS>
int launch_ts(const FusedArgs &a, const FusedParams &p) {
  if (a.HV == 2 * a.H) {   // two value heads per k-head: paired CTAs
    // one token with the row-major state: staged in shared memory while the conv runs
    if (!a.trans && a.T == 1 && (reinterpret_cast<uintptr_t>(a.state) & 15u) == 0) return launch_pair_sst<TIO, TS>(a, p);
    return launch_pair<TIO, TS>(a, p);
  }
  switch (a.HV / a.H) {   // 256 threads per value head: at most 512 per CTA keeps the state in registers
    case 1: return launch_r<TIO, TS, 1>(a, p);
    case 2: return launch_r<TIO, TS, 2>(a, p);
  }
  return set_error(YB_ERR_UNSUPPORTED, "gdn decode fused: HV / H = %lld not built (1, 2)",
                   (long long)(a.HV / a.H));
}

template <typename TIO>
int launch_io(const FusedArgs &a, const FusedParams &p) {
  if (a.state_dtype == YB_F16) return launch_ts<TIO, __half>(a, p);
  if (a.state_dtype == YB_BF16) return launch_ts<TIO, __nv_bfloat16>(a, p);
  return launch_ts<TIO, float>(a, p);
}

}  // namespace

int launch_gdn_decode_fused(const FusedArgs &a) {
  if (a.K != KD || a.V != VD || a.conv_ks != CONV_KS || a.conv_width != CONV_KS)
    return set_error(YB_ERR_UNSUPPORTED, "gdn decode fused: built for K = V = 128 and a width-4 conv state");
  if (a.N * a.H == 0 || a.T == 0) return YB_OK;
  FusedParams p;
  p.mixed = a.mixed; p.mixed_ts = a.mixed_ts; p.z = a.z; p.z_ts = a.z_ts; p.a = a.a; p.b = a.b; p.ab_ts = a.ab_ts;
  p.conv_state = a.conv_state; p.conv_bs = a.conv_bs; p.conv_w = a.conv_w; p.conv_b = a.conv_b;
  p.state = a.state; p.A_log = a.A_log; p.dt_bias = a.dt_bias; p.norm_w = a.norm_w; p.norm_eps = a.norm_eps;
  p.scale = a.scale; p.o = a.o; p.T = a.T; p.N = a.N; p.H = int(a.H); p.HV = int(a.HV);
  switch (a.io_dtype) {
    case YB_BF16: return launch_io<__nv_bfloat16>(a, p);
    case YB_F16: return launch_io<__half>(a, p);
  }
  return set_error(YB_ERR_UNSUPPORTED, "gdn decode fused: activations must be bf16 or fp16");
}

int read_device_error_fused(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(tc::g_device_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace yb
