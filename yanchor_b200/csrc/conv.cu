// Causal depthwise conv1d in front of the GDN recurrence (the short
// convolution over the fused q/k/v projection), decode update and prefill.
//
//   y[t, c] = act(sum_{j < KS} w[c, j] * x[t - (KS - 1) + j, c] + bias[c])
//
// with inputs before the segment taken from the conv state (zeros without
// one).  Decode: runtime/model/inference_kernels.py:339-355 (the graph-safe
// Triton update: fp32 arithmetic, one rounding, state shifted left and the
// new input appended) and modeling_yanchor.py:349-353.  Prefill: transformers
// qwen3_5 modeling_qwen3_5.py:462-480 (the cached state prepended, the new
// state = the last inputs, zero-padded on the left).
//
// Layout: activations token-major with channels contiguous ([B, T, C], the
// memory behind the reference's [B, C, T] transposed view); state [B, C, W]
// with W = KS (the cache's convention) or KS - 1 (the causal-conv1d
// package's `initial_states`), only its last KS - 1 entries feed outputs.
// One thread per channel: a warp reads 32 consecutive channels of a token.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace yb {
namespace {

constexpr int kConvThreads = 128;
constexpr int kConvTile = 32;   // tokens per thread in prefill

__device__ __forceinline__ float conv_act(float y, bool silu) { return silu ? y * sigmoidf_(y) : y; }

// The common decode case (width-4 cache state, 16-bit activations, C a
// multiple of 4): a thread owns 4 consecutive channels of kConvRows batch
// rows, so the weights stay in registers, and issues every load of its rows
// before its first store.  Two rows per thread in 256-thread CTAs (256 CTAs
// at B=64, C=8192) measured fastest inside the decode step's CUDA graph:
// 1.322 ms/step against 1.357 with one row in 128-thread CTAs, 1.327 with
// two rows in 128-thread CTAs and 1.365 with four.
constexpr int kConvRows = 2;
constexpr int kConv4Threads = 256;

template <typename T>
__global__ void __launch_bounds__(kConv4Threads) conv_update4_kernel(const ConvArgs a) {
  const int64_t c = (int64_t(blockIdx.x) * kConv4Threads + threadIdx.x) * 4;
  const int64_t b0 = int64_t(blockIdx.y) * kConvRows;
  if (c < a.C && (threadIdx.x & 1) == 0) {
    // warm L2 with this thread pair's state row pieces and weights before the wait (an L2 prefetch is
    // safe even if the previous kernel writes them); the input comes from the previous kernel
    for (int rr = 0; rr < kConvRows && b0 + rr < a.B; ++rr)
      prefetch_l2(static_cast<const T *>(a.state) + (b0 + rr) * a.state_bs + c * 4);
    prefetch_l2(a.weight + c * 4);
  }
  pdl_wait();
  pdl_release();
  if (c >= a.C) return;
  float4 w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) w[j] = __ldg(reinterpret_cast<const float4 *>(a.weight + (c + j) * 4));
  float bias[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.bias) {
#pragma unroll
    for (int j = 0; j < 4; ++j) bias[j] = a.bias[c + j];
  }
  // every row's loads before any store (the compiler cannot move a load above a store that might
  // alias it), so a thread's rows cost one memory latency
  uint2 xv[kConvRows];
  uint4 sv[kConvRows][2];   // 4 channels x 4 taps per row
#pragma unroll
  for (int rr = 0; rr < kConvRows; ++rr) {
    const int64_t b = b0 + rr;
    if (b >= a.B) break;
    const T *st = static_cast<const T *>(a.state) + b * a.state_bs + c * 4;
    xv[rr] = *reinterpret_cast<const uint2 *>(static_cast<const T *>(a.x) + b * a.x_bs + c);
    sv[rr][0] = *reinterpret_cast<const uint4 *>(st);
    sv[rr][1] = *reinterpret_cast<const uint4 *>(st + 8);
  }
#pragma unroll
  for (int rr = 0; rr < kConvRows; ++rr) {
    const int64_t b = b0 + rr;
    if (b >= a.B) break;
    T *st = static_cast<T *>(a.state) + b * a.state_bs + c * 4;
    const T *xin = reinterpret_cast<const T *>(&xv[rr]);
    T *h = reinterpret_cast<T *>(sv[rr]);
    T yo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      T *s4 = h + 4 * j;
      float y = bias[j];
      y = fmaf(w[j].x, to_f(s4[1]), y);
      y = fmaf(w[j].y, to_f(s4[2]), y);
      y = fmaf(w[j].z, to_f(s4[3]), y);
      y = fmaf(w[j].w, to_f(xin[j]), y);
      s4[0] = s4[1];
      s4[1] = s4[2];
      s4[2] = s4[3];
      s4[3] = xin[j];
      yo[j] = from_f<T>(conv_act(y, a.silu));
    }
    *reinterpret_cast<uint4 *>(st) = sv[rr][0];
    *reinterpret_cast<uint4 *>(st + 8) = sv[rr][1];
    *reinterpret_cast<uint2 *>(static_cast<T *>(a.out) + b * a.out_bs + c) = *reinterpret_cast<const uint2 *>(yo);
  }
}

template <typename T, int KS>
__global__ void __launch_bounds__(kConvThreads) conv_update_kernel(const ConvArgs a) {
  const int64_t b = blockIdx.y;
  const int64_t c = int64_t(blockIdx.x) * kConvThreads + threadIdx.x;
  pdl_wait();
  pdl_release();
  if (c >= a.C) return;
  const T *x = static_cast<const T *>(a.x) + b * a.x_bs;
  T *st = static_cast<T *>(a.state) + b * a.state_bs + c * a.state_cs;
  if constexpr (KS == 4) {
    // the common case (width-4 cache state): the channel's state and weights
    // move as single vectors
    using V = typename std::conditional<sizeof(T) == 4, float4, uint2>::type;
    if (a.W == 4 && a.state_ts == 1 && (reinterpret_cast<uintptr_t>(st) % sizeof(V)) == 0 &&
        (reinterpret_cast<uintptr_t>(a.weight + c * 4) % 16) == 0) {
      V sv = *reinterpret_cast<const V *>(st);
      T *h = reinterpret_cast<T *>(&sv);
      const T xin = x[c];
      const float4 w4 = *reinterpret_cast<const float4 *>(a.weight + c * 4);
      float y = a.bias ? a.bias[c] : 0.f;
      y = fmaf(w4.x, to_f(h[1]), y);
      y = fmaf(w4.y, to_f(h[2]), y);
      y = fmaf(w4.z, to_f(h[3]), y);
      y = fmaf(w4.w, to_f(xin), y);
      h[0] = h[1];
      h[1] = h[2];
      h[2] = h[3];
      h[3] = xin;
      *reinterpret_cast<V *>(st) = sv;
      static_cast<T *>(a.out)[b * a.out_bs + c] = from_f<T>(conv_act(y, a.silu));
      return;
    }
  }
  float win[KS];
#pragma unroll
  for (int j = 0; j < KS - 1; ++j) win[j] = to_f(st[(a.W - (KS - 1) + j) * a.state_ts]);
  const T xin = x[c];
  win[KS - 1] = to_f(xin);
  float y = a.bias ? a.bias[c] : 0.f;
#pragma unroll
  for (int j = 0; j < KS; ++j) y = fmaf(a.weight[c * KS + j], win[j], y);
  // shift the state left by one and append the input (stored values are inputs: no rounding)
  for (int j = 0; j + 1 < a.W; ++j) st[j * a.state_ts] = st[(j + 1) * a.state_ts];
  st[(a.W - 1) * a.state_ts] = xin;
  static_cast<T *>(a.out)[b * a.out_bs + c] = from_f<T>(conv_act(y, a.silu));
}

template <typename T, int KS>
__global__ void __launch_bounds__(kConvThreads) conv_fwd_kernel(const ConvArgs a) {
  const int64_t b = blockIdx.z;
  const int64_t c = int64_t(blockIdx.x) * kConvThreads + threadIdx.x;
  const int64_t t0 = int64_t(blockIdx.y) * kConvTile;
  if (c >= a.C) return;
  const T *x = static_cast<const T *>(a.x) + b * a.x_bs + c;
  const T *st_in = a.state_in ? static_cast<const T *>(a.state_in) + b * a.state_bs + c * a.state_cs : nullptr;
  float w[KS];
#pragma unroll
  for (int j = 0; j < KS; ++j) w[j] = a.weight[c * KS + j];
  const float bias = a.bias ? a.bias[c] : 0.f;
  // the KS - 1 inputs before t0
  auto input = [&](int64_t t) -> float {
    if (t >= 0) return to_f(x[t * a.x_ts]);
    const int64_t back = -t;   // 1 .. KS - 1 (or more, before the state: zero)
    if (st_in && back <= a.W) return to_f(st_in[(a.W - back) * a.state_ts]);
    return 0.f;
  };
  float win[KS];
#pragma unroll
  for (int j = 0; j < KS - 1; ++j) win[j] = input(t0 - (KS - 1) + j);
  const int64_t t1 = t0 + kConvTile < a.T ? t0 + kConvTile : a.T;
  T *out = static_cast<T *>(a.out) + b * a.out_bs + c;
  for (int64_t t = t0; t < t1; ++t) {
    win[KS - 1] = to_f(x[t * a.x_ts]);
    float y = bias;
#pragma unroll
    for (int j = 0; j < KS; ++j) y = fmaf(w[j], win[j], y);
    out[t * a.out_ts] = from_f<T>(conv_act(y, a.silu));
#pragma unroll
    for (int j = 0; j < KS - 1; ++j) win[j] = win[j + 1];
  }
  // final state: the last W inputs of [state | x] (zeros before both); tile 0
  // is the only reader of the initial state, so the two may alias
  if (blockIdx.y == 0 && a.state_out) {
    T *so = static_cast<T *>(a.state_out) + b * a.state_bs + c * a.state_cs;
    T vals[8];
    for (int j = 0; j < a.W; ++j) {
      const int64_t t = a.T - a.W + j;
      if (t >= 0) vals[j] = x[t * a.x_ts];
      else if (st_in && -t <= a.W) vals[j] = st_in[(a.W + t) * a.state_ts];
      else vals[j] = from_f<T>(0.f);
    }
    for (int j = 0; j < a.W; ++j) so[j * a.state_ts] = vals[j];
  }
}

template <typename T>
int conv_dispatch(const ConvArgs &a, bool update) {
  if constexpr (sizeof(T) == 2) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.state) |
                         reinterpret_cast<uintptr_t>(a.out) | reinterpret_cast<uintptr_t>(a.weight);
    if (update && a.KS == 4 && a.W == 4 && a.state_cs == 4 && a.state_ts == 1 && a.C % 4 == 0 && (al % 16) == 0 &&
        (a.x_bs % 4) == 0 &&
        (a.out_bs % 4) == 0 && (a.state_bs % 8) == 0) {
      const dim3 grid(unsigned((a.C / 4 + kConv4Threads - 1) / kConv4Threads),
                      unsigned((a.B + kConvRows - 1) / kConvRows));
      const cudaError_t e = launch_pdl(conv_update4_kernel<T>, grid, dim3(kConv4Threads), 0, a.stream, a);
      if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "conv_update4_kernel: %s", cudaGetErrorString(e));
      return check_launch("conv_update4_kernel");
    }
  }
  switch (a.KS) {
#define YB_CONV_CASE(K)                                                                                 \
  case K:                                                                                               \
    if (update) {                                                                                       \
      const cudaError_t e = launch_pdl(conv_update_kernel<T, K>,                                        \
                                       dim3(unsigned((a.C + kConvThreads - 1) / kConvThreads), unsigned(a.B)), \
                                       dim3(kConvThreads), 0, a.stream, a);                             \
      if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "conv_update_kernel: %s", cudaGetErrorString(e)); \
      return check_launch("conv_update_kernel");                                                        \
    }                                                                                                   \
    conv_fwd_kernel<T, K><<<dim3(unsigned((a.C + kConvThreads - 1) / kConvThreads),                     \
                                 unsigned((a.T + kConvTile - 1) / kConvTile), unsigned(a.B)),           \
                            kConvThreads, 0, a.stream>>>(a);                                            \
    return check_launch("conv_fwd_kernel");
    YB_CONV_CASE(2)
    YB_CONV_CASE(3)
    YB_CONV_CASE(4)
#undef YB_CONV_CASE
  }
  return set_error(YB_ERR_UNSUPPORTED, "conv1d: kernel width %lld not built (2, 3, 4)", (long long)a.KS);
}

}  // namespace

int launch_conv1d(const ConvArgs &a, bool update) {
  if (a.B == 0 || a.C == 0 || (!update && a.T == 0 && !a.state_out)) return YB_OK;
  if (!update && a.T == 0) {
    // nothing to convolve; the state is unchanged
    return YB_OK;
  }
  switch (a.dtype) {
    case YB_F32: return conv_dispatch<float>(a, update);
    case YB_BF16: return conv_dispatch<__nv_bfloat16>(a, update);
    case YB_F16: return conv_dispatch<__half>(a, update);
  }
  return set_error(YB_ERR_ARGUMENT, "conv1d: bad dtype %d", a.dtype);
}

}  // namespace yb
