// Shared device helpers for the yanchor_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/yanchor_b200.h"

namespace yb {

// ---- element conversion --------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Round a float through T and back (identity for float).
template <typename T> __device__ __forceinline__ float round_to(float x) { return to_f<T>(from_f<T>(x)); }

// Load 4 consecutive elements (8-byte aligned for 16-bit types, 16-byte for float).
template <typename T> __device__ __forceinline__ void load4(const T *p, float out[4]);
template <> __device__ __forceinline__ void load4<float>(const float *p, float out[4]) {
  float4 v = *reinterpret_cast<const float4 *>(p);
  out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}
template <> __device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16 *p, float out[4]) {
  uint2 raw = *reinterpret_cast<const uint2 *>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&raw.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&raw.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  out[0] = fa.x; out[1] = fa.y; out[2] = fb.x; out[3] = fb.y;
}
template <> __device__ __forceinline__ void load4<__half>(const __half *p, float out[4]) {
  uint2 raw = *reinterpret_cast<const uint2 *>(p);
  __half2 a = *reinterpret_cast<__half2 *>(&raw.x);
  __half2 b = *reinterpret_cast<__half2 *>(&raw.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  out[0] = fa.x; out[1] = fa.y; out[2] = fb.x; out[3] = fb.y;
}

template <typename T> __device__ __forceinline__ void store4(T *p, const float v[4]);
template <> __device__ __forceinline__ void store4<float>(float *p, const float v[4]) {
  *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <> __device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16 *p, const float v[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 raw;
  raw.x = *reinterpret_cast<uint32_t *>(&a);
  raw.y = *reinterpret_cast<uint32_t *>(&b);
  *reinterpret_cast<uint2 *>(p) = raw;
}
template <> __device__ __forceinline__ void store4<__half>(__half *p, const float v[4]) {
  __half2 a = __floats2half2_rn(v[0], v[1]);
  __half2 b = __floats2half2_rn(v[2], v[3]);
  uint2 raw;
  raw.x = *reinterpret_cast<uint32_t *>(&a);
  raw.y = *reinterpret_cast<uint32_t *>(&b);
  *reinterpret_cast<uint2 *>(p) = raw;
}

// 8 consecutive elements (16-byte aligned for 16-bit types and for float).
template <typename T> __device__ __forceinline__ void load8(const T *p, float out[8]) {
  load4(p, out);
  load4(p + 4, out + 4);
}
template <typename T> __device__ __forceinline__ void store8(T *p, const float v[8]) {
  store4(p, v);
  store4(p + 4, v + 4);
}

// ---- reductions ------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Sum over groups of `width` consecutive lanes (width a power of two <= 32).
template <int WIDTH> __device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- math ------------------------------------------------------------------
// softplus with the torch / Triton threshold: x itself above 20.
__device__ __forceinline__ float softplus20(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

}  // namespace yb

// ---- programmatic dependent launch -------------------------------------------
// A kernel launched with launch_pdl may start while the previous kernel in
// its stream is still running.  Before pdl_wait() it must read nothing that
// kernel may write (an L2 prefetch is always safe: a later write lands in L2
// first); pdl_release() lets the next kernel begin launching.  Both are no-ops
// for a normal launch.  A kernel releases only after its own wait, so when it
// runs its pre-wait part every kernel before its predecessor has finished,
// and a dependent can only be scheduled once every CTA of its predecessor is.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- host-side error plumbing (defined in capi.cu) ---------------------------
namespace yb {
int set_error(int code, const char *fmt, ...);
int check_launch(const char *what);
}  // namespace yb
