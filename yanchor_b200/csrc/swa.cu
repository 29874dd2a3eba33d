// Sliding-window attention decode over the physical ring cache
// (runtime/model/inference_kernels.py:1828-1897).
//
// Ring: key / value [B, KVH, W, D] (positions contiguous rows of D), valid
// [B, W], one device-resident write index for the batch.  Update: the new
// token's key / value / valid go to position `index`, then the index
// advances modulo W (a second one-thread launch, so no block of the write
// sees a moved index).
//
// Attention: each query head attends to every ring position whose valid
// flag is set (order does not matter to a softmax), scale D^-1/2, query head
// h reading KV head h / R (R = QH / KVH).  Split over the window: one CTA per
// (row, KV head, 64-position slice) stages the slice's K and V rows by
// cp.async into padded shared rows, computes the R heads' logits (one
// (position, head) pair per thread), their slice max and exp-sum, and the
// exp-weighted value sums (one feature column per thread); a combine kernel
// rescales the slices to the global max and normalises.  Memory-bound: every
// K / V byte is read once.
#include "common.cuh"
#include "kernels.h"

namespace yb {
namespace {

constexpr int kSwaThreads = 256;
constexpr int kSwaSlice = 64;

__device__ __forceinline__ void cp_async16_swa(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ int64_t ring_index_of(const SwaArgs &a) {
  return a.index_i64 ? *static_cast<const int64_t *>(a.ring_index) : int64_t(*static_cast<const int32_t *>(a.ring_index));
}

template <typename T>
__global__ void swa_ring_write_kernel(const SwaArgs a) {
  constexpr int VEC = 16 / int(sizeof(T));
  pdl_wait();
  pdl_release();
  const int64_t idx = ring_index_of(a);
  if (idx < 0 || idx >= a.W) return;   // a corrupt index writes nothing (the advance restarts it at 0)
  const int64_t pieces = a.B * a.KVH * (a.D / VEC);
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e < 2 * pieces) {
    const bool is_v = e >= pieces;
    const int64_t f = is_v ? e - pieces : e;
    const int64_t d = (f % (a.D / VEC)) * VEC, bh = f / (a.D / VEC), b = bh / a.KVH, h = bh % a.KVH;
    const T *src = static_cast<const T *>(is_v ? a.new_v : a.new_k) + b * a.new_bs + h * a.new_hs + d;
    T *dst = static_cast<T *>(is_v ? a.ring_v : a.ring_k) + b * a.ring_bs + h * a.ring_hs + idx * a.D + d;
    *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
  } else if (e < 2 * pieces + a.B) {
    const int64_t b = e - 2 * pieces;
    a.ring_valid[b * a.valid_bs + idx] = a.new_valid[b];
  }
}

__global__ void swa_ring_advance_kernel(const SwaArgs a) {
  pdl_wait();   // every write of the previous kernel has read the index
  pdl_release();
  const int64_t i = ring_index_of(a);
  const int64_t next = (i < 0 || i + 1 >= a.W) ? 0 : i + 1;
  if (a.index_i64) *static_cast<int64_t *>(a.ring_index) = next;
  else *static_cast<int32_t *>(a.ring_index) = int32_t(next);
}

template <typename T, int R, int D>
__global__ void __launch_bounds__(kSwaThreads) swa_partial_kernel(const SwaArgs a, float *part) {
  constexpr int ROWB = D * int(sizeof(T)) + 16;   // padded shared row (bank spread)
  constexpr int PIECES = D * int(sizeof(T)) / 16;
  constexpr int QP = D + 4;
  extern __shared__ __align__(16) unsigned char swa_raw[];
  unsigned char *sk = swa_raw;                                        // [slice][ROWB]
  unsigned char *sv = sk + kSwaSlice * ROWB;                          // [slice][ROWB]
  float *sq = reinterpret_cast<float *>(sv + kSwaSlice * ROWB);       // [R][QP]
  float *sp = sq + R * QP;                                            // [R][slice] logits -> weights
  float *sm = sp + R * kSwaSlice;                                     // [R] max, [R] sum
  const int tid = threadIdx.x;
  const int64_t bh = blockIdx.x, b = bh / a.KVH, kvh = bh % a.KVH;
  const int64_t slice = blockIdx.y, p0 = slice * kSwaSlice;
  const int np = int(a.W - p0 < kSwaSlice ? a.W - p0 : kSwaSlice);
  const unsigned char *kb = reinterpret_cast<const unsigned char *>(static_cast<const T *>(a.ring_k) + b * a.ring_bs +
                                                                      kvh * a.ring_hs + p0 * D);
  const unsigned char *vb = reinterpret_cast<const unsigned char *>(static_cast<const T *>(a.ring_v) + b * a.ring_bs +
                                                                      kvh * a.ring_hs + p0 * D);
  for (int e = tid; e < np * PIECES; e += kSwaThreads)
    cp_async16_swa(sk + (e / PIECES) * ROWB + (e % PIECES) * 16, kb + size_t(e / PIECES) * D * sizeof(T) +
                                                                     (e % PIECES) * 16);
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int e = tid; e < np * PIECES; e += kSwaThreads)
    cp_async16_swa(sv + (e / PIECES) * ROWB + (e % PIECES) * 16, vb + size_t(e / PIECES) * D * sizeof(T) +
                                                                     (e % PIECES) * 16);
  asm volatile("cp.async.commit_group;" ::: "memory");
  const T *q = static_cast<const T *>(a.query) + (b * a.QH + kvh * R) * D;
  for (int e = tid; e < R * D; e += kSwaThreads) sq[(e / D) * QP + e % D] = to_f(q[e]);
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  const float scale = rsqrtf(float(D));
  for (int e = tid; e < kSwaSlice * R; e += kSwaThreads) {
    const int pos = e / R, r = e % R;
    float acc = -INFINITY;
    if (pos < np && a.ring_valid[b * a.valid_bs + p0 + pos]) {
      const T *krow = reinterpret_cast<const T *>(sk + pos * ROWB);
      const float *qr = sq + r * QP;
      acc = 0.f;
#pragma unroll 4
      for (int d = 0; d < D; d += 8) {
        float kx[8];
        load8(krow + d, kx);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(qr[d + j], kx[j], acc);
      }
      acc *= scale;
    }
    sp[r * kSwaSlice + pos] = acc;
  }
  __syncthreads();
  // per head: slice max and exp-sum (a warp per head)
  const int warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < R; r += kSwaThreads / 32) {
    float m = -INFINITY;
    for (int j = lane; j < kSwaSlice; j += 32) m = fmaxf(m, sp[r * kSwaSlice + j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < kSwaSlice; j += 32) {
      const float x = sp[r * kSwaSlice + j];
      const float w = x == -INFINITY ? 0.f : __expf(x - m);
      sp[r * kSwaSlice + j] = w;
      l += w;
    }
    l = warp_sum(l);
    if (lane == 0) {
      sm[r] = m;
      sm[R + r] = l;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // exp-weighted value sums: one feature column per thread, all R heads
  float *out = part + (bh * gridDim.y + slice) * (R * (D + 2));
  for (int d = tid; d < D; d += kSwaThreads) {
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int pos = 0; pos < np; ++pos) {
      const float x = to_f(reinterpret_cast<const T *>(sv + pos * ROWB)[d]);
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = fmaf(sp[r * kSwaSlice + pos], x, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) out[r * (D + 2) + d] = acc[r];
  }
  if (tid < R) {
    out[tid * (D + 2) + D] = sm[tid];
    out[tid * (D + 2) + D + 1] = sm[R + tid];
  }
}

// The combine of one (row, KV head): for each of its HN query heads, every slice's factor
// e^{m_s - M} once per CTA (a slice with nothing valid is skipped), then one output feature per
// thread for all HN heads, with the slices' partial sums for it loaded 16 at a time (16 / HN slices
// of every head) before they are summed in slice order.
__host__ __device__ constexpr size_t combine_smem(int slices, int R) { return size_t(2) * R * slices * sizeof(float); }

template <typename T, int HN>
__global__ void swa_combine_kernel(const SwaArgs a, const float *part, int slices) {
  extern __shared__ float comb[];   // per head: [slices] factor (-1: skip), then per head: [slices] exp-sum
  __shared__ float s_den[HN];
  const int64_t bh = blockIdx.x, b = bh / a.KVH, kvh = bh % a.KVH;
  const int D = int(a.D), tid = threadIdx.x, nt = blockDim.x;
  pdl_wait();   // the slices are written
  pdl_release();
  const int64_t stride = int64_t(HN) * (D + 2);
  const float *pb = part + bh * slices * stride;
  float *fac = comb, *lsum = comb + HN * slices;
  for (int i = tid; i < HN * slices; i += nt) {
    const int hr = i / slices, s = i - hr * slices;
    fac[i] = pb[s * stride + hr * (D + 2) + D];
    lsum[i] = pb[s * stride + hr * (D + 2) + D + 1];
  }
  __syncthreads();
  if (tid < HN) {   // this head's max over the slices, its factors, and its denominator in slice order
    float *fh = fac + tid * slices;
    const float *lh = lsum + tid * slices;
    float M = -INFINITY;
    for (int s = 0; s < slices; ++s) M = fmaxf(M, fh[s]);
    float den = 0.f;
    for (int s = 0; s < slices; ++s) {
      const float f = (M == -INFINITY || fh[s] == -INFINITY) ? -1.f : __expf(fh[s] - M);
      fh[s] = f;
      if (f >= 0.f) den = fmaf(lh[s], f, den);
    }
    s_den[tid] = den;
  }
  __syncthreads();
  for (int d = tid; d < D; d += nt) {
    float num[HN];
#pragma unroll
    for (int hr = 0; hr < HN; ++hr) num[hr] = 0.f;
    constexpr int BATCH = HN >= 8 ? 2 : 16 / HN;   // 16 loads in flight per thread
    for (int s0 = 0; s0 < slices; s0 += BATCH) {
      float x[HN][BATCH];
#pragma unroll
      for (int hr = 0; hr < HN; ++hr)
#pragma unroll
        for (int j = 0; j < BATCH; ++j)
          x[hr][j] = s0 + j < slices ? pb[(s0 + j) * stride + hr * (D + 2) + d] : 0.f;
#pragma unroll
      for (int hr = 0; hr < HN; ++hr)
#pragma unroll
        for (int j = 0; j < BATCH; ++j)
          if (s0 + j < slices && fac[hr * slices + s0 + j] >= 0.f)
            num[hr] = fmaf(x[hr][j], fac[hr * slices + s0 + j], num[hr]);
    }
#pragma unroll
    for (int hr = 0; hr < HN; ++hr) {
      const float den = s_den[hr];
      static_cast<T *>(a.out)[(b * a.QH + kvh * HN + hr) * D + d] = from_f<T>(den > 0.f ? num[hr] / den : 0.f);
    }
  }
}

// the combine of every (row, KV head), one CTA each; its dynamic shared memory beyond the default
// 48 KB (R x slices > 6144) needs the attribute
template <typename T, int HN>
int combine_launch_hn(const SwaArgs &a, const float *part, int slices, bool pdl) {
  const size_t smem = combine_smem(slices, HN);
  auto k = swa_combine_kernel<T, HN>;
  if (smem > 227 * 1024) return set_error(YB_ERR_UNSUPPORTED, "swa combine: %d slices exceed shared memory", slices);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "swa combine: smem attribute: %s", cudaGetErrorString(e));
  }
  const dim3 grid(unsigned(a.B * a.KVH)), block(unsigned(a.D < 256 ? a.D : 256));
  if (pdl) {
    const cudaError_t e = launch_pdl(k, grid, block, smem, a.stream, a, part, slices);
    if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "swa_combine_kernel: %s", cudaGetErrorString(e));
  } else {
    k<<<grid, block, smem, a.stream>>>(a, part, slices);
  }
  return check_launch("swa_combine_kernel");
}

template <typename T>
int combine_launch(const SwaArgs &a, const float *part, int R, int slices, bool pdl) {
  switch (R) {
    case 1: return combine_launch_hn<T, 1>(a, part, slices, pdl);
    case 2: return combine_launch_hn<T, 2>(a, part, slices, pdl);
    case 4: return combine_launch_hn<T, 4>(a, part, slices, pdl);
    case 8: return combine_launch_hn<T, 8>(a, part, slices, pdl);
  }
  return set_error(YB_ERR_UNSUPPORTED, "swa combine: QH / KVH = %d not built (1/2/4/8)", R);
}

template <typename T, int R, int D>
int attn_launch(const SwaArgs &a, float *part, int slices) {
  const size_t smem = size_t(2) * kSwaSlice * (D * sizeof(T) + 16) + sizeof(float) * (R * (D + 4) + R * kSwaSlice + 2 * R);
  auto k = swa_partial_kernel<T, R, D>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "swa attention: smem attribute: %s", cudaGetErrorString(e));
  k<<<dim3(unsigned(a.B * a.KVH), unsigned(slices)), kSwaThreads, smem, a.stream>>>(a, part);
  int rc = check_launch("swa_partial_kernel");
  if (rc) return rc;
  return combine_launch<T>(a, part, R, slices, false);
}

template <typename T, int R>
int attn_r(const SwaArgs &a, float *part, int slices) {
  switch (a.D) {
    case 32: return attn_launch<T, R, 32>(a, part, slices);
    case 64: return attn_launch<T, R, 64>(a, part, slices);
    case 128: return attn_launch<T, R, 128>(a, part, slices);
    case 256: return attn_launch<T, R, 256>(a, part, slices);
  }
  return set_error(YB_ERR_UNSUPPORTED, "swa attention: head dim %lld not built (32/64/128/256)", (long long)a.D);
}

template <typename T>
int attn_t(const SwaArgs &a, float *part, int slices) {
  switch (a.QH / a.KVH) {
    case 1: return attn_r<T, 1>(a, part, slices);
    case 2: return attn_r<T, 2>(a, part, slices);
    case 4: return attn_r<T, 4>(a, part, slices);
    case 8: return attn_r<T, 8>(a, part, slices);
  }
  return set_error(YB_ERR_UNSUPPORTED, "swa attention: QH / KVH = %lld not built (1/2/4/8)",
                   (long long)(a.QH / a.KVH));
}

}  // namespace

int64_t swa_workspace_bytes(int64_t B, int64_t KVH, int64_t QH, int64_t W, int64_t D) {
  const int64_t slices = (W + kSwaSlice - 1) / kSwaSlice;
  return B * KVH * slices * (QH / (KVH > 0 ? KVH : 1)) * (D + 2) * int64_t(sizeof(float));
}

int launch_swa_ring_write(const SwaArgs &a) {
  if (a.B == 0) return YB_OK;
  const int64_t elem = a.dtype == YB_F32 ? 4 : 2;
  const int64_t n = 2 * a.B * a.KVH * (a.D * elem / 16) + a.B;
  const unsigned blocks = unsigned((n + 255) / 256);
  cudaError_t e;
  switch (a.dtype) {
    case YB_F32: e = launch_pdl(swa_ring_write_kernel<float>, dim3(blocks), dim3(256), 0, a.stream, a); break;
    case YB_BF16: e = launch_pdl(swa_ring_write_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, a.stream, a); break;
    case YB_F16: e = launch_pdl(swa_ring_write_kernel<__half>, dim3(blocks), dim3(256), 0, a.stream, a); break;
    default: return set_error(YB_ERR_ARGUMENT, "swa ring: bad dtype %d", a.dtype);
  }
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "swa_ring_write_kernel: %s", cudaGetErrorString(e));
  int rc = check_launch("swa_ring_write_kernel");
  if (rc) return rc;
  e = launch_pdl(swa_ring_advance_kernel, dim3(1), dim3(1), 0, a.stream, a);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "swa_ring_advance_kernel: %s", cudaGetErrorString(e));
  return check_launch("swa_ring_advance_kernel");
}

int launch_swa_decode_attention(const SwaArgs &a, void *workspace) {
  if (a.B * a.KVH == 0) return YB_OK;
  const int slices = int((a.W + kSwaSlice - 1) / kSwaSlice);
  float *part = static_cast<float *>(workspace);
  const auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (gqa_decode_mma_supported(a.dtype, a.QH, a.KVH, a.D) && a.ring_bs % 8 == 0 && a.ring_hs % 8 == 0 &&
      al16(a.query) && al16(a.ring_k) && al16(a.ring_v)) {
    // tensor-core slices, then the same combine pass
    GqaDecodeArgs g{};
    g.query = a.query;
    g.keys = a.ring_k;
    g.values = a.ring_v;
    g.kv_bs = a.ring_bs;
    g.kv_gs = a.ring_hs;
    g.valid = a.ring_valid;
    g.valid_bs = a.valid_bs;
    g.partial = part;
    g.B = a.B;
    g.G = a.KVH;
    g.QH = a.QH;
    g.D = a.D;
    g.P = a.W;
    g.dtype = a.dtype;
    g.stream = a.stream;
    int rc = launch_gqa_decode_mma(g);
    if (rc) return rc;
    const int R = int(a.QH / a.KVH);
    return a.dtype == YB_BF16 ? combine_launch<__nv_bfloat16>(a, part, R, slices, true)
                              : combine_launch<__half>(a, part, R, slices, true);
  }
  switch (a.dtype) {
    case YB_F32: return attn_t<float>(a, part, slices);
    case YB_BF16: return attn_t<__nv_bfloat16>(a, part, slices);
    case YB_F16: return attn_t<__half>(a, part, slices);
  }
  return set_error(YB_ERR_ARGUMENT, "swa attention: bad dtype %d", a.dtype);
}

}  // namespace yb
