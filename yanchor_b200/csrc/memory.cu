// Anchor memory ("independent GQA memory") kernels: decode read, decode
// write/commit and the prefill indexed read.
//
// Semantics follow modeling_yanchor.py:22-42 (indexed read), :51-63 (top-k
// selection order) and :277-313 (decode read / commit), and the Triton
// kernels of runtime/model/independent_memory.py.  Every softmax includes
// the null slot: one extra logit 0 whose value row is zero.
#include "common.cuh"
#include "kernels.h"
#include "mem_commit.cuh"

namespace yb {
namespace {

// ---------------------------------------------------------------------------
// Decode read: one CTA per (request row, group).  R = H / G query rows read
// the CAP committed slots of their group.
// ---------------------------------------------------------------------------
constexpr int kReadThreads = 128;

template <typename T, int R, int D>
__global__ void __launch_bounds__(kReadThreads) mem_decode_read_kernel(const MemReadArgs a) {
  constexpr int NW = kReadThreads / 32;
  constexpr int DL = D / 8;  // lanes covering one row (8 elements each)
  static_assert(D % 8 == 0 && DL <= 32, "D must be a multiple of 8, at most 256");
  extern __shared__ __align__(16) float rsm[];
  const int CAP = int(a.CAP);
  float *sq = rsm;                // [R][D]
  float *sw = sq + R * D;         // [R][CAP] logits -> weights
  float *part = sw + R * CAP;     // [NW][R][D] partial outputs
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x / a.G;
  const int g = int(blockIdx.x % a.G);
  const int64_t s = a.indices ? a.indices[row] : row;
  const T *qp = static_cast<const T *>(a.query) + (row * a.H + int64_t(g) * R) * D;
  T *outp = static_cast<T *>(a.out) + (row * a.H + int64_t(g) * R) * D;
  if (s < 0) {  // skipped request: zeros
    for (int e = tid; e < R * D; e += kReadThreads) outp[e] = from_f<T>(0.f);
    return;
  }
  const T *kp = static_cast<const T *>(a.keys) + s * a.kv_s0 + int64_t(g) * CAP * D;
  const T *vp = static_cast<const T *>(a.values) + s * a.kv_s0 + int64_t(g) * CAP * D;
  const int32_t *pp = a.positions + s * a.pos_s0 + int64_t(g) * CAP;
  for (int e = tid; e < R * D; e += kReadThreads) sq[e] = to_f(qp[e]);
  __syncthreads();
  const float scale = rsqrtf(float(D));
  // logits: a warp per slot, lanes split D
  for (int slot = warp; slot < CAP; slot += NW) {
    float kv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (lane < DL) load8(kp + int64_t(slot) * D + lane * 8, kv);
    const bool valid = pp[slot] >= 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float acc = 0.f;
      if (lane < DL) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(sq[r * D + lane * 8 + j], kv[j], acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) sw[r * CAP + slot] = valid ? acc * scale : -INFINITY;
    }
  }
  __syncthreads();
  // softmax with the null logit 0: a warp per query row
  for (int r = warp; r < R; r += NW) {
    float m = 0.f;
    for (int j = lane; j < CAP; j += 32) m = fmaxf(m, sw[r * CAP + j]);
    m = warp_max(m);
    float den = 0.f;
    for (int j = lane; j < CAP; j += 32) {
      const float e = expf(sw[r * CAP + j] - m);
      sw[r * CAP + j] = e;
      den += e;
    }
    den = warp_sum(den) + expf(-m);
    const float inv = 1.f / den;
    for (int j = lane; j < CAP; j += 32) sw[r * CAP + j] *= inv;
  }
  __syncthreads();
  // weighted values: each warp takes a strided subset of slots; lanes split D
  if (lane < DL) {
    float acc[R][8];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[r][j] = 0.f;
    for (int slot = warp; slot < CAP; slot += NW) {
      float vv[8];
      load8(vp + int64_t(slot) * D + lane * 8, vv);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float w = sw[r * CAP + slot];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[r][j] = fmaf(w, vv[j], acc[r][j]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < 8; ++j) part[(warp * R + r) * D + lane * 8 + j] = acc[r][j];
  }
  __syncthreads();
  for (int e = tid; e < R * D; e += kReadThreads) {
    float x = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) x += part[w * R * D + e];
    outp[e] = from_f<T>(x);
  }
}

// ---------------------------------------------------------------------------
// Decode read, staged: the same read with the whole bank of a (row, group)
// (CAP key rows and CAP value rows) put in flight at once by cp.async into
// padded shared-memory rows, so one CTA's 2*CAP*D*sizeof(T) bytes stream at
// once instead of one dependent row load per warp iteration.  Logits: one
// (slot, head) pair per thread (the 16-byte row padding makes the 8 slots a
// warp touches hit different banks); softmax: a warp per head; weighted
// values: one feature column per thread for all R heads.  Used whenever the
// staged bank fits in shared memory.
// ---------------------------------------------------------------------------
constexpr int kStageThreads = 256;

__device__ __forceinline__ void cp_async16_mem(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

template <typename T, int R, int D>
__global__ void __launch_bounds__(kStageThreads) mem_decode_read_staged_kernel(const MemReadArgs a) {
  constexpr int ROWB = D * int(sizeof(T)) + 16;   // padded row bytes
  constexpr int PIECES = D * int(sizeof(T)) / 16;
  constexpr int QP = D + 4;                       // padded q row (floats)
  extern __shared__ __align__(16) unsigned char st_raw[];
  const int CAP = int(a.CAP);
  unsigned char *sk = st_raw;                                     // [CAP][ROWB]
  unsigned char *sv = sk + size_t(CAP) * ROWB;                    // [CAP][ROWB]
  float *sq = reinterpret_cast<float *>(sv + size_t(CAP) * ROWB); // [R][QP]
  float *sw = sq + R * QP;                                        // [R][CAP]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x / a.G;
  const int g = int(blockIdx.x % a.G);
  if (!a.indices) {   // the bank's rows are known before the wait: warm L2 with them
    const unsigned char *k0 = reinterpret_cast<const unsigned char *>(static_cast<const T *>(a.keys) + row * a.kv_s0 +
                                                                       int64_t(g) * a.CAP * D);
    const unsigned char *v0 = reinterpret_cast<const unsigned char *>(static_cast<const T *>(a.values) + row * a.kv_s0 +
                                                                       int64_t(g) * a.CAP * D);
    for (int64_t off = int64_t(tid) * 128; off < a.CAP * D * int64_t(sizeof(T)); off += kStageThreads * 128) {
      prefetch_l2(k0 + off);
      prefetch_l2(v0 + off);
    }
  }
  pdl_wait();
  pdl_release();
  const int64_t s = a.indices ? a.indices[row] : row;
  const T *qp = static_cast<const T *>(a.query) + (row * a.H + int64_t(g) * R) * D;
  T *outp = static_cast<T *>(a.out) + (row * a.H + int64_t(g) * R) * D;
  if (s < 0) {  // skipped request: zeros
    for (int e = tid; e < R * D; e += kStageThreads) outp[e] = from_f<T>(0.f);
    return;
  }
  const unsigned char *kp =
      reinterpret_cast<const unsigned char *>(static_cast<const T *>(a.keys) + s * a.kv_s0 + int64_t(g) * CAP * D);
  const unsigned char *vp =
      reinterpret_cast<const unsigned char *>(static_cast<const T *>(a.values) + s * a.kv_s0 + int64_t(g) * CAP * D);
  const int32_t *pp = a.positions + s * a.pos_s0 + int64_t(g) * CAP;
  for (int e = tid; e < CAP * PIECES; e += kStageThreads) {
    const int slot = e / PIECES, pc = e % PIECES;
    cp_async16_mem(sk + slot * ROWB + pc * 16, kp + (size_t(slot) * D * sizeof(T) + pc * 16));
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int e = tid; e < CAP * PIECES; e += kStageThreads) {
    const int slot = e / PIECES, pc = e % PIECES;
    cp_async16_mem(sv + slot * ROWB + pc * 16, vp + (size_t(slot) * D * sizeof(T) + pc * 16));
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int e = tid; e < R * D; e += kStageThreads) sq[(e / D) * QP + e % D] = to_f(qp[e]);
  asm volatile("cp.async.wait_group 1;" ::: "memory");   // keys are in
  __syncthreads();
  const float scale = rsqrtf(float(D));
  for (int e = tid; e < CAP * R; e += kStageThreads) {
    const int slot = e / R, r = e % R;
    const T *krow = reinterpret_cast<const T *>(sk + slot * ROWB);
    const float *qr = sq + r * QP;
    float acc = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; d += 8) {
      float kx[8];
      load8(krow + d, kx);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = fmaf(qr[d + j], kx[j], acc);
    }
    sw[r * CAP + slot] = pp[slot] >= 0 ? acc * scale : -INFINITY;
  }
  __syncthreads();
  // softmax with the null logit 0: a warp per head
  for (int r = warp; r < R; r += kStageThreads / 32) {
    float m = 0.f;
    for (int j = lane; j < CAP; j += 32) m = fmaxf(m, sw[r * CAP + j]);
    m = warp_max(m);
    float den = 0.f;
    for (int j = lane; j < CAP; j += 32) {
      const float e = expf(sw[r * CAP + j] - m);
      sw[r * CAP + j] = e;
      den += e;
    }
    den = warp_sum(den) + expf(-m);
    const float inv = 1.f / den;
    for (int j = lane; j < CAP; j += 32) sw[r * CAP + j] *= inv;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");   // values are in
  __syncthreads();
  for (int d = tid; d < D; d += kStageThreads) {
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int slot = 0; slot < CAP; ++slot) {
      const float x = to_f(reinterpret_cast<const T *>(sv + slot * ROWB)[d]);
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = fmaf(sw[r * CAP + slot], x, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) outp[r * D + d] = from_f<T>(acc[r]);
  }
}

template <typename T, int R>
int launch_read_r(const MemReadArgs &a) {
  const size_t smem = sizeof(float) * (R * a.D + R * a.CAP + (kReadThreads / 32) * R * a.D);
  const size_t staged = size_t(a.CAP) * 2 * (a.D * sizeof(T) + 16) + sizeof(float) * (R * (a.D + 4) + R * a.CAP);
  dim3 grid(unsigned(a.B * a.G));
  switch (a.D) {
#define YB_READ_CASE(DD)                                                                           \
  case DD: {                                                                                       \
    if (staged <= 160 * 1024) {                                                                    \
      auto sk = mem_decode_read_staged_kernel<T, R, DD>;                                           \
      cudaError_t e = cudaFuncSetAttribute(sk, cudaFuncAttributeMaxDynamicSharedMemorySize, int(staged)); \
      if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "memory read: smem attribute: %s", cudaGetErrorString(e)); \
      e = launch_pdl(sk, grid, dim3(kStageThreads), staged, a.stream, a);                           \
      if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "memory read: %s", cudaGetErrorString(e)); \
      return check_launch("mem_decode_read_staged_kernel");                                        \
    }                                                                                              \
    auto kern = mem_decode_read_kernel<T, R, DD>;                                                  \
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)); \
    kern<<<grid, kReadThreads, smem, a.stream>>>(a);                                               \
    return check_launch("mem_decode_read_kernel");                                                 \
  }
    YB_READ_CASE(32)
    YB_READ_CASE(64)
    YB_READ_CASE(128)
    YB_READ_CASE(256)
#undef YB_READ_CASE
  }
  return set_error(YB_ERR_UNSUPPORTED, "memory read: D=%lld not built (32/64/128/256)", (long long)a.D);
}

template <typename T>
int launch_read_t(const MemReadArgs &a) {
  switch (a.H / a.G) {
    case 1: return launch_read_r<T, 1>(a);
    case 2: return launch_read_r<T, 2>(a);
    case 4: return launch_read_r<T, 4>(a);
    case 8: return launch_read_r<T, 8>(a);
  }
  return set_error(YB_ERR_UNSUPPORTED, "memory read: H/G=%lld not built (1/2/4/8)", (long long)(a.H / a.G));
}

// ---------------------------------------------------------------------------
// Decode commit: one CTA per request row (the row's work is
// memcommit::commit_row; the memory step's commit warps merge by the same order).
// ---------------------------------------------------------------------------
constexpr int kCommitThreads = 256;
constexpr int kMaxCand = memcommit::kMaxCand;

template <typename T>
__global__ void __launch_bounds__(kCommitThreads) mem_decode_commit_kernel(const MemCommitArgs a) {
  pdl_wait();
  pdl_release();
  __shared__ float c_score[kMaxCand];
  __shared__ int64_t c_pkey[kMaxCand];  // position, INT64_MAX for an invalid slot
  __shared__ int sel[kMaxCand];         // new slot -> winning candidate
  extern __shared__ __align__(16) unsigned char cm_raw[];
  memcommit::commit_row<T>(a, blockIdx.x, c_score, c_pkey, sel, reinterpret_cast<T *>(cm_raw));
}

template <typename T>
int launch_commit_t(const MemCommitArgs &a) {
  const size_t smem = sizeof(T) * a.CAP * a.D;
  auto kern = mem_decode_commit_kernel<T>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "memory commit: smem attribute: %s", cudaGetErrorString(e));
  }
  const cudaError_t le = launch_pdl(kern, dim3(unsigned(a.B)), dim3(kCommitThreads), smem, a.stream, a);
  if (le != cudaSuccess) return set_error(YB_ERR_CUDA, "memory commit: %s", cudaGetErrorString(le));
  return check_launch("mem_decode_commit_kernel");
}

// ---------------------------------------------------------------------------
// Prefill indexed read: one CTA per (row, block, group).  The referenced key
// and value rows are gathered once into shared memory; each warp then takes
// one chunk position at a time and computes the R heads of the group.
// ---------------------------------------------------------------------------
constexpr int kIdxThreads = 256;
constexpr int kIdxMaxCap = 128;

template <typename T, int R, int D>
__global__ void __launch_bounds__(kIdxThreads) mem_indexed_read_kernel(const MemIndexedArgs a) {
  constexpr int PITCH = D + 16 / int(sizeof(T));  // pad each row by 16 bytes (bank spread)
  constexpr int NW = kIdxThreads / 32;
  constexpr int DL = D / 8;
  constexpr int SL = kIdxMaxCap / 32;  // slots per lane (max)
  extern __shared__ __align__(16) unsigned char ir_raw[];
  const int CAP = int(a.CAP);
  T *sk = reinterpret_cast<T *>(ir_raw);     // [CAP][PITCH]
  T *sv = sk + CAP * PITCH;                  // [CAP][PITCH]
  float *sq = reinterpret_cast<float *>(sv + CAP * PITCH);  // [NW][R][D]
  __shared__ int svalid[kIdxMaxCap];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t gid = blockIdx.x;
  const int g = int(gid % a.G);
  const int64_t blk = (gid / a.G) % a.blocks;
  const int64_t b = gid / (a.G * a.blocks);
  const int64_t kb = a.KB == 1 ? 0 : b;
  const int64_t *refs = a.refs + gid * CAP;
  const T *kbase = static_cast<const T *>(a.key);
  const T *vbase = static_cast<const T *>(a.value);
  // gather referenced rows (16-byte vectors)
  for (int e = tid; e < CAP * (D / 8); e += kIdxThreads) {
    const int slot = e / (D / 8), d8 = (e % (D / 8)) * 8;
    const int64_t ref = refs[slot];
    float kx[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, vx[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const bool ok_ref = ref >= 0 && ref < a.S + a.S2;  // out-of-range references read as empty
    if (ok_ref) {
      if (ref < a.S) {
        const int64_t off = ((kb * a.S + ref) * a.G + g) * D + d8;
        load8(kbase + off, kx);
        load8(vbase + off, vx);
      } else {   // the second source (key batch 1)
        const int64_t off = ((ref - a.S) * a.G + g) * D + d8;
        load8(static_cast<const T *>(a.key2) + off, kx);
        load8(static_cast<const T *>(a.value2) + off, vx);
      }
    }
    store8(sk + slot * PITCH + d8, kx);
    store8(sv + slot * PITCH + d8, vx);
    if (d8 == 0) svalid[slot] = ok_ref;
  }
  __syncthreads();
  const float scale = rsqrtf(float(D));
  const T *qbase = static_cast<const T *>(a.query);
  T *obase = static_cast<T *>(a.out);
  float *myq = sq + warp * R * D;
  for (int c = warp; c < a.chunk; c += NW) {
    int64_t qrow = ((b * a.blocks + blk) * a.chunk + c) * a.H + int64_t(g) * R;  // first head row
    if (a.tok_shift) {           // timeline mode: slot -> token; only the write range is computed
      const int64_t s = blk * a.chunk + c, tok = s + a.tok_shift[b];
      if (s < a.w_lo[b] || s >= a.w_hi[b] || tok < 0 || tok >= a.T) continue;
      qrow = (b * a.T + tok) * a.H + int64_t(g) * R;
    }
    for (int e = lane; e < R * D; e += 32) myq[e] = to_f(qbase[qrow * D + e]);
    __syncwarp();
    // logits: lane owns slots lane, lane + 32, ...
    float lg[R][SL];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < SL; ++j) lg[r][j] = -INFINITY;
#pragma unroll
    for (int j = 0; j < SL; ++j) {
      const int slot = lane + 32 * j;
      if (slot < CAP && svalid[slot]) {
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.f;
        for (int d = 0; d < D; d += 8) {
          float kx[8];
          load8(sk + slot * PITCH + d, kx);
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[r] = fmaf(myq[r * D + d + t], kx[t], acc[r]);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) lg[r][j] = acc[r] * scale;
      }
    }
    // softmax with the null logit 0
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < SL; ++j) m = fmaxf(m, lg[r][j]);
      m = warp_max(m);
      float den = 0.f;
#pragma unroll
      for (int j = 0; j < SL; ++j) {
        lg[r][j] = expf(lg[r][j] - m);
        den += lg[r][j];
      }
      const float inv = 1.f / (warp_sum(den) + expf(-m));
#pragma unroll
      for (int j = 0; j < SL; ++j) lg[r][j] *= inv;
    }
    // weighted values: lanes split D
    float acc[R][8];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[r][t] = 0.f;
#pragma unroll
    for (int j = 0; j < SL; ++j) {
      for (int src = 0; src < 32; ++src) {
        const int slot = src + 32 * j;
        if (slot >= CAP) break;
        float w[R];
#pragma unroll
        for (int r = 0; r < R; ++r) w[r] = __shfl_sync(0xffffffffu, lg[r][j], src);
        if (lane < DL) {
          float vx[8];
          load8(sv + slot * PITCH + lane * 8, vx);
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[r][t] = fmaf(w[r], vx[t], acc[r][t]);
        }
      }
    }
    if (lane < DL) {
#pragma unroll
      for (int r = 0; r < R; ++r) store8(obase + (qrow + r) * D + lane * 8, acc[r]);
    }
    __syncwarp();
  }
}

template <typename T, int R>
int launch_indexed_r(const MemIndexedArgs &a) {
  dim3 grid(unsigned(a.B * a.blocks * a.G));
  switch (a.D) {
#define YB_IDX_CASE(DD)                                                                                 \
  case DD: {                                                                                            \
    constexpr int PITCH = DD + 16 / int(sizeof(T));                                                     \
    const size_t smem = 2 * sizeof(T) * a.CAP * PITCH + sizeof(float) * (kIdxThreads / 32) * R * DD;    \
    auto kern = mem_indexed_read_kernel<T, R, DD>;                                                      \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)); \
    if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "indexed read: smem attribute: %s", cudaGetErrorString(e)); \
    kern<<<grid, kIdxThreads, smem, a.stream>>>(a);                                                     \
    return check_launch("mem_indexed_read_kernel");                                                     \
  }
    YB_IDX_CASE(32)
    YB_IDX_CASE(64)
    YB_IDX_CASE(128)
    YB_IDX_CASE(256)
#undef YB_IDX_CASE
  }
  return set_error(YB_ERR_UNSUPPORTED, "indexed read: D=%lld not built (32/64/128/256)", (long long)a.D);
}

template <typename T>
int launch_indexed_t(const MemIndexedArgs &a) {
  switch (a.H / a.G) {
    case 1: return launch_indexed_r<T, 1>(a);
    case 2: return launch_indexed_r<T, 2>(a);
    case 4: return launch_indexed_r<T, 4>(a);
    case 8: return launch_indexed_r<T, 8>(a);
  }
  return set_error(YB_ERR_UNSUPPORTED, "indexed read: H/G=%lld not built (1/2/4/8)", (long long)(a.H / a.G));
}

}  // namespace

// a bank of at most 64 slots, 16-bit, aligned: the tensor-core read (one CTA per (row, group))
static bool mma_read_args(const MemReadArgs &a, GqaDecodeArgs &g) {
  const auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!(a.CAP <= 64 && gqa_decode_mma_supported(a.dtype, a.H, a.G, a.D) && a.kv_s0 % 8 == 0 && al16(a.query) &&
        al16(a.keys) && al16(a.values) && al16(a.out)))
    return false;
  g = GqaDecodeArgs{};
  g.query = a.query;
  g.keys = a.keys;
  g.values = a.values;
  g.kv_bs = a.kv_s0;
  g.kv_gs = a.CAP * a.D;
  g.positions = a.positions;
  g.pos_bs = a.pos_s0;
  g.pos_gs = a.CAP;
  g.indices = a.indices;
  g.out = a.out;
  g.null_slot = 1;
  g.B = a.B;
  g.G = a.G;
  g.QH = a.H;
  g.D = a.D;
  g.P = a.CAP;
  g.dtype = a.dtype;
  g.stream = a.stream;
  return true;
}

int launch_mem_decode_read(const MemReadArgs &a) {
  if (a.B * a.G == 0) return YB_OK;
  GqaDecodeArgs g;
  if (mma_read_args(a, g)) return launch_gqa_decode_mma(g);
  switch (a.dtype) {
    case YB_F32: return launch_read_t<float>(a);
    case YB_BF16: return launch_read_t<__nv_bfloat16>(a);
    case YB_F16: return launch_read_t<__half>(a);
  }
  return set_error(YB_ERR_ARGUMENT, "memory read: bad dtype %d", a.dtype);
}

int launch_mem_decode_commit(const MemCommitArgs &a) {
  if (a.B == 0) return YB_OK;
  if (a.CAP + a.chunk > kMaxCand)
    return set_error(YB_ERR_UNSUPPORTED, "memory commit: CAP + chunk = %lld exceeds %d",
                     (long long)(a.CAP + a.chunk), kMaxCand);
  switch (a.dtype) {
    case YB_F32: return launch_commit_t<float>(a);
    case YB_BF16: return launch_commit_t<__nv_bfloat16>(a);
    case YB_F16: return launch_commit_t<__half>(a);
  }
  return set_error(YB_ERR_ARGUMENT, "memory commit: bad dtype %d", a.dtype);
}

int launch_mem_decode_step(const MemReadArgs &r, const MemCommitArgs &c, int32_t *arrive) {
  GqaDecodeArgs g;
  if (r.B * r.G > 0 && arrive && c.CAP + c.chunk <= kMaxCand && mma_read_args(r, g) && gqa_decode_commit_fits(g, c))
    return launch_gqa_decode_commit(g, c, arrive);
  const int rc = launch_mem_decode_read(r);
  return rc != YB_OK ? rc : launch_mem_decode_commit(c);
}

int launch_mem_indexed_read(const MemIndexedArgs &a) {
  if (a.B * a.blocks * a.G == 0) return YB_OK;
  if (mem_indexed_tc_supported(a)) return launch_mem_indexed_tc(a);
  if (a.CAP > kIdxMaxCap)
    return set_error(YB_ERR_UNSUPPORTED, "indexed read: CAP=%lld exceeds %d", (long long)a.CAP, kIdxMaxCap);
  switch (a.dtype) {
    case YB_F32: return launch_indexed_t<float>(a);
    case YB_BF16: return launch_indexed_t<__nv_bfloat16>(a);
    case YB_F16: return launch_indexed_t<__half>(a);
  }
  return set_error(YB_ERR_ARGUMENT, "indexed read: bad dtype %d", a.dtype);
}

}  // namespace yb
