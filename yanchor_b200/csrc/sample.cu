// Final-logit sampling: greedy argmax and the top-k / top-p counter sampler,
// plus the dense presence penalty and the GDN gate kernel.
//
// Sampling follows runtime/model/inference_kernels.py:24-88: top-k of the
// (temperature-scaled) scores, softmax, top-p truncation (keep while the
// running sum before an entry is below top_p), renormalise, then the inverse
// CDF with the stateless counter uniform of (attempt id, step, seed, stream).
// Ties inside the top-k are ordered by ascending vocabulary index.
//
// Both samplers split each row over several CTAs: the first pass writes
// per-split candidates to the caller's workspace and the second reduces them
// per row, so a batch of 64 rows still fills the GPU.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace yb {
// Built-in scratch of the no-allocation greedy entry point: 16 bytes per
// (row, split) partial; 64 KiB covers up to 4096 rows.
constexpr int64_t kGreedyScratchBytes = 64 * 1024;
constexpr int kMaxDevices = 64;
static __device__ __align__(256) unsigned char g_greedy_scratch[kGreedyScratchBytes];
}  // namespace yb

namespace yb {
namespace {

constexpr int kNT = 256;
constexpr int kMaxTopK = 256;
constexpr int kTopkSpan = 16384;  // elements per CTA in the top-k first pass

struct Cand {
  float v;
  int32_t pad;
  int64_t i;
};
static_assert(sizeof(Cand) == 16, "candidate record is 16 bytes");

// Order-preserving map float -> uint32 (larger float, larger key).
__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ bool better(float v, int64_t i, float bv, int64_t bi) {
  return v > bv || (v == bv && i < bi);
}

int greedy_splits(int64_t B, int64_t vocab) {
  int64_t s = (1184 + B - 1) / B;   // ~8 CTAs per SM: enough loads in flight to stream the scores
  const int64_t cap = (vocab + 2047) / 2048;
  if (s > cap) s = cap;
  return int(s < 1 ? 1 : s);
}
int topk_splits(int64_t vocab, int64_t k) {
  int64_t s = (vocab + kTopkSpan - 1) / kTopkSpan;
  while (s > 1 && vocab / s < k) --s;  // every split holds at least k entries
  return int(s < 1 ? 1 : s);
}

// Range [lo, hi) of split `split` out of `splits` over n elements.
__host__ __device__ __forceinline__ void split_range(int64_t n, int splits, int split, int64_t &lo, int64_t &hi) {
  lo = n * split / splits;
  hi = n * (split + 1) / splits;
}

// ---------------------------------------------------------------- greedy ----
template <typename T>
__global__ void __launch_bounds__(kNT) greedy_partial_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                             int splits, Cand *ws) {
  pdl_wait();
  pdl_release();
  const int split = blockIdx.x;
  const int64_t b = blockIdx.y;
  int64_t lo, hi;
  split_range(vocab, splits, split, lo, hi);
  const T *row = scores + b * row_stride;
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  constexpr int VEC = 16 / sizeof(T);
  // align the vector part to 16 bytes
  int64_t head = lo;
  while (head < hi && (reinterpret_cast<uintptr_t>(row + head) & 15)) ++head;
  for (int64_t j = lo + threadIdx.x; j < head; j += kNT) {
    const float x = to_f(row[j]);
    if (better(x, j, best, bi)) { best = x; bi = j; }
  }
  const int64_t nvec = (hi - head) / VEC;
  // four vectors per pass, all loads issued before the compares
  int64_t u = threadIdx.x;
  for (; u + 3 * kNT < nvec; u += 4 * kNT) {
    float x[4][VEC];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int64_t i = head + (u + w * kNT) * VEC;
      if constexpr (VEC == 4) load4(reinterpret_cast<const float *>(row + i), x[w]);
      else load8(row + i, x[w]);
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int64_t i = head + (u + w * kNT) * VEC;
#pragma unroll
      for (int t = 0; t < VEC; ++t)
        if (better(x[w][t], i + t, best, bi)) { best = x[w][t]; bi = i + t; }
    }
  }
  for (; u < nvec; u += kNT) {
    const int64_t i = head + u * VEC;
    float x[VEC];
    if constexpr (VEC == 4) load4(reinterpret_cast<const float *>(row + i), x);
    else load8(row + i, x);
#pragma unroll
    for (int t = 0; t < VEC; ++t)
      if (better(x[t], i + t, best, bi)) { best = x[t]; bi = i + t; }
  }
  for (int64_t j = head + nvec * VEC + threadIdx.x; j < hi; j += kNT) {
    const float x = to_f(row[j]);
    if (better(x, j, best, bi)) { best = x; bi = j; }
  }
  __shared__ float sv[kNT / 32];
  __shared__ int64_t si[kNT / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, best, bi)) { best = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kNT / 32; ++w)
      if (better(sv[w], si[w], best, bi)) { best = sv[w]; bi = si[w]; }
    Cand c;
    c.v = best; c.pad = 0; c.i = bi;
    ws[b * splits + split] = c;
  }
}

__global__ void greedy_final_kernel(const Cand *ws, int splits, int64_t B, int64_t *out) {
  pdl_wait();
  pdl_release();
  const int64_t b = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int s = lane; s < splits; s += 32) {
    const Cand c = ws[b * splits + s];
    if (better(c.v, c.i, best, bi)) { best = c.v; bi = c.i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, best, bi)) { best = ov; bi = oi; }
  }
  if (lane == 0) out[b] = bi == INT64_MAX ? 0 : bi;
}

// ------------------------------------------------------ block radix select ---
// Among the n keys in shared memory find the K-th largest key `thr` (1 <= K
// <= n) and the number `gt` of keys strictly above it.  Four 8-bit passes;
// warp-aggregated shared-memory histograms.
__device__ void radix_select(const uint32_t *keys, int n, int K, int *hist, uint32_t &thr, int &gt) {
  __shared__ int s_digit, s_above;
  uint32_t prefix = 0, mask = 0;
  int remaining = K, above = 0;
  const int lane = threadIdx.x & 31;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kNT) hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < n; base += kNT) {
      const int i = base + threadIdx.x;
      int digit = -1;
      if (i < n) {
        const uint32_t k = keys[i];
        if ((k & mask) == prefix) digit = int((k >> shift) & 255u);
      }
      const unsigned peers = __match_any_sync(0xffffffffu, digit);
      if (digit >= 0 && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0, d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= remaining) break;
        acc += hist[d];
      }
      s_digit = d;
      s_above = acc;
    }
    __syncthreads();
    prefix |= uint32_t(s_digit) << shift;
    mask |= 255u << shift;
    remaining -= s_above;
    above += s_above;
    __syncthreads();
  }
  thr = prefix;
  gt = above;
}

// Exclusive block scan of one int per thread; returns the block total.
__device__ int block_exclusive_scan(int x, int &total) {
  __shared__ int warp_tot[kNT / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  int offset = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kNT / 32; ++w) {
    if (w < warp) offset += warp_tot[w];
    tot += warp_tot[w];
  }
  __syncthreads();
  total = tot;
  return offset + inc - x;
}

// Select the K largest of n (value, index) entries held in shared memory
// (keys = fkey(value)); ties at the threshold go to the smallest indices.
// Entries are scanned in the given order; when `index_ordered` is true the
// storage order is ascending index, so the first `need` ties in storage order
// are the smallest indices.  Writes K candidates to `outc` (any order).
__device__ void select_k(const uint32_t *keys, const float *vals, const int64_t *idx, int n, int K,
                         bool index_ordered, int *hist, Cand *outc) {
  uint32_t thr;
  int gt;
  radix_select(keys, n, K, hist, thr, gt);
  const int need = K - gt;  // ties to take
  const int per = (n + kNT - 1) / kNT;
  const int lo = min(n, int(threadIdx.x) * per), hi = min(n, lo + per);
  int cg = 0, ce = 0;
  for (int i = lo; i < hi; ++i) {
    cg += keys[i] > thr;
    ce += keys[i] == thr;
  }
  int tg, te;
  int og = block_exclusive_scan(cg, tg);
  int oe = block_exclusive_scan(ce, te);
  for (int i = lo; i < hi; ++i) {
    const uint32_t k = keys[i];
    if (k > thr) {
      Cand c;
      c.v = vals[i]; c.pad = 0; c.i = idx[i];
      outc[og++] = c;
    } else if (k == thr) {
      int rank = oe;
      if (!index_ordered) {  // rank among ties by index
        rank = 0;
        for (int j = 0; j < n; ++j) rank += keys[j] == thr && idx[j] < idx[i];
      }
      if (rank < need) {
        Cand c;
        c.v = vals[i]; c.pad = 0; c.i = idx[i];
        outc[gt + rank] = c;
      }
      ++oe;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kNT) topk_partial_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                           int splits, int K, Cand *ws) {
  extern __shared__ __align__(16) unsigned char tk_raw[];
  uint32_t *keys = reinterpret_cast<uint32_t *>(tk_raw);       // [span]
  float *vals = reinterpret_cast<float *>(keys + kTopkSpan);   // [span]
  __shared__ int hist[256];
  const int split = blockIdx.x;
  const int64_t b = blockIdx.y;
  int64_t lo, hi;
  split_range(vocab, splits, split, lo, hi);
  const int n = int(hi - lo);
  const T *row = scores + b * row_stride;
  for (int i = threadIdx.x; i < n; i += kNT) {
    const float x = to_f(row[lo + i]);
    vals[i] = x;
    keys[i] = fkey(x);
  }
  __syncthreads();
  // indices are implicit (lo + i): pass a null index array through a lambda-free path
  uint32_t thr;
  int gt;
  radix_select(keys, n, K, hist, thr, gt);
  const int need = K - gt;
  const int per = (n + kNT - 1) / kNT;
  const int a0 = min(n, int(threadIdx.x) * per), a1 = min(n, a0 + per);
  int cg = 0, ce = 0;
  for (int i = a0; i < a1; ++i) {
    cg += keys[i] > thr;
    ce += keys[i] == thr;
  }
  int tg, te;
  int og = block_exclusive_scan(cg, tg);
  int oe = block_exclusive_scan(ce, te);
  Cand *outc = ws + (b * splits + split) * int64_t(K);
  for (int i = a0; i < a1; ++i) {
    const uint32_t k = keys[i];
    if (k > thr || (k == thr && oe < need)) {
      Cand c;
      c.v = vals[i]; c.pad = 0; c.i = lo + i;
      outc[k > thr ? og : gt + oe] = c;
    }
    og += k > thr;
    oe += k == thr;
  }
}

// counter uniform of (attempt id, step, seed, stream): uint32 hash -> (w + 0.5) / 2^32
__device__ __forceinline__ float counter_uniform(int64_t attempt, int64_t step, int64_t seed, int64_t stream) {
  const uint32_t id = uint32_t(attempt), st = uint32_t(step);
  uint32_t state = id * 747796405u + st * 289133645u + uint32_t(seed) * 277803737u + uint32_t(stream) * 144269504u;
  const uint32_t shift = (state >> 28) + 4u;
  uint32_t word = ((state >> shift) ^ state) * 277803737u;
  word = (word >> 22) ^ word;
  const float u = float((double(word) + 0.5) / 4294967296.0);
  const float limit = 1.0f - 5.9604645e-08f;  // 1 - eps(float32) / 2
  return fminf(u, limit);
}

__global__ void __launch_bounds__(kNT) topk_final_kernel(const Cand *ws, int splits, int K, const int64_t *attempt,
                                                         const int64_t *steps, int64_t scalar_step, int64_t seed,
                                                         int64_t stream_id, float temperature, float top_p,
                                                         int64_t *out) {
  extern __shared__ __align__(16) unsigned char tf_raw[];
  const int M = splits * K;
  uint32_t *keys = reinterpret_cast<uint32_t *>(tf_raw);      // [M] at byte 0
  float *vals = reinterpret_cast<float *>(tf_raw + 4 * M);      // [M] at byte 4M
  int64_t *idx = reinterpret_cast<int64_t *>(tf_raw + 8 * M);   // [M] at byte 8M (8-byte aligned)
  __shared__ int hist[256];
  __shared__ Cand sel[kMaxTopK];
  __shared__ float sv[kMaxTopK];
  __shared__ int64_t si[kMaxTopK];
  const int64_t b = blockIdx.x;
  for (int i = threadIdx.x; i < M; i += kNT) {
    const Cand c = ws[b * M + i];
    vals[i] = c.v;
    idx[i] = c.i;
    keys[i] = fkey(c.v);
  }
  __syncthreads();
  select_k(keys, vals, idx, M, K, false, hist, sel);
  __syncthreads();
  // sort the K winners: value descending, index ascending
  for (int i = threadIdx.x; i < K; i += kNT) {
    const float v = sel[i].v;
    const int64_t ix = sel[i].i;
    int rank = 0;
    for (int j = 0; j < K; ++j) rank += better(sel[j].v, sel[j].i, v, ix);
    sv[rank] = v;
    si[rank] = ix;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // softmax of values / temperature (the division is monotone, so top-k is unchanged)
    const float m = sv[0] / temperature;
    float tot = 0.f;
    for (int i = 0; i < K; ++i) {
      const float e = expf(sv[i] / temperature - m);
      sv[i] = e;
      tot += e;
    }
    for (int i = 0; i < K; ++i) sv[i] /= tot;
    // top-p: keep while the running sum before the entry is below top_p
    double run = 0.0;
    float kept = 0.f;
    for (int i = 0; i < K; ++i) {
      const float p = sv[i];
      const bool keep = float(float(run + p) - p) < top_p;
      run += p;
      sv[i] = keep ? p : 0.f;
      kept += sv[i];
    }
    for (int i = 0; i < K; ++i) sv[i] /= kept;
    float tot2 = 0.f;
    for (int i = 0; i < K; ++i) tot2 += sv[i];
    for (int i = 0; i < K; ++i) sv[i] /= tot2;
    // inverse CDF with the counter uniform
    double cum = 0.0;
    float last = 0.f;
    for (int i = 0; i < K; ++i) {
      cum += sv[i];
      sv[i] = float(cum);
      last = sv[i];
    }
    const float u = counter_uniform(attempt[b], steps ? steps[b] : scalar_step, seed, stream_id);
    const float thr = fminf(u * last, nextafterf(last, 0.f));
    int rank = 0;
    while (rank < K - 1 && sv[rank] < thr) ++rank;
    out[b] = si[rank];
  }
}

// ---------------------------------------------------------------- misc ------
template <typename T>
__global__ void presence_kernel(T *scores, const uint8_t *seen, int64_t n, float penalty) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    if (seen[i]) scores[i] = from_f<T>(to_f(scores[i]) - penalty);
}

template <typename T>
__global__ void gates_kernel(const T *b, const T *a, int64_t b_rs, int64_t a_rs, const float *A_log,
                             const float *dt_bias, T *beta, float *g, int64_t rows, int64_t heads) {
  const int64_t n = rows * heads;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / heads, h = i % heads;
    const float bb = to_f(b[r * b_rs + h]);
    const float aa = to_f(a[r * a_rs + h]);
    beta[i] = from_f<T>(sigmoidf_(bb));
    g[i] = -expf(A_log[h]) * softplus20(aa + (dt_bias ? dt_bias[h] : 0.f));
  }
}

// ------------------------------------------------ whole-vocabulary CDF ------
// top_k <= 0 with top_p == 1 (runtime/model/inference_kernels.py:77-80):
// softmax(scores / temperature) over the whole vocabulary in index order,
// then the first index whose running sum reaches min(u * total,
// nextafter(total, 0)).  Pass 1: per (row, span) the max of x / T and the
// exp-sum relative to it (online, one read).  Pass 2, one CTA per row: join
// the spans, find the span where the running sum crosses the threshold, and
// scan that span in index order (block-wide prefix sums) for the index.
// The running sums are fp32 in a different order than a sequential cumsum;
// ids can differ only where the threshold lies within rounding distance of a
// CDF step.
struct SoftPart {
  float m, z;
};

__device__ __forceinline__ void join_soft(float &m, float &z, float m2, float z2) {
  const float mm = fmaxf(m, m2);
  z = (mm == -INFINITY) ? 0.f : z * __expf(m - mm) + z2 * __expf(m2 - mm);
  m = mm;
}

template <typename T>
__global__ void __launch_bounds__(kNT) cdf_partial_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                          int splits, float temperature, SoftPart *ws) {
  __shared__ float red_m[kNT / 32], red_z[kNT / 32];
  const int64_t b = blockIdx.y;
  const int64_t lo = int64_t(blockIdx.x) * kTopkSpan;
  const int64_t hi = lo + kTopkSpan < vocab ? lo + kTopkSpan : vocab;
  const T *row = scores + b * row_stride;
  float m = -INFINITY, z = 0.f;
  for (int64_t i = lo + threadIdx.x; i < hi; i += kNT) {
    const float x = to_f(row[i]) / temperature;
    if (x == -INFINITY) continue;              // masked logits add nothing (and -inf - -inf is NaN)
    if (x > m) {
      z = z * __expf(m - x) + 1.f;
      m = x;
    } else {
      z += __expf(x - m);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), z2 = __shfl_xor_sync(0xffffffffu, z, o);
    join_soft(m, z, m2, z2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_m[warp] = m;
    red_z[warp] = z;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY, Z = 0.f;
    for (int w = 0; w < kNT / 32; ++w) join_soft(M, Z, red_m[w], red_z[w]);
    ws[b * splits + blockIdx.x] = SoftPart{M, Z};
  }
}

template <typename T>
__global__ void __launch_bounds__(kNT) cdf_final_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                        int splits, float temperature, const SoftPart *ws,
                                                        const int64_t *attempt, const int64_t *steps,
                                                        int64_t scalar_step, int64_t seed, int64_t stream_id,
                                                        int64_t *out) {
  constexpr int PER = 8;                      // consecutive elements per thread per tile
  constexpr int TILE = kNT * PER;
  __shared__ float s_base, s_thr, s_M;
  __shared__ int s_split;
  __shared__ float warp_tot[kNT / 32];
  __shared__ int s_found;
  const int64_t b = blockIdx.x;
  const T *row = scores + b * row_stride;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, ws[b * splits + s].m);
    float Z = 0.f;
    for (int s = 0; s < splits; ++s) {
      const SoftPart p = ws[b * splits + s];
      Z += p.m == -INFINITY ? 0.f : p.z * __expf(p.m - M);
    }
    const float u = counter_uniform(attempt[b], steps ? steps[b] : scalar_step, seed, stream_id);
    const float thr = fminf(u * Z, nextafterf(Z, 0.f));
    // the span whose running sum first reaches the threshold
    float base = 0.f;
    int split = splits - 1;
    for (int s = 0; s < splits; ++s) {
      const SoftPart p = ws[b * splits + s];
      const float zs = p.m == -INFINITY ? 0.f : p.z * __expf(p.m - M);
      if (base + zs >= thr) {
        split = s;
        break;
      }
      base += zs;
    }
    s_base = base;
    s_thr = thr;
    s_M = M;
    s_split = split;
    s_found = 0x7fffffff;
  }
  __syncthreads();
  const float M = s_M, thr = s_thr;
  float base = s_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // scan from the chosen span onward (later spans only if rounding moved the crossing)
  for (int64_t t0 = int64_t(s_split) * kTopkSpan; t0 < vocab; t0 += TILE) {
    const int64_t i0 = t0 + int64_t(threadIdx.x) * PER;
    float e[PER], mine = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      e[j] = (i0 + j < vocab) ? __expf(to_f(row[i0 + j]) / temperature - M) : 0.f;
      mine += e[j];
    }
    // exclusive prefix of `mine` over the block
    float incl = mine;
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    float before = 0.f, tile_tot = 0.f;
    for (int w = 0; w < kNT / 32; ++w) {
      if (w < warp) before += warp_tot[w];
      tile_tot += warp_tot[w];
    }
    float run = base + before + (incl - mine);
    if (i0 < vocab && run + mine >= thr) {     // the crossing is in this thread's elements
      int hit = PER - 1;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        run += e[j];
        if (run >= thr) {
          hit = j;
          break;
        }
      }
      const int64_t idx = i0 + hit < vocab ? i0 + hit : vocab - 1;
      atomicMin(&s_found, int(idx));
    }
    __syncthreads();
    if (s_found != 0x7fffffff) break;
    base += tile_tot;
    __syncthreads();                           // warp_tot is rewritten by the next tile
  }
  if (threadIdx.x == 0) out[b] = s_found != 0x7fffffff ? int64_t(s_found) : vocab - 1;
}

template <typename T>
int cdf_t(const SampleArgs &a) {
  const int splits = int((a.vocab + kTopkSpan - 1) / kTopkSpan);
  SoftPart *ws = static_cast<SoftPart *>(a.workspace);
  cdf_partial_kernel<T><<<dim3(splits, unsigned(a.B)), kNT, 0, a.stream>>>(
      static_cast<const T *>(a.scores), a.row_stride, a.vocab, splits, a.temperature, ws);
  int rc = check_launch("cdf_partial_kernel");
  if (rc) return rc;
  cdf_final_kernel<T><<<unsigned(a.B), kNT, 0, a.stream>>>(static_cast<const T *>(a.scores), a.row_stride, a.vocab,
                                                          splits, a.temperature, ws, a.attempt_ids, a.steps,
                                                          a.scalar_step, a.seed, a.stream_id, a.out);
  return check_launch("cdf_final_kernel");
}

template <typename T>
int greedy_t(const SampleArgs &a) {
  const int splits = greedy_splits(a.B, a.vocab);
  Cand *ws = static_cast<Cand *>(a.workspace);
  cudaError_t e = launch_pdl(greedy_partial_kernel<T>, dim3(splits, unsigned(a.B)), dim3(kNT), 0, a.stream,
                             static_cast<const T *>(a.scores), a.row_stride, a.vocab, splits, ws);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "greedy_partial_kernel: %s", cudaGetErrorString(e));
  int rc = check_launch("greedy_partial_kernel");
  if (rc) return rc;
  e = launch_pdl(greedy_final_kernel, dim3(unsigned((a.B + 7) / 8)), dim3(256), 0, a.stream,
                 static_cast<const Cand *>(ws), splits, a.B, a.out);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "greedy_final_kernel: %s", cudaGetErrorString(e));
  return check_launch("greedy_final_kernel");
}

template <typename T>
int topk_t(const SampleArgs &a) {
  const int K = int(a.top_k);
  const int splits = topk_splits(a.vocab, K);
  Cand *ws = static_cast<Cand *>(a.workspace);
  const size_t smem1 = size_t(kTopkSpan) * 8;
  auto k1 = topk_partial_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem1));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "topk: smem attribute: %s", cudaGetErrorString(e));
  k1<<<dim3(splits, unsigned(a.B)), kNT, smem1, a.stream>>>(static_cast<const T *>(a.scores), a.row_stride, a.vocab,
                                                           splits, K, ws);
  int rc = check_launch("topk_partial_kernel");
  if (rc) return rc;
  const int M = splits * K;
  const size_t smem2 = size_t(M) * 8 + size_t(M + 1) * 8;
  e = cudaFuncSetAttribute(topk_final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem2));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "topk: smem attribute: %s", cudaGetErrorString(e));
  topk_final_kernel<<<unsigned(a.B), kNT, smem2, a.stream>>>(ws, splits, K, a.attempt_ids, a.steps, a.scalar_step,
                                                            a.seed, a.stream_id, a.temperature, a.top_p, a.out);
  return check_launch("topk_final_kernel");
}

// ------------------------------------------------- sorted nucleus ----------
// top_k > kMaxTopK, or top_k <= 0 with top_p < 1 (runtime/model/
// inference_kernels.py:85-88 through top_k_top_p_distribution :42-56 and
// sample_probabilities_counter :58-71): the reference sorts the top-k of
// z = x / T, takes their softmax, keeps the entries whose running mass before
// them is below top_p, renormalises and picks with the counter uniform in
// that sorted order.  Nothing is sorted here.  Every question about the
// sorted order is a quantile: "the element at which the running count (or
// mass) crosses a target".  Each is answered by a radix descent over the
// order-preserving 32-bit keys of z, 8 bits per level, with per-row
// histograms of counts and masses.  A mass is exp(z - z_max) in 2^-26 fixed
// point (the largest is 2^26), so every sum is an exact integer whatever the
// order of the atomic additions, and repeated calls give the same ids.
// Equal z are ordered by ascending index (a tie group has one mass per
// element, so which tie the target falls on is integer arithmetic; its index
// comes from one counting pass).  The steps, per row:
//   1. z_max (the largest key);
//   2. top_k < vocab: the k-th largest key kappa by count; Z = mass of the
//      top k (keys above kappa plus the first `need` ties of kappa);
//      otherwise Z = the mass of every element;
//   3. top_p < 1: the element where the running mass crosses ceil(top_p Z):
//      the kept set ends there; E = its mass up to and including that
//      element; otherwise E = Z;
//   4. theta = ceil(u E) (u the counter uniform), at most E: the element
//      where the running mass crosses theta is the sample.
// Elements outside the top-k set or beyond the kept set come later in the
// sorted order, so they never change where a target below Z (or E) falls,
// and the descents need no exclusion.  The running sums are exact where the
// reference's are fp32 in sorted order; ids can differ only where a target
// lies within that rounding of a boundary.  NaN scores count as -inf.
constexpr int kNucMaxSplits = 64;
constexpr float kNucScale = 67108864.f;   // 2^26

struct NucRow {
  unsigned maxkey, prefix, mask, found;
  int stage, pad;
  long long want, above_count, need, tie_rank;
  unsigned long long above_mass, Z, E;
  int hist_count[256];
  unsigned long long hist_mass[256];
  int split_ties[kNucMaxSplits];
};

__device__ __forceinline__ float nuc_z(float x, float temperature) {
  const float z = temperature == 1.f ? x : x / temperature;
  return z != z ? -INFINITY : z;
}
// inverse of fkey
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ uint32_t nuc_mass(float z, float zmax) {
  return zmax == -INFINITY ? 0u : uint32_t(rintf(__expf(z - zmax) * kNucScale));
}

__global__ void nuc_init_kernel(NucRow *rows, int64_t B) {
  const int64_t b = blockIdx.x;
  if (b >= B) return;
  NucRow &r = rows[b];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    r.hist_count[i] = 0;
    r.hist_mass[i] = 0ull;
  }
  if (threadIdx.x == 0) {
    r.maxkey = 0u; r.prefix = 0u; r.mask = 0u; r.found = 0u; r.stage = 0;
    r.want = 0; r.above_count = 0; r.need = 0; r.tie_rank = 0;
    r.above_mass = 0ull; r.Z = 0ull; r.E = 0ull;
  }
}

template <typename T>
__global__ void __launch_bounds__(kNT) nuc_max_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                      float temperature, NucRow *rows) {
  const int64_t b = blockIdx.y;
  const int64_t lo = int64_t(blockIdx.x) * kTopkSpan, hi = lo + kTopkSpan < vocab ? lo + kTopkSpan : vocab;
  const T *row = scores + b * row_stride;
  uint32_t best = 0u;
  for (int64_t i = lo + threadIdx.x; i < hi; i += kNT) best = max(best, fkey(nuc_z(to_f(row[i]), temperature)));
  best = __reduce_max_sync(0xffffffffu, best);
  if ((threadIdx.x & 31) == 0) atomicMax(&rows[b].maxkey, best);
}

// Histogram of the 8-bit digit at `shift` of the keys that match the row's prefix so far.
template <typename T>
__global__ void __launch_bounds__(kNT) nuc_hist_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                       float temperature, int shift, NucRow *rows) {
  __shared__ int h_count[256];
  __shared__ unsigned long long h_mass[256];
  const int64_t b = blockIdx.y;
  NucRow &r = rows[b];
  for (int i = threadIdx.x; i < 256; i += kNT) {
    h_count[i] = 0;
    h_mass[i] = 0ull;
  }
  __syncthreads();
  const uint32_t prefix = r.prefix, mask = r.mask;
  const float zmax = key_value(r.maxkey);
  const int64_t lo = int64_t(blockIdx.x) * kTopkSpan, hi = lo + kTopkSpan < vocab ? lo + kTopkSpan : vocab;
  const T *row = scores + b * row_stride;
  const int lane = threadIdx.x & 31;
  for (int64_t base = lo; base < hi; base += kNT) {
    const int64_t i = base + threadIdx.x;
    int digit = -1;
    uint32_t m = 0u;
    if (i < hi) {
      const float z = nuc_z(to_f(row[i]), temperature);
      const uint32_t k = fkey(z);
      if ((k & mask) == prefix) {
        digit = int((k >> shift) & 255u);
        m = nuc_mass(z, zmax);
      }
    }
    // one shared-memory update per distinct digit in the warp (peers share it; their masses fit 32 bits)
    const unsigned peers = __match_any_sync(0xffffffffu, digit);
    const unsigned msum = __reduce_add_sync(peers, m);
    if (digit >= 0 && lane == __ffs(peers) - 1) {
      atomicAdd(&h_count[digit], __popc(peers));
      atomicAdd(&h_mass[digit], (unsigned long long)msum);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += kNT) {
    if (h_count[i]) {
      atomicAdd(&r.hist_count[i], h_count[i]);
      atomicAdd(&r.hist_mass[i], h_mass[i]);
    }
  }
}

// One thread per row: pick the digit where the target falls, move the descent on, and after the last
// level finish the current question and set up the next one.
__global__ void nuc_pick_kernel(NucRow *rows, int64_t B, int level, int64_t top_k, int64_t vocab, float top_p,
                                const int64_t *attempt, const int64_t *steps, int64_t scalar_step, int64_t seed,
                                int64_t stream_id) {
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= B) return;
  NucRow &r = rows[b];
  const int shift = 24 - 8 * level;
  if (level == 0 && r.stage > 0 && r.Z == 0ull && top_k >= vocab) {
    // no top-k cut: Z is the mass of every element (the level-0 histogram covers them all)
    unsigned long long z = 0ull;
    for (int d = 0; d < 256; ++d) z += r.hist_mass[d];
    r.Z = z;
  }
  if (level == 0 && r.stage == 1) {
    const double t = ceil(double(top_p) * double(r.Z));
    r.want = (long long)(t < 1.0 ? 1.0 : t);
  }
  if (level == 0 && r.stage == 2) {
    if (r.E == 0ull) r.E = r.Z;
    const float u = counter_uniform(attempt[b], steps ? steps[b] : scalar_step, seed, stream_id);
    double t = ceil(double(u) * double(r.E));
    if (t < 1.0) t = 1.0;
    if (t > double(r.E)) t = double(r.E);
    r.want = (long long)t;
  }
  long long acc_c = 0;
  unsigned long long acc_m = 0ull;
  int d = 255;
  for (; d > 0; --d) {
    const long long c = r.hist_count[d];
    const unsigned long long m = r.hist_mass[d];
    if (r.stage == 0 ? (acc_c + c >= r.want) : (acc_m + m >= (unsigned long long)r.want)) break;
    acc_c += c;
    acc_m += m;
  }
  const long long ties = r.hist_count[d];
  const unsigned long long tie_mass = r.hist_mass[d];
  r.prefix |= uint32_t(d) << shift;
  r.mask |= 255u << shift;
  r.above_count += acc_c;
  r.above_mass += acc_m;
  r.want -= r.stage == 0 ? acc_c : (long long)acc_m;
  for (int i = 0; i < 256; ++i) {
    r.hist_count[i] = 0;
    r.hist_mass[i] = 0ull;
  }
  if (shift != 0) return;
  // the descent reached one key: r.prefix; `ties` elements share it, each of mass tie_mass / ties
  const unsigned long long each = ties > 0 ? tie_mass / (unsigned long long)ties : 0ull;
  const long long t = each ? (long long)(((unsigned long long)r.want + each - 1ull) / each) - 1 : 0;
  if (r.stage == 0) {
    r.need = r.want;                                   // ties of kappa inside the top k
    r.Z = r.above_mass + (unsigned long long)r.need * each;
    r.stage = top_p < 1.f ? 1 : 2;
  } else if (r.stage == 1) {
    r.E = r.above_mass + (unsigned long long)(t + 1) * each;
    r.stage = 2;
  } else {
    r.found = r.prefix;
    r.tie_rank = t < 0 ? 0 : t;
    r.stage = 3;
  }
  if (r.stage != 3) {
    r.prefix = r.mask = 0u;
    r.above_count = 0;
    r.above_mass = 0ull;
  }
}

// The first question of every row: `stage` 0 (the k-th largest by count, want = k) or a mass question.
__global__ void nuc_stage_kernel(NucRow *rows, int64_t B, int stage, int64_t k) {
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= B) return;
  rows[b].stage = stage;
  rows[b].want = stage == 0 ? k : 0;
}

// Ties of the selected key per split (in index order), then the row's pick.
template <typename T>
__global__ void __launch_bounds__(kNT) nuc_ties_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                       float temperature, NucRow *rows) {
  const int64_t b = blockIdx.y;
  const uint32_t found = rows[b].found;
  const int64_t lo = int64_t(blockIdx.x) * kTopkSpan, hi = lo + kTopkSpan < vocab ? lo + kTopkSpan : vocab;
  const T *row = scores + b * row_stride;
  int n = 0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += kNT) n += fkey(nuc_z(to_f(row[i]), temperature)) == found;
  int total;
  block_exclusive_scan(n, total);
  if (threadIdx.x == 0) rows[b].split_ties[blockIdx.x] = total;
}

template <typename T>
__global__ void __launch_bounds__(kNT) nuc_final_kernel(const T *scores, int64_t row_stride, int64_t vocab,
                                                        float temperature, int splits, NucRow *rows, int64_t *out) {
  const int64_t b = blockIdx.x;
  const NucRow &r = rows[b];
  long long rank = r.tie_rank;
  int s = 0;
  for (; s < splits - 1; ++s) {
    if (rank < r.split_ties[s]) break;
    rank -= r.split_ties[s];
  }
  const int64_t lo = int64_t(s) * kTopkSpan, hi = lo + kTopkSpan < vocab ? lo + kTopkSpan : vocab;
  const T *row = scores + b * row_stride;
  __shared__ long long pick;
  if (threadIdx.x == 0) pick = -1;
  __syncthreads();
  // walk the split in index order, kNT elements at a time, counting the ties before each
  long long seen = 0;
  for (int64_t base = lo; base < hi; base += kNT) {
    const int64_t i = base + threadIdx.x;
    const int hit = (i < hi && fkey(nuc_z(to_f(row[i]), temperature)) == r.found) ? 1 : 0;
    int total;
    const int before = block_exclusive_scan(hit, total);
    if (hit && seen + before == rank) pick = i;
    seen += total;
    __syncthreads();
    if (pick >= 0 || seen > rank) break;
  }
  if (threadIdx.x == 0) out[b] = pick >= 0 ? pick : lo;
}

template <typename T>
int nucleus_t(const SampleArgs &a) {
  const int splits = int((a.vocab + kTopkSpan - 1) / kTopkSpan);
  if (splits > kNucMaxSplits) return set_error(YB_ERR_UNSUPPORTED, "sample: vocabulary too large for the nucleus path");
  NucRow *rows = static_cast<NucRow *>(a.workspace);
  const T *sc = static_cast<const T *>(a.scores);
  const dim3 grid(unsigned(splits), unsigned(a.B));
  const unsigned pick_blocks = unsigned((a.B + 63) / 64);
  nuc_init_kernel<<<unsigned(a.B), 256, 0, a.stream>>>(rows, a.B);
  nuc_max_kernel<T><<<grid, kNT, 0, a.stream>>>(sc, a.row_stride, a.vocab, a.temperature, rows);
  const int64_t k_eff = a.top_k > 0 ? a.top_k : a.vocab;
  // the questions in order: [k-th by count] [top-p cut by mass] sample by mass; each is 4 levels
  const int first = k_eff < a.vocab ? 0 : (a.top_p < 1.f ? 1 : 2);
  // without a count question Z comes from the first mass histogram (it covers every element)
  nuc_stage_kernel<<<pick_blocks, 64, 0, a.stream>>>(rows, a.B, first, k_eff);
  for (int q = first; q <= 2; ++q) {
    if (q == 1 && a.top_p >= 1.f) continue;
    for (int level = 0; level < 4; ++level) {
      nuc_hist_kernel<T><<<grid, kNT, 0, a.stream>>>(sc, a.row_stride, a.vocab, a.temperature, 24 - 8 * level, rows);
      nuc_pick_kernel<<<pick_blocks, 64, 0, a.stream>>>(rows, a.B, level, k_eff, a.vocab, a.top_p, a.attempt_ids,
                                                        a.steps, a.scalar_step, a.seed, a.stream_id);
    }
  }
  nuc_ties_kernel<T><<<grid, kNT, 0, a.stream>>>(sc, a.row_stride, a.vocab, a.temperature, rows);
  nuc_final_kernel<T><<<unsigned(a.B), kNT, 0, a.stream>>>(sc, a.row_stride, a.vocab, a.temperature, splits, rows,
                                                          a.out);
  return check_launch("nuc_final_kernel");
}

}  // namespace

int64_t sample_workspace_bytes(int64_t B, int64_t vocab, int64_t top_k) {
  const int64_t g = int64_t(greedy_splits(B, vocab)) * B * int64_t(sizeof(Cand));
  int64_t t = 0;
  if (top_k > 1 && top_k <= kMaxTopK) t = int64_t(topk_splits(vocab, top_k)) * top_k * B * int64_t(sizeof(Cand));
  if (top_k <= 0) t = (vocab + kTopkSpan - 1) / kTopkSpan * B * int64_t(sizeof(SoftPart));
  if (top_k <= 0 || top_k > kMaxTopK) {   // the sorted-nucleus path
    const int64_t n = B * int64_t(sizeof(NucRow));
    t = t > n ? t : n;
  }
  return g > t ? g : t;
}

int launch_sample_cdf(const SampleArgs &a) {
  if (a.B == 0) return YB_OK;
  if (a.vocab >= 0x7fffffffLL) return set_error(YB_ERR_UNSUPPORTED, "sample: vocabulary too large");
  switch (a.dtype) {
    case YB_F32: return cdf_t<float>(a);
    case YB_BF16: return cdf_t<__nv_bfloat16>(a);
    case YB_F16: return cdf_t<__half>(a);
  }
  return set_error(YB_ERR_ARGUMENT, "sample: bad dtype %d", a.dtype);
}

int launch_sample_greedy(const SampleArgs &a) {
  if (a.B == 0) return YB_OK;
  switch (a.dtype) {
    case YB_F32: return greedy_t<float>(a);
    case YB_BF16: return greedy_t<__nv_bfloat16>(a);
    case YB_F16: return greedy_t<__half>(a);
  }
  return set_error(YB_ERR_ARGUMENT, "sample: bad dtype %d", a.dtype);
}

// ---- greedy argmax for callers that cannot allocate device memory ----------
// The per-split partial maxima live in this fixed array instead of a
// caller-provided workspace.  Every GPU that loads the library holds it until
// the process exits; all calls on a device share it, so calls that overlap on
// the GPU (different streams, no ordering between them) race on it.  Nothing
// in it needs to start at zero: every call writes each partial it reads.
int64_t greedy_builtin_scratch_bytes() { return kGreedyScratchBytes; }

namespace {
// Host code may not use g_greedy_scratch's address directly (the host-side
// name is only a stand-in); the device address comes from
// cudaGetSymbolAddress, looked up with the device current.  The lookup is
// cached per device together with the unique id of the CUDA context it was
// made in (cuCtxGetId: never reused within a process).  A context created
// later on that device, e.g. after cudaDeviceReset or by a caller's own
// driver-API context, has another id, so its first call looks the address up
// again instead of using one from a context that no longer exists.
typedef int (*CtxGetCurrentFn)(void **);
typedef int (*CtxGetIdFn)(void *, unsigned long long *);
std::mutex g_scratch_mu;
void *g_scratch_addr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

// unique id of the calling thread's current context, 0 if the driver cannot tell
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
    looked_up = true;
  }
  void *ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, &id) == 0) return id;
  return 0;
}
}  // namespace

int launch_sample_greedy_noalloc(const SampleArgs &a) {
  const int64_t need = sample_workspace_bytes(a.B, a.vocab, 1);
  if (need > kGreedyScratchBytes)
    return set_error(YB_ERR_UNSUPPORTED,
                     "sample_greedy_noalloc: %lld rows need %lld bytes of scratch; the built-in scratch holds %lld "
                     "(use yb_sample_greedy with a workspace)",
                     (long long)a.B, (long long)need, (long long)kGreedyScratchBytes);
  if (a.B == 0) return YB_OK;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "sample_greedy_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(YB_ERR_UNSUPPORTED, "sample_greedy_noalloc: device %d", dev);
  void *scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    const unsigned long long ctx = current_context_id();
    if (!g_scratch_addr[dev] || ctx == 0 || ctx != g_scratch_ctx[dev]) {
      void *p = nullptr;
      e = cudaGetSymbolAddress(&p, g_greedy_scratch);
      if (e != cudaSuccess)
        return set_error(YB_ERR_CUDA, "sample_greedy_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_scratch_addr[dev] = p;
      g_scratch_ctx[dev] = ctx;
    }
    scratch = g_scratch_addr[dev];
  }
  SampleArgs b = a;
  b.workspace = scratch;
  b.workspace_bytes = kGreedyScratchBytes;
  return launch_sample_greedy(b);
}

int launch_sample_nucleus(const SampleArgs &a) {
  if (a.B == 0) return YB_OK;
  if (a.vocab >= 0x7fffffffLL) return set_error(YB_ERR_UNSUPPORTED, "sample: vocabulary too large");
  switch (a.dtype) {
    case YB_F32: return nucleus_t<float>(a);
    case YB_BF16: return nucleus_t<__nv_bfloat16>(a);
    case YB_F16: return nucleus_t<__half>(a);
  }
  return set_error(YB_ERR_ARGUMENT, "sample: bad dtype %d", a.dtype);
}

int launch_sample_topk_topp(const SampleArgs &a) {
  if (a.B == 0) return YB_OK;
  if (a.top_k < 2) return set_error(YB_ERR_UNSUPPORTED, "sample: top_k=%lld below 2", (long long)a.top_k);
  if (a.top_k > kMaxTopK) return launch_sample_nucleus(a);   // beyond the sorted top-k buffers
  const int M = topk_splits(a.vocab, a.top_k) * int(a.top_k);
  if (size_t(M) * 16 + 8 > 200 * 1024) return launch_sample_nucleus(a);
  switch (a.dtype) {
    case YB_F32: return topk_t<float>(a);
    case YB_BF16: return topk_t<__nv_bfloat16>(a);
    case YB_F16: return topk_t<__half>(a);
  }
  return set_error(YB_ERR_ARGUMENT, "sample: bad dtype %d", a.dtype);
}

int launch_presence_penalty(void *scores, const uint8_t *seen, int64_t n, float penalty, int dtype,
                            cudaStream_t stream) {
  if (n == 0 || penalty == 0.f) return YB_OK;
  const unsigned grid = unsigned(((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16));
  switch (dtype) {
    case YB_F32: presence_kernel<float><<<grid, 256, 0, stream>>>(static_cast<float *>(scores), seen, n, penalty); break;
    case YB_BF16: presence_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<__nv_bfloat16 *>(scores), seen, n, penalty); break;
    case YB_F16: presence_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<__half *>(scores), seen, n, penalty); break;
    default: return set_error(YB_ERR_ARGUMENT, "presence penalty: bad dtype %d", dtype);
  }
  return check_launch("presence_kernel");
}

int launch_gdn_gates(const void *b, const void *a, int64_t b_rs, int64_t a_rs, const float *A_log,
                     const float *dt_bias, void *beta_out, float *g_out, int64_t rows, int64_t heads, int io_dtype,
                     cudaStream_t stream) {
  const int64_t n = rows * heads;
  if (n == 0) return YB_OK;
  const unsigned grid = unsigned(((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16));
  switch (io_dtype) {
#define YB_GATES(T) \
  gates_kernel<T><<<grid, 256, 0, stream>>>(static_cast<const T *>(b), static_cast<const T *>(a), b_rs, a_rs, A_log, dt_bias, static_cast<T *>(beta_out), g_out, rows, heads)
    case YB_F32: YB_GATES(float); break;
    case YB_BF16: YB_GATES(__nv_bfloat16); break;
    case YB_F16: YB_GATES(__half); break;
#undef YB_GATES
    default: return set_error(YB_ERR_ARGUMENT, "gates: bad dtype %d", io_dtype);
  }
  return check_launch("gates_kernel");
}

}  // namespace yb
