// Grouped-query decode attention on warp-level tensor cores (mma.sync
// m16n8k16, bf16 / fp16 in, fp32 accumulate): the R query heads of one KV
// group attend to a slice of up to 64 stored positions.  Shared by the
// anchor-memory decode read (one 64-slot slice per (row, group), the null
// slot folded into the softmax, output written directly; semantics of
// modeling_yanchor.py:283-290 and runtime/model/independent_memory.py:47-88)
// and the sliding-window ring decode (64-position slices, partial results
// merged by swa_combine_kernel; runtime/model/inference_kernels.py:1881-1897).
//
// Per CTA (4 warps): K, V slice rows arrive by cp.async in padded shared rows
// (row stride D*2+16 bytes: every ldmatrix phase touches 8 distinct banks
// groups).  Warp w computes S^T = K Q^T for positions 16w..16w+15 (A = K rows,
// B = Q padded to 8 heads), the CTA takes the per-head max and exp-sum, P goes
// to shared memory as bf16 hi + lo, and O^T = V^T P^T (A = V rows through
// ldmatrix.trans, B = P) gives each warp a quarter of the D columns.
#include "common.cuh"
#include "kernels.h"
#include "mem_commit.cuh"

namespace yb {

namespace {

constexpr int kGqaThreads = 128;
constexpr int kGqaSlice = 64;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t *r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t *r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t *r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
template <typename T>
__device__ __forceinline__ void mma16816(float *c, const uint32_t *a, const uint32_t *b);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float *c, const uint32_t *a, const uint32_t *b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float *c, const uint32_t *a, const uint32_t *b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void cp16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// The commit of group g after its read, in the read's CTA.  Push (key, value, score) into pending
// slot `count`; when the chunk fills, rank the CAP bank slots and the `chunk` pending slots (score
// descending, position ascending with empty slots last, then candidate index: the stable double
// argsort of select_topk, modeling_yanchor.py:51-55) and write the new bank.  The old bank's key and
// value rows are still in shared memory from the read (rows of ROW elements in sk / sv): a new slot won
// by an old row is one bulk copy from there to the bank; the slots won by pending rows are copied by
// the threads, all their loads in flight together.
// Candidate arrays live over the query / P rows (`cand`, free once the read's MMAs are done).
// What the commit needs that does not depend on the read, loaded by every thread at the start of the
// kernel so that its memory latency hides behind the read: the row's flags and counters, this thread's
// piece of the new key / value row and, when the chunk fills, this thread's merge candidate (the
// pending rows are prefetched into L2 for the bank write).
struct CommitPrefetch {
  bool active;
  int64_t count, total;
  float new_score;
  uint4 kpiece, vpiece;
  float cand_score;
  int64_t cand_key;
};

template <typename T, int D>
__device__ CommitPrefetch commit_prefetch(const MemCommitArgs &a, int64_t row, int64_t s, int g) {
  const int tid = threadIdx.x, nt = blockDim.x;
  constexpr int VEC = 16 / int(sizeof(T));
  constexpr int DV = D / VEC;
  CommitPrefetch f{};
  f.active = a.active[row] != 0;
  if (!f.active) return f;
  f.count = a.count[s * a.count_s0];
  f.total = a.total[s * a.count_s0];
  f.new_score = a.scores[row * a.G + g];
  if (tid < DV) {
    f.kpiece = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.key) + (row * a.G + g) * D + tid * VEC);
    f.vpiece = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.value) + (row * a.G + g) * D + tid * VEC);
  }
  if (f.count + 1 != a.chunk) return f;
  const int CAP = int(a.CAP);
  if (tid < CAP) {
    const int32_t pos = a.positions[s * a.meta_s0 + int64_t(g) * CAP + tid];
    f.cand_score = a.bank_scores[s * a.meta_s0 + int64_t(g) * CAP + tid];
    f.cand_key = pos < 0 ? INT64_MAX : int64_t(pos);
  } else if (tid < CAP + a.chunk) {
    const int i = tid - CAP;
    f.cand_score = i == f.count ? f.new_score : a.pscores[s * a.pmeta_s0 + int64_t(g) * a.PC + i];
    f.cand_key = f.total - f.count + i;
  }
  const char *pk = reinterpret_cast<const char *>(static_cast<const T *>(a.pkeys) + s * a.pkv_s0 + int64_t(g) * a.PC * D);
  const char *pv = reinterpret_cast<const char *>(static_cast<const T *>(a.pvalues) + s * a.pkv_s0 + int64_t(g) * a.PC * D);
  for (int64_t off = int64_t(tid) * 128; off < a.chunk * D * int64_t(sizeof(T)); off += int64_t(nt) * 128) {
    prefetch_l2(pk + off);
    prefetch_l2(pv + off);
  }
  return f;
}

template <typename T, int D, int ROW>
__device__ void commit_after_read(const MemCommitArgs &a, int64_t row, int64_t s, int g, const CommitPrefetch &f,
                                  const T *sk, const T *sv, unsigned char *cand) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int64_t count = f.count, total = f.total;
  const int CAP = int(a.CAP), chunk = int(a.chunk), G = int(a.G), PC = int(a.PC);
  T *bank_k = static_cast<T *>(a.keys) + s * a.kv_s0 + int64_t(g) * CAP * D;
  T *bank_v = static_cast<T *>(a.values) + s * a.kv_s0 + int64_t(g) * CAP * D;
  T *pend_k = static_cast<T *>(a.pkeys) + s * a.pkv_s0 + int64_t(g) * PC * D;
  T *pend_v = static_cast<T *>(a.pvalues) + s * a.pkv_s0 + int64_t(g) * PC * D;
  float *bscore = a.bank_scores + s * a.meta_s0 + int64_t(g) * CAP;
  int32_t *bpos = a.positions + s * a.meta_s0 + int64_t(g) * CAP;
  float *pscore = a.pscores + s * a.pmeta_s0 + int64_t(g) * PC;
  constexpr int VEC = 16 / int(sizeof(T));
  constexpr int DV = D / VEC;
  // push (16-byte pieces, loaded at the start: row starts are 16-byte aligned)
  if (tid < DV) {
    *reinterpret_cast<uint4 *>(pend_k + count * D + tid * VEC) = f.kpiece;
    *reinterpret_cast<uint4 *>(pend_v + count * D + tid * VEC) = f.vpiece;
  }
  const float new_score = f.new_score;
  if (tid == 0) pscore[count] = new_score;
  if (count + 1 != chunk) return;
  const int n = CAP + chunk;
  float *c_score = reinterpret_cast<float *>(cand);
  int64_t *c_pkey = reinterpret_cast<int64_t *>(cand + ((4 * n + 15) & ~15));
  int *sel = reinterpret_cast<int *>(reinterpret_cast<unsigned char *>(c_pkey) + 8 * n);
  if (tid < n) {   // this thread's candidate, loaded at the start
    c_score[tid] = f.cand_score;
    c_pkey[tid] = f.cand_key;
  }
  for (int c = nt + tid; c < n; c += nt) {   // any beyond one per thread
    if (c < CAP) {
      const int32_t pos = bpos[c];
      c_score[c] = bscore[c];
      c_pkey[c] = pos < 0 ? INT64_MAX : int64_t(pos);
    } else {
      const int i = c - CAP;   // every pending slot is filled when the chunk commits; slot `count` is new
      c_score[c] = i == count ? new_score : pscore[i];
      c_pkey[c] = total - count + i;
    }
  }
  __syncthreads();
  for (int c = tid; c < n; c += nt) {
    const float sc = c_score[c];
    const int64_t pkc = c_pkey[c];
    int r0 = 0, r1 = 0;
    int o = 0;
#pragma unroll 4
    for (; o + 1 < n; o += 2) {
      r0 += memcommit::cand_before(c_score[o], c_pkey[o], o, sc, pkc, c);
      r1 += memcommit::cand_before(c_score[o + 1], c_pkey[o + 1], o + 1, sc, pkc, c);
    }
    if (o < n) r0 += memcommit::cand_before(c_score[o], c_pkey[o], o, sc, pkc, c);
    if (r0 + r1 < CAP) sel[r0 + r1] = c;
  }
  __syncthreads();   // sel complete
  // the new slots whose winner is a pending row, in slot order (warp 0; CAP <= 64)
  int *plist = sel + CAP;
  int *npend = plist + CAP;
  if (tid < 32) {
    int base = 0;
    for (int r0 = 0; r0 < CAP; r0 += 32) {
      const int r = r0 + tid;
      bool from_pend = false;
      if (r < CAP) {
        const int c = sel[r];
        from_pend = c_pkey[c] != INT64_MAX && c >= CAP;
      }
      const unsigned m = __ballot_sync(0xffffffffu, from_pend);
      if (from_pend) plist[base + __popc(m & ((1u << tid) - 1u))] = r;
      base += __popc(m);
    }
    if (tid == 0) *npend = base;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the old bank rows are read below by bulk copies
  __syncthreads();      // sel, plist complete; every thread's push is visible to the pending loads below
  // (1) slots won by an old bank row (an empty winner copies old bank slot 0, as the reference): one
  //     bulk copy per row straight from the shared-memory row the read used
  if (tid < 2 * CAP) {
    const int r = tid % CAP, half = tid / CAP;
    const int c = sel[r];
    const int src = c_pkey[c] == INT64_MAX ? 0 : c;
    if (src < CAP) {
      T *dst = (half ? bank_v : bank_k) + r * D;
      const T *from = (half ? sv : sk) + src * ROW;
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                   "r"(static_cast<uint32_t>(__cvta_generic_to_shared(from))), "r"(uint32_t(D * sizeof(T)))
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  // (2) slots won by a pending row: each thread loads all its pieces (key and value rows together)
  //     before it stores them
  const int np = *npend;
  constexpr int PER = 8;
  for (int base = 0; base < np * 2 * DV; base += nt * PER) {
    uint4 buf[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = base + tid + i * nt;
      if (e < np * 2 * DV) {
        const int r = plist[e / (2 * DV)], rem = e % (2 * DV), half = rem / DV, d = (rem % DV) * VEC;
        buf[i] = *reinterpret_cast<const uint4 *>((half ? pend_v : pend_k) + (sel[r] - CAP) * D + d);
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = base + tid + i * nt;
      if (e < np * 2 * DV) {
        const int r = plist[e / (2 * DV)], rem = e % (2 * DV), half = rem / DV, d = (rem % DV) * VEC;
        *reinterpret_cast<uint4 *>((half ? bank_v : bank_k) + r * D + d) = buf[i];
      }
    }
  }
  for (int r = tid; r < CAP; r += nt) {
    const int c = sel[r];
    bscore[r] = c_score[c];
    bpos[r] = c_pkey[c] == INT64_MAX ? -1 : int32_t(c_pkey[c]);
  }
  // the bulk copies have read their rows and written the bank before the CTA goes on or exits
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <typename T, int R, int D, bool COMMIT>
__global__ void __launch_bounds__(kGqaThreads) gqa_decode_mma_kernel(const GqaDecodeArgs a, const MemCommitTail ct) {
  static_assert(R <= 8 && D % 64 == 0, "R <= 8 heads, D a multiple of 64");
  constexpr int ROW = D + 8;          // padded K / V / Q row (elements)
  constexpr int PROW = kGqaSlice + 8; // padded P row
  extern __shared__ __align__(16) unsigned char gqa_raw[];
  T *sk = reinterpret_cast<T *>(gqa_raw);                 // [64][ROW]
  T *sv = sk + kGqaSlice * ROW;                           // [64][ROW]
  T *sq = sv + kGqaSlice * ROW;                           // [8][ROW]
  T *sp = sq + 8 * ROW;                                   // [2][8][PROW]  P hi, P lo
  float *red = reinterpret_cast<float *>(sp + 2 * 8 * PROW);   // [4 warps][8] max, then [4][8] sums
  float *fin = red + 2 * 4 * 8;                                // [8] max, [8] 1 / denominator
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  const int64_t unit = blockIdx.x;                        // (row, group)
  const int64_t slice = blockIdx.y, p0 = slice * kGqaSlice;
  const int64_t b = unit / a.G, g = unit % a.G;
  if (!a.indices) {   // the slice's rows are known before the wait: warm L2 with them
    const char *k0 = reinterpret_cast<const char *>(static_cast<const T *>(a.keys) + b * a.kv_bs + g * a.kv_gs + p0 * D);
    const char *v0 = reinterpret_cast<const char *>(static_cast<const T *>(a.values) + b * a.kv_bs + g * a.kv_gs + p0 * D);
    const int64_t nb = (a.P - p0 < kGqaSlice ? a.P - p0 : kGqaSlice) * D * int64_t(sizeof(T));
    for (int64_t off = int64_t(tid) * 128; off < nb; off += kGqaThreads * 128) {
      prefetch_l2(k0 + off);
      prefetch_l2(v0 + off);
    }
  }
  // the stored row this CTA reads; a memory row may be skipped (index -1)
  pdl_wait();
  pdl_release();
  const int64_t s = a.indices ? a.indices[b] : b;
  const int np = int(a.P - p0 < kGqaSlice ? a.P - p0 : kGqaSlice);
  if (s < 0) {   // skipped request (memory read): zero output
    T *o = static_cast<T *>(a.out) + (b * a.QH + g * R) * D;
    for (int e = tid; e < R * D; e += kGqaThreads) o[e] = from_f<T>(0.f);
    return;
  }
  CommitPrefetch pre{};
  if constexpr (COMMIT) pre = commit_prefetch<T, D>(ct.c, b, s, int(g));
  const T *kb = static_cast<const T *>(a.keys) + s * a.kv_bs + g * a.kv_gs + p0 * D;
  const T *vb = static_cast<const T *>(a.values) + s * a.kv_bs + g * a.kv_gs + p0 * D;
  constexpr int PIECES = D / 8;
  for (int e = tid; e < np * PIECES; e += kGqaThreads) cp16(sk + (e / PIECES) * ROW + (e % PIECES) * 8, kb + e * 8);
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int e = tid; e < np * PIECES; e += kGqaThreads) cp16(sv + (e / PIECES) * ROW + (e % PIECES) * 8, vb + e * 8);
  asm volatile("cp.async.commit_group;" ::: "memory");
  // zero the rows a short slice leaves empty (their logits are masked; V must not hold NaNs)
  for (int e = np * PIECES + tid; e < kGqaSlice * PIECES; e += kGqaThreads) {
    *reinterpret_cast<uint4 *>(sk + (e / PIECES) * ROW + (e % PIECES) * 8) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4 *>(sv + (e / PIECES) * ROW + (e % PIECES) * 8) = make_uint4(0, 0, 0, 0);
  }
  const T *qg = static_cast<const T *>(a.query) + (b * a.QH + g * R) * D;
  for (int e = tid; e < 8 * PIECES; e += kGqaThreads) {
    const int h = e / PIECES, c = (e % PIECES) * 8;
    *reinterpret_cast<uint4 *>(sq + h * ROW + c) =
        h < R ? *reinterpret_cast<const uint4 *>(qg + h * D + c) : make_uint4(0, 0, 0, 0);
  }
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();

  // ---- S^T (16 positions x 8 heads per warp) ----
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const int pr = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), kc = 8 * (lane >> 4);
    const int qr = lane & 7, qc = 8 * ((lane >> 3) & 1);
#pragma unroll
    for (int k = 0; k < D; k += 16) {
      uint32_t af[4], bfr[2];
      ldsm_x4(smem_addr(sk + pr * ROW + k + kc), af);
      ldsm_x2(smem_addr(sq + qr * ROW + k + qc), bfr);
      mma16816<T>(sc, af, bfr);
    }
  }
  // this thread's entries: positions warp*16 + g8 (+8), heads 2 t4, 2 t4 + 1
  const float scale = rsqrtf(float(D));
  float m2[2];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int pos = warp * 16 + g8 + (j >> 1) * 8;
    bool ok = pos < np;
    if (ok) {
      if (a.positions) ok = a.positions[s * a.pos_bs + g * a.pos_gs + p0 + pos] >= 0;
      else ok = a.valid[b * a.valid_bs + p0 + pos] != 0;
    }
    sc[j] = ok ? sc[j] * scale : -INFINITY;
  }
  m2[0] = fmaxf(sc[0], sc[2]);
  m2[1] = fmaxf(sc[1], sc[3]);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    m2[0] = fmaxf(m2[0], __shfl_xor_sync(0xffffffffu, m2[0], o));
    m2[1] = fmaxf(m2[1], __shfl_xor_sync(0xffffffffu, m2[1], o));
  }
  if (g8 == 0) {
    red[warp * 8 + 2 * t4] = m2[0];
    red[warp * 8 + 2 * t4 + 1] = m2[1];
  }
  __syncthreads();
  if (tid < 8) {
    float m = fmaxf(fmaxf(red[tid], red[8 + tid]), fmaxf(red[16 + tid], red[24 + tid]));
    if (a.null_slot) m = fmaxf(m, 0.f);
    fin[tid] = m;
  }
  __syncthreads();
  // ---- P = exp(S - m) as bf16 hi + lo, and the exp-sums ----
  float l2[2] = {0.f, 0.f};
  T *phi = sp, *plo = sp + 8 * PROW;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int pos = warp * 16 + g8 + (j >> 1) * 8, h = 2 * t4 + (j & 1);
    const float m = fin[h];
    const float p = (sc[j] == -INFINITY || m == -INFINITY) ? 0.f : expf(sc[j] - m);
    l2[j & 1] += p;
    const T hi = from_f<T>(p);
    phi[h * PROW + pos] = hi;
    plo[h * PROW + pos] = from_f<T>(p - to_f(hi));
  }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l2[0] += __shfl_xor_sync(0xffffffffu, l2[0], o);
    l2[1] += __shfl_xor_sync(0xffffffffu, l2[1], o);
  }
  if (g8 == 0) {
    red[32 + warp * 8 + 2 * t4] = l2[0];
    red[32 + warp * 8 + 2 * t4 + 1] = l2[1];
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (tid < 8) {
    float l = red[32 + tid] + red[40 + tid] + red[48 + tid] + red[56 + tid];
    if (a.null_slot) l += expf(-fin[tid]);         // the null slot: logit 0, value 0
    fin[8 + tid] = l;
  }
  __syncthreads();

  // ---- O^T = V^T P^T: warp w owns D columns [w D/4, (w+1) D/4) ----
  constexpr int DW = D / 4, TILES = DW / 16;
  float acc[TILES][4];
#pragma unroll
  for (int t = 0; t < TILES; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
  {
    const int vp = (lane & 7) + 8 * (lane >> 4), vd = 8 * ((lane >> 3) & 1);
    const int pr = lane & 7, pc = 8 * ((lane >> 3) & 1);
#pragma unroll
    for (int k = 0; k < kGqaSlice; k += 16) {
      uint32_t bh[2], bl[2];
      ldsm_x2(smem_addr(phi + pr * PROW + k + pc), bh);
      ldsm_x2(smem_addr(plo + pr * PROW + k + pc), bl);
#pragma unroll
      for (int t = 0; t < TILES; ++t) {
        uint32_t af[4];
        ldsm_x4_t(smem_addr(sv + (k + vp) * ROW + warp * DW + t * 16 + vd), af);
        mma16816<T>(acc[t], af, bh);
        mma16816<T>(acc[t], af, bl);
      }
    }
  }
  // acc[t]: rows (D columns) warp*DW + 16 t + g8 (+8), cols (heads) 2 t4, 2 t4 + 1
  if (a.partial) {
    // SWA slice: unnormalised sums + the slice's max and exp-sum, for the combine pass
    float *part = a.partial + (unit * gridDim.y + slice) * (R * (D + 2));
#pragma unroll
    for (int t = 0; t < TILES; ++t)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int h = 2 * t4 + (j & 1), d = warp * DW + 16 * t + g8 + (j >> 1) * 8;
        if (h < R) part[h * (D + 2) + d] = acc[t][j];
      }
    if (tid < R) {
      part[tid * (D + 2) + D] = fin[tid];
      part[tid * (D + 2) + D + 1] = fin[8 + tid];
    }
  } else {
    T *o = static_cast<T *>(a.out) + (b * a.QH + g * R) * D;
#pragma unroll
    for (int t = 0; t < TILES; ++t)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int h = 2 * t4 + (j & 1), d = warp * DW + 16 * t + g8 + (j >> 1) * 8;
        if (h < R) {
          const float l = fin[8 + h];
          o[h * D + d] = from_f<T>(l > 0.f ? acc[t][j] / l : 0.f);
        }
      }
    if constexpr (COMMIT) {
      // This group's commit (push, and the merge when the chunk fills), right after its read: the
      // group's bank is read by this CTA alone, so every read of the step still sees the bank
      // from before the commit, as with a read launch followed by a commit launch.  The last of
      // the row's G CTAs to finish updates count / total, which all of them read first; its
      // arrival counter goes back to 0 for the next call.  The commit's buffers reuse the K / V
      // rows, which every warp is done with after the first barrier.
      const MemCommitArgs &c = ct.c;
      if (pre.active) {   // the same for the row's G CTAs
        const int64_t count = pre.count, total = pre.total;
        __syncthreads();   // every warp is done with the query / P rows and the V rows
        commit_after_read<T, D, ROW>(c, b, s, int(g), pre, sk, sv, reinterpret_cast<unsigned char *>(sq));
        __syncthreads();
        if (tid == 0) {
          __threadfence();
          if (atomicAdd(ct.arrive + b, 1) == int(a.G) - 1) {
            ct.arrive[b] = 0;
            c.count[s * c.count_s0] = count + 1 == c.chunk ? 0 : count + 1;
            c.total[s * c.count_s0] = total + 1;
          }
        }
      }
    }
  }
}

template <typename T, int R, int D, bool COMMIT>
int launch_gqa(const GqaDecodeArgs &a, const MemCommitTail &ct, unsigned slices) {
  constexpr int ROW = D + 8, PROW = kGqaSlice + 8;
  static_assert(kGqaSlice * ROW * sizeof(T) >= (sizeof(float) + sizeof(int64_t) + sizeof(int)) * memcommit::kMaxCand,
                "the commit's candidate arrays fit in the V rows");
  const size_t smem = sizeof(T) * (2 * kGqaSlice * ROW + 8 * ROW + 2 * 8 * PROW) + sizeof(float) * (64 + 16);
  auto k = gqa_decode_mma_kernel<T, R, D, COMMIT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gqa decode: smem attribute: %s", cudaGetErrorString(e));
  e = launch_pdl(k, dim3(unsigned(a.B * a.G), slices), dim3(kGqaThreads), smem, a.stream, a, ct);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gqa decode: %s", cudaGetErrorString(e));
  return check_launch("gqa_decode_mma_kernel");
}

template <typename T, int R, bool COMMIT>
int gqa_d(const GqaDecodeArgs &a, const MemCommitTail &ct, unsigned slices) {
  switch (a.D) {
    case 64: return launch_gqa<T, R, 64, COMMIT>(a, ct, slices);
    case 128: return launch_gqa<T, R, 128, COMMIT>(a, ct, slices);
    case 256: return launch_gqa<T, R, 256, COMMIT>(a, ct, slices);
  }
  return -1;
}

template <typename T, bool COMMIT>
int gqa_r(const GqaDecodeArgs &a, const MemCommitTail &ct, unsigned slices) {
  switch (a.QH / a.G) {
    case 1: return gqa_d<T, 1, COMMIT>(a, ct, slices);
    case 2: return gqa_d<T, 2, COMMIT>(a, ct, slices);
    case 4: return gqa_d<T, 4, COMMIT>(a, ct, slices);
    case 8: return gqa_d<T, 8, COMMIT>(a, ct, slices);
  }
  return -1;
}

}  // namespace

bool gqa_decode_mma_supported(int dtype, int64_t QH, int64_t G, int64_t D) {
  const int64_t R = G > 0 ? QH / G : 0;
  return (dtype == YB_BF16 || dtype == YB_F16) && (D == 64 || D == 128 || D == 256) &&
         (R == 1 || R == 2 || R == 4 || R == 8) && QH % G == 0;
}

int launch_gqa_decode_mma(const GqaDecodeArgs &a) {
  if (a.B * a.G == 0) return YB_OK;
  const unsigned slices = unsigned((a.P + kGqaSlice - 1) / kGqaSlice);
  if (!a.partial && slices != 1) return set_error(YB_ERR_UNSUPPORTED, "gqa decode: a direct read covers <= 64 slots");
  const MemCommitTail none{};
  const int rc = a.dtype == YB_BF16 ? gqa_r<__nv_bfloat16, false>(a, none, slices) : gqa_r<__half, false>(a, none, slices);
  if (rc < 0) return set_error(YB_ERR_UNSUPPORTED, "gqa decode: shape not built");
  return rc;
}

bool gqa_decode_commit_fits(const GqaDecodeArgs &a, const MemCommitArgs &c) {
  const int64_t n = c.CAP + c.chunk;
  const int64_t cand_bytes = ((4 * n + 15) & ~int64_t(15)) + 8 * n + 4 * c.CAP + 4 * c.CAP + 4;   // + plist, npend
  const int64_t room = 2 * (8 * (a.D + 8) + 2 * 8 * (kGqaSlice + 8));   // the query and P rows (16-bit)
  const uintptr_t al = reinterpret_cast<uintptr_t>(c.key) | reinterpret_cast<uintptr_t>(c.value) |
                       reinterpret_cast<uintptr_t>(c.keys) | reinterpret_cast<uintptr_t>(c.values) |
                       reinterpret_cast<uintptr_t>(c.pkeys) | reinterpret_cast<uintptr_t>(c.pvalues);
  return !a.partial && a.P <= kGqaSlice && a.B == c.B && a.G == c.G && a.indices == c.indices &&
         cand_bytes <= room && c.CAP == a.P && c.D == a.D && c.dtype == a.dtype && (al % 16) == 0 &&
         (c.kv_s0 % 8) == 0 && (c.pkv_s0 % 8) == 0;
}

int launch_gqa_decode_commit(const GqaDecodeArgs &a, const MemCommitArgs &c, int32_t *arrive) {
  if (a.B * a.G == 0) return YB_OK;
  if (!arrive || !gqa_decode_commit_fits(a, c))
    return set_error(YB_ERR_UNSUPPORTED, "gqa decode + commit: arguments do not describe one memory layer");
  const MemCommitTail ct{c, arrive};
  const int rc = a.dtype == YB_BF16 ? gqa_r<__nv_bfloat16, true>(a, ct, 1) : gqa_r<__half, true>(a, ct, 1);
  if (rc < 0) return set_error(YB_ERR_UNSUPPORTED, "gqa decode + commit: shape not built");
  return rc;
}

}  // namespace yb
