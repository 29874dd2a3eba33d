// Anchor-memory decode commit of one request row, for the commit kernel
// (memory.cu); the memory step's commit warps (gqa_decode_mma.cu) rank by
// the same order (`cand_before`)
// (runtime/model/independent_memory.py:190 `commit_decode`,
// modeling_yanchor.py:186-216 `_commit`, :229-251 `select_topk`).
//
// Push (key, value, score) of every group into pending slot `count`; when the
// chunk fills, merge the CAP bank slots and the `chunk` pending slots of each
// group into the new top-CAP bank.  Groups are independent: commit_group does
// one.  Order:
// score descending with NaN first (NaNs tie with each other, as in torch's
// descending sort), then position ascending (invalid last), then candidate
// index — the stable double argsort of select_topk.  It is a strict total
// order, so the ranks of the candidates are a permutation.  Invalid winners get
// position -1 and copy bank slot 0, as the reference's gather with references
// clamped at 0 does.  Every thread of the CTA calls these; loops stride by the
// CTA's thread count.
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace yb {
namespace memcommit {

constexpr int kMaxCand = 512;

__device__ __forceinline__ bool cand_before(float sa, int64_t pa, int ia, float sb, int64_t pb, int ib) {
  const bool na = sa != sa, nb = sb != sb;
  if (na != nb) return na;                 // NaN ahead of every number
  if (!na && sa != sb) return sa > sb;     // -0.0 == 0.0, as in a float sort
  if (pa != pb) return pa < pb;
  return ia < ib;
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

// The winning rows (bank slot or pending slot per new bank slot) into `stage`, then back over the
// bank.  With 16-byte aligned rows every piece is fetched by cp.async, all of them in flight at
// once, so the gather costs about one memory latency instead of one per piece a thread handles.
template <typename T>
__device__ void commit_gather(T *bank, const T *pend, T *stage, const int *sel, const int64_t *pkey, int g,
                              int CAP, int PC, int D) {
  const int tid = threadIdx.x, nt = blockDim.x;
  constexpr int VEC = 16 / int(sizeof(T));
  const bool vec = (D % VEC) == 0 && (reinterpret_cast<uintptr_t>(bank) % 16) == 0 &&
                   (reinterpret_cast<uintptr_t>(pend) % 16) == 0;
  if (vec) {
    const int DV = D / VEC;
    for (int e = tid; e < CAP * DV; e += nt) {
      const int r = e / DV, d = (e % DV) * VEC;
      const int c = sel[r];
      const int src = pkey[c] == INT64_MAX ? 0 : c;
      const T *from = src < CAP ? bank + (int64_t(g) * CAP + src) * D : pend + (int64_t(g) * PC + src - CAP) * D;
      cp_async16(stage + r * D + d, from + d);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    for (int e = tid; e < CAP * DV; e += nt)
      *reinterpret_cast<uint4 *>(bank + int64_t(g) * CAP * D + e * VEC) = *reinterpret_cast<const uint4 *>(stage + e * VEC);
    __syncthreads();
    return;
  }
  for (int e = tid; e < CAP * D; e += nt) {
    const int r = e / D, d = e % D;
    const int c = sel[r];
    const int src = pkey[c] == INT64_MAX ? 0 : c;
    stage[e] = src < CAP ? bank[(int64_t(g) * CAP + src) * D + d] : pend[(int64_t(g) * PC + src - CAP) * D + d];
  }
  __syncthreads();
  for (int e = tid; e < CAP * D; e += nt) bank[int64_t(g) * CAP * D + e] = stage[e];
  __syncthreads();
}

// Both banks at once: the key rows by cp.async into `stage`, the value rows into registers, all
// of them in flight together, then both written back.  Used when every thread holds at most
// kRegPieces value pieces (the YANchor shape: CAP 64, D 256, 128 threads -> 16); otherwise the
// two banks go one after the other through `stage`.
constexpr int kRegPieces = 16;

template <typename T>
__device__ void commit_gather_kv(T *bank_k, T *bank_v, const T *pend_k, const T *pend_v, T *stage, const int *sel,
                                 const int64_t *pkey, int g, int CAP, int PC, int D) {
  const int tid = threadIdx.x, nt = blockDim.x;
  constexpr int VEC = 16 / int(sizeof(T));
  const int DV = D / VEC;
  const bool vec = (D % VEC) == 0 && ((reinterpret_cast<uintptr_t>(bank_k) | reinterpret_cast<uintptr_t>(bank_v) |
                                       reinterpret_cast<uintptr_t>(pend_k) | reinterpret_cast<uintptr_t>(pend_v)) %
                                      16) == 0;
  if (!vec || CAP * DV > nt * kRegPieces) {
    commit_gather(bank_k, pend_k, stage, sel, pkey, g, CAP, PC, D);
    commit_gather(bank_v, pend_v, stage, sel, pkey, g, CAP, PC, D);
    return;
  }
  uint4 vreg[kRegPieces];
#pragma unroll
  for (int i = 0; i < kRegPieces; ++i) {
    const int e = tid + i * nt;
    if (e < CAP * DV) {
      const int r = e / DV, d = (e % DV) * VEC;
      const int c = sel[r];
      const int src = pkey[c] == INT64_MAX ? 0 : c;
      const int64_t off = src < CAP ? (int64_t(g) * CAP + src) * D : (int64_t(g) * PC + src - CAP) * D;
      cp_async16(stage + r * D + d, (src < CAP ? bank_k : pend_k) + off + d);
      vreg[i] = *reinterpret_cast<const uint4 *>((src < CAP ? bank_v : pend_v) + off + d);
    }
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kRegPieces; ++i) {
    const int e = tid + i * nt;
    if (e < CAP * DV) {
      *reinterpret_cast<uint4 *>(bank_k + int64_t(g) * CAP * D + e * VEC) = *reinterpret_cast<const uint4 *>(stage + e * VEC);
      *reinterpret_cast<uint4 *>(bank_v + int64_t(g) * CAP * D + e * VEC) = vreg[i];
    }
  }
  __syncthreads();
}

// Group g of request row `row` (state row s, active): push into pending slot `count` (unless
// PUSH is false: the caller pushed every group already), and merge when the chunk fills.
// count / total are read by the caller and not updated here.
// c_score, c_pkey, sel: kMaxCand entries each; stage: CAP * D elements (all shared memory).
template <typename T, bool PUSH = true>
__device__ void commit_group(const MemCommitArgs &a, int64_t row, int64_t s, int g, int64_t count, int64_t total,
                             float *c_score, int64_t *c_pkey, int *sel, T *stage) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int CAP = int(a.CAP), D = int(a.D), chunk = int(a.chunk), G = int(a.G), PC = int(a.PC);
  const bool commit = count + 1 == chunk;
  const T *key = static_cast<const T *>(a.key) + (row * G + g) * D;
  const T *val = static_cast<const T *>(a.value) + (row * G + g) * D;
  T *bank_k = static_cast<T *>(a.keys) + s * a.kv_s0;
  T *bank_v = static_cast<T *>(a.values) + s * a.kv_s0;
  T *pend_k = static_cast<T *>(a.pkeys) + s * a.pkv_s0;
  T *pend_v = static_cast<T *>(a.pvalues) + s * a.pkv_s0;
  float *bscore = a.bank_scores + s * a.meta_s0;
  int32_t *bpos = a.positions + s * a.meta_s0;
  float *pscore = a.pscores + s * a.pmeta_s0;

  if constexpr (PUSH) {
    // push into pending slot `count` (16-byte pieces when every row start is aligned)
    T *pk = pend_k + (int64_t(g) * PC + count) * D, *pv = pend_v + (int64_t(g) * PC + count) * D;
    constexpr int VEC = 16 / int(sizeof(T));
    const bool vec = (D % VEC) == 0 && (reinterpret_cast<uintptr_t>(key) % 16) == 0 &&
                     (reinterpret_cast<uintptr_t>(val) % 16) == 0 && (reinterpret_cast<uintptr_t>(pk) % 16) == 0 &&
                     (reinterpret_cast<uintptr_t>(pv) % 16) == 0;
    if (vec) {
      for (int e = tid * VEC; e < D; e += nt * VEC) {
        *reinterpret_cast<uint4 *>(pk + e) = *reinterpret_cast<const uint4 *>(key + e);
        *reinterpret_cast<uint4 *>(pv + e) = *reinterpret_cast<const uint4 *>(val + e);
      }
    } else {
      for (int e = tid; e < D; e += nt) {
        pk[e] = key[e];
        pv[e] = val[e];
      }
    }
    if (tid == 0) pscore[int64_t(g) * PC + count] = a.scores[row * G + g];
  }
  if (!commit) return;
  const int n = CAP + chunk;
  __syncthreads();  // the push is visible; the previous group's use of the candidate arrays is over
  for (int c = tid; c < n; c += nt) {
    if (c < CAP) {
      const int32_t pos = bpos[int64_t(g) * CAP + c];
      c_score[c] = bscore[int64_t(g) * CAP + c];
      c_pkey[c] = pos < 0 ? INT64_MAX : int64_t(pos);
    } else {
      const int i = c - CAP;  // every pending slot is filled when committing
      c_score[c] = pscore[int64_t(g) * PC + i];
      c_pkey[c] = total - count + i;
    }
  }
  __syncthreads();
  for (int c = tid; c < n; c += nt) {
    const float sc = c_score[c];
    const int64_t pkc = c_pkey[c];
    int rank = 0;
    for (int o = 0; o < n; ++o) rank += cand_before(c_score[o], c_pkey[o], o, sc, pkc, c);
    if (rank < CAP) sel[rank] = c;
  }
  __syncthreads();
  commit_gather_kv(bank_k, bank_v, pend_k, pend_v, stage, sel, c_pkey, g, CAP, PC, D);
  for (int r = tid; r < CAP; r += nt) {
    const int c = sel[r];
    bscore[int64_t(g) * CAP + r] = c_score[c];
    bpos[int64_t(g) * CAP + r] = c_pkey[c] == INT64_MAX ? -1 : int32_t(c_pkey[c]);
  }
}

// the whole row, every group in turn, then its count / total
template <typename T>
__device__ void commit_row(const MemCommitArgs &a, int64_t row, float *c_score, int64_t *c_pkey, int *sel,
                           T *stage) {
  const int64_t s = a.indices ? a.indices[row] : row;
  if (s < 0 || !a.active[row]) return;
  const int64_t count = a.count[s * a.count_s0];
  const int64_t total = a.total[s * a.count_s0];
  // push every group into pending slot `count` at once (16-byte pieces when every row start is aligned)
  const int tid = threadIdx.x, nt = blockDim.x, G = int(a.G), D = int(a.D), PC = int(a.PC);
  const T *key = static_cast<const T *>(a.key) + row * G * D;
  const T *val = static_cast<const T *>(a.value) + row * G * D;
  T *pend_k = static_cast<T *>(a.pkeys) + s * a.pkv_s0;
  T *pend_v = static_cast<T *>(a.pvalues) + s * a.pkv_s0;
  constexpr int VEC = 16 / int(sizeof(T));
  const bool vec = (D % VEC) == 0 && (reinterpret_cast<uintptr_t>(key) % 16) == 0 &&
                   (reinterpret_cast<uintptr_t>(val) % 16) == 0 && (reinterpret_cast<uintptr_t>(pend_k) % 16) == 0 &&
                   (reinterpret_cast<uintptr_t>(pend_v) % 16) == 0;
  if (vec) {
    for (int e = tid * VEC; e < G * D; e += nt * VEC) {
      const int g = e / D, d = e % D;
      const int64_t dst = (int64_t(g) * PC + count) * D + d;
      *reinterpret_cast<uint4 *>(pend_k + dst) = *reinterpret_cast<const uint4 *>(key + e);
      *reinterpret_cast<uint4 *>(pend_v + dst) = *reinterpret_cast<const uint4 *>(val + e);
    }
  } else {
    for (int e = tid; e < G * D; e += nt) {
      const int g = e / D, d = e % D;
      pend_k[(int64_t(g) * PC + count) * D + d] = key[e];
      pend_v[(int64_t(g) * PC + count) * D + d] = val[e];
    }
  }
  if (tid < G) a.pscores[s * a.pmeta_s0 + int64_t(tid) * PC + count] = a.scores[row * G + tid];
  for (int g = 0; g < G; ++g) commit_group<T, false>(a, row, s, g, count, total, c_score, c_pkey, sel, stage);
  __syncthreads();  // every thread has read count / total
  if (threadIdx.x == 0) {
    a.count[s * a.count_s0] = count + 1 == a.chunk ? 0 : count + 1;
    a.total[s * a.count_s0] = total + 1;
  }
}

}  // namespace memcommit
}  // namespace yb
