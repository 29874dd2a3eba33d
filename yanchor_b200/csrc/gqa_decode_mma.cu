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

// Named barriers of the memory step's CTA (barrier 0 is __syncthreads): the read warps (0-3) sync
// among themselves on 1, the commit warps (4-7) on 2, and the read warps arrive on 3 once the K / V
// rows have landed, where the commit warps wait for them.
constexpr int kBarRead = 1, kBarCommit = 2, kBarLanded = 3;
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// The commit of group g, run by four warps of the read's CTA beside the read (the memory step:
// committed_gqa then commit_decode in one launch).  Push (key, value, score) into pending slot
// `count`; when the chunk fills, rank the CAP bank slots and the `chunk` pending slots (score
// descending with NaN first, position ascending with empty slots last, then candidate index: the
// stable double argsort of select_topk, modeling_yanchor.py:51-55) and write the new bank.
//
// The rank needs nothing from the read, so it runs while the read computes: each candidate's
// (score, key) sits in the 16 spare bytes at the end of a K row (candidates 0..63) or V row
// (64..127), which no load, MMA or copy touches.  The bank is rewritten once the read's K / V rows
// have landed (so the read still sees the bank from before the commit): a new slot won by an old row
// is one bulk copy from the row the read holds in shared memory, the slots won by pending rows are
// copied by the threads, all their loads in flight together.  The read warps only read those rows,
// and read the positions they mask with before they arrive, so nothing the read uses is written
// under it.  The last of the row's G CTAs to finish updates count / total, which all of them read
// first; its arrival counter goes back to 0 for the next call.
struct CommitPrefetch {
  bool active;
  int64_t count, total;
  float new_score;
  uint4 kpiece, vpiece;
  float cand_score;
  int64_t cand_key;
};

// What the commit reads before it can do anything else (thread `t` of `nt` commit threads): the
// row's flags and counters, this thread's piece of the new key / value row and, when the chunk
// fills, this thread's merge candidate (the pending rows are prefetched into L2 for the bank write).
template <typename T, int D>
__device__ CommitPrefetch commit_prefetch(const MemCommitArgs &a, int64_t row, int64_t s, int g, int t, int nt) {
  constexpr int VEC = 16 / int(sizeof(T));
  constexpr int DV = D / VEC;
  CommitPrefetch f{};
  // every load in one round trip: the merge candidate is loaded before it is known whether the
  // chunk fills (a few bytes per thread, every address valid for a stored row)
  const int CAP = int(a.CAP);
  f.active = a.active[row] != 0;
  f.count = a.count[s * a.count_s0];
  f.total = a.total[s * a.count_s0];
  f.new_score = a.scores[row * a.G + g];
  if (t < DV) {
    f.kpiece = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.key) + (row * a.G + g) * D + t * VEC);
    f.vpiece = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.value) + (row * a.G + g) * D + t * VEC);
  }
  int32_t bpos = -1;
  float sc = 0.f;
  if (t < CAP) {
    bpos = a.positions[s * a.meta_s0 + int64_t(g) * CAP + t];
    sc = a.bank_scores[s * a.meta_s0 + int64_t(g) * CAP + t];
  } else if (t < CAP + a.chunk) {
    sc = a.pscores[s * a.pmeta_s0 + int64_t(g) * a.PC + (t - CAP)];
  }
  if (!f.active || f.count + 1 != a.chunk) return f;
  if (t < CAP) {
    f.cand_score = sc;
    f.cand_key = bpos < 0 ? INT64_MAX : int64_t(bpos);
  } else if (t < CAP + a.chunk) {
    const int i = t - CAP;
    f.cand_score = i == f.count ? f.new_score : sc;
    f.cand_key = f.total - f.count + i;
  }
  const char *pk = reinterpret_cast<const char *>(static_cast<const T *>(a.pkeys) + s * a.pkv_s0 + int64_t(g) * a.PC * D);
  const char *pv = reinterpret_cast<const char *>(static_cast<const T *>(a.pvalues) + s * a.pkv_s0 + int64_t(g) * a.PC * D);
  for (int64_t off = int64_t(t) * 128; off < a.chunk * D * int64_t(sizeof(T)); off += int64_t(nt) * 128) {
    prefetch_l2(pk + off);
    prefetch_l2(pv + off);
  }
  return f;
}

// candidate c's (score, key): the spare bytes of K row c or V row c - 64
template <typename T, int D, int ROW>
__device__ __forceinline__ unsigned char *cand_pad(const T *sk, const T *sv, int c) {
  return reinterpret_cast<unsigned char *>(const_cast<T *>((c < kGqaSlice ? sk + c * ROW : sv + (c - kGqaSlice) * ROW) + D));
}

// Shared memory of the commit warps beyond the rows: the candidates' order keys (padded to a
// multiple of 32), sel (the candidate of each new slot), plist (the new slots won by pending rows, in
// slot order) and their count.
constexpr int kCommitBytes = 2 * kGqaSlice * 8 + (2 * kGqaSlice + 4) * 4;

// One 64-bit key per candidate whose unsigned order is the merge order, up to the candidate index:
// the score (NaN first, then descending, -0.0 with 0.0) above the position (empty slots last).  Exact
// for positions below 2^32 - 1; `ok` is false otherwise, and the CTA then ranks by cand_before.
__device__ __forceinline__ uint64_t order_key(float sc, int64_t pk, bool &ok) {
  uint32_t ks = 0u;                                             // NaN
  if (sc == sc) {
    const uint32_t bits = __float_as_uint(sc == 0.f ? 0.f : sc);
    ks = ~((bits & 0x80000000u) ? ~bits : (bits | 0x80000000u));   // larger score, smaller key; never 0
  }
  ok = pk == INT64_MAX || (pk >= 0 && pk < 0xFFFFFFFFll);
  return (uint64_t(ks) << 32) | (pk == INT64_MAX ? 0xFFFFFFFFull : uint64_t(uint32_t(pk)));
}
__device__ __forceinline__ bool commit_red_and(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(p)), "r"(kBarCommit), "r"(kGqaThreads)
      : "memory");
  return r != 0;
}

// Every path through here reaches the landed barrier exactly once (the read warps arrive on it
// exactly once) and the commit warps' own barriers the same number of times in every thread.
template <typename T, int D, int ROW>
__device__ void commit_group(const MemCommitTail &ct, int64_t row, int64_t s, int g, const T *sk, const T *sv,
                             int *cm, int t) {
  constexpr int NT = kGqaThreads;
  const MemCommitArgs &a = ct.c;
  const CommitPrefetch f = commit_prefetch<T, D>(a, row, s, g, t, NT);
  if (!f.active) {   // the same for the row's G CTAs: no push, no arrival
    named_sync(kBarLanded, 2 * NT);
    return;
  }
  const int64_t count = f.count, total = f.total;
  const int CAP = int(a.CAP), chunk = int(a.chunk), PC = int(a.PC);
  T *bank_k = static_cast<T *>(a.keys) + s * a.kv_s0 + int64_t(g) * CAP * D;
  T *bank_v = static_cast<T *>(a.values) + s * a.kv_s0 + int64_t(g) * CAP * D;
  T *pend_k = static_cast<T *>(a.pkeys) + s * a.pkv_s0 + int64_t(g) * PC * D;
  T *pend_v = static_cast<T *>(a.pvalues) + s * a.pkv_s0 + int64_t(g) * PC * D;
  float *bscore = a.bank_scores + s * a.meta_s0 + int64_t(g) * CAP;
  int32_t *bpos = a.positions + s * a.meta_s0 + int64_t(g) * CAP;
  float *pscore = a.pscores + s * a.pmeta_s0 + int64_t(g) * PC;
  constexpr int VEC = 16 / int(sizeof(T));
  constexpr int DV = D / VEC;
  // push (16-byte pieces: row starts are 16-byte aligned); the read does not look at pending rows
  if (t < DV) {
    *reinterpret_cast<uint4 *>(pend_k + count * D + t * VEC) = f.kpiece;
    *reinterpret_cast<uint4 *>(pend_v + count * D + t * VEC) = f.vpiece;
  }
  if (t == 0) pscore[count] = f.new_score;
  const bool merge = count + 1 == chunk;   // the same for the whole CTA
  const int n = CAP + chunk;                // at most 2 * kGqaSlice = NT (checked on the host)
  uint64_t *okey = reinterpret_cast<uint64_t *>(cm);
  int *sel = reinterpret_cast<int *>(okey + 2 * kGqaSlice), *plist = sel + kGqaSlice, *npend = plist + kGqaSlice;
  constexpr int PER = 8;
  uint4 buf[PER];
  int np = 0;
  if (merge) {
    bool key_ok = true;
    const int n32 = (n + 31) & ~31;
    if (t < n) {
      unsigned char *pd = cand_pad<T, D, ROW>(sk, sv, t);
      *reinterpret_cast<float *>(pd) = f.cand_score;
      *reinterpret_cast<int64_t *>(pd + 8) = f.cand_key;
      okey[t] = order_key(f.cand_score, f.cand_key, key_ok);
    } else if (t < n32) {
      okey[t] = ~0ull;   // padding: after every candidate
    }
    key_ok = commit_red_and(key_ok);   // also the barrier after the keys
    if (key_ok && t < n) {
      // rank = keys below this one + equal keys at a lower index; blocks of 32 candidates below (above)
      // this warp's own compare with key + 1 (key), the warp's own block candidate by candidate
      const uint64_t kc = okey[t], kc1 = kc + 1;   // no overflow: the score part is at most 0xFF800000
      const int w = t >> 5;
      int r0 = 0, r1 = 0;
      for (int jb = 0; jb < n32 / 32; ++jb) {
        const ulonglong2 *kp = reinterpret_cast<const ulonglong2 *>(okey + jb * 32);
        if (jb != w) {
          const uint64_t lim = jb < w ? kc1 : kc;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const ulonglong2 k2 = kp[i];
            r0 += k2.x < lim;
            r1 += k2.y < lim;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const ulonglong2 k2 = kp[i];
            const int o = jb * 32 + 2 * i;
            r0 += k2.x < (o < t ? kc1 : kc);
            r1 += k2.y < (o + 1 < t ? kc1 : kc);
          }
        }
      }
      if (r0 + r1 < CAP) sel[r0 + r1] = t;   // the order is strict and total: the ranks are a permutation
    } else if (t < n) {
      const float sc = f.cand_score;
      const int64_t pk = f.cand_key;
      int r0 = 0, r1 = 0, o = 0;
#pragma unroll 4
      for (; o + 1 < n; o += 2) {
        const unsigned char *q0 = cand_pad<T, D, ROW>(sk, sv, o), *q1 = cand_pad<T, D, ROW>(sk, sv, o + 1);
        r0 += memcommit::cand_before(*reinterpret_cast<const float *>(q0), *reinterpret_cast<const int64_t *>(q0 + 8),
                                     o, sc, pk, t);
        r1 += memcommit::cand_before(*reinterpret_cast<const float *>(q1), *reinterpret_cast<const int64_t *>(q1 + 8),
                                     o + 1, sc, pk, t);
      }
      if (o < n) {
        const unsigned char *q0 = cand_pad<T, D, ROW>(sk, sv, o);
        r0 += memcommit::cand_before(*reinterpret_cast<const float *>(q0), *reinterpret_cast<const int64_t *>(q0 + 8),
                                     o, sc, pk, t);
      }
      if (r0 + r1 < CAP) sel[r0 + r1] = t;
    }
    named_sync(kBarCommit, NT);   // sel complete
    // the new slots whose winner is a pending row, in slot order (first commit warp; CAP <= 64)
    if (t < 32) {
      int base = 0;
      for (int r0 = 0; r0 < CAP; r0 += 32) {
        const int r = r0 + t;
        bool from_pend = false;
        if (r < CAP) {
          const int c = sel[r];
          from_pend = c >= CAP;   // pending candidates are never empty
        }
        const unsigned m = __ballot_sync(0xffffffffu, from_pend);
        if (from_pend) plist[base + __popc(m & ((1u << t) - 1u))] = r;
        base += __popc(m);
      }
      if (t == 0) *npend = base;
    }
    named_sync(kBarCommit, NT);   // plist complete
    np = *npend;
    // the first round of pending-row loads (they read pending rows only, which the read never touches)
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = t + i * NT;
      if (e < np * 2 * DV) {
        const int r = plist[e / (2 * DV)], rem = e % (2 * DV), half = rem / DV, d = (rem % DV) * VEC;
        buf[i] = *reinterpret_cast<const uint4 *>((half ? pend_v : pend_k) + (sel[r] - CAP) * D + d);
      }
    }
  }
  // the read's K / V rows have landed (its warps arrive here after their last row wait and a proxy
  // fence): the bank may be overwritten, and the rows in shared memory are final
  named_sync(kBarLanded, 2 * NT);
  if (merge) {
    // (1) slots won by an old bank row (an empty winner copies old bank slot 0, as the reference):
    //     one bulk copy per row straight from the shared-memory row the read holds
    if (t < 2 * CAP) {
      const int r = t % CAP, half = t / CAP;
      const int c = sel[r];
      const int src = *reinterpret_cast<const int64_t *>(cand_pad<T, D, ROW>(sk, sv, c) + 8) == INT64_MAX ? 0 : c;
      if (src < CAP) {
        T *dst = (half ? bank_v : bank_k) + r * D;
        const T *from = (half ? sv : sk) + src * ROW;
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                     "r"(static_cast<uint32_t>(__cvta_generic_to_shared(from))), "r"(uint32_t(D * sizeof(T)))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
    }
    // (2) slots won by a pending row: each thread loads all its pieces of a round (key and value rows
    //     together) before it stores them; the first round's loads were issued before the wait
    for (int base = 0; base < np * 2 * DV; base += NT * PER) {
      if (base > 0) {
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const int e = base + t + i * NT;
          if (e < np * 2 * DV) {
            const int r = plist[e / (2 * DV)], rem = e % (2 * DV), half = rem / DV, d = (rem % DV) * VEC;
            buf[i] = *reinterpret_cast<const uint4 *>((half ? pend_v : pend_k) + (sel[r] - CAP) * D + d);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = base + t + i * NT;
        if (e < np * 2 * DV) {
          const int r = plist[e / (2 * DV)], rem = e % (2 * DV), half = rem / DV, d = (rem % DV) * VEC;
          *reinterpret_cast<uint4 *>((half ? bank_v : bank_k) + r * D + d) = buf[i];
        }
      }
    }
    for (int r = t; r < CAP; r += NT) {
      const int c = sel[r];
      const unsigned char *pd = cand_pad<T, D, ROW>(sk, sv, c);
      const int64_t key = *reinterpret_cast<const int64_t *>(pd + 8);
      bscore[r] = *reinterpret_cast<const float *>(pd);
      bpos[r] = key == INT64_MAX ? -1 : int32_t(key);
    }
    // the bulk copies have read their rows and written the bank before the CTA goes on or exits
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  named_sync(kBarCommit, NT);   // every commit store of this CTA is issued
  if (t == 0) {
    __threadfence();
    if (atomicAdd(ct.arrive + row, 1) == int(a.G) - 1) {
      ct.arrive[row] = 0;
      a.count[s * a.count_s0] = merge ? 0 : count + 1;
      a.total[s * a.count_s0] = total + 1;
    }
  }
}

template <typename T, int R, int D, bool COMMIT>
__global__ void __launch_bounds__(COMMIT ? 2 * kGqaThreads : kGqaThreads, 3)
    gqa_decode_mma_kernel(const GqaDecodeArgs a, const MemCommitTail ct) {
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
  int *cm = reinterpret_cast<int *>(fin + 16);                 // the commit warps' arrays (memory step)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  const int64_t unit = blockIdx.x;                        // (row, group)
  const int64_t slice = blockIdx.y, p0 = slice * kGqaSlice;
  const int64_t b = unit / a.G, g = unit % a.G;
  if (!a.indices && tid < kGqaThreads) {   // the slice's rows are known before the wait: warm L2 with them
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
    if (tid < kGqaThreads)
      for (int e = tid; e < R * D; e += kGqaThreads) o[e] = from_f<T>(0.f);
    return;
  }
  if constexpr (COMMIT) {
    if (tid >= kGqaThreads) {   // warps 4-7: this group's commit, beside the read
      commit_group<T, D, ROW>(ct, b, s, int(g), sk, sv, cm, tid - kGqaThreads);
      return;
    }
  }
  // warps 0-3: the read
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
  named_sync(kBarRead, kGqaThreads);

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
  named_sync(kBarRead, kGqaThreads);
  if (tid < 8) {
    float m = fmaxf(fmaxf(red[tid], red[8 + tid]), fmaxf(red[16 + tid], red[24 + tid]));
    if (a.null_slot) m = fmaxf(m, 0.f);
    fin[tid] = m;
  }
  named_sync(kBarRead, kGqaThreads);
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
  if constexpr (COMMIT) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the commit's bulk copies read these rows
    named_arrive(kBarLanded, 2 * kGqaThreads);
  }
  named_sync(kBarRead, kGqaThreads);
  if (tid < 8) {
    float l = red[32 + tid] + red[40 + tid] + red[48 + tid] + red[56 + tid];
    if (a.null_slot) l += expf(-fin[tid]);         // the null slot: logit 0, value 0
    fin[8 + tid] = l;
  }
  named_sync(kBarRead, kGqaThreads);

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
  }
}

template <typename T, int R, int D, bool COMMIT>
int launch_gqa(const GqaDecodeArgs &a, const MemCommitTail &ct, unsigned slices) {
  constexpr int ROW = D + 8, PROW = kGqaSlice + 8;
  const size_t smem = sizeof(T) * (2 * kGqaSlice * ROW + 8 * ROW + 2 * 8 * PROW) + sizeof(float) * (64 + 16) +
                      (COMMIT ? kCommitBytes : 0);
  auto k = gqa_decode_mma_kernel<T, R, D, COMMIT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gqa decode: smem attribute: %s", cudaGetErrorString(e));
  e = launch_pdl(k, dim3(unsigned(a.B * a.G), slices), dim3(COMMIT ? 2 * kGqaThreads : kGqaThreads), smem, a.stream,
                 a, ct);
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
  const int64_t n = c.CAP + c.chunk;   // one merge candidate per commit thread, in the rows' spare bytes
  const uintptr_t al = reinterpret_cast<uintptr_t>(c.key) | reinterpret_cast<uintptr_t>(c.value) |
                       reinterpret_cast<uintptr_t>(c.keys) | reinterpret_cast<uintptr_t>(c.values) |
                       reinterpret_cast<uintptr_t>(c.pkeys) | reinterpret_cast<uintptr_t>(c.pvalues);
  return !a.partial && a.P <= kGqaSlice && a.B == c.B && a.G == c.G && a.indices == c.indices &&
         n <= 2 * kGqaSlice && c.CAP == a.P && c.D == a.D && c.dtype == a.dtype && (al % 16) == 0 &&
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
