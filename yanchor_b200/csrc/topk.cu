// Top-CAP selection of anchor candidates: select_topk / merge_topk and the
// exclusive prefix over chunk blocks (modeling_yanchor.py:51-78).
//
// Order of every selection (the reference's two stable argsorts): score
// descending with NaN first (torch's descending sort ranks NaN highest) and
// -0.0 equal to 0.0, then position ascending with invalid entries
// (reference < 0) last, then candidate index.  Each candidate gets one
// 128-bit key that sorts ascending in that order:
//   hi = score_key << 32 | pos_key >> 32,   lo = pos_key << 32 | index.
// Invalid entries report position -1; missing entries (fewer candidates than
// CAP) come out as (-inf, -1, -1).
//
// select: one CTA per row, bitonic sort of the keys in shared memory.
// exclusive prefix: phase 1 selects each block's own top-CAP (sorted) into
// output slot blk + 1 (only a block's top-CAP can survive any later merge).
// Merging two sorted top-CAP lists (binary-search ranks; on equal keys the
// earlier list goes first, as it precedes the later one in the reference's
// concatenation) is associative, so the scan over the blocks runs as a
// two-level scan: phase 2 merges, inside each segment of 1024 / (2 CAP)
// blocks, the blocks' lists into local prefixes (one CTA per segment); phase
// 3 runs one CTA per (row, group) down the segments, merging the running
// prefix with all of a segment's local prefixes at once.  A sequential depth
// of seg + blocks / seg merges instead of blocks.  An optional initial bank
// seeds the running prefix, which equals the reference's merge of every
// prefix entry with the state's bank (modeling_yanchor.py:206-208).
#include "common.cuh"
#include "kernels.h"

namespace yb {
namespace {

constexpr int kSelMaxN = 4096;
constexpr int kScanMaxCap = 512;

__device__ __forceinline__ uint32_t score_key(float s) {
  if (s != s) return 0u;                       // NaN first
  uint32_t u = __float_as_uint(s);
  if ((u << 1) == 0u) u = 0u;                  // -0.0 == 0.0
  const uint32_t asc = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ~asc;                                 // descending; never 0 for a number
}

__device__ __forceinline__ uint64_t pos_key(int64_t pos, int64_t ref) {
  return ref < 0 ? ~0ull : (uint64_t(pos) ^ 0x8000000000000000ull);
}

__device__ __forceinline__ int64_t load_pos(const void *p, int dtype, int64_t i) {
  return dtype == YB_I32 ? int64_t(static_cast<const int32_t *>(p)[i]) : static_cast<const int64_t *>(p)[i];
}

struct Key {
  uint64_t hi, lo;
};
__device__ __forceinline__ bool key_less(const Key &a, const Key &b) {
  return a.hi < b.hi || (a.hi == b.hi && a.lo < b.lo);
}
__device__ __forceinline__ Key make_key(float s, int64_t pos, int64_t ref, uint32_t idx) {
  const uint64_t pk = pos_key(pos, ref);
  return Key{(uint64_t(score_key(s)) << 32) | (pk >> 32), (pk << 32) | idx};
}

struct SelArgs {
  const float *scores;
  const void *positions;
  const int64_t *refs;
  int pos_dtype;
  int64_t rows, n, cap;
  int64_t group_rows, skip;  // out_row = row + (row / group_rows + 1) * skip
  float *out_s;
  int64_t *out_p, *out_r;
};

__global__ void select_topk_kernel(const SelArgs a, int n2) {
  extern __shared__ __align__(16) unsigned char sel_raw[];
  Key *key = reinterpret_cast<Key *>(sel_raw);
  const int64_t row = blockIdx.x;
  const int n = int(a.n);
  const float *s = a.scores + row * a.n;
  const int64_t *r = a.refs + row * a.n;
  for (int i = threadIdx.x; i < n2; i += blockDim.x)
    key[i] = i < n ? make_key(s[i], load_pos(a.positions, a.pos_dtype, row * a.n + i), r[i], uint32_t(i))
                   : Key{~0ull, ~0ull};
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const Key x = key[i], y = key[ixj];
          const bool up = (i & k) == 0;
          if (key_less(y, x) == up) {
            key[i] = y;
            key[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  const int64_t orow = a.skip ? row + (row / a.group_rows + 1) * a.skip : row;
  for (int64_t t = threadIdx.x; t < a.cap; t += blockDim.x) {
    float os = -INFINITY;
    int64_t op = -1, oref = -1;
    if (t < n) {
      const int idx = int(key[t].lo & 0xffffffffu);
      os = s[idx];
      oref = r[idx];
      op = oref < 0 ? -1 : load_pos(a.positions, a.pos_dtype, row * a.n + idx);
    }
    a.out_s[orow * a.cap + t] = os;
    a.out_p[orow * a.cap + t] = op;
    a.out_r[orow * a.cap + t] = oref;
  }
}

struct ScanArgs {
  const float *init_s;
  const void *init_p;
  const int64_t *init_r;  // null: slot index where the position is >= 0, else -1
  int init_pos_dtype;
  int64_t B, blocks, G, cap;
  float *out_s;
  int64_t *out_p, *out_r;  // [B, blocks + 1, G, cap]; slots 1.. hold each block's own top-cap on entry
};

struct Entry {
  float s;
  int64_t p, r;
};

// Merge of two sorted top-cap lists into the first cap of their union (the
// left list first on equal keys), by the group of 2 * cap threads t: thread
// t < cap places left[t], thread cap + t places right[t], at their ranks.
__device__ __forceinline__ void merge_place(const Key *lk, const Entry *le, const Key *rk, const Entry *re, Key *nk,
                                            Entry *ne, int cap, int t) {
  const bool from_left = t < cap;
  const int i = from_left ? t : t - cap;
  const Key mine = from_left ? lk[i] : rk[i];
  const Key *other = from_left ? rk : lk;
  // from the left: count other < mine;  from the right: count other <= mine
  int lo = 0, hi = cap;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    const bool before = from_left ? key_less(other[mid], mine) : !key_less(mine, other[mid]);
    if (before) lo = mid + 1; else hi = mid;
  }
  const int rank = i + lo;
  if (rank < cap) {
    nk[rank] = mine;
    ne[rank] = from_left ? le[i] : re[i];
  }
}

__device__ __forceinline__ Entry load_entry(const ScanArgs &a, int64_t o) {
  return Entry{a.out_s[o], a.out_p[o], a.out_r[o]};
}
__device__ __forceinline__ void store_entry(const ScanArgs &a, int64_t o, const Entry &e) {
  a.out_s[o] = e.s;
  a.out_p[o] = e.p;
  a.out_r[o] = e.r;
}
// keys of a list entry: the index bits stay 0, so equal keys keep list order
__device__ __forceinline__ Key entry_key(const Entry &e) { return make_key(e.s, e.p, e.r, 0u); }

// Phase A: within each segment of `seg` blocks, the inclusive prefix of the
// blocks' own top-cap lists (slots blk + 1), written back in place.  One CTA
// of 2 * cap threads per (row, group, segment).
__global__ void prefix_segment_kernel(const ScanArgs a, int seg) {
  extern __shared__ __align__(16) unsigned char scan_raw[];
  const int cap = int(a.cap);
  Key *acc_k = reinterpret_cast<Key *>(scan_raw);
  Key *cand_k = acc_k + cap;
  Key *new_k = cand_k + cap;
  Entry *acc_e = reinterpret_cast<Entry *>(new_k + cap);
  Entry *cand_e = acc_e + cap;
  Entry *new_e = cand_e + cap;
  const int tid = threadIdx.x;
  const int64_t nseg = (a.blocks + seg - 1) / seg;
  const int64_t bg = blockIdx.x / nseg, sg = blockIdx.x % nseg;
  const int64_t b = bg / a.G, g = bg % a.G;
  auto slot = [&](int64_t i) { return ((b * (a.blocks + 1) + i) * a.G + g) * a.cap; };
  const int64_t first = sg * seg, last = (first + seg < a.blocks ? first + seg : a.blocks) - 1;
  if (tid < cap) {
    const Entry e = load_entry(a, slot(first + 1) + tid);
    acc_e[tid] = e;
    acc_k[tid] = entry_key(e);
  }
  Entry nxt{-INFINITY, -1, -1};   // the next block's entry, loaded one merge ahead
  if (tid < cap && first + 1 <= last) nxt = load_entry(a, slot(first + 2) + tid);
  for (int64_t blk = first + 1; blk <= last; ++blk) {
    if (tid < cap) {
      cand_e[tid] = nxt;
      cand_k[tid] = entry_key(nxt);
      if (blk + 1 <= last) nxt = load_entry(a, slot(blk + 2) + tid);
    }
    __syncthreads();
    if (tid < 2 * cap) merge_place(acc_k, acc_e, cand_k, cand_e, new_k, new_e, cap, tid);
    __syncthreads();
    if (tid < cap) {
      acc_k[tid] = new_k[tid];
      acc_e[tid] = new_e[tid];
      store_entry(a, slot(blk + 1) + tid, new_e[tid]);
    }
    __syncthreads();
  }
}

// Phase B: one CTA per (row, group) walks the segments: the running prefix
// (the sorted initial bank first, written to slot 0) is merged with every
// local prefix of the segment at once (groups of 2 * cap threads, one block
// each), which gives those blocks' exclusive prefixes; the segment's last
// result carries on.  Every merge keeps the earlier blocks first on equal
// keys, so the result is the sequential scan's.
__global__ void prefix_carry_kernel(const ScanArgs a, int seg) {
  extern __shared__ __align__(16) unsigned char scan_raw[];
  const int cap = int(a.cap);
  Key *acc_k = reinterpret_cast<Key *>(scan_raw);               // [cap]
  Key *cand_k = acc_k + cap;                                     // [seg][cap]
  Key *new_k = cand_k + seg * cap;                               // [seg][cap]
  Entry *acc_e = reinterpret_cast<Entry *>(new_k + seg * cap);   // [cap]
  Entry *cand_e = acc_e + cap;                                   // [seg][cap]
  Entry *new_e = cand_e + seg * cap;                             // [seg][cap]
  const int tid = threadIdx.x, q = tid / (2 * cap), t = tid % (2 * cap);
  const int64_t b = blockIdx.x / a.G, g = blockIdx.x % a.G;
  auto slot = [&](int64_t i) { return ((b * (a.blocks + 1) + i) * a.G + g) * a.cap; };

  // entry 0: the (sorted) initial bank, or nothing
  if (tid < cap) {
    Entry e{-INFINITY, -1, -1};
    if (a.init_s) {
      const int64_t i = (b * a.G + g) * a.cap + tid;
      const int64_t p = load_pos(a.init_p, a.init_pos_dtype, i);
      e.s = a.init_s[i];
      e.r = a.init_r ? a.init_r[i] : (p < 0 ? -1 : tid);
      e.p = e.r < 0 ? -1 : p;
    }
    cand_e[tid] = e;
    cand_k[tid] = make_key(e.s, e.p, e.r, uint32_t(tid));
  }
  __syncthreads();
  if (tid < cap) {
    int rank = 0;
    const Key mine = cand_k[tid];
    for (int j = 0; j < cap; ++j) rank += key_less(cand_k[j], mine);
    acc_e[rank] = cand_e[tid];
    acc_k[rank] = Key{mine.hi, mine.lo & ~0xffffffffull};   // index no longer needed: list order breaks ties
    store_entry(a, slot(0) + rank, cand_e[tid]);
  }
  __syncthreads();
  // the local prefix of each segment up to block first + q, loaded one segment ahead
  Entry nxt{-INFINITY, -1, -1};
  if (q < seg && q < a.blocks && t < cap) nxt = load_entry(a, slot(q + 1) + t);
  for (int64_t first = 0; first < a.blocks; first += seg) {
    const int64_t blk = first + q;
    const bool active = q < seg && blk < a.blocks;
    if (active && t < cap) {
      cand_e[q * cap + t] = nxt;
      cand_k[q * cap + t] = entry_key(nxt);
      if (blk + seg < a.blocks) nxt = load_entry(a, slot(blk + seg + 1) + t);
    }
    __syncthreads();
    if (active)
      merge_place(acc_k, acc_e, cand_k + q * cap, cand_e + q * cap, new_k + q * cap, new_e + q * cap, cap, t);
    __syncthreads();
    if (active && t < cap) store_entry(a, slot(blk + 1) + t, new_e[q * cap + t]);
    const int64_t lastq = (first + seg < a.blocks ? seg : a.blocks - first) - 1;
    if (tid < cap) {
      acc_k[tid] = new_k[lastq * cap + tid];
      acc_e[tid] = new_e[lastq * cap + tid];
    }
    __syncthreads();
  }
}

int select_threads(int n2) { return n2 >= 512 ? 256 : (n2 / 2 >= 32 ? n2 / 2 : 32); }

int next_pow2(int64_t n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

int launch_select(const SelArgs &a, cudaStream_t stream) {
  if (a.rows == 0 || a.cap == 0) return YB_OK;
  const int n2 = next_pow2(a.n > 1 ? a.n : 1);
  const size_t smem = size_t(n2) * sizeof(Key);
  cudaError_t e = cudaFuncSetAttribute(select_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "select_topk: smem attribute: %s", cudaGetErrorString(e));
  select_topk_kernel<<<unsigned(a.rows), select_threads(n2), smem, stream>>>(a, n2);
  return check_launch("select_topk_kernel");
}

}  // namespace

int launch_select_topk(const TopkArgs &t) {
  if (t.n > kSelMaxN)
    return set_error(YB_ERR_UNSUPPORTED, "select_topk: %lld candidates per row exceed %d", (long long)t.n, kSelMaxN);
  SelArgs a{t.scores, t.positions, t.refs, t.pos_dtype, t.rows, t.n, t.cap, 1, 0, t.out_s, t.out_p, t.out_r};
  return launch_select(a, t.stream);
}

int launch_exclusive_prefix_topk(const PrefixTopkArgs &t) {
  if (t.chunk > kSelMaxN)
    return set_error(YB_ERR_UNSUPPORTED, "exclusive_prefix_topk: chunk %lld exceeds %d", (long long)t.chunk,
                     kSelMaxN);
  if (t.cap > kScanMaxCap)
    return set_error(YB_ERR_UNSUPPORTED, "exclusive_prefix_topk: capacity %lld exceeds %d", (long long)t.cap,
                     kScanMaxCap);
  if (t.B * t.G == 0 || t.cap == 0) return YB_OK;
  if (t.blocks > 0) {
    SelArgs a{t.scores, t.positions, t.refs, t.pos_dtype, t.B * t.blocks * t.G, t.chunk, t.cap,
              t.blocks * t.G, t.G, t.out_s, t.out_p, t.out_r};
    const int rc = launch_select(a, t.stream);
    if (rc) return rc;
  }
  ScanArgs s{t.init_s, t.init_p, t.init_r, t.init_pos_dtype, t.B, t.blocks, t.G, t.cap, t.out_s, t.out_p, t.out_r};
  // segments of `seg` blocks: as many merges side by side as fit in 1024 threads (8 at cap 64)
  const int seg = int(1024 / (2 * t.cap) > 0 ? 1024 / (2 * t.cap) : 1);
  const int64_t nseg = (t.blocks + seg - 1) / seg;
  const int group = int((2 * t.cap + 31) / 32 * 32);
  if (seg > 1 && t.blocks > 1) {
    const size_t smem_a = size_t(t.cap) * 3 * (sizeof(Key) + sizeof(Entry));
    cudaError_t e = cudaFuncSetAttribute(prefix_segment_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem_a));
    if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "prefix scan: smem attribute: %s", cudaGetErrorString(e));
    prefix_segment_kernel<<<unsigned(t.B * t.G * nseg), group, smem_a, t.stream>>>(s, seg);
    const int rc = check_launch("prefix_segment_kernel");
    if (rc) return rc;
  }
  const int seg_b = t.blocks > 1 ? seg : 1;   // one block per segment: phase A is the identity
  const size_t smem_b = size_t(t.cap) * (1 + 2 * seg_b) * (sizeof(Key) + sizeof(Entry));
  cudaError_t e = cudaFuncSetAttribute(prefix_carry_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(smem_b));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "prefix scan: smem attribute: %s", cudaGetErrorString(e));
  const int threads = int(((2 * t.cap * seg_b) + 31) / 32 * 32);
  prefix_carry_kernel<<<unsigned(t.B * t.G), threads, smem_b, t.stream>>>(s, seg_b);
  return check_launch("prefix_carry_kernel");
}

}  // namespace yb
