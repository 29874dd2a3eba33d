// Anchor-memory prefill orchestration on the device: the index work of
// IndependentGQAMemory._sequence (modeling_yanchor.py:178-275) around the
// selection and read kernels, as four small kernels in place of the
// reference's ~150 torch indexing launches.
//
//   timeline   each row's slots [the state's pending tokens | new tokens, valid
//              first] padded to whole blocks of `chunk`: the slot's score (the
//              new token's, or the pending chunk's), position and reference,
//              written in the selection's blocked layout [B, blocks, G, chunk],
//              and the token index of every slot (modeling_yanchor.py:186-205);
//   table      which new tokens need a writer row (they enter a block-end
//              top-CAP, or stay pending) and the slot -> source-row table
//              (modeling_yanchor.py:206-244);
//   read refs  each block's prefix top-CAP as source rows (modeling_yanchor.py:
//              245-255);
//   state      the new bank (the top-CAP after the last complete block) and
//              pending chunk (the incomplete tail), gathered from the two row
//              sources, and the counters (modeling_yanchor.py:266-275).
// Source rows: [old bank + pending rows of every row | the writer's new rows];
// reference x < offset reads old row x, else new row x - offset.
#include "common.cuh"
#include "kernels.h"

namespace yb {
namespace {

constexpr int kGlueThreads = 256;

__device__ __forceinline__ void snapshot(const PrefillGlueArgs &a, int64_t b, int64_t &c0, int64_t &t0,
                                         int64_t &nn) {
  c0 = a.snap[b];
  t0 = a.snap[a.B + b];
  nn = a.snap[2 * a.B + b];
}

__global__ void glue_timeline_kernel(const PrefillGlueArgs a) {
  const int64_t n = a.B * a.extent * a.G;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = e / (a.extent * a.G), rem = e % (a.extent * a.G), slot = rem / a.G, g = rem % a.G;
    const int64_t c0 = a.has_state ? a.count[b * a.count_s0] : 0;
    const int64_t t0 = a.has_state ? a.total[b * a.count_s0] : 0;
    const int64_t nn = a.n_new ? a.n_new[b] : a.T;
    const int64_t fill = c0 + nn;
    const bool live = slot < fill, is_new = slot >= c0;
    int64_t j = slot - c0;
    j = j < 0 ? 0 : (j > a.T - 1 ? a.T - 1 : j);
    const int64_t tk = a.order ? a.order[b * a.T + j] : j;
    float sv;
    if (is_new) sv = a.scores[(b * a.T + tk) * a.G + g];
    else sv = a.pend_scores[b * a.pmeta_s0 + g * a.PC + (slot < a.chunk - 1 ? slot : a.chunk - 1)];
    if (!live) sv = -INFINITY;
    const int64_t dst = ((b * a.blocks + slot / a.chunk) * a.G + g) * a.chunk + slot % a.chunk;
    a.s_blk[dst] = sv;
    a.pos_blk[dst] = t0 - c0 + slot;
    a.ref_blk[dst] = live ? slot + a.shift : -1;
    if (g == 0) a.tok[b * a.extent + slot] = tk;
    if (slot == 0 && g == 0) {   // the counters before the prefill, for the later phases
      a.snap[b] = c0;
      a.snap[a.B + b] = t0;
      a.snap[2 * a.B + b] = nn;
    }
  }
}

// a new slot that enters the top-CAP at the end of its own block (a block that
// some later block reads, or the bank) needs a writer row
__global__ void glue_needed_kernel(const PrefillGlueArgs a) {
  const int64_t n = a.B * a.blocks * a.G * a.cap;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = e / (a.blocks * a.G * a.cap), i = (e / (a.G * a.cap)) % a.blocks, gk = e % (a.G * a.cap);
    const int64_t r = a.pre_r[(b * (a.blocks + 1) + i + 1) * a.G * a.cap + gk];
    int64_t c0, t0, nn;
    snapshot(a, b, c0, t0, nn);
    const int64_t fill = c0 + nn, bound = (i + 1) * a.chunk, ent = r - a.shift;
    const bool used = a.has_state ? bound <= fill : bound < fill;
    if (ent >= bound - a.chunk && ent < bound && used) a.needed[b * a.extent + ent] = 1;
  }
}

// the tail that stays pending needs rows too; only live new slots do; then the table
__global__ void glue_table_kernel(const PrefillGlueArgs a) {
  const int64_t width = a.shift + a.extent, per = a.cap + a.chunk, offset = a.has_state ? a.B * per : 0;
  const int64_t n = a.B * width;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = e / width, s = e % width;
    if (s < a.shift) {   // the old bank slots
      a.table[e] = b * per + s;
      continue;
    }
    const int64_t slot = s - a.shift;
    int64_t c0, t0, nn;
    snapshot(a, b, c0, t0, nn);
    const int64_t fill = c0 + nn;
    const bool live = slot < fill, is_new = slot >= c0;
    bool nd = a.needed[b * a.extent + slot] != 0;
    if (a.has_state) nd = nd || (live && slot >= (fill / a.chunk) * a.chunk);
    nd = nd && live && is_new;
    a.needed[b * a.extent + slot] = nd ? 1 : 0;
    int64_t t = (a.has_state && !is_new) ? b * per + a.cap + slot : -1;
    if (a.capture_safe && nd) t = offset + b * a.extent + slot;   // the writer ran on every slot
    a.table[e] = t;
  }
}

__global__ void glue_read_refs_kernel(const PrefillGlueArgs a) {
  const int64_t width = a.shift + a.extent;
  const int64_t n = a.B * a.blocks * a.G * a.cap;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = e / (a.blocks * a.G * a.cap), rest = e % (a.blocks * a.G * a.cap);
    const int64_t r = a.pre_r[b * (a.blocks + 1) * a.G * a.cap + rest];   // prefix entry blk = entries 0 .. blocks-1
    a.read_refs[e] = r < 0 ? -1 : a.table[b * width + r];
  }
}

// 16-byte piece d of row x, group g, of the joint source
template <typename T>
__device__ __forceinline__ uint4 source_piece(const PrefillGlueArgs a, const void *old_rows, const void *new_rows,
                                              int64_t x, int64_t g, int64_t d) {
  const int64_t offset = a.has_state ? a.B * (a.cap + a.chunk) : 0;
  const T *src = x < offset ? static_cast<const T *>(old_rows) + (x * a.G + g) * a.D
                            : static_cast<const T *>(new_rows) + ((x - offset) * a.G + g) * a.D;
  return *reinterpret_cast<const uint4 *>(src + d);
}

template <typename T>
__global__ void glue_state_kernel(const PrefillGlueArgs a) {
  constexpr int VEC = 16 / int(sizeof(T));
  const int64_t DV = a.D / VEC, width = a.shift + a.extent;
  const int64_t nbank = a.B * a.G * a.cap * DV, npend = a.B * a.G * a.PC * DV;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < nbank + npend + a.B;
       e += int64_t(gridDim.x) * blockDim.x) {
    if (e < nbank) {
      // bank slot k of group g: the prefix entry after the last complete block
      const int64_t b = e / (a.G * a.cap * DV), gk = (e / DV) % (a.G * a.cap), d = (e % DV) * VEC;
      const int64_t g = gk / a.cap, k = gk % a.cap;
      int64_t c0, t0, nn;
      snapshot(a, b, c0, t0, nn);
      const int64_t full = (c0 + nn) / a.chunk;
      const int64_t pe = (b * (a.blocks + 1) + full) * a.G * a.cap + gk;
      const int64_t r = a.pre_r[pe];
      uint4 v = make_uint4(0, 0, 0, 0), w = make_uint4(0, 0, 0, 0);
      if (r >= 0) {
        int64_t x = a.table[b * width + r];
        x = x < 0 ? 0 : x;
        v = source_piece<T>(a, a.old_k, a.new_k, x, g, d);
        w = source_piece<T>(a, a.old_v, a.new_v, x, g, d);
      }
      *reinterpret_cast<uint4 *>(static_cast<T *>(a.keys) + b * a.kv_s0 + gk * a.D + d) = v;
      *reinterpret_cast<uint4 *>(static_cast<T *>(a.values) + b * a.kv_s0 + gk * a.D + d) = w;
      if (d == 0) {
        a.bank_scores[b * a.meta_s0 + gk] = a.pre_s[pe];
        a.positions[b * a.meta_s0 + gk] = int32_t(a.pre_p[pe]);
      }
    } else if (e < nbank + npend) {
      // pending slot p of group g: the incomplete tail of the timeline
      const int64_t f = e - nbank;
      const int64_t b = f / (a.G * a.PC * DV), gp = (f / DV) % (a.G * a.PC), d = (f % DV) * VEC;
      const int64_t g = gp / a.PC, p = gp % a.PC;
      int64_t c0, t0, nn;
      snapshot(a, b, c0, t0, nn);
      const int64_t fill = c0 + nn, full = fill / a.chunk;
      const bool keep = p < fill % a.chunk;
      int64_t tail = full * a.chunk + p;
      tail = tail < a.extent - 1 ? tail : a.extent - 1;
      uint4 v = make_uint4(0, 0, 0, 0), w = make_uint4(0, 0, 0, 0);
      if (keep) {
        int64_t x = a.table[b * width + tail + a.shift];
        x = x < 0 ? 0 : x;
        v = source_piece<T>(a, a.old_k, a.new_k, x, g, d);
        w = source_piece<T>(a, a.old_v, a.new_v, x, g, d);
      }
      *reinterpret_cast<uint4 *>(static_cast<T *>(a.pkeys) + b * a.pkv_s0 + gp * a.D + d) = v;
      *reinterpret_cast<uint4 *>(static_cast<T *>(a.pvalues) + b * a.pkv_s0 + gp * a.D + d) = w;
      if (d == 0)
        a.pscores[b * a.pmeta_s0 + gp] =
            keep ? a.s_blk[((b * a.blocks + tail / a.chunk) * a.G + g) * a.chunk + tail % a.chunk] : -INFINITY;
    } else {
      const int64_t b = e - nbank - npend;
      int64_t c0, t0, nn;
      snapshot(a, b, c0, t0, nn);
      a.count_out[b * a.count_s0] = (c0 + nn) % a.chunk;
      a.total_out[b * a.count_s0] = t0 + nn;
    }
  }
}

unsigned glue_grid(int64_t n) {
  const int64_t blocks = (n + kGlueThreads - 1) / kGlueThreads;
  return unsigned(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

}  // namespace

int launch_prefill_glue(const PrefillGlueArgs &a, int phase) {
  switch (phase) {
    case 0:
      glue_timeline_kernel<<<glue_grid(a.B * a.extent * a.G), kGlueThreads, 0, a.stream>>>(a);
      return check_launch("glue_timeline_kernel");
    case 1: {
      const cudaError_t e = cudaMemsetAsync(a.needed, 0, size_t(a.B * a.extent), a.stream);
      if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "prefill table: %s", cudaGetErrorString(e));
      glue_needed_kernel<<<glue_grid(a.B * a.blocks * a.G * a.cap), kGlueThreads, 0, a.stream>>>(a);
      int rc = check_launch("glue_needed_kernel");
      if (rc) return rc;
      glue_table_kernel<<<glue_grid(a.B * (a.shift + a.extent)), kGlueThreads, 0, a.stream>>>(a);
      return check_launch("glue_table_kernel");
    }
    case 2:
      glue_read_refs_kernel<<<glue_grid(a.B * a.blocks * a.G * a.cap), kGlueThreads, 0, a.stream>>>(a);
      return check_launch("glue_read_refs_kernel");
    case 3: {
      const int64_t n = a.B * a.G * (a.cap + a.PC) * (a.D / (16 / (a.dtype == YB_F32 ? 4 : 2))) + a.B;
      if (a.dtype == YB_BF16) glue_state_kernel<__nv_bfloat16><<<glue_grid(n), kGlueThreads, 0, a.stream>>>(a);
      else if (a.dtype == YB_F16) glue_state_kernel<__half><<<glue_grid(n), kGlueThreads, 0, a.stream>>>(a);
      else glue_state_kernel<float><<<glue_grid(n), kGlueThreads, 0, a.stream>>>(a);
      return check_launch("glue_state_kernel");
    }
  }
  return set_error(YB_ERR_ARGUMENT, "prefill glue: bad phase %d", phase);
}

}  // namespace yb
