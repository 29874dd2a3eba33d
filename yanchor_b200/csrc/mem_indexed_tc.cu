// Prefill anchor read (indexed GQA) on the tcgen05 tensor cores, bf16,
// D = 256, CAP = 64 referenced rows, 256 query rows per unit (chunk 64 x 4
// heads per group) — the YANchor memory shape.
//
// A persistent CTA per SM walks the units (row b, block, group g) in
// turn.  A unit's 256 query rows are the (position, head) pairs of the
// block's 64 positions and the group's 4 heads, taken as two halves of 128
// rows (32 positions); TMA brings each half in as one 3-D box per 64-column
// slice, already in (position, head) row order.  The 64 referenced key /
// value rows are gathered with cp.async (empty references become zero
// rows).  Per half:
//   S = Q K^T (TMEM, fp32)  ->  softmax over the 64 slots plus the null slot
//   (logit 0, value 0), masked where the reference is empty  ->  P as bf16
//   hi + lo parts in TMEM  ->  O = (P_hi + P_lo) V (TMEM)  ->  O / den in
//   bf16  ->  TMA store through two 16 KB staging tiles.
// Warp roles: warp 0 loads the Q halves (TMA) and the K rows (cp.async), warp
// 6 the V rows (cp.async), warp 1 issues the MMAs, warps 2-5 run the softmax
// and the output.  Each buffer is
// refilled for the next unit as soon as its last reader is done: a Q half
// after its S MMA, K after the second S MMA, V after the second O MMA, so
// the next unit's loads overlap this unit's softmax and output.
// (modeling_yanchor.py:22-42 indexed_gqa_torch; runtime/model/
// independent_memory.py:6-45 indexed_gqa, which also splits p into bf16
// hi + lo.)
//
// Timeline mode (the prefill orchestration): query and output are the
// prompt's own [B, T, H, D] tensors and block slot s of row b is token
// s + token_shift[b]; a 4-D tensor map loads the block's rows straight from
// there (tokens outside [0, T) read as zeros) and only slots in
// [write_lo[b], write_hi[b]) are written — whole 32-position halves by TMA
// store, ragged halves by each thread's own predicated stores.  This
// replaces two gathers of the whole query / output through a timeline copy.
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace yb {
namespace {

using namespace tc;

constexpr int D = 256, CAPS = 64, ROWS = 256, NT = 224;
constexpr uint32_t OFF_Q = 0;           // two Q halves: 4 column blocks x 128 rows x 128 B each (64 KB)
constexpr uint32_t OFF_K = 131072;      // K: 4 column blocks x 64 rows x 128 B
constexpr uint32_t OFF_V = 163840;      // V: same
constexpr uint32_t OFF_OS = 196608;     // two output staging tiles, 128 rows x 128 B
constexpr uint32_t OFF_BAR = 229376;    // 16 mbarriers
constexpr uint32_t OFF_MISC = OFF_BAR + 16 * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16;
constexpr uint32_t T_S = 0;      // S of half h at columns 64 h
constexpr uint32_t T_P = 128;    // P of half h at 128 + 64 h: hi parts, then lo parts (32 columns each)
constexpr uint32_t T_O = 256;    // O (256 columns)
constexpr uint32_t ID_S = idesc_bf16(128, 64, false, false);
constexpr uint32_t ID_O = idesc_bf16(128, 256, false, true);
constexpr int ERR_WAIT_Q = 0x201, ERR_WAIT_S = 0x202, ERR_WAIT_O = 0x203, ERR_WAIT_KV = 0x204, ERR_WAIT_P = 0x205,
              ERR_WAIT_FREE = 0x206, ERR_WAIT_DONE = 0x207;
// barrier slots
enum { B_QFULL = 0, B_QEMPTY = 2, B_KFULL = 4, B_KEMPTY, B_VFULL, B_VEMPTY, B_SFULL, B_PFULL = 10, B_OFULL = 12,
       B_OEMPTY, B_DONE, B_COUNT };
static_assert(B_COUNT <= 16, "barrier slots");

struct IdxParams {
  const __nv_bfloat16 *key, *value;
  const int64_t *refs;
  int64_t blocks, chunk, H, G, S, KB;
  float scale;
  // timeline mode (tok_shift != nullptr)
  const int64_t *tok_shift, *w_lo, *w_hi;
  int64_t T;
  __nv_bfloat16 *out;
  int64_t units;
  // second source: references S .. S + S2 - 1 are rows of key2 / value2 (key batch 1)
  const __nv_bfloat16 *key2, *value2;
  int64_t S2;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y),
      "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
// 64 floats -> 64 bf16 (128 contiguous bytes) in global memory
__device__ __forceinline__ void st_global_row64_bf16(__nv_bfloat16 *dst, const float *v) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
    w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    reinterpret_cast<uint4 *>(dst)[j] = w;
  }
}

// Named barrier 1 over the 128 softmax / output threads, AND-reducing `ok`.
__device__ __forceinline__ bool epi_sync_and(bool ok) {
  uint32_t res;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.and.pred po, 1, 128, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(res)
      : "r"(uint32_t(ok))
      : "memory");
  return res != 0;
}

struct Unit {
  int64_t b, blk, kb;
  int g;
  int tok0, ttok0;   // first token of the block (packed layout) / of its timeline slots
};
__device__ __forceinline__ Unit unit_of(const IdxParams &p, int64_t unit) {
  Unit u;
  u.g = int(unit % p.G);
  u.blk = (unit / p.G) % p.blocks;
  u.b = unit / (p.G * p.blocks);
  u.kb = p.KB == 1 ? 0 : u.b;
  u.tok0 = int((u.b * p.blocks + u.blk) * p.chunk);
  u.ttok0 = int(u.blk * CAPS + (p.tok_shift ? p.tok_shift[u.b] : 0));
  return u;
}

__global__ void __launch_bounds__(NT, 1)
    mem_indexed_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_o,
                          const IdxParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);
  const int R = int(p.H / p.G);
  const bool timeline = p.tok_shift != nullptr;
  const int64_t stride = gridDim.x;

  if (tid == 0) {
    *abort_flag = (smem_u32(smem) & 1023u) ? 1 : 0;
    for (int i = 0; i < B_COUNT; ++i) {
      uint32_t count = 1;
      if (i == B_KFULL || i == B_VFULL) count = 32;                    // one arrival per producer lane
      if (i == B_PFULL || i == B_PFULL + 1 || i == B_OEMPTY) count = 4;   // one per softmax / output warp
      mbar_init(&bars[i], count);
    }
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_smem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_smem;

  if (warp == 0 || warp == 6) {
    // ===================== loads: Q halves by TMA (warp 0, lane 0) and K rows by cp.async (warp 0);
    //                       V rows by cp.async (warp 6), so the two gathers run side by side =====================
    const bool kq = warp == 0;
    if (kq && lane == 0 && !*abort_flag) prefetch_tensormap(&map_q);
    int issued = 0;
    int phases[4] = {0, 0, 0, 0};   // loads issued on Q half 0, Q half 1, K, V
    bool ok = !*abort_flag;
    const int cb = lane >> 3, j = lane & 7;   // this lane's 16-byte piece of every row
    for (int64_t unit = blockIdx.x; unit < p.units && ok; unit += stride, ++issued) {
      const Unit u = unit_of(p, unit);
      const int n = issued;
      const int64_t *refs = p.refs + unit * CAPS;
      const int64_t r0 = refs[lane], r1 = refs[lane + 32];
      auto load_q = [&](int h) {
        if (n > 0) ok = ok && mbar_wait(&bars[B_QEMPTY + h], (n - 1) & 1, abort_flag, ERR_WAIT_FREE);
        if (ok) ++phases[h];
        if (ok && lane == 0) {
          mbar_arrive_expect_tx(&bars[B_QFULL + h], 4 * 16384);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint8_t *dst = smem + OFF_Q + h * 65536 + c * 16384;
            if (timeline)
              tma_load_4d(dst, &map_q, &bars[B_QFULL + h], c * 64, u.g * R, u.ttok0 + h * 32, int(u.b));
            else
              tma_load_3d(dst, &map_q, &bars[B_QFULL + h], c * 64, u.g * R, u.tok0 + h * 32);
          }
        }
        ok = __all_sync(0xffffffffu, ok);
      };
      // K / V rows: 64 slots x 32 pieces of 16 bytes, lane = piece; the lane
      // waits for its own copies and makes them visible to the tensor core
      // before it arrives on the full barrier
      auto gather = [&](int empty_bar, const __nv_bfloat16 *src, const __nv_bfloat16 *src2, uint32_t off,
                        int &phase) {
        if (n > 0) ok = ok && mbar_wait(&bars[empty_bar], (n - 1) & 1, abort_flag, ERR_WAIT_FREE);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) return;
        ++phase;
        if (p.S2 == 0) {
#pragma unroll 4
          for (int slot = 0; slot < CAPS; ++slot) {
            const int64_t ref = __shfl_sync(0xffffffffu, slot < 32 ? r0 : r1, slot & 31);
            const bool ok_ref = ref >= 0 && ref < p.S;   // out-of-range references read as empty
            const int64_t row = ((u.kb * p.S + (ok_ref ? ref : 0)) * p.G + u.g) * D + lane * 8;
            cp_async16(smem + off + sw128_off(64, cb, slot, j), src + row, ok_ref);
          }
        } else {   // references from S on read the second source (key batch 1)
#pragma unroll 4
          for (int slot = 0; slot < CAPS; ++slot) {
            const int64_t ref = __shfl_sync(0xffffffffu, slot < 32 ? r0 : r1, slot & 31);
            const bool ok_ref = ref >= 0 && ref < p.S + p.S2;
            const bool second = ok_ref && ref >= p.S;
            const int64_t row = ((second ? ref - p.S : (ok_ref ? ref : 0)) * p.G + u.g) * D + lane * 8;
            cp_async16(smem + off + sw128_off(64, cb, slot, j), (second ? src2 : src) + row, ok_ref);
          }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      };
      auto publish = [&](int full_bar) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        fence_async_smem();
        mbar_arrive(&bars[full_bar]);
      };
      if (kq) {
        load_q(0);
        if (ok) gather(B_KEMPTY, p.key, p.key2, OFF_K, phases[2]);
        if (ok) load_q(1);
        if (ok) publish(B_KFULL);
      } else {
        gather(B_VEMPTY, p.value, p.value2, OFF_V, phases[3]);
        if (ok) publish(B_VFULL);
      }
    }
    // drain: every copy issued must have landed before the CTA may exit
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    volatile int drain_flag = 0;
    for (int h = 0; h < 2; ++h)
      if (phases[h] > 0) mbar_wait(&bars[B_QFULL + h], (phases[h] - 1) & 1, &drain_flag, ERR_WAIT_DONE);
    __syncwarp();
  } else if (warp == 1) {
    // ===================== MMA issuer (one thread) =====================
    if (lane == 0) {
      bool ok = !*abort_flag;
      auto wait = [&](int bar, uint32_t parity, int code) {
        ok = ok && mbar_wait(&bars[bar], parity, abort_flag, code);
        tc_fence_after();
        return ok;
      };
      const uint32_t k = smem_u32(smem + OFF_K), v = smem_u32(smem + OFF_V);
      int n = 0;
      for (int64_t unit = blockIdx.x; unit < p.units && ok; unit += stride, ++n) {
        // S of both halves: Q_h K^T (M=128, N=64, K=256)
        if (!wait(B_KFULL, n & 1, ERR_WAIT_KV)) break;
        for (int h = 0; h < 2; ++h) {
          if (!wait(B_QFULL + h, n & 1, ERR_WAIT_Q)) break;
          const uint32_t q = smem_u32(smem + OFF_Q + h * 65536);
#pragma unroll
          for (int kk = 0; kk < 16; ++kk)
            mma_bf16(tmem + T_S + h * 64, sdesc(q + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                     sdesc(k + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), ID_S, kk > 0);
          mma_commit(&bars[B_SFULL + h]);
          mma_commit(&bars[B_QEMPTY + h]);
        }
        if (!ok) break;
        mma_commit(&bars[B_KEMPTY]);
        // O = (P_hi + P_lo) V per half (M=128, N=256, K=64); O is free once the
        // output warps have read the previous half
        if (!wait(B_VFULL, n & 1, ERR_WAIT_KV)) break;
        for (int h = 0; h < 2; ++h) {
          if (!wait(B_PFULL + h, n & 1, ERR_WAIT_P)) break;
          if ((n > 0 || h > 0) && !wait(B_OEMPTY, (h + 1) & 1, ERR_WAIT_FREE)) break;
          const uint32_t ph = tmem + T_P + h * 64;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ts(tmem + T_O, ph + kk * 8, sdesc(v + kk * 2048, 8192, 1024), ID_O, kk > 0);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ts(tmem + T_O, ph + 32 + kk * 8, sdesc(v + kk * 2048, 8192, 1024), ID_O, true);
          mma_commit(&bars[B_OFULL]);
        }
        if (!ok) break;
        mma_commit(&bars[B_VEMPTY]);
      }
      // every MMA issued has finished before TMEM is released
      mma_commit(&bars[B_DONE]);
      volatile int drain_flag = 0;
      mbar_wait(&bars[B_DONE], 0, &drain_flag, ERR_WAIT_DONE);
    }
    __syncwarp();
  } else {
    // ===================== softmax and output: one query row of the half per thread =====================
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    bool ok = !*abort_flag;
    int n = 0, stores = 0;
    for (int64_t unit = blockIdx.x; unit < p.units && ok; unit += stride, ++n) {
      const Unit u = unit_of(p, unit);
      // the valid slots as a 64-bit mask (bit s: reference s is in range)
      const int64_t *refs = p.refs + unit * CAPS;
      const int64_t r0 = refs[lane], r1 = refs[lane + 32];
      const int64_t nrows = p.S + p.S2;
      const uint64_t mask = uint64_t(__ballot_sync(0xffffffffu, r0 >= 0 && r0 < nrows)) |
                            (uint64_t(__ballot_sync(0xffffffffu, r1 >= 0 && r1 < nrows)) << 32);
      float inv_den[2];
      for (int h = 0; h < 2; ++h) {
        ok = ok && mbar_wait(&bars[B_SFULL + h], n & 1, abort_flag, ERR_WAIT_S);
        tc_fence_after();
        if (!ok) break;
        float l[64];
        tmem_ld32(lane_base + T_S + h * 64, l);
        tmem_ld32(lane_base + T_S + h * 64 + 32, l + 32);
        tmem_wait_ld();
        float mx = 0.f;   // the null slot's logit
#pragma unroll
        for (int s = 0; s < 64; ++s) {
          l[s] = (mask >> s) & 1 ? l[s] * p.scale : -INFINITY;
          mx = fmaxf(mx, l[s]);
        }
        float den = __expf(-mx);
#pragma unroll
        for (int s = 0; s < 64; ++s) {
          l[s] = __expf(l[s] - mx);
          den += l[s];
        }
        inv_den[h] = 1.f / den;
        float pw[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) pw[c] = __uint_as_float(pack_bf16x2(l[2 * c], l[2 * c + 1]));
        tmem_st32(lane_base + T_P + h * 64, pw);                                    // P_hi
#pragma unroll
        for (int s = 0; s < 64; ++s) l[s] -= __bfloat162float(__float2bfloat16_rn(l[s]));
#pragma unroll
        for (int c = 0; c < 32; ++c) pw[c] = __uint_as_float(pack_bf16x2(l[2 * c], l[2 * c + 1]));
        tmem_st32(lane_base + T_P + h * 64 + 32, pw);                               // P_lo
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_PFULL + h]);
      }
      ok = epi_sync_and(ok);
      if (!ok) break;
      // ---- O / den -> bf16 -> two staging tiles -> TMA store, per 64-column block ----
      // (timeline halves that are not wholly inside the write range: each
      // thread stores its own row if its slot is in range; a TMA store never
      // starts at a negative or out-of-range token)
      const int64_t shift = timeline ? p.tok_shift[u.b] : 0;
      const int64_t w_lo = timeline ? p.w_lo[u.b] : 0, w_hi = timeline ? p.w_hi[u.b] : 0;
      for (int h = 0; h < 2 && ok; ++h) {
        ok = mbar_wait(&bars[B_OFULL], h, abort_flag, ERR_WAIT_O);
        tc_fence_after();
        ok = epi_sync_and(ok);
        if (!ok) break;
        const int64_t s0 = u.blk * CAPS + h * 32;
        const bool direct = timeline && (s0 < w_lo || s0 + 32 > w_hi || s0 + shift < 0 || s0 + shift + 32 > p.T);
        const int64_t my_slot = s0 + (r >> 2);
        const bool mine = direct && my_slot >= w_lo && my_slot < w_hi && my_slot + shift >= 0 && my_slot + shift < p.T;
        __nv_bfloat16 *my_out = mine ? p.out + (((u.b * p.T + my_slot + shift) * p.H) + u.g * R + (r & 3)) * D : nullptr;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[64];
          tmem_ld32(lane_base + T_O + c * 64, o);
          tmem_ld32(lane_base + T_O + c * 64 + 32, o + 32);
          tmem_wait_ld();
          if (c == 3) {
            // every read of O for this half is done: the next O MMA may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_OEMPTY]);
          }
#pragma unroll
          for (int t = 0; t < 64; ++t) o[t] *= inv_den[h];
          if (direct) {
            if (mine) st_global_row64_bf16(my_out + c * 64, o);
            continue;
          }
          // staging tile stores & 1 is free once the store issued from it two stores ago has read it
          uint8_t *stage = smem + OFF_OS + (stores & 1) * 16384;
          if (r == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          epi_sync_and(true);
          st_row64_bf16(stage, 128, 0, r, o);
          fence_async_smem();
          epi_sync_and(true);
          if (r == 0) {
            if (timeline)
              tma_store_4d(&map_o, stage, c * 64, u.g * R, u.ttok0 + h * 32, int(u.b));
            else
              tma_store_3d(&map_o, stage, c * 64, u.g * R, u.tok0 + h * 32);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          ++stores;
        }
      }
    }
    if (r == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [tokens, H, 256] bf16 with boxes of `pos` positions x R heads x 64 features
int make_map(CUtensorMap *map, const void *base, int64_t ntok, int64_t H, int R, int pos) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(YB_ERR_CUDA, "indexed read tc: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(H), cuuint64_t(ntok)};
  const cuuint64_t strides[2] = {cuuint64_t(D) * 2, cuuint64_t(H) * D * 2};
  const cuuint32_t box[3] = {64, cuuint32_t(R), cuuint32_t(pos)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(YB_ERR_CUDA, "indexed read tc: tensor map encode failed (%d)", int(r));
  return YB_OK;
}

// [B, T, H, 256] bf16 with boxes of `pos` positions x R heads x 64 features of one row
int make_map_4d(CUtensorMap *map, const void *base, int64_t B, int64_t T, int64_t H, int R, int pos) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(YB_ERR_CUDA, "indexed read tc: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(H), cuuint64_t(T), cuuint64_t(B)};
  const cuuint64_t strides[3] = {cuuint64_t(D) * 2, cuuint64_t(H) * D * 2, cuuint64_t(T) * H * D * 2};
  const cuuint32_t box[4] = {64, cuuint32_t(R), cuuint32_t(pos), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(YB_ERR_CUDA, "indexed read tc: tensor map encode failed (%d)", int(r));
  return YB_OK;
}

int idx_sm_count() {
  static int count[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!count[dev] && cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    count[dev] = 148;
  return count[dev];
}

}  // namespace

bool mem_indexed_tc_supported(const MemIndexedArgs &a) {
  // TMA needs 16-byte aligned global bases; cp.async moves 16-byte pieces.
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.query) | reinterpret_cast<uintptr_t>(a.out) |
                         reinterpret_cast<uintptr_t>(a.key) | reinterpret_cast<uintptr_t>(a.value) |
                         reinterpret_cast<uintptr_t>(a.key2) | reinterpret_cast<uintptr_t>(a.value2)) & 15u) == 0;
  return a.dtype == YB_BF16 && a.D == D && a.CAP == CAPS && a.chunk * (a.H / a.G) == ROWS && a.chunk == 64 &&
         a.B * a.blocks * a.G > 0 && aligned;
}

int launch_mem_indexed_tc(const MemIndexedArgs &a) {
  const int64_t ntok = a.B * a.blocks * a.chunk;
  const int R = int(a.H / a.G);
  CUtensorMap mq, mo;
  int rc;
  if (a.tok_shift) {
    rc = make_map_4d(&mq, a.query, a.B, a.T, a.H, R, 32);
    if (!rc) rc = make_map_4d(&mo, a.out, a.B, a.T, a.H, R, 32);
  } else {
    rc = make_map(&mq, a.query, ntok, a.H, R, 32);
    if (!rc) rc = make_map(&mo, a.out, ntok, a.H, R, 32);
  }
  if (rc) return rc;
  IdxParams p;
  p.key = static_cast<const __nv_bfloat16 *>(a.key);
  p.value = static_cast<const __nv_bfloat16 *>(a.value);
  p.refs = a.refs;
  p.blocks = a.blocks; p.chunk = a.chunk; p.H = a.H; p.G = a.G; p.S = a.S; p.KB = a.KB;
  p.scale = 1.0f / sqrtf(float(D));
  p.tok_shift = a.tok_shift; p.w_lo = a.w_lo; p.w_hi = a.w_hi; p.T = a.T;
  p.out = static_cast<__nv_bfloat16 *>(a.out);
  p.key2 = static_cast<const __nv_bfloat16 *>(a.key2);
  p.value2 = static_cast<const __nv_bfloat16 *>(a.value2);
  p.S2 = a.key2 ? a.S2 : 0;
  cudaError_t e = cudaFuncSetAttribute(mem_indexed_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SMEM_BYTES));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "indexed read tc: smem attribute: %s", cudaGetErrorString(e));
  p.units = a.B * a.blocks * a.G;
  const int64_t sms = idx_sm_count();
  mem_indexed_tc_kernel<<<unsigned(p.units < sms ? p.units : sms), NT, SMEM_BYTES, a.stream>>>(mq, mo, p);
  return check_launch("mem_indexed_tc_kernel");
}

int read_device_error_idx(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(tc::g_device_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace yb
