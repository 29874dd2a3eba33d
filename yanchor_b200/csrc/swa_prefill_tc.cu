// Sliding-window prefill attention on the tcgen05 tensor cores, bf16, D = 256
// (the YANchor SWA layer): queries [B, Tq, QH, D] at absolute positions
// query_start + i attend to keys [B, Tk, KVH, D] at positions j with
// i_abs - window < j <= i_abs and key_valid[b, j]; scale D^-1/2; grouped
// query heads (R = QH / KVH); a query whose own key_valid entry is false, or
// that admits no key, gives zeros.  (modeling_yanchor.py:412-427
// reference_swa; flash_swa :429-449 over each row's valid tokens.)
//
// One CTA per (row b, KV head, P = 128 / R query positions): its 128 query
// rows are the (position, head) pairs of the group's R heads, brought in by
// TMA in that order.  The keys the tile can see (at most window + P - 1)
// stream through in 64-key tiles:
//   warp 0   TMA producer of Q (once) and the K tiles (4 stages, each
//            released when its S MMA is done)
//   warp 6   TMA producer of the V tiles (3 stages, each released when its
//            PV MMA is done)
//   warp 1   TMEM allocator and S issuer: S(t) = Q K(t)^T (M=128, N=64,
//            K=256) with Q resident in TMEM, issued as soon as the softmax
//            warps have read S(t-1), so it runs under their softmax
//   warp 7   PV issuer: O += P(t) V(t) (N=256) with P in TMEM, issued as soon
//            as P(t) is there (two issuing threads, so neither waits behind
//            the other's MMAs; they write disjoint TMEM and commit their own)
//   warps 2-5  one query row per thread: copy the Q row into TMEM once; per
//            tile mask, online softmax in base 2 (O is rescaled only when the
//            row max grows by more than 2^8), P as bf16 (as FlashAttention
//            rounds it) into one of two TMEM buffers; at the end O / l staged
//            in shared memory and TMA-stored.
// Shared memory holds only the K / V stages (224 KB), deep enough to hide
// the ~2 us a tile's copy takes.  Every barrier a role can lag on is indexed
// by stage or tile parity, so no parity wait can see a barrier two phases
// ahead.  Every wait is bounded in time; a CTA that gives up records an
// error code, drains its copies and MMAs, frees TMEM and exits.
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace yb {
namespace {

using namespace tc;

constexpr int D = 256, NT = 256, KT = 64, KST = 4, VST = 3;
constexpr uint32_t OFF_K = 0;              // K: 4 stages x 4 column blocks x 64 rows x 128 B (later the O staging)
constexpr uint32_t OFF_V = 131072;         // V: 3 stages (the first two hold Q until it is in TMEM)
constexpr uint32_t OFF_BAR = 229376;
constexpr uint32_t OFF_MISC = OFF_BAR + 24 * 8;   // 24 mbarriers
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16;
static_assert(OFF_V + VST * 32768 <= OFF_BAR && SMEM_BYTES <= 232448, "shared memory budget");
constexpr uint32_t T_Q = 0;                // Q: 128 columns of packed bf16 pairs
constexpr uint32_t T_S = 128;              // S: 64 columns
constexpr uint32_t T_P = 192;              // P: 2 x 32 columns of packed bf16 pairs
constexpr uint32_t T_O = 256;              // O: 256 columns
constexpr uint32_t ID_S = idesc_bf16(128, 64, false, false);
constexpr uint32_t ID_O = idesc_bf16(128, 256, false, true);
constexpr float kRescale = 8.f;            // log2 of the largest exp2 factor P may carry before O is rescaled
constexpr int ERR_SP_Q = 0x501, ERR_SP_FULL = 0x502, ERR_SP_EMPTY = 0x503, ERR_SP_S = 0x504, ERR_SP_P = 0x505,
              ERR_SP_O = 0x506, ERR_SP_DONE = 0x507, ERR_SP_FREE = 0x508;

struct SpParams {
  const uint8_t *key_valid;
  int64_t valid_bs;
  int64_t Tq, Tk, KVH, window, query_start, qtiles;
  int R, P;
  float scale_log2;
};

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
// 2^x on the special-function unit (PTX ex2.approx.ftz; 2^-inf = +0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// the softmax warps' named barrier (barrier 1, 128 threads), ANDing a status
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

__global__ void __launch_bounds__(NT, 1)
    swa_prefill_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                          const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                          const SpParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint64_t *qbar = bars + 0;       // Q landed in shared memory (1 + tx)
  uint64_t *q_ready = bars + 1;    // the softmax warps copied Q into TMEM (128)
  uint64_t *full_k = bars + 2;     // [4] K tile landed (1 + tx)
  uint64_t *empty_k = bars + 6;    // [4] the tile's S MMA finished (1)
  uint64_t *full_v = bars + 10;    // [3] V tile landed (1 + tx)
  uint64_t *empty_v = bars + 13;   // [3] the tile's PV MMA finished (1)
  uint64_t *s_full = bars + 16;    // S of the tile in TMEM (1)
  uint64_t *s_free = bars + 17;    // the softmax warps have read S (128)
  uint64_t *p_ready = bars + 18;   // [2] P of the tile in TMEM, O rescaled if needed (128)
  uint64_t *o_done = bars + 20;    // [2] O += P V of the tile finished (1)
  uint64_t *done_bar = bars + 22;   // [2] all MMAs of the S / PV issuer finished
  uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

  const int64_t unit = blockIdx.x;
  const int64_t qt = unit % p.qtiles;
  const int kvh = int((unit / p.qtiles) % p.KVH);
  const int b = int(unit / (p.qtiles * p.KVH));
  const int64_t qp0 = qt * p.P;                                     // first query of the tile
  const int64_t qabs0 = p.query_start + qp0;
  const int64_t qlast = p.query_start + (p.Tq < qp0 + p.P ? p.Tq : qp0 + p.P) - 1;
  const int64_t lo = qabs0 - p.window + 1 > 0 ? qabs0 - p.window + 1 : 0;
  const int64_t hi = qlast < p.Tk - 1 ? qlast : p.Tk - 1;
  const int ntiles = hi >= lo ? int((hi - lo) / KT + 1) : 0;

  if (tid == 0) {
    *abort_flag = (smem_u32(smem) & 1023u) ? 1 : 0;  // SW128 tiles need a 1024-byte aligned base
    if (*abort_flag) atomicCAS(&g_device_error, 0, ERR_SP_Q);
    mbar_init(qbar, 1);
    mbar_init(q_ready, 128);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&full_k[s], 1);
      mbar_init(&empty_k[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&full_v[s], 1);
      mbar_init(&empty_v[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&p_ready[s], 128);
      mbar_init(&o_done[s], 1);
    }
    mbar_init(&done_bar[0], 1);
    mbar_init(&done_bar[1], 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_smem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_smem;

  if (warp == 0 || warp == 6) {
    // ===================== producers: Q and K (warp 0), V (warp 6) =====================
    if (lane == 0) {
      const bool is_k = warp == 0;
      if (is_k && ntiles > 0 && !*abort_flag) {
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_k);
        mbar_arrive_expect_tx(qbar, 4 * 16384);
#pragma unroll
        for (int cb = 0; cb < 4; ++cb)
          tma_load_4d(smem + OFF_V + cb * 16384, &map_q, qbar, cb * 64, kvh * p.R, int(qp0), b);
      }
      const int nst = is_k ? KST : VST;
      uint64_t *fullb = is_k ? full_k : full_v, *emptyb = is_k ? empty_k : empty_v;
      const CUtensorMap *map = is_k ? &map_k : &map_v;
      uint8_t *base = smem + (is_k ? OFF_K : OFF_V);
      int issued = 0;
      bool ok = true;
      // V's first stages hold Q until the softmax warps have copied it into TMEM
      if (!is_k && ntiles > 0) {
        prefetch_tensormap(&map_v);
        ok = mbar_wait(q_ready, 0, abort_flag, ERR_SP_Q);
      }
      for (int t = 0; t < ntiles && ok && !*abort_flag; ++t) {
        const int s = t % nst;
        if (t >= nst && !mbar_wait(&emptyb[s], (t / nst - 1) & 1, abort_flag, ERR_SP_EMPTY)) break;
        mbar_arrive_expect_tx(&fullb[s], 4 * 8192);
        const int kt0 = int(lo + int64_t(t) * KT);
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) tma_load_4d(base + s * 32768 + cb * 8192, map, &fullb[s], cb * 64, kvh, kt0, b);
        issued = t + 1;
      }
      // drain: every issued copy must have landed before the CTA may exit
      volatile int drain_flag = 0;
      if (is_k && ntiles > 0) mbar_wait(qbar, 0, &drain_flag, ERR_SP_Q);
      for (int t = (issued > nst ? issued - nst : 0); t < issued; ++t)
        mbar_wait(&fullb[t % nst], (t / nst) & 1, &drain_flag, ERR_SP_FULL);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 7) {
    // ===================== MMA issuers: S (warp 1), PV (warp 7), one thread each =====================
    if (lane == 0 && ntiles > 0) {
      const bool is_s = warp == 1;
      bool ok = true;
      auto wait = [&](uint64_t *bar, uint32_t parity, int code) {
        ok = ok && mbar_wait(bar, parity, abort_flag, code);
        tc_fence_after();
        return ok;
      };
      if (is_s) {
        wait(q_ready, 0, ERR_SP_Q);
        for (int t = 0; t < ntiles && ok; ++t) {
          const int s = t % KST;
          if (!wait(&full_k[s], (t / KST) & 1, ERR_SP_FULL)) break;
          if (t >= 1 && !wait(s_free, (t - 1) & 1, ERR_SP_FREE)) break;
          const uint32_t k = smem_u32(smem + OFF_K + s * 32768);
#pragma unroll
          for (int kk = 0; kk < 16; ++kk)
            mma_bf16_ts(tmem + T_S, tmem + T_Q + kk * 8, sdesc(k + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024),
                        ID_S, kk > 0);
          mma_commit(s_full);
          mma_commit(&empty_k[s]);
        }
      } else {
        for (int u = 0; u < ntiles && ok; ++u) {
          const int pb = u & 1, sv = u % VST;
          if (!wait(&p_ready[pb], (u >> 1) & 1, ERR_SP_P) || !wait(&full_v[sv], (u / VST) & 1, ERR_SP_FULL)) break;
          const uint32_t v = smem_u32(smem + OFF_V + sv * 32768);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ts(tmem + T_O, tmem + T_P + pb * 32 + kk * 8, sdesc(v + kk * 2048, 8192, 1024), ID_O,
                        u > 0 || kk > 0);
          mma_commit(&o_done[pb]);
          mma_commit(&empty_v[sv]);
        }
      }
      // all MMAs this thread issued finished before TMEM is released
      mma_commit(&done_bar[is_s ? 0 : 1]);
      mbar_wait(&done_bar[is_s ? 0 : 1], 0, abort_flag, ERR_SP_DONE);
    }
    __syncwarp();
  } else {
    // ===================== softmax and output (one query row per thread) =====================
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    const int64_t qp = qp0 + r / p.R;
    const int64_t qabs = p.query_start + qp;
    const bool has_valid = p.key_valid != nullptr;
    bool ok = true;
    // ---- this row of Q into TMEM (packed bf16 pairs, as they sit in memory) ----
    if (ntiles > 0) {
      ok = mbar_wait(qbar, 0, abort_flag, ERR_SP_Q);
      if (ok) {
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
          float w[32];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 c4 = *reinterpret_cast<const uint4 *>(smem + OFF_V + sw128_off(128, cb, r, j));
            w[4 * j] = __uint_as_float(c4.x);
            w[4 * j + 1] = __uint_as_float(c4.y);
            w[4 * j + 2] = __uint_as_float(c4.z);
            w[4 * j + 3] = __uint_as_float(c4.w);
          }
          tmem_st32(lane_base + T_Q + cb * 32, w);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(q_ready);
    }
    float m_run = -INFINITY, l = 0.f;
    for (int t = 0; t < ntiles; ++t) {
      const int s = t & 1;
      const int64_t kt0 = lo + int64_t(t) * KT;
      ok = ok && mbar_wait(s_full, t & 1, abort_flag, ERR_SP_S);
      tc_fence_after();
      if (!ok) break;
      float x[64];
      tmem_ld32(lane_base + T_S, x);
      tmem_ld32(lane_base + T_S + 32, x + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_free);
      // key c of the tile sits d0 - c positions before this query: admitted when
      // 0 <= d0 - c < window, it exists (kt0 + c < Tk) and its key_valid flag is
      // set.  The window leaves a contiguous range of c, so the admitted keys
      // are one 64-bit mask and every tile runs the same loop.
      const int d0 = int(qabs - kt0);
      int c_lo = d0 - p.window + 1, c_hi = d0;                       // window: c in [c_lo, c_hi]
      const int nk = int(p.Tk - kt0 < KT ? p.Tk - kt0 : KT);
      c_hi = c_hi < nk - 1 ? c_hi : nk - 1;
      c_lo = c_lo > 0 ? c_lo : 0;
      // pass 1: the admitted keys' largest raw logit (masked keys become -inf);
      // a tile wholly inside the window needs no mask
      float mx[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx[u] = -INFINITY;
      if (has_valid) {
        uint64_t adm = 0;
        if (c_lo <= c_hi) adm = (~uint64_t(0) >> (63 - c_hi)) & (~uint64_t(0) << c_lo);
        if (adm) {
          const uint8_t *kv = p.key_valid + int64_t(b) * p.valid_bs + kt0;
          uint64_t vm = 0;
#pragma unroll 1
          for (int c = 0; c < nk; ++c) vm |= uint64_t(kv[c] != 0) << c;
          adm &= vm;
        }
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          x[c] = (adm >> c) & 1 ? x[c] : -INFINITY;
          mx[c & 7] = fmaxf(mx[c & 7], x[c]);
        }
      } else if (c_lo == 0 && c_hi == KT - 1) {
#pragma unroll
        for (int c = 0; c < 64; ++c) mx[c & 7] = fmaxf(mx[c & 7], x[c]);
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          x[c] = c >= c_lo && c <= c_hi ? x[c] : -INFINITY;
          mx[c & 7] = fmaxf(mx[c & 7], x[c]);
        }
      }
      // the running max in the scaled base-2 domain (scale_log2 > 0 keeps the order)
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * p.scale_log2;
      const float m_new = fmaxf(m_run, mt);
      if (m_new > m_run + kRescale) {
        // the running max grows by more than 2^8: rescale O (once the previous
        // tile's PV has landed) and l to the new max
        if (m_run != -INFINITY) {
          const float f = ex2(m_run - m_new);
          ok = mbar_wait(&o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, ERR_SP_O);
          tc_fence_after();
          if (!ok) break;
#pragma unroll 1
          for (int q4 = 0; q4 < 8; ++q4) {
            float o[32];
            tmem_ld32(lane_base + T_O + q4 * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 32; ++d) o[d] *= f;
            tmem_st32(lane_base + T_O + q4 * 32, o);
          }
          tmem_wait_st();
          l *= f;
        }
        m_run = m_new;
      }
      // pass 2: p = 2^(x scale_log2 - m_run), one FFMA and one ex2 per key
      // (m_run is -inf only while every key so far was masked: then all p are 0)
      float ls[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) ls[u] = 0.f;
      if (m_run != -INFINITY) {
        const float nm = -m_run;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          x[c] = ex2(fmaf(x[c], p.scale_log2, nm));
          ls[c & 7] += x[c];
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] = 0.f;
      }
      l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
      // P buffer t & 1 was last read by the PV MMA of tile t - 2
      if (t >= 2) ok = mbar_wait(&o_done[s], ((t - 2) >> 1) & 1, abort_flag, ERR_SP_O);
      if (!ok) break;
      float pw[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) pw[c] = __uint_as_float(pack_bf16x2(x[2 * c], x[2 * c + 1]));
      tmem_st32(lane_base + T_P + s * 32, pw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_ready[s]);
    }
    if (ok && ntiles > 0) {
      ok = mbar_wait(&o_done[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1, abort_flag, ERR_SP_O);
      tc_fence_after();
    }
    // ---- O / l (zero for a query without admitted keys or marked invalid) staged over the K stages
    //      (every S MMA, the last reader of K, is done) ----
    bool row_valid = qp < p.Tq && l > 0.f;
    if (row_valid && p.key_valid) row_valid = qabs < p.Tk && p.key_valid[int64_t(b) * p.valid_bs + qabs] != 0;
    const float inv = row_valid ? 1.f / l : 0.f;
    const bool use_o = ok && ntiles > 0;
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      float o[64];
      if (use_o) {
        tmem_ld32(lane_base + T_O + cb * 64, o);
        tmem_ld32(lane_base + T_O + cb * 64 + 32, o + 32);
        tmem_wait_ld();
      }
#pragma unroll
      for (int d = 0; d < 64; ++d) o[d] = use_o ? o[d] * inv : 0.f;
      st_row64_bf16(smem + OFF_K + cb * 16384, 128, 0, r, o);
    }
    fence_async_smem();
    ok = epi_sync_and(ok);
    if (r == 0 && ok) {
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) tma_store_4d(&map_o, smem + OFF_K + cb * 16384, cb * 64, kvh * p.R, int(qp0), b);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      // the CTA may exit once the store has read its staging tile; the
      // writes to global memory complete on their own
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
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

// [B, T, H, 256] bf16, boxes of `pos` positions x `heads` heads x 64 features of one row
int make_map(CUtensorMap *map, const void *base, int64_t B, int64_t T, int64_t H, int heads, int pos) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(YB_ERR_CUDA, "swa prefill: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(H), cuuint64_t(T), cuuint64_t(B)};
  const cuuint64_t strides[3] = {cuuint64_t(D) * 2, cuuint64_t(H) * D * 2, cuuint64_t(T) * H * D * 2};
  const cuuint32_t box[4] = {64, cuuint32_t(heads), cuuint32_t(pos), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(YB_ERR_CUDA, "swa prefill: tensor map encode failed (%d)", int(r));
  return YB_OK;
}

}  // namespace

bool swa_prefill_tc_supported(const SwaPrefillArgs &a) {
  const int64_t R = a.KVH > 0 ? a.QH / a.KVH : 0;
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                         reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out)) & 15u) == 0;
  return a.dtype == YB_BF16 && a.D == D && a.QH % a.KVH == 0 && (R == 1 || R == 2 || R == 4 || R == 8) &&
         a.window >= 1 && aligned && a.Tq <= (int64_t(1) << 30) && a.Tk <= (int64_t(1) << 30);
}

int launch_swa_prefill_tc(const SwaPrefillArgs &a) {
  if (a.B * a.Tq == 0) return YB_OK;
  if (!swa_prefill_tc_supported(a))
    return set_error(YB_ERR_UNSUPPORTED, "swa prefill: bf16, D = 256, QH / KVH in 1/2/4/8, 16-byte aligned only");
  const int R = int(a.QH / a.KVH), P = 128 / R;
  CUtensorMap mq, mk, mv, mo;
  int rc = make_map(&mq, a.q, a.B, a.Tq, a.QH, R, P);
  if (!rc) rc = make_map(&mo, a.out, a.B, a.Tq, a.QH, R, P);
  if (!rc) rc = make_map(&mk, a.k, a.B, a.Tk, a.KVH, 1, KT);
  if (!rc) rc = make_map(&mv, a.v, a.B, a.Tk, a.KVH, 1, KT);
  if (rc) return rc;
  SpParams p{};
  p.key_valid = a.key_valid;
  p.valid_bs = a.valid_bs;
  p.Tq = a.Tq; p.Tk = a.Tk; p.KVH = a.KVH; p.window = a.window; p.query_start = a.query_start;
  p.R = R; p.P = P;
  p.qtiles = (a.Tq + P - 1) / P;
  p.scale_log2 = float(1.4426950408889634 / sqrt(double(D)));
  cudaError_t e = cudaFuncSetAttribute(swa_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SMEM_BYTES));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "swa prefill: smem attribute: %s", cudaGetErrorString(e));
  const int64_t grid = a.B * a.KVH * p.qtiles;
  swa_prefill_tc_kernel<<<unsigned(grid), NT, SMEM_BYTES, a.stream>>>(mq, mk, mv, mo, p);
  return check_launch("swa_prefill_tc_kernel");
}

int read_device_error_swa(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(tc::g_device_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace yb
