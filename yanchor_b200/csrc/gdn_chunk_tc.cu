// Chunked gated delta rule on the 5th-generation tensor cores (tcgen05 +
// TMEM + TMA), bf16 inputs, K = V = 128, chunk C = 64, fp32 state.
//
// One CTA owns one (sequence, value head) and walks the sequence chunk by
// chunk.  Per chunk, with raw (unnormalised) bf16 q, k, v tiles straight
// from TMA and the L2 norms folded into fp32 scale factors (kn_j = 1/|k_j|,
// qn_i = scale/|q_i|), G the in-chunk cumulative log decay:
//
//   MMA1  [K;Q][K;Q]^T            -> k_i.k_j, q_i.k_j, and |k|^2, |q|^2 on the diagonal
//   A     L_ij = beta_i e^{G_i-G_j} kn_i kn_j k_i.k_j   (j < i),
//         P_ij = qn_i kn_j e^{G_i-G_j} q_i.k_j           (j <= i)
//   A     T = (I + L)^-1 in fp32 (16x16 blocked forward substitution)
//   MMA2  W^T = k^T Tw^T, U^T = v^T Tu^T   with Tw_ij = T_ij beta_j e^{G_j} kn_j,
//                                                Tu_ij = T_ij beta_j   (bf16 hi + lo)
//   MMA3  X^T = S^T W^T, Y^T = S^T q^T                          (state bf16)
//   B     v_new^T = U^T - X^T  (S^T in TMEM already holds e^{G_last} S^T)
//   MMA4  O^T = v_new^T P^T
//   MMA5  S^T += (v_new^T * e^{G_last-G} kn) k     (that operand as bf16 hi + lo)
//   B     o = e^{G} qn Y + O
//
// (the chunk form of transformers qwen3_5 modeling_qwen3_5.py:234-311 and
// of fla's chunk_gated_delta_rule_fwd).  Every state-dependent product is
// computed transposed ("value lanes"): TMEM lane v holds value column v, so
// each thread of group B owns one column of the state, of v_new and of o, and
// all element-wise work stays in registers.  The state lives in TMEM as
// fp32 for the whole sequence and enters the MMAs as a bf16 copy.
//
// Roles: warp 0 = TMA producer (+ gates, cumulative decay), warp 1 = TMEM
// allocator and single-thread MMA issuer, warps 2..5 = group A (the
// state-independent work of a chunk: norms, L, P, T, Tw / Tu, W), warps 6..9
// = group B (the state chain: v_new, the state update, o).  Thread row
// r = 32*(warp%4) + lane is the TMEM lane it may access.  Group A works on
// chunk c + 1 while group B finishes chunk c: MMA1 of chunk c + 1 is issued
// right after MMA2 of chunk c, into the other of two alternating TMEM
// regions, and the shared tiles the two groups touch are distinct or ordered
// by the MMA barriers.
// Every wait is bounded in time; a CTA that gives up records an error code,
// drains its in-flight copies and MMAs, frees TMEM and exits.
#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace yb {
namespace {

using namespace tc;

constexpr int C = 64;       // chunk length
constexpr int KD = 128;     // key dim
constexpr int VD = 128;     // value dim
constexpr int NTHREADS = 320;   // warp 0 TMA, warp 1 MMA, warps 2..5 group A, warps 6..9 group B
constexpr int LP = 68;      // row pitch (floats) of the fp32 L and T matrices: 16-byte aligned rows

// shared memory (byte offsets; SW128 tiles start on 1024-byte boundaries)
constexpr uint32_t OFF_KQ0 = 0;            // [K;Q] stage 0: 2 column blocks of (K 64 rows, Q 64 rows)
constexpr uint32_t OFF_KQ1 = 32768;        // stage 1
constexpr uint32_t OFF_V = 65536;          // V 64 x 128 (one buffer: only MMA2 reads it)
constexpr uint32_t OFF_LF = 81920;         // L fp32 64 x LP; once solved: Tw_lo / Tu_lo
constexpr uint32_t OFF_TWLO = OFF_LF;      // Tw_lo bf16 64x64 (SW128)
constexpr uint32_t OFF_TULO = OFF_LF + 8192;
constexpr uint32_t OFF_TF = 99328;         // raw q.k rows fp32 64 x LP, then T fp32
constexpr uint32_t OFF_P = 116736;         // P bf16 64x64 (SW128)
constexpr uint32_t OFF_TW = 124928;        // Tw bf16 64x64 (SW128); solve scratch before that
constexpr uint32_t OFF_TU = 133120;        // Tu bf16 64x64 (SW128)
constexpr uint32_t OFF_VN = 141312;        // W^T bf16 128x64 (MMA3), then v_new^T (MMA4) of the same chunk
constexpr uint32_t OFF_WT = OFF_VN;
constexpr uint32_t OFF_OST = 157696;       // v~^T hi (MMA5), then the o staging tile [64][128] bf16
constexpr uint32_t OFF_VHI = OFF_OST;      // v~^T bf16 128x64, high part
constexpr uint32_t OFF_VLO = 174080;       // v~^T, low part
constexpr uint32_t OFF_ST = 190464;        // S^T bf16 128x128 (2 column blocks)
constexpr uint32_t OFF_GST = 223232;       // 3 slots: G, beta, e^G, e^{G_last-G} (4 x 64 floats)
constexpr uint32_t OFF_NORM = OFF_GST + 3 * 1024;   // 3 slots: kn[64], qn[64]
constexpr uint32_t OFF_FW = OFF_NORM + 3 * 512;     // Tw column factors beta e^G kn of group A's chunk
constexpr uint32_t OFF_BAR = OFF_FW + 256;          // 17 mbarriers
constexpr uint32_t OFF_MISC = OFF_BAR + 20 * 8;     // tmem base, abort flag
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16;
static_assert(OFF_LF + 64 * LP * 4 <= OFF_TF && OFF_TF + 64 * LP * 4 <= OFF_P, "L / T regions");
static_assert(OFF_TULO + 8192 <= OFF_TF && OFF_TF % 1024 == 0, "tiles inside L");
static_assert(OFF_P % 1024 == 0 && OFF_VN % 1024 == 0 && OFF_ST % 1024 == 0 && OFF_ST + 32768 <= OFF_GST, "tiles");
static_assert(3 * 320 * 4 <= 8192, "solve scratch fits the Tw tile");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

// TMEM columns (fp32, 128 lanes).  Chunk c uses region R(c) = c even ? T_R0 : T_R1
// for [K;Q][K;Q]^T, then U^T (first 64 columns) and W^T / X^T (last 64).
constexpr uint32_t T_R0 = 0;
constexpr uint32_t T_R1 = 128;
constexpr uint32_t T_Y = 256;    // Y^T
constexpr uint32_t T_O = 320;    // O^T
constexpr uint32_t T_S = 384;    // S^T fp32 state (128 columns)

constexpr uint32_t ID_N64_KK = idesc_bf16(128, 64, false, false);
constexpr uint32_t ID_N128_KK = idesc_bf16(128, 128, false, false);
constexpr uint32_t ID_N64_MK = idesc_bf16(128, 64, true, false);
constexpr uint32_t ID_N64_KM = idesc_bf16(128, 64, false, true);
constexpr uint32_t ID_N128_KM = idesc_bf16(128, 128, false, true);

// error codes recorded in g_device_error
constexpr int ERR_WAIT_FULL = 0x101, ERR_WAIT_EMPTY = 0x102, ERR_WAIT_MMA = 0x103, ERR_WAIT_EPI = 0x104,
              ERR_ALIGN = 0x105, ERR_WAIT_DONE = 0x106;

struct TcParams {
  const void *g, *beta;
  int64_t g_ts, beta_ts;
  int g_dtype, beta_dtype;
  const float *A_log, *dt_bias;
  const float *h0;
  float *ht;
  __nv_bfloat16 *o;
#ifdef YB_TC_DEBUG
  float *dbg;  // test-only build: intermediates of CTA 0, chunk 0
#endif
  const int64_t *cu;
  int64_t T;
  int H, HV;
  float scale;
  uint32_t flags;
};

__device__ __forceinline__ float load_scalar(const void *p, int64_t idx, int dtype) {
  if (dtype == YB_F32) return static_cast<const float *>(p)[idx];
  if (dtype == YB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[idx]);
  return __half2float(static_cast<const __half *>(p)[idx]);
}


__device__ __forceinline__ uint32_t to_tf32(float x) {
  // the raw fp32 bits: the tf32 MMA reads the top 19 bits (truncation), which
  // saves a conversion per operand on the inverse's latency-bound chains
  return __float_as_uint(x);
}

// acc (16x16 as two 16x8 tiles, m16n8 accumulator fragments) += A (16x16) B (16x16),
// both fp32 row-major in shared memory (pitches lda, ldb), on the warp-level tf32
// tensor-core path (these 16x16 blocks are far below tcgen05's 128-row tiles).
__device__ __forceinline__ void block_mma16_tf32(float acc[2][4], const float *pa, int lda, const float *pb, int ldb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < 16; k0 += 8) {
    const uint32_t a0 = to_tf32(pa[g * lda + k0 + t]), a1 = to_tf32(pa[(g + 8) * lda + k0 + t]);
    const uint32_t a2 = to_tf32(pa[g * lda + k0 + t + 4]), a3 = to_tf32(pa[(g + 8) * lda + k0 + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint32_t b0 = to_tf32(pb[(k0 + t) * ldb + nt * 8 + g]), b1 = to_tf32(pb[(k0 + t + 4) * ldb + nt * 8 + g]);
      asm volatile(
          "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%0,%1,%2,%3};"
          : "+f"(acc[nt][0]), "+f"(acc[nt][1]), "+f"(acc[nt][2]), "+f"(acc[nt][3])
          : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
  }
}

// dst (16x16 fp32, pitch ld) = sign * acc
__device__ __forceinline__ void store_block16(float *dst, int ld, const float acc[2][4], float sign) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    dst[g * ld + nt * 8 + 2 * t] = sign * acc[nt][0];
    dst[g * ld + nt * 8 + 2 * t + 1] = sign * acc[nt][1];
    dst[(g + 8) * ld + nt * 8 + 2 * t] = sign * acc[nt][2];
    dst[(g + 8) * ld + nt * 8 + 2 * t + 1] = sign * acc[nt][3];
  }
}

constexpr int DBG_D1 = 0, DBG_W = 16384, DBG_U = 24576, DBG_X = 32768, DBG_Y = 40960, DBG_O = 49152,
              DBG_S1 = 57344, DBG_T = 73728, DBG_NORM = 77824, DBG_TS = 78000;
#ifdef YB_TC_DEBUG
// Test-only: copy `n` values of TMEM row r (already in registers) into the
// debug buffer at tile offset `off` (row-major, `n` columns).
#define YB_DBG_ROW(off, width, base, n, vals)                                          \
  do {                                                                                 \
    if (p.dbg && blockIdx.x == 0 && c == 0)                                            \
      for (int _i = 0; _i < (n); ++_i) p.dbg[(off) + r * (width) + (base) + _i] = (vals)[_i]; \
  } while (0)
// Test-only: phase timestamps (ns since the thread started) of thread 0 of
// each epilogue group of CTA 0 for the first 32 chunks, 16 events per chunk
// (group A events 0..7, group B events 8..13).
#define YB_DBG_TS(ev)                                                                   \
  do {                                                                                  \
    if (p.dbg && blockIdx.x == 0 && r == 0 && c < 32)                                   \
      p.dbg[DBG_TS + c * 16 + (ev)] = float(globaltimer_ns() - dbg_t0);                 \
  } while (0)
#else
#define YB_DBG_ROW(off, width, base, n, vals) \
  do {                                        \
  } while (0)
#define YB_DBG_TS(ev) \
  do {                \
  } while (0)
#endif

// 64 values -> one SW128 row of bf16 (8 x 16-byte stores), and as two
// 32-value halves (one per TMEM load) for the state copy.
__device__ __forceinline__ void st_half_bf16(uint8_t *tile, int rows, int cb, int r, int jbase, const float *v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
    w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4 *>(tile + sw128_off(rows, cb, r, jbase + j)) = w;
  }
}

// 64 values of one row as packed bf16 pairs -> one SW128 row half (jbase 0) or
// second half (jbase 4) from 16 packed words.
__device__ __forceinline__ void st_half_packed(uint8_t *tile, int rows, int cb, int r, int jbase, const uint32_t *pk) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4 *>(tile + sw128_off(rows, cb, r, jbase + j)) =
        make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
}

// Named barrier of group A (warps 2..5, barrier 1).  The *_and forms also AND
// a status across the group, so that a wait that gave up ends the
// loop in every thread of the group together (none is left at a barrier).
__device__ __forceinline__ bool a_sync_and(bool ok) {
  uint32_t res;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.and.pred po, 1, 128, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(res)
      : "r"(uint32_t(ok))
      : "memory");
  return res != 0;
}
// group B (warps 6..9, barrier 3)
__device__ __forceinline__ bool b_sync_and(bool ok) {
  uint32_t res;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.and.pred po, 3, 128, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(res)
      : "r"(uint32_t(ok))
      : "memory");
  return res != 0;
}

__global__ void __launch_bounds__(NTHREADS, 1)
    gdn_chunk_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint64_t *full_kq = bars + 0;    // [2] K, Q tiles of a stage landed + its gates written (32 + tx)
  uint64_t *empty_kq = bars + 2;   // [2] the stage's last MMA (MMA5) finished (1)
  uint64_t *full_v = bars + 4;     // V landed (1 + tx)
  uint64_t *empty_v = bars + 5;    // MMA2 read V (1)
  uint64_t *mma1_bar = bars + 6;   // [2] [K;Q][K;Q]^T of chunk c in TMEM (c & 1 selects)
  uint64_t *mma2_bar = bars + 8;   // W in TMEM
  uint64_t *mma3_bar = bars + 9;   // X, Y in TMEM
  uint64_t *mma45_bar = bars + 10; // O in TMEM, state updated
  uint64_t *a_wt = bars + 11;      // group A: P and W^T tiles written (128)
  uint64_t *b_vn = bars + 12;      // group B: v_new, v~ tiles written (128)
  uint64_t *b_done = bars + 13;    // group B: state copy for the next MMA3 written, Y / O consumed, the
                                   //          state scaled by the next chunk's decay (128)
  uint64_t *done_bar = bars + 14;
  uint64_t *a_tw = bars + 15;      // [2] group A: Tw / Tu tiles and the norms written, [K;Q][K;Q]^T
                                   //     consumed (128; c & 1 selects)
  uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

  const int n = blockIdx.x / p.HV, hv = blockIdx.x % p.HV;
  const int h = hv / (p.HV / p.H);
  int64_t bos, len;
  if (p.cu) {
    bos = p.cu[n];
    len = p.cu[n + 1] - bos;
  } else {
    bos = int64_t(n) * p.T;
    len = p.T;
  }
  const int nchunks = int((len + C - 1) / C);
  const int64_t head = (int64_t(n) * p.HV + hv) * int64_t(KD) * VD;
  const bool trans = p.flags & YB_GDN_TRANSPOSE_STATE;

  if (tid == 0) {
    *abort_flag = (smem_u32(smem) & 1023u) ? 1 : 0;  // SW128 tiles need a 1024-byte aligned base
    if (*abort_flag) atomicCAS(&g_device_error, 0, ERR_ALIGN);
    mbar_init(&full_kq[0], 32);
    mbar_init(&full_kq[1], 32);
    mbar_init(&empty_kq[0], 1);
    mbar_init(&empty_kq[1], 1);
    mbar_init(full_v, 1);
    mbar_init(empty_v, 1);
    mbar_init(&mma1_bar[0], 1);
    mbar_init(&mma1_bar[1], 1);
    mbar_init(mma2_bar, 1);
    mbar_init(mma3_bar, 1);
    mbar_init(mma45_bar, 1);
    mbar_init(&a_tw[0], 128);
    mbar_init(&a_tw[1], 128);
    mbar_init(a_wt, 128);
    mbar_init(b_vn, 128);
    mbar_init(b_done, 128);
    mbar_init(done_bar, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_smem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_smem;

  if (warp == 0) {
    // ===================== producer: TMA and gates =====================
    if (lane == 0) {
      prefetch_tensormap(&map_q);
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
    }
    const bool gate_in = p.flags & YB_GDN_GATE_IN_KERNEL;
    const bool beta_sig = p.flags & YB_GDN_BETA_SIGMOID;
    const float a_coef = gate_in ? -expf(p.A_log[hv]) : 0.f;
    const float dtb = (gate_in && p.dt_bias) ? p.dt_bias[hv] : 0.f;
    int issued_kq = 0, issued_v = 0;
    for (int c = 0; c < nchunks && !*abort_flag; ++c) {
      const int s = c & 1;
      const int tok0 = int(bos + int64_t(c) * C);
      if (c >= 2 && !mbar_wait(&empty_kq[s], ((c >> 1) - 1) & 1, abort_flag, ERR_WAIT_EMPTY)) break;
      if (lane == 0) {
        uint8_t *kq = smem + (s ? OFF_KQ1 : OFF_KQ0);
        mbar_expect_tx(&full_kq[s], 4 * 8192);
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
          tma_load_3d(kq + cb * 16384, &map_k, &full_kq[s], cb * 64, h, tok0);
          tma_load_3d(kq + cb * 16384 + 8192, &map_q, &full_kq[s], cb * 64, h, tok0);
        }
      }
      issued_kq = c + 1;
      // gates, masked beyond the sequence, and the cumulative decay (slot c % 3:
      // its previous user, chunk c - 3, finished before this stage came free)
      float gv[2], bv[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = lane + 32 * half;
        const int64_t t = int64_t(c) * C + i;
        float gl = 0.f, b = 0.f;
        if (t < len) {
          const int64_t tok = bos + t;
          gl = load_scalar(p.g, tok * p.g_ts + hv, p.g_dtype);
          if (gate_in) gl = a_coef * softplus20(gl + dtb);
          b = load_scalar(p.beta, tok * p.beta_ts + hv, p.beta_dtype);
          if (beta_sig) b = round_to<__nv_bfloat16>(sigmoidf_(b));   // beta in the input dtype, as the reference stores it
        }
        gv[half] = gl;
        bv[half] = b;
      }
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y0 = __shfl_up_sync(0xffffffffu, gv[0], off), y1 = __shfl_up_sync(0xffffffffu, gv[1], off);
        if (lane >= off) {
          gv[0] += y0;
          gv[1] += y1;
        }
      }
      gv[1] += __shfl_sync(0xffffffffu, gv[0], 31);
      const float glast = __shfl_sync(0xffffffffu, gv[1], 31);
      float *gst = reinterpret_cast<float *>(smem + OFF_GST + (c % 3) * 1024);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = lane + 32 * half;
        gst[i] = gv[half];
        gst[64 + i] = bv[half];
        gst[128 + i] = expf(gv[half]);
        gst[192 + i] = expf(glast - gv[half]);
      }
      __syncwarp();
      mbar_arrive(&full_kq[s]);
      // V of chunk c once MMA2 of chunk c - 1 has read the buffer
      if (c >= 1 && !mbar_wait(empty_v, (c - 1) & 1, abort_flag, ERR_WAIT_EMPTY)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(full_v, 2 * 8192);
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) tma_load_3d(smem + OFF_V + cb * 8192, &map_v, full_v, cb * 64, hv, tok0);
      }
      issued_v = c + 1;
    }
    // drain: every issued copy must have landed before the CTA may exit (bounded
    // in time, but not cut short by another role's abort)
    volatile int drain_flag = 0;
    for (int c = (issued_kq > 2 ? issued_kq - 2 : 0); c < issued_kq; ++c)
      mbar_wait(&full_kq[c & 1], (c >> 1) & 1, &drain_flag, ERR_WAIT_FULL);
    if (issued_v > 0) mbar_wait(full_v, (issued_v - 1) & 1, &drain_flag, ERR_WAIT_FULL);
  } else if (warp == 1) {
    // ===================== MMA issuer (one thread) =====================
    if (lane == 0) {
      bool ok = true;
      auto wait = [&](uint64_t *bar, uint32_t parity, int code) {
        ok = ok && mbar_wait(bar, parity, abort_flag, code);
        tc_fence_after();
        return ok;
      };
      auto mma1 = [&](int c) {   // [K;Q] [K;Q]^T  (M=128, N=128, K=128) into R(c)
        const uint32_t kq = smem_u32(smem + ((c & 1) ? OFF_KQ1 : OFF_KQ0));
        const uint32_t d = tmem + ((c & 1) ? T_R1 : T_R0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_bf16(d, sdesc(kq + off, 16, 1024), sdesc(kq + off, 16, 1024), ID_N128_KK, kk > 0);
        }
        mma_commit(&mma1_bar[c & 1]);
      };
      if (nchunks > 0 && wait(&full_kq[0], 0, ERR_WAIT_FULL)) mma1(0);
      for (int c = 0; c < nchunks && ok; ++c) {
        const int s = c & 1;
        const uint32_t kq = smem_u32(smem + (s ? OFF_KQ1 : OFF_KQ0));
        const uint32_t R = tmem + (s ? T_R1 : T_R0);
        // MMA2: W^T = k^T (Tw_hi + Tw_lo)^T -> R + 64, committed on its own so group A can copy W^T
        // while U^T = v^T (Tu_hi + Tu_lo)^T -> R runs   (M=128, N=64, K=64)
        if (!wait(&a_tw[s], (c >> 1) & 1, ERR_WAIT_EPI)) break;
        const uint32_t vt = smem_u32(smem + OFF_V);
        const uint32_t tw = smem_u32(smem + OFF_TW), tu = smem_u32(smem + OFF_TU);
        const uint32_t twl = smem_u32(smem + OFF_TWLO), tul = smem_u32(smem + OFF_TULO);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(R + 64, sdesc(kq + kk * 2048, 16384, 1024), sdesc(tw + kk * 32, 16, 1024), ID_N64_MK, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(R + 64, sdesc(kq + kk * 2048, 16384, 1024), sdesc(twl + kk * 32, 16, 1024), ID_N64_MK, true);
        mma_commit(mma2_bar);
        if (!wait(full_v, c & 1, ERR_WAIT_FULL)) break;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(R, sdesc(vt + kk * 2048, 8192, 1024), sdesc(tu + kk * 32, 16, 1024), ID_N64_MK, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(R, sdesc(vt + kk * 2048, 8192, 1024), sdesc(tul + kk * 32, 16, 1024), ID_N64_MK, true);
        mma_commit(empty_v);
        // MMA1 of chunk c + 1 into R(c + 1): group B read U, X of chunk c - 1 there before its b_vn;
        // the stage's copy was issued a whole group-A phase ago (after MMA5 of chunk c - 1)
        if (c + 1 < nchunks) {
          if (!wait(&full_kq[s ^ 1], ((c + 1) >> 1) & 1, ERR_WAIT_FULL)) break;
          mma1(c + 1);
        }
        // MMA3: X^T = S^T W^T -> R + 64 ;  Y^T = S^T q^T -> T_Y   (M=128, N=64, K=128)
        if (!wait(a_wt, c & 1, ERR_WAIT_EPI) || !wait(b_done, c & 1, ERR_WAIT_EPI)) break;
        const uint32_t st = smem_u32(smem + OFF_ST), wt = smem_u32(smem + OFF_WT);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = sdesc(st + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          mma_bf16(R + 64, a, sdesc(wt + kk * 2048, 16384, 1024), ID_N64_KM, kk > 0);
          mma_bf16(tmem + T_Y, a, sdesc(kq + 8192 + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), ID_N64_KK,
                   kk > 0);
        }
        mma_commit(mma3_bar);
        // MMA4: O^T = v_new^T P^T (N=64, K=64) ;  MMA5: S^T += (v~_hi + v~_lo)^T k (N=128, K=64), the
        // state already scaled by the chunk's decay (group B did it with the previous state copy)
        if (!wait(b_vn, c & 1, ERR_WAIT_EPI)) break;
        const uint32_t vn = smem_u32(smem + OFF_VN), pp = smem_u32(smem + OFF_P);
        const uint32_t vhi = smem_u32(smem + OFF_VHI), vlo = smem_u32(smem + OFF_VLO);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16(tmem + T_O, sdesc(vn + kk * 32, 16, 1024), sdesc(pp + kk * 32, 16, 1024), ID_N64_KK, kk > 0);
          mma_bf16(tmem + T_S, sdesc(vhi + kk * 32, 16, 1024), sdesc(kq + kk * 2048, 16384, 1024), ID_N128_KM,
                   true);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(tmem + T_S, sdesc(vlo + kk * 32, 16, 1024), sdesc(kq + kk * 2048, 16384, 1024), ID_N128_KM,
                   true);
        mma_commit(mma45_bar);
        mma_commit(&empty_kq[s]);
      }
      // all issued MMAs finished before TMEM is released
      mma_commit(done_bar);
      mbar_wait(done_bar, 0, abort_flag, ERR_WAIT_DONE);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ===================== group A: the state-independent work of a chunk =====================
    // thread r = TMEM lane r: rows r < 64 are L rows (and the solve), rows 64..127 P rows
    const int r = (warp & 3) * 32 + lane;
#ifdef YB_TC_DEBUG
    const uint64_t dbg_t0 = globaltimer_ns();
#endif
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    const bool l2 = p.flags & YB_GDN_QK_L2NORM;
    float *LF = reinterpret_cast<float *>(smem + OFF_LF);
    bool ok = true;
    auto signal = [&](uint64_t *bar) {
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(bar);
    };
    for (int c = 0; c < nchunks && ok; ++c) {
      const int s = c & 1;
      const uint32_t R = s ? T_R1 : T_R0;
      const float *gst = reinterpret_cast<const float *>(smem + OFF_GST + (c % 3) * 1024);
      const float *G = gst, *BT = gst + 64, *EG = gst + 128;
      float *kn = reinterpret_cast<float *>(smem + OFF_NORM + (c % 3) * 512);
      float *qn = kn + 64;
      float *fw = reinterpret_cast<float *>(smem + OFF_FW);
      YB_DBG_TS(0);
      ok = mbar_wait(&full_kq[s], (c >> 1) & 1, abort_flag, ERR_WAIT_FULL);
      ok = ok && mbar_wait(&mma1_bar[s], (c >> 1) & 1, abort_flag, ERR_WAIT_MMA);
      tc_fence_after();
      YB_DBG_TS(1);
      // ---------- norms from the diagonal of [K;Q][K;Q]^T; the raw k_i.k_j rows (threads r < 64)
      //            into the L buffer, the raw q_i.k_j rows (r >= 64) into the T buffer ----------
      if (ok) {
        float dg[32];
        tmem_ld32(lane_base + R + uint32_t(r & ~31), dg);
        tmem_wait_ld();
#ifdef YB_TC_DEBUG
        if (p.dbg && blockIdx.x == 0 && c == 0) {
          float full_row[32];
          for (int q4 = 0; q4 < 4; ++q4) {
            tmem_ld32(lane_base + R + q4 * 32, full_row);
            tmem_wait_ld();
            for (int t = 0; t < 32; ++t) p.dbg[DBG_D1 + r * 128 + q4 * 32 + t] = full_row[t];
          }
        }
#endif
        float diag = 0.f;
#pragma unroll
        for (int t = 0; t < 32; ++t) diag = (t == lane) ? dg[t] : diag;
        const float nrm = l2 ? rsqrtf(diag + 1e-6f) : 1.f;
        if (r < 64) {
          kn[r] = nrm;
          fw[r] = BT[r] * EG[r] * nrm;
        } else {
          qn[r - 64] = nrm * p.scale;
        }
        float *raw = (r < 64 ? LF : reinterpret_cast<float *>(smem + OFF_TF)) + (r & 63) * LP;
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          float d1[32];
          tmem_ld32(lane_base + R + uint32_t(32 * hf), d1);
          tmem_wait_ld();
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            *reinterpret_cast<float4 *>(raw + 32 * hf + 4 * j4) =
                make_float4(d1[4 * j4], d1[4 * j4 + 1], d1[4 * j4 + 2], d1[4 * j4 + 3]);
        }
      }
      if (!(ok = a_sync_and(ok))) break;
      YB_DBG_TS(2);
      // ---------- L and P of row i = r & 63, columns 32 (r >> 6) .. +31, sharing one
      //            e^{g_i - g_j} per entry: L in place (k_i.k_j, j < i), P packed into registers
      //            (q_i.k_j, j <= i) and stored once MMA2 shows that MMA4 of chunk c - 1 has
      //            read the P tile.  Branch-free masks; the exponent is clamped so masked entries
      //            stay finite.  Rows i < 32 have nothing in columns 32..63 (L is never read there). ----------
      float *TF = reinterpret_cast<float *>(smem + OFF_TF);   // raw q.k, then T fp32, pitch LP
      uint32_t pk[16];
      {
        const int i = r & 63, jb = 32 * (r >> 6);
        if (jb > i) {   // uniform across a warp: its lanes share r >> 5
#pragma unroll
          for (int t = 0; t < 16; ++t) pk[t] = 0u;
        } else {
          const float ci = BT[i] * kn[i], qi = qn[i], gi = G[i];
          float4 *row4 = reinterpret_cast<float4 *>(LF + i * LP + jb);
          const float4 *qk4 = reinterpret_cast<const float4 *>(TF + i * LP + jb);
          const float4 *kn4 = reinterpret_cast<const float4 *>(kn + jb);
          const float4 *g4 = reinterpret_cast<const float4 *>(G + jb);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            float4 d = row4[j4];
            const float4 qq = qk4[j4], kk = kn4[j4], gg = g4[j4];
            const int j = jb + 4 * j4;
            const float e0 = __expf(fminf(gi - gg.x, 0.f)), e1 = __expf(fminf(gi - gg.y, 0.f));
            const float e2 = __expf(fminf(gi - gg.z, 0.f)), e3 = __expf(fminf(gi - gg.w, 0.f));
            d.x *= ci * kk.x * e0 * float(j < i);
            d.y *= ci * kk.y * e1 * float(j + 1 < i);
            d.z *= ci * kk.z * e2 * float(j + 2 < i);
            d.w *= ci * kk.w * e3 * float(j + 3 < i);
            row4[j4] = d;
            pk[2 * j4] = pack_bf16x2(qi * kk.x * e0 * qq.x * float(j <= i), qi * kk.y * e1 * qq.y * float(j + 1 <= i));
            pk[2 * j4 + 1] =
                pack_bf16x2(qi * kk.z * e2 * qq.z * float(j + 2 <= i), qi * kk.w * e3 * qq.w * float(j + 3 <= i));
          }
        }
      }
      if (!(ok = a_sync_and(ok))) break;
      YB_DBG_TS(3);
      // ---------- T = (I + L)^-1 by 16x16 blocks: the diagonal blocks D_j = (I + L_jj)^-1 by
      //            forward substitution (thread r < 64 solves column r of its block in registers),
      //            then T_ij = -D_i sum_{m=j}^{i-1} L_im T_mj for i > j, one warp per column
      //            block j walking down its blocks, so a warp only reads the T blocks it wrote ----------
      if (r < 64) {
        const int j = r, b = j >> 4, jj = j & 15;
        float x[16];
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) {
          const float4 *L4 = reinterpret_cast<const float4 *>(LF + (b * 16 + ii) * LP + b * 16);
          float a0 = 0.f, a1 = 0.f;
#pragma unroll
          for (int q = 0; 4 * q < ii; ++q) {
            const float4 l = L4[q];
            if (4 * q < ii) a0 = fmaf(l.x, x[4 * q], a0);
            if (4 * q + 1 < ii) a1 = fmaf(l.y, x[4 * q + 1], a1);
            if (4 * q + 2 < ii) a0 = fmaf(l.z, x[4 * q + 2], a0);
            if (4 * q + 3 < ii) a1 = fmaf(l.w, x[4 * q + 3], a1);
          }
          x[ii] = ii < jj ? 0.f : (ii == jj ? 1.f : -(a0 + a1));
        }
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) TF[(b * 16 + ii) * LP + j] = x[ii];
      }
      if (!(ok = a_sync_and(ok))) break;
      {
        const int jc = r >> 5;   // this warp's column block
        if (jc < 3) {
          float *scr = reinterpret_cast<float *>(smem + OFF_TW) + jc * 320;   // 16x16, pitch 20
          auto lblk = [&](int i, int m) { return LF + (i * 16) * LP + m * 16; };
          auto tblk = [&](int i, int m) { return TF + (i * 16) * LP + m * 16; };
          // acc[n]: sum_m L_im T_mj for block row i = jc + 1 + n, over the T_mj known so far
          float acc[3][2][4] = {};
#pragma unroll
          for (int n = 0; n < 3; ++n)
            if (jc + 1 + n < 4) block_mma16_tf32(acc[n], lblk(jc + 1 + n, jc), LP, tblk(jc, jc), LP);
#pragma unroll
          for (int n = 0; n < 3; ++n) {
            const int i = jc + 1 + n;
            if (i < 4) {
              store_block16(scr, 20, acc[n], 1.f);
              __syncwarp();
              float t[2][4] = {};
              block_mma16_tf32(t, tblk(i, i), LP, scr, 20);
              store_block16(tblk(i, jc), LP, t, -1.f);
              __syncwarp();
#pragma unroll
              for (int n2 = n + 1; n2 < 3; ++n2)
                if (jc + 1 + n2 < 4) block_mma16_tf32(acc[n2], lblk(jc + 1 + n2, i), LP, tblk(i, jc), LP);
            }
          }
        }
      }
      if (!(ok = a_sync_and(ok))) break;
      YB_DBG_TS(4);
      // ---------- Tw (rows of threads r < 64) and Tu (r >= 64) from T, as bf16 hi + lo tiles:
      //            both factors enter MMA2 as hi + lo, since a single bf16 rounding of T alone
      //            costs ~2e-3 relative on the state ----------
      {
        const int i = r & 63;
        const float *fac = r < 64 ? fw : BT;   // Tw = T diag(beta e^G kn), Tu = T diag(beta)
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            // blocks above the diagonal are zero (the buffer holds stale data there)
            float4 t4 = *reinterpret_cast<const float4 *>(TF + i * LP + 32 * hf + 4 * j4);
            if (((32 * hf + 4 * j4) >> 4) > (i >> 4)) t4 = make_float4(0.f, 0.f, 0.f, 0.f);
#ifdef YB_TC_DEBUG
            if (p.dbg && blockIdx.x == 0 && c == 0 && r < 64) {
              float *d = p.dbg + DBG_T + r * 64 + 32 * hf + 4 * j4;
              d[0] = t4.x, d[1] = t4.y, d[2] = t4.z, d[3] = t4.w;
            }
#endif
            const float4 f4 = *reinterpret_cast<const float4 *>(fac + 32 * hf + 4 * j4);
            t4.x *= f4.x, t4.y *= f4.y, t4.z *= f4.z, t4.w *= f4.w;
            const uint32_t h0 = pack_bf16x2(t4.x, t4.y), h1 = pack_bf16x2(t4.z, t4.w);
            hi[2 * j4] = h0;
            hi[2 * j4 + 1] = h1;
            lo[2 * j4] = pack_bf16x2(t4.x - __uint_as_float(h0 << 16), t4.y - __uint_as_float(h0 & 0xffff0000u));
            lo[2 * j4 + 1] = pack_bf16x2(t4.z - __uint_as_float(h1 << 16), t4.w - __uint_as_float(h1 & 0xffff0000u));
          }
          st_half_packed(smem + (r < 64 ? OFF_TW : OFF_TU), 64, 0, i, 4 * hf, hi);
          st_half_packed(smem + (r < 64 ? OFF_TWLO : OFF_TULO), 64, 0, i, 4 * hf, lo);
        }
#ifdef YB_TC_DEBUG
        if (p.dbg && blockIdx.x == 0 && c == 0) p.dbg[DBG_NORM + r] = r < 64 ? kn[r] : qn[r - 64];
#endif
      }
      signal(&a_tw[s]);
      YB_DBG_TS(5);
      // ---------- P, and W^T (MN-major B operand of MMA3) over the v_new tile ----------
      // MMA2 of this chunk was issued after MMA4 / MMA5 of the previous one, so
      // once it is done the P and v_new tiles of chunk c - 1 have been read
      ok = mbar_wait(mma2_bar, c & 1, abort_flag, ERR_WAIT_MMA);
      tc_fence_after();
      if (!(ok = a_sync_and(ok))) break;
      YB_DBG_TS(6);
      st_half_packed(smem + OFF_P, 64, 0, r & 63, 4 * (r >> 6), pk);
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        float w[32];
        tmem_ld32(lane_base + R + 64 + uint32_t(32 * hf), w);
        tmem_wait_ld();
        YB_DBG_ROW(DBG_W, 64, 32 * hf, 32, w);
        st_half_bf16(smem + OFF_WT, 128, 0, r, 4 * hf, w);
      }
      signal(a_wt);
      YB_DBG_TS(7);
    }
  } else {
    // ===================== group B: the state chain of a chunk =====================
    // thread r = TMEM lane r = value column r of the state, of v_new and of o
    const int r = (warp & 3) * 32 + lane;
#ifdef YB_TC_DEBUG
    const uint64_t dbg_t0 = globaltimer_ns();
#endif
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    uint8_t *st_tile = smem + OFF_ST;
    bool ok = true;
    auto signal = [&](uint64_t *bar) {
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(bar);
    };
    // ---- initial state: bf16 copy for the first MMA3, and fp32 into TMEM scaled by
    //      the first chunk's decay (MMA5 of a chunk accumulates into e^{G_last} S) ----
    float decay0 = 1.f;
    if (nchunks > 0) {
      ok = mbar_wait(&full_kq[0], 0, abort_flag, ERR_WAIT_FULL);   // gates of chunk 0
      decay0 = reinterpret_cast<const float *>(smem + OFF_GST)[128 + 63];
    }
#pragma unroll 1
    for (int q4 = 0; q4 < 4; ++q4) {
      float row[32];
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        const int dd = q4 * 32 + d;
        row[d] = p.h0 ? (trans ? p.h0[head + int64_t(r) * KD + dd] : p.h0[head + int64_t(dd) * VD + r]) : 0.f;
      }
      if (nchunks == 0 && p.ht) {
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          const int dd = q4 * 32 + d;
          if (trans) p.ht[head + int64_t(r) * KD + dd] = row[d];
          else p.ht[head + int64_t(dd) * VD + r] = row[d];
        }
      }
      st_half_bf16(st_tile, 128, q4 >> 1, r, (q4 & 1) * 4, row);
#pragma unroll
      for (int d = 0; d < 32; ++d) row[d] *= decay0;
      tmem_st32(lane_base + T_S + q4 * 32, row);
    }
    tmem_wait_st();
    if (ok) signal(b_done);

    for (int c = 0; c < nchunks; ++c) {
      // every thread of the group has finished the previous chunk (its reads of
      // the o staging tile included); a wait that gave up ends the loop for all
      if (!(ok = b_sync_and(ok))) break;
      const int s = c & 1;
      const uint32_t R = s ? T_R1 : T_R0;
      const float *gst = reinterpret_cast<const float *>(smem + OFF_GST + (c % 3) * 1024);
      const float *EG = gst + 128, *TAIL = gst + 192;
      const float *kn = reinterpret_cast<const float *>(smem + OFF_NORM + (c % 3) * 512);
      const float *qn = kn + 64;
      const int m = int(len - int64_t(c) * C < C ? len - int64_t(c) * C : C);
      const bool last = c == nchunks - 1;
      YB_DBG_TS(8);
      ok = mbar_wait(mma3_bar, c & 1, abort_flag, ERR_WAIT_MMA);
      // the chunk's gates and norms: acquired from group A's release (it wrote the
      // norms after acquiring the gates); that barrier's next phase is chunk c + 2
      ok = ok && mbar_wait(&a_tw[s], (c >> 1) & 1, abort_flag, ERR_WAIT_EPI);
      tc_fence_after();
      YB_DBG_TS(9);
      // ---------- v_new = U - X; v~ = v_new e^{G_last-G} kn as bf16 hi + lo ----------
      if (ok) {
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          float u[32], x[32];
          tmem_ld32(lane_base + R + uint32_t(32 * hf), u);
          tmem_ld32(lane_base + R + 64 + uint32_t(32 * hf), x);
          tmem_wait_ld();
          YB_DBG_ROW(DBG_U, 64, 32 * hf, 32, u);
          YB_DBG_ROW(DBG_X, 64, 32 * hf, 32, x);
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] -= x[i];
          st_half_bf16(smem + OFF_VN, 128, 0, r, 4 * hf, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] *= TAIL[32 * hf + i] * kn[32 * hf + i];
          st_half_bf16(smem + OFF_VHI, 128, 0, r, 4 * hf, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] -= __bfloat162float(__float2bfloat16_rn(u[i]));
          st_half_bf16(smem + OFF_VLO, 128, 0, r, 4 * hf, u);
        }
        signal(b_vn);
      }
      YB_DBG_TS(10);
      ok = ok && mbar_wait(mma45_bar, c & 1, abort_flag, ERR_WAIT_MMA);
      // the next chunk's decay scales the state now (its gates were written two chunks ahead)
      if (!last) ok = ok && mbar_wait(&full_kq[s ^ 1], ((c + 1) >> 1) & 1, abort_flag, ERR_WAIT_FULL);
      tc_fence_after();
      YB_DBG_TS(11);
      if (ok) {
        // ---------- o = e^{G} qn Y + O for this value column, staged as [token][value]
        //            rows over the v~_hi tile (MMA5 has read it) ----------
        __nv_bfloat16 *ostage = reinterpret_cast<__nv_bfloat16 *>(smem + OFF_OST);
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          float y[32], oo[32];
          tmem_ld32(lane_base + T_Y + uint32_t(32 * hf), y);
          tmem_ld32(lane_base + T_O + uint32_t(32 * hf), oo);
          tmem_wait_ld();
          YB_DBG_ROW(DBG_Y, 64, 32 * hf, 32, y);
          YB_DBG_ROW(DBG_O, 64, 32 * hf, 32, oo);
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int a = 32 * hf + t;
            ostage[a * 128 + r] = __float2bfloat16_rn(EG[a] * qn[a] * y[t] + oo[t]);
          }
        }
        // ---------- the updated state: bf16 copy for the next MMA3 (ht after the last chunk),
        //            then fp32 scaled by the next chunk's decay back into TMEM ----------
        const float dnext =
            last ? 1.f : reinterpret_cast<const float *>(smem + OFF_GST + ((c + 1) % 3) * 1024)[128 + 63];
#pragma unroll 1
        for (int q4 = 0; q4 < 4; ++q4) {
          float sv[32];
          tmem_ld32(lane_base + T_S + q4 * 32, sv);
          tmem_wait_ld();
#ifdef YB_TC_DEBUG
          if (p.dbg && blockIdx.x == 0 && c == 0)
            for (int d = 0; d < 32; ++d) p.dbg[DBG_S1 + r * 128 + q4 * 32 + d] = sv[d];
#endif
          st_half_bf16(st_tile, 128, q4 >> 1, r, (q4 & 1) * 4, sv);
          if (last) {
            if (p.ht) {
#pragma unroll
              for (int d = 0; d < 32; ++d) {
                const int dd = q4 * 32 + d;
                if (trans) p.ht[head + int64_t(r) * KD + dd] = sv[d];
                else p.ht[head + int64_t(dd) * VD + r] = sv[d];
              }
            }
          } else {
#pragma unroll
            for (int d = 0; d < 32; ++d) sv[d] *= dnext;
            tmem_st32(lane_base + T_S + q4 * 32, sv);
          }
        }
        tmem_wait_st();
        signal(b_done);
        YB_DBG_TS(12);
      }
      if (!(ok = b_sync_and(ok))) break;
      // ---------- o out: 16-byte piece q = r + 128 t covers token q / 16, bytes 16 (q % 16) ----------
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int q = r + 128 * t, i = q >> 4, piece = q & 15;
        if (i < m) {
          const uint4 v = *reinterpret_cast<const uint4 *>(smem + OFF_OST + q * 16);
          *reinterpret_cast<uint4 *>(p.o + ((bos + int64_t(c) * C + i) * p.HV + hv) * VD + piece * 8) = v;
        }
      }
      YB_DBG_TS(13);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---- host side ----------------------------------------------------------------
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

// [tokens, heads, 128] bf16 -> boxes of 64 tokens x 1 head x 64 features, 128-byte swizzle
int make_map(CUtensorMap *map, const void *base, int64_t ntok, int64_t heads, int64_t tok_stride) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(YB_ERR_CUDA, "gdn chunk tc: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {128, cuuint64_t(heads), cuuint64_t(ntok)};
  const cuuint64_t strides[2] = {128 * 2, cuuint64_t(tok_stride) * 2};
  const cuuint32_t box[3] = {64, 1, 64};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(YB_ERR_CUDA, "gdn chunk tc: tensor map encode failed (%d)", int(r));
  return YB_OK;
}

}  // namespace

bool gdn_chunk_tc_supported(const GdnArgs &a) {
  return a.io_dtype == YB_BF16 && a.K == KD && a.V == VD && a.B * a.T > 0;
}

int launch_gdn_chunk_tc_impl(const GdnArgs &a, float *dbg) {
  const int64_t ntok = a.B * a.T;
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, a.q, ntok, a.H, a.q_ts);
  if (!rc) rc = make_map(&mk, a.k, ntok, a.H, a.k_ts);
  if (!rc) rc = make_map(&mv, a.v, ntok, a.HV, a.v_ts);
  if (rc) return rc;
  TcParams p;
  p.g = a.g; p.beta = a.beta; p.g_ts = a.g_ts; p.beta_ts = a.beta_ts;
  p.g_dtype = a.g_dtype; p.beta_dtype = a.beta_dtype;
  p.A_log = a.A_log; p.dt_bias = a.dt_bias;
  p.h0 = a.h0; p.ht = a.ht; p.o = static_cast<__nv_bfloat16 *>(a.o);
  p.cu = a.cu_seqlens; p.T = a.T; p.H = int(a.H); p.HV = int(a.HV);
  p.scale = a.scale; p.flags = a.flags;
#ifdef YB_TC_DEBUG
  p.dbg = dbg;
#else
  (void)dbg;
#endif
  cudaError_t e = cudaFuncSetAttribute(gdn_chunk_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SMEM_BYTES));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gdn chunk tc: smem attribute: %s", cudaGetErrorString(e));
  gdn_chunk_tc_kernel<<<unsigned(a.N * a.HV), NTHREADS, SMEM_BYTES, a.stream>>>(mq, mk, mv, p);
  return check_launch("gdn_chunk_tc_kernel");
}

int launch_gdn_chunk_tc(const GdnArgs &a) { return launch_gdn_chunk_tc_impl(a, nullptr); }

int read_device_error(int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int));
  if (e != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(tc::g_device_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace yb
