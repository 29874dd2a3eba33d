// Prefill anchor read (indexed GQA) on the tcgen05 tensor cores, bf16,
// D = 256, CAP = 64 referenced rows, 256 query rows per unit (chunk 64 x 4
// heads per group) — the YANchor memory shape.
//
// One CTA handles one unit (row b, block, group g).  Its 256 query rows are
// the (position, head) pairs of the block's 64 positions and the group's 4
// heads; TMA brings them in as one 3-D box per 64-column slice, already in
// (position, head) row order.  The 64 referenced key / value rows are
// gathered with cp.async (empty references become zero rows).  Per 128-row
// half:
//   S = Q K^T (TMEM, fp32)  ->  softmax over the 64 slots plus the null slot
//   (logit 0, value 0), masked where the reference is empty  ->  P as bf16
//   hi + lo parts  ->  O = (P_hi + P_lo) V (TMEM)  ->  O / den in bf16 ->
//   TMA store.
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

constexpr int D = 256, CAPS = 64, ROWS = 256, NT = 128;
constexpr uint32_t OFF_QO = 0;          // Q (then P, then O staging): 4 column blocks x 256 rows x 128 B
constexpr uint32_t OFF_K = 131072;      // K: 4 column blocks x 64 rows x 128 B
constexpr uint32_t OFF_V = 163840;      // V: same
constexpr uint32_t OFF_BAR = 196608;
constexpr uint32_t OFF_MISC = OFF_BAR + 32;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 64 * 4;   // + valid[64]
constexpr uint32_t T_S = 0;      // S half 0 / half 1 at cols 0 / 64
constexpr uint32_t T_O = 256;    // O (256 columns)
constexpr uint32_t ID_S = idesc_bf16(128, 64, false, false);
constexpr uint32_t ID_O = idesc_bf16(128, 256, false, true);
constexpr int ERR_WAIT_Q = 0x201, ERR_WAIT_S = 0x202, ERR_WAIT_O = 0x203;

struct IdxParams {
  const __nv_bfloat16 *key, *value;
  const int64_t *refs;
  int64_t blocks, chunk, H, G, S, KB;
  float scale;
  // timeline mode (tok_shift != nullptr)
  const int64_t *tok_shift, *w_lo, *w_hi;
  int64_t T;
  __nv_bfloat16 *out;
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

__global__ void __launch_bounds__(NT, 1)
    mem_indexed_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_o,
                          const IdxParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t *qbar = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint64_t *mbar = qbar + 1;
  uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);
  float *valid = reinterpret_cast<float *>(smem + OFF_MISC + 16);

  const int64_t unit = blockIdx.x;
  const int g = int(unit % p.G);
  const int64_t blk = (unit / p.G) % p.blocks;
  const int64_t b = unit / (p.G * p.blocks);
  const int64_t kb = p.KB == 1 ? 0 : b;
  const int R = int(p.H / p.G);
  const int tok0 = int((b * p.blocks + blk) * p.chunk);
  const int64_t *refs = p.refs + unit * CAPS;
  const bool timeline = p.tok_shift != nullptr;
  const int64_t shift = timeline ? p.tok_shift[b] : 0;
  const int64_t w_lo = timeline ? p.w_lo[b] : 0, w_hi = timeline ? p.w_hi[b] : 0;
  const int ttok0 = int(blk * CAPS + shift);        // timeline: token of the block's first slot

  if (tid == 0) {
    *abort_flag = (smem_u32(smem) & 1023u) ? 1 : 0;
    mbar_init(qbar, 1);
    mbar_init(mbar, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_base_smem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_smem;
  const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
  bool ok = !*abort_flag;

  if (tid == 0 && ok) {
    prefetch_tensormap(&map_q);
    mbar_arrive_expect_tx(qbar, 4 * 32768);
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      if (timeline)
        tma_load_4d(smem + OFF_QO + cb * 32768, &map_q, qbar, cb * 64, g * R, ttok0, int(b));
      else
        tma_load_3d(smem + OFF_QO + cb * 32768, &map_q, qbar, cb * 64, g * R, tok0);
    }
  }
  // gather the referenced key / value rows (16-byte pieces, swizzled rows)
  for (int e = tid; e < CAPS * 32; e += NT) {
    const int slot = e >> 5, piece = e & 31, cb = piece >> 3, j = piece & 7;
    const int64_t ref = refs[slot];
    const bool ok_ref = ref >= 0 && ref < p.S;   // out-of-range references read as empty
    const int64_t row = ((kb * p.S + (ok_ref ? ref : 0)) * p.G + g) * D + piece * 8;
    const uint32_t off = sw128_off(64, cb, slot, j);
    cp_async16(smem + OFF_K + off, p.key + row, ok_ref);
    cp_async16(smem + OFF_V + off, p.value + row, ok_ref);
    if (piece == 0) valid[slot] = ok_ref ? 1.f : 0.f;
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  fence_async_smem();
  __syncthreads();
  int mphase = 0;
  auto wait_mma = [&](int code) {
    ok = ok && mbar_wait(mbar, mphase & 1, abort_flag, code);
    ++mphase;
    tc_fence_after();
    ok = !__syncthreads_or(!ok);   // every thread takes the same branch after a wait
  };
  if (ok) ok = mbar_wait(qbar, 0, abort_flag, ERR_WAIT_Q);
  ok = !__syncthreads_or(!ok);

  // S for both halves: Q_h K^T (M=128, N=64, K=256)
  if (tid == 0 && ok) {
    tc_fence_after();
    const uint32_t q = smem_u32(smem + OFF_QO), k = smem_u32(smem + OFF_K);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)
        mma_bf16(tmem + T_S + h * 64, sdesc(q + (kk >> 2) * 32768 + h * 16384 + (kk & 3) * 32, 16, 1024),
                 sdesc(k + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), ID_S, kk > 0);
    mma_commit(mbar);
  }
  wait_mma(ERR_WAIT_S);

  for (int h = 0; h < 2 && ok; ++h) {
    // ---- softmax of row `tid` of half h; P hi / lo into the dead Q rows ----
    float inv_den;
    {
      float l[64];
      tmem_ld32(lane_base + T_S + h * 64, l);
      tmem_ld32(lane_base + T_S + h * 64 + 32, l + 32);
      tmem_wait_ld();
      float mx = 0.f;   // the null slot's logit
#pragma unroll
      for (int s = 0; s < 64; ++s) {
        l[s] = valid[s] > 0.f ? l[s] * p.scale : -INFINITY;
        mx = fmaxf(mx, l[s]);
      }
      float den = __expf(-mx);
#pragma unroll
      for (int s = 0; s < 64; ++s) {
        l[s] = __expf(l[s] - mx);
        den += l[s];
      }
      inv_den = 1.f / den;
      st_row64_bf16(smem + OFF_QO + h * 16384, 128, 0, tid, l);            // P_hi (column block 0)
#pragma unroll
      for (int s = 0; s < 64; ++s) l[s] -= __bfloat162float(__float2bfloat16_rn(l[s]));
      st_row64_bf16(smem + OFF_QO + 32768 + h * 16384, 128, 0, tid, l);    // P_lo (column block 1)
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- O = (P_hi + P_lo) V (M=128, N=256, K=64) ----
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ph = smem_u32(smem + OFF_QO + h * 16384), pl = smem_u32(smem + OFF_QO + 32768 + h * 16384);
      const uint32_t v = smem_u32(smem + OFF_V);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_bf16(tmem + T_O, sdesc(ph + kk * 32, 16, 1024), sdesc(v + kk * 2048, 8192, 1024), ID_O, kk > 0);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_bf16(tmem + T_O, sdesc(pl + kk * 32, 16, 1024), sdesc(v + kk * 2048, 8192, 1024), ID_O, true);
      mma_commit(mbar);
    }
    wait_mma(ERR_WAIT_O);
    if (!ok) break;
    // ---- O / den -> bf16 staging (rows of half h, 4 column blocks) -> TMA store ----
    // (timeline halves that are not wholly inside the write range: each
    // thread stores its own row if its slot is in range)
    // (a TMA store never starts at a negative or out-of-range token)
    const int64_t s0 = blk * CAPS + h * 32;
    const bool direct = timeline && (s0 < w_lo || s0 + 32 > w_hi || s0 + shift < 0 || s0 + shift + 32 > p.T);
    const int64_t my_slot = s0 + (tid >> 2);
    const bool mine = direct && my_slot >= w_lo && my_slot < w_hi && my_slot + shift >= 0 && my_slot + shift < p.T;
    __nv_bfloat16 *my_out =
        mine ? p.out + (((b * p.T + my_slot + shift) * p.H) + g * R + (tid & 3)) * D : nullptr;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      float o[64];
      tmem_ld32(lane_base + T_O + cb * 64, o);
      tmem_ld32(lane_base + T_O + cb * 64 + 32, o + 32);
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < 64; ++t) o[t] *= inv_den;
      if (direct) {
        if (mine) st_global_row64_bf16(my_out + cb * 64, o);
      } else {
        st_row64_bf16(smem + OFF_QO + cb * 32768 + h * 16384, 128, 0, tid, o);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && !direct) {
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        if (timeline)
          tma_store_4d(&map_o, smem + OFF_QO + cb * 32768 + h * 16384, cb * 64, g * R, ttok0 + h * 32, int(b));
        else
          tma_store_3d(&map_o, smem + OFF_QO + cb * 32768 + h * 16384, cb * 64, g * R, tok0 + h * 32);
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  if (tid == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
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

}  // namespace

bool mem_indexed_tc_supported(const MemIndexedArgs &a) {
  // TMA needs 16-byte aligned global bases; cp.async moves 16-byte pieces.
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.query) | reinterpret_cast<uintptr_t>(a.out) |
                         reinterpret_cast<uintptr_t>(a.key) | reinterpret_cast<uintptr_t>(a.value)) & 15u) == 0;
  return a.dtype == YB_BF16 && a.D == D && a.CAP == CAPS && a.chunk * (a.H / a.G) == ROWS && a.chunk == 64 &&
         a.B * a.blocks * a.G > 0 && aligned;
}

int launch_mem_indexed_tc(const MemIndexedArgs &a) {
  const int64_t ntok = a.B * a.blocks * a.chunk;
  const int R = int(a.H / a.G);
  CUtensorMap mq, mo;
  int rc;
  if (a.tok_shift) {
    rc = make_map_4d(&mq, a.query, a.B, a.T, a.H, R, 64);
    if (!rc) rc = make_map_4d(&mo, a.out, a.B, a.T, a.H, R, 32);
  } else {
    rc = make_map(&mq, a.query, ntok, a.H, R, 64);
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
  cudaError_t e = cudaFuncSetAttribute(mem_indexed_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SMEM_BYTES));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "indexed read tc: smem attribute: %s", cudaGetErrorString(e));
  mem_indexed_tc_kernel<<<unsigned(a.B * a.blocks * a.G), NT, SMEM_BYTES, a.stream>>>(mq, mo, p);
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
