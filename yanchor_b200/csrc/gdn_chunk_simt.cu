// Chunked gated delta rule, fp32 SIMT version.  Used for fp32 inputs and for
// head sizes the tensor-core kernel does not cover; it also serves as an
// independent fp32 GPU cross-check of the tensor-core kernel.
//
// One CTA owns one (sequence, value head, 64-wide value slice) and walks the
// sequence chunk by chunk (C = 64 tokens), keeping its state slice S[K][64]
// in shared memory.  Per chunk, with G the in-chunk cumulative log decay and
// Tm = (I + L)^-1, L[i][j] = beta_i k_i.k_j e^{G_i-G_j} (j < i):
//   Y     = beta * (v - e^{G} * (k S))            (C x BV)
//   v_new = Tm Y                                   (= U - W S of the WY form)
//   o     = e^{G} * (q S) + P v_new,  P[i][j] = q_i.k_j e^{G_i-G_j} (j <= i)
//   S    <- e^{G_last} S + (k * e^{G_last - G})^T v_new
// (transformers qwen3_5 modeling_qwen3_5.py:234-311; the Y form folds
// W = Tm (beta e^G k) into one triangular product.)
#include "common.cuh"
#include "kernels.h"

namespace yb {
namespace {

constexpr int C = 64;    // chunk length
constexpr int NT = 256;  // threads

struct ChunkParams {
  const void *q, *k, *v;
  int64_t q_ts, k_ts, v_ts;
  const void *g, *beta;
  int64_t g_ts, beta_ts;
  int g_dtype, beta_dtype;
  const float *A_log, *dt_bias;
  const float *h0;
  float *ht;
  void *o;
  const int64_t *cu;
  int64_t T;
  int H, HV, V;
  float scale;
  uint32_t flags;
};

__device__ __forceinline__ float load_scalar(const void *p, int64_t idx, int dtype) {
  if (dtype == YB_F32) return static_cast<const float *>(p)[idx];
  if (dtype == YB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[idx]);
  return __half2float(static_cast<const __half *>(p)[idx]);
}

template <int K, int BV>
struct Smem {
  static constexpr int KP = K + 1;  // padded row pitch for q / k
  static constexpr int CP = C + 1;
  float S[K][BV];
  float q[C][KP];
  float k[C][KP];
  float vv[C][BV];  // v -> Y -> v_new
  float L[C][CP];
  float Tm[C][CP];
  float P[C][CP];
  float G[C], eG[C], bet[C], tail[C];
};

template <typename TIO, int K, int BV>
__global__ void __launch_bounds__(NT) gdn_chunk_simt_kernel(const ChunkParams p) {
  constexpr int TXN = BV / 4;             // threads across a C x BV tile row (4 columns each)
  constexpr int RT = C * BV / (4 * NT);   // tile rows per thread
  constexpr int RD = K * BV / (4 * NT);   // state rows per thread
  static_assert(RT >= 1 && RD >= 1, "tile must cover the block");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem<K, BV> &sm = *reinterpret_cast<Smem<K, BV> *>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = blockIdx.x / p.HV, hv = blockIdx.x % p.HV;
  const int v0 = blockIdx.y * BV;
  const int h = hv / (p.HV / p.H);
  const bool trans = p.flags & YB_GDN_TRANSPOSE_STATE;
  const bool l2 = p.flags & YB_GDN_QK_L2NORM;
  const bool gate_in = p.flags & YB_GDN_GATE_IN_KERNEL;
  const bool beta_sig = p.flags & YB_GDN_BETA_SIGMOID;
  int64_t bos, len;
  if (p.cu) {
    bos = p.cu[n];
    len = p.cu[n + 1] - bos;
  } else {
    bos = int64_t(n) * p.T;
    len = p.T;
  }
  const int64_t head = (int64_t(n) * p.HV + hv) * int64_t(K) * p.V;

  // initial state slice
  for (int e = tid; e < K * BV; e += NT) {
    const int d = e / BV, c = e % BV;
    float x = 0.f;
    if (p.h0) x = trans ? p.h0[head + int64_t(v0 + c) * K + d] : p.h0[head + int64_t(d) * p.V + v0 + c];
    sm.S[d][c] = x;
  }

  const TIO *qp = static_cast<const TIO *>(p.q);
  const TIO *kp = static_cast<const TIO *>(p.k);
  const TIO *vp = static_cast<const TIO *>(p.v);
  TIO *op = static_cast<TIO *>(p.o);
  // C x BV products: rows RT*ty.., cols 4*tx..;  C x C products: 4x4 at (4*py, 4*px)
  const int tx = tid % TXN, ty = tid / TXN;
  const int px = tid % 16, py = tid / 16;

  for (int64_t c0 = 0; c0 < len; c0 += C) {
    const int m = int(len - c0 < C ? len - c0 : C);
    __syncthreads();  // previous chunk fully consumed
    // ---- load chunk ----
    for (int e = tid; e < C * K; e += NT) {
      const int i = e / K, d = e % K;
      float qx = 0.f, kx = 0.f;
      if (i < m) {
        const int64_t tok = bos + c0 + i;
        qx = to_f(qp[tok * p.q_ts + int64_t(h) * K + d]);
        kx = to_f(kp[tok * p.k_ts + int64_t(h) * K + d]);
      }
      sm.q[i][d] = qx;
      sm.k[i][d] = kx;
    }
    for (int e = tid; e < C * BV; e += NT) {
      const int i = e / BV, c = e % BV;
      float vx = 0.f;
      if (i < m) vx = to_f(vp[(bos + c0 + i) * p.v_ts + int64_t(hv) * p.V + v0 + c]);
      sm.vv[i][c] = vx;
    }
    if (tid < C) {
      float gl = 0.f, b = 0.f;
      if (tid < m) {
        const int64_t tok = bos + c0 + tid;
        gl = load_scalar(p.g, tok * p.g_ts + hv, p.g_dtype);
        if (gate_in) gl = -expf(p.A_log[hv]) * softplus20(gl + (p.dt_bias ? p.dt_bias[hv] : 0.f));
        b = load_scalar(p.beta, tok * p.beta_ts + hv, p.beta_dtype);
        if (beta_sig) b = round_to<TIO>(sigmoidf_(b));   // beta in the input dtype, as the reference stores it
      }
      sm.G[tid] = gl;
      sm.bet[tid] = b;
    }
    __syncthreads();
    // ---- normalise q, k; scale q; cumulative decay ----
    for (int i = warp; i < C; i += NT / 32) {
      float qs2 = 0.f, ks2 = 0.f;
      for (int d = lane; d < K; d += 32) {
        qs2 += sm.q[i][d] * sm.q[i][d];
        ks2 += sm.k[i][d] * sm.k[i][d];
      }
      const float qn = (l2 ? rsqrtf(warp_sum(qs2) + 1e-6f) : 1.f) * p.scale;
      const float kn = l2 ? rsqrtf(warp_sum(ks2) + 1e-6f) : 1.f;
      for (int d = lane; d < K; d += 32) {
        sm.q[i][d] *= qn;
        sm.k[i][d] *= kn;
      }
    }
    if (warp == 0) {
      float a = sm.G[lane], b = sm.G[lane + 32];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float ya = __shfl_up_sync(0xffffffffu, a, o), yb = __shfl_up_sync(0xffffffffu, b, o);
        if (lane >= o) { a += ya; b += yb; }
      }
      b += __shfl_sync(0xffffffffu, a, 31);
      sm.G[lane] = a;
      sm.G[lane + 32] = b;
    }
    __syncthreads();
    if (tid < C) {
      sm.eG[tid] = expf(sm.G[tid]);
      sm.tail[tid] = expf(sm.G[C - 1] - sm.G[tid]);
    }
    // ---- L (strict lower) and P (lower incl. diagonal): 64 x 64, 4x4 per thread ----
    {
      float kk[4][4] = {}, qk[4][4] = {};
      for (int d = 0; d < K; ++d) {
        float ki[4], qi[4], kj[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          ki[a] = sm.k[py * 4 + a][d];
          qi[a] = sm.q[py * 4 + a][d];
          kj[a] = sm.k[px * 4 + a][d];
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            kk[a][b] = fmaf(ki[a], kj[b], kk[a][b]);
            qk[a][b] = fmaf(qi[a], kj[b], qk[a][b]);
          }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int i = py * 4 + a, j = px * 4 + b;
          const float dec = j <= i ? expf(sm.G[i] - sm.G[j]) : 0.f;
          sm.L[i][j] = j < i ? sm.bet[i] * kk[a][b] * dec : 0.f;
          sm.P[i][j] = qk[a][b] * dec;
        }
    }
    __syncthreads();
    // ---- Tm = (I + L)^-1: 4 threads per column, forward substitution ----
    {
      const int j = tid >> 2, part = tid & 3;
      for (int i = 0; i < C; ++i) {
        float acc = 0.f;
        for (int mm = j + part; mm < i; mm += 4) acc = fmaf(sm.L[i][mm], sm.Tm[mm][j], acc);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        if (part == 0) sm.Tm[i][j] = i < j ? 0.f : (i == j ? 1.f : -acc);
        __syncwarp();
      }
    }
    // ---- Y = beta (v - e^G (k S));  QS = q S kept in registers ----
    float qs[RT][4] = {};
    {
      float ks[RT][4] = {};
      for (int d = 0; d < K; ++d) {
        float4 sv = *reinterpret_cast<const float4 *>(&sm.S[d][tx * 4]);
        const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
        float ki[RT], qi[RT];
#pragma unroll
        for (int a = 0; a < RT; ++a) {
          ki[a] = sm.k[ty * RT + a][d];
          qi[a] = sm.q[ty * RT + a][d];
        }
#pragma unroll
        for (int a = 0; a < RT; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            ks[a][b] = fmaf(ki[a], s4[b], ks[a][b]);
            qs[a][b] = fmaf(qi[a], s4[b], qs[a][b]);
          }
      }
#pragma unroll
      for (int a = 0; a < RT; ++a) {
        const int i = ty * RT + a;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int c = tx * 4 + b;
          sm.vv[i][c] = sm.bet[i] * (sm.vv[i][c] - sm.eG[i] * ks[a][b]);
        }
      }
    }
    __syncthreads();
    // ---- v_new = Tm Y ----
    float vn[RT][4] = {};
    for (int j = 0; j < C; ++j) {
      float4 yv = *reinterpret_cast<const float4 *>(&sm.vv[j][tx * 4]);
      const float y4[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
      for (int a = 0; a < RT; ++a) {
        const float t = sm.Tm[ty * RT + a][j];
#pragma unroll
        for (int b = 0; b < 4; ++b) vn[a][b] = fmaf(t, y4[b], vn[a][b]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < RT; ++a)
      *reinterpret_cast<float4 *>(&sm.vv[ty * RT + a][tx * 4]) = make_float4(vn[a][0], vn[a][1], vn[a][2], vn[a][3]);
    __syncthreads();
    // ---- o = e^G QS + P v_new ----
    {
      float ov[RT][4];
#pragma unroll
      for (int a = 0; a < RT; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) ov[a][b] = sm.eG[ty * RT + a] * qs[a][b];
      for (int j = 0; j < C; ++j) {
        float4 xv = *reinterpret_cast<const float4 *>(&sm.vv[j][tx * 4]);
        const float x4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int a = 0; a < RT; ++a) {
          const float pp = sm.P[ty * RT + a][j];
#pragma unroll
          for (int b = 0; b < 4; ++b) ov[a][b] = fmaf(pp, x4[b], ov[a][b]);
        }
      }
#pragma unroll
      for (int a = 0; a < RT; ++a) {
        const int i = ty * RT + a;
        if (i < m) {
          TIO *dst = op + (bos + c0 + i) * int64_t(p.HV) * p.V + int64_t(hv) * p.V + v0 + tx * 4;
          store4(dst, ov[a]);
        }
      }
    }
    // ---- S <- e^{G_last} S + (k e^{G_last - G})^T v_new : K x BV, RD x 4 per thread ----
    {
      const float gl = expf(sm.G[C - 1]);
      float acc[RD][4];
#pragma unroll
      for (int a = 0; a < RD; ++a) {
        float4 sv = *reinterpret_cast<const float4 *>(&sm.S[ty * RD + a][tx * 4]);
        acc[a][0] = gl * sv.x; acc[a][1] = gl * sv.y; acc[a][2] = gl * sv.z; acc[a][3] = gl * sv.w;
      }
      for (int i = 0; i < C; ++i) {
        float4 xv = *reinterpret_cast<const float4 *>(&sm.vv[i][tx * 4]);
        const float x4[4] = {xv.x, xv.y, xv.z, xv.w};
        const float tl = sm.tail[i];
#pragma unroll
        for (int a = 0; a < RD; ++a) {
          const float kd = sm.k[i][ty * RD + a] * tl;
#pragma unroll
          for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(kd, x4[b], acc[a][b]);
        }
      }
      __syncthreads();  // every thread done reading S (q S / k S above) — safe to overwrite
#pragma unroll
      for (int a = 0; a < RD; ++a)
        *reinterpret_cast<float4 *>(&sm.S[ty * RD + a][tx * 4]) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    }
  }
  __syncthreads();
  if (p.ht) {
    for (int e = tid; e < K * BV; e += NT) {
      const int d = e / BV, c = e % BV;
      if (trans)
        p.ht[head + int64_t(v0 + c) * K + d] = sm.S[d][c];
      else
        p.ht[head + int64_t(d) * p.V + v0 + c] = sm.S[d][c];
    }
  }
}

template <typename TIO, int K, int BV>
int launch_kb(const GdnArgs &a, const ChunkParams &p) {
  const size_t smem = sizeof(Smem<K, BV>);
  auto kern = gdn_chunk_simt_kernel<TIO, K, BV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "gdn chunk simt: smem attribute: %s", cudaGetErrorString(e));
  dim3 grid(unsigned(a.N * a.HV), unsigned(a.V / BV));
  kern<<<grid, NT, smem, a.stream>>>(p);
  return check_launch("gdn_chunk_simt_kernel");
}

template <typename TIO, int K>
int launch_k(const GdnArgs &a, const ChunkParams &p) {
  return a.V % 64 == 0 ? launch_kb<TIO, K, 64>(a, p) : launch_kb<TIO, K, 32>(a, p);
}

template <typename TIO>
int launch_io(const GdnArgs &a, const ChunkParams &p) {
  if (a.K == 32) return launch_k<TIO, 32>(a, p);
  if (a.K == 64) return launch_k<TIO, 64>(a, p);
  return launch_k<TIO, 128>(a, p);
}

}  // namespace

int launch_gdn_chunk_simt(const GdnArgs &a) {
  ChunkParams p;
  p.q = a.q; p.k = a.k; p.v = a.v;
  p.q_ts = a.q_ts; p.k_ts = a.k_ts; p.v_ts = a.v_ts;
  p.g = a.g; p.beta = a.beta; p.g_ts = a.g_ts; p.beta_ts = a.beta_ts;
  p.g_dtype = a.g_dtype; p.beta_dtype = a.beta_dtype;
  p.A_log = a.A_log; p.dt_bias = a.dt_bias;
  p.h0 = a.h0; p.ht = a.ht; p.o = a.o;
  p.cu = a.cu_seqlens; p.T = a.T;
  p.H = int(a.H); p.HV = int(a.HV); p.V = int(a.V);
  p.scale = a.scale; p.flags = a.flags;
  if (a.N * a.HV == 0) return YB_OK;
  if (a.V % 32) return set_error(YB_ERR_UNSUPPORTED, "gdn chunk: V=%lld must be a multiple of 32", (long long)a.V);
  if (a.K != 32 && a.K != 64 && a.K != 128)
    return set_error(YB_ERR_UNSUPPORTED, "gdn chunk: K=%lld not built; supported 32/64/128", (long long)a.K);
  switch (a.io_dtype) {
    case YB_F32: return launch_io<float>(a, p);
    case YB_BF16: return launch_io<__nv_bfloat16>(a, p);
    case YB_F16: return launch_io<__half>(a, p);
  }
  return set_error(YB_ERR_ARGUMENT, "gdn chunk: bad io dtype %d", a.io_dtype);
}

}  // namespace yb
