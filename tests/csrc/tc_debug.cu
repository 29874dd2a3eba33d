// Test-only build of the tensor-core chunk kernel with its intermediate-dump
// hooks enabled (YB_TC_DEBUG).  Compiled into tests/_build/libyb_tc_debug.so,
// in its own namespace so nothing clashes with libyanchor_b200.so; used by
// tests/test_gpu_tc_stages.py to compare every stage of the first chunk
// against numpy.
#include <cstdarg>
#include <cstdio>

#define yb yb_dbg
#define YB_TC_DEBUG 1
#include "../../yanchor_b200/csrc/gdn_chunk_tc.cu"

namespace yb_dbg {
static char g_err[512] = "";
int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
int check_launch(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return YB_OK;
}
}  // namespace yb_dbg

extern "C" const char *ybdbg_last_error(void) { return yb_dbg::g_err; }
extern "C" int ybdbg_device_error(int clear) { return yb_dbg::read_device_error(clear); }

extern "C" int ybdbg_gdn_chunk_tc(const void *q, const void *k, const void *v, int64_t qs, int64_t ks, int64_t vs,
                                  const void *g, const void *beta, int64_t gs, int64_t bs, const float *h0,
                                  float *ht, void *o, int64_t B, int64_t T, int64_t H, int64_t HV, float scale,
                                  int g_dtype, int beta_dtype, uint32_t flags, float *dbg, void *stream) {
  yb_dbg::GdnArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_ts = qs; a.k_ts = ks; a.v_ts = vs;
  a.g = g; a.beta = beta; a.g_ts = gs; a.beta_ts = bs;
  a.h0 = h0; a.ht = ht; a.o = o;
  a.B = B; a.T = T; a.H = H; a.HV = HV; a.K = 128; a.V = 128; a.N = B; a.scale = scale;
  a.io_dtype = YB_BF16; a.g_dtype = g_dtype; a.beta_dtype = beta_dtype; a.flags = flags;
  a.stream = static_cast<cudaStream_t>(stream);
  return yb_dbg::launch_gdn_chunk_tc_impl(a, dbg);
}
