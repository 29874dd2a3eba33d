// Dispatcher for the chunked gated delta rule: the tcgen05 tensor-core kernel
// for bf16 inputs with K = V = 128 (the YANchor shape), the fp32 SIMT kernel
// otherwise.
#include "common.cuh"
#include "kernels.h"

namespace yb {

int64_t gdn_chunk_workspace_bytes(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int) { return 0; }

int launch_gdn_chunk(const GdnArgs &a) {
  if (gdn_chunk_tc_supported(a)) return launch_gdn_chunk_tc(a);
  return launch_gdn_chunk_simt(a);
}

}  // namespace yb
