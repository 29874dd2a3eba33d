// Dispatcher for the chunked gated delta rule.
#include "common.cuh"
#include "kernels.h"

namespace yb {

int64_t gdn_chunk_workspace_bytes(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int) { return 0; }

int launch_gdn_chunk(const GdnArgs &a) { return launch_gdn_chunk_simt(a); }

}  // namespace yb
