// Decode-loop bookkeeping after each sampled token: one launch updates the
// slot table of a batched decode (token storage, seen-token table, lengths,
// finish flags, steps, positions, next decode ids, useful-event counter).
// Semantics of runtime/model/inference_kernels.py:1701-1717 (torch path) and
// :1169-1204 (`_qwen35_decode_state_update_kernel`), with any number of EOS
// ids up to kMaxEos.
//
// Rows are independent: row r reads and writes its own slot entries and one
// storage / length / eos entry at its write row (its slot row when active,
// its private sink row otherwise), so threads never collide.  The only
// reduction is the active count, summed per block and added once.  An index
// that would leave a table (token outside the vocabulary, write row or
// column outside storage) skips that store and records ERR_DECODE_INDEX in
// the error word that yb_device_error() reads.
#include "common.cuh"
#include "kernels.h"

namespace yb {

namespace {

constexpr int kLoopThreads = 256;
constexpr int ERR_DECODE_INDEX = 0x401;
__device__ int g_loop_error = 0;

template <typename TS>
__global__ void __launch_bounds__(kLoopThreads) decode_state_update_kernel(const DecodeStateArgs a) {
  __shared__ long long warp_active[kLoopThreads / 32];
  pdl_wait();
  pdl_release();
  long long mine = 0;
  for (int64_t r = threadIdx.x; r < a.slots; r += kLoopThreads) {
    const int64_t sampled = a.sampled[r * a.sampled_stride];
    const bool finished = a.finished[r] != 0;
    const int64_t slot_row = a.slot_rows[r];
    const bool active = !finished && slot_row >= 0;
    const int64_t write_row = active ? slot_row : a.sink_rows[r];
    const int64_t step = a.row_steps[r];
    const int64_t write_col = active ? step : a.max_new;
    const int64_t tok = active ? sampled : a.pad;
    bool bad = false;
    const bool row_ok = write_row >= 0 && write_row < a.storage_rows;
    if (row_ok && write_col >= 0 && write_col < a.storage_cols)
      static_cast<TS *>(a.storage)[write_row * a.storage_stride + write_col] = TS(tok);
    else
      bad = true;
    if (tok >= 0 && tok < a.vocab) a.dense_seen[r * a.seen_stride + tok] = 1;
    else bad = true;
    const int64_t next_step = step + (active ? 1 : 0);
    bool is_eos = false;
    for (int e = 0; e < a.eos_count; ++e) is_eos |= tok == a.eos[e];
    if (active && row_ok) {
      a.generated_lengths[write_row] = next_step;
      if (is_eos) a.finished_by_eos[write_row] = 1;
    }
    const bool next_finished = finished || (active && (is_eos || next_step >= a.slot_caps[r]));
    a.finished[r] = next_finished ? 1 : 0;
    a.row_steps[r] = next_step;
    a.row_positions[r] += active ? 1 : 0;
    a.decode_ids[r * a.decode_ids_stride] = next_finished ? a.pad : tok;
    mine += active ? 1 : 0;
    if (bad) atomicCAS(&g_loop_error, 0, ERR_DECODE_INDEX);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if ((threadIdx.x & 31) == 0) warp_active[threadIdx.x >> 5] = mine;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long s = 0;
#pragma unroll
    for (int w = 0; w < kLoopThreads / 32; ++w) s += warp_active[w];
    *a.useful_events += s;
  }
}

}  // namespace

int launch_decode_state_update(const DecodeStateArgs &a) {
  if (a.slots == 0) return YB_OK;
  if (a.eos_count < 0 || a.eos_count > kMaxEos)
    return set_error(YB_ERR_UNSUPPORTED, "decode state: %d EOS ids (at most %d)", a.eos_count, kMaxEos);
  cudaError_t e = a.storage_i64 ? launch_pdl(decode_state_update_kernel<int64_t>, dim3(1), dim3(kLoopThreads), 0,
                                             a.stream, a)
                                : launch_pdl(decode_state_update_kernel<int32_t>, dim3(1), dim3(kLoopThreads), 0,
                                             a.stream, a);
  if (e != cudaSuccess) return set_error(YB_ERR_CUDA, "decode state: %s", cudaGetErrorString(e));
  return check_launch("decode_state_update_kernel");
}

int read_device_error_loop(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_loop_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_loop_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace yb
