// Device-side timing stamps for the light-timing profiler.
//
// One single-thread kernel writes %globaltimer (ns) into slot `col` of the
// current row of a device ring int64[rows, width]; the row index lives in
// device memory (`cursor`), so a stamp recorded inside a captured CUDA graph
// writes into whichever row the replay opened, with no host work per step.
// `open_row` advances the cursor (wrapping) and clears the new row.  The
// reference stamps the same way from a Triton kernel
// (vllm_sm80/worker/light_timing.py:1-60, LightTimer :183).
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace {

__global__ void stamp_kernel(int64_t* ring, const int* cursor, int width, int col) {
  pdl_prologue();
  const int row = *cursor;
  ring[(int64_t)row * width + col] = (int64_t)globaltimer();
}

__global__ void open_row_kernel(int64_t* ring, int* cursor, int rows, int width, int64_t* step_counter) {
  pdl_prologue();
  __shared__ int s_row;
  if (threadIdx.x == 0) {
    const int r = (*cursor + 1) % rows;
    *cursor = r;
    s_row = r;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < width; c += blockDim.x) ring[(int64_t)s_row * width + c] = 0;
  if (threadIdx.x == 0 && step_counter) ring[(int64_t)s_row * width] = ++(*step_counter);
}

}  // namespace

cudaError_t timing_stamp(int64_t* ring, const int* cursor, int width, int col, cudaStream_t stream) {
  if (col < 1 || col >= width) return cudaErrorInvalidValue;  // column 0 holds the row's step number
  launch_pdl(stamp_kernel, dim3(1), dim3(1), 0, stream, ring, cursor, width, col);
  return cudaGetLastError();
}

cudaError_t timing_open_row(int64_t* ring, int* cursor, int rows, int width, int64_t* step_counter,
                            cudaStream_t stream) {
  launch_pdl(open_row_kernel, dim3(1), dim3(128), 0, stream, ring, cursor, rows, width, step_counter);
  return cudaGetLastError();
}

}  // namespace b200
