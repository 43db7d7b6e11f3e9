// Plain C++ interface between the torch glue (*.cpp, compiled by the host
// compiler) and the kernel translation units (*.cu).  Nothing here includes
// torch, so the .cu files compile in seconds.  Launchers take raw device
// pointers and a stream and return a cudaError_t; the glue turns errors into
// exceptions.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

int device_sm_count();

// ---------------------------------------------------------------- gemm_bf16.cu
// C[M, N] = X[M, K] . W[N, K]^T (+ bias[N]); bf16 in/out, fp32 accumulate.
// `partial` (fp32, >= splits * M * N elements) is required when splits > 1;
// pass splits = 0 to let the launcher choose (then `partial_cap` elements are
// available).  Returns the number of splits used through *splits_used.
struct GemmArgs {
  const void* x;
  int64_t ldx;
  const void* w;
  int64_t ldw;
  const void* bias;
  void* c;
  int64_t ldc;
  int M, N, K;
  int splits;
  float* partial;
  int64_t partial_cap;
  uint32_t* status;
};
int gemm_bf16_splits(int M, int N, int K, int splits_req);
cudaError_t gemm_bf16(const GemmArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- norm.cu
cudaError_t rms_norm(void* out, int64_t ld_out, const void* x, int64_t ld_x, const void* w, int T, int H, float eps,
                     cudaStream_t stream);
cudaError_t fused_add_rms_norm(void* x, int64_t ld_x, void* residual, int64_t ld_res, const void* w, int T, int H,
                               float eps, cudaStream_t stream);

}  // namespace b200
