// Torch glue of the `_C` extension: argument checks, stream/device guards and
// scratch allocation around the plain launchers of launch.h.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "launch.h"
#include "ops.h"

#define B200_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define B200_CHECK_DTYPE(x, t) TORCH_CHECK((x).scalar_type() == (t), #x " has dtype ", (x).scalar_type())
#define B200_LAUNCH(expr)                                                                          \
  do {                                                                                             \
    cudaError_t _e = (expr);                                                                       \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));                      \
  } while (0)

namespace b200 {

static inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

static inline uint32_t* status_ptr(const at::Tensor& status) {
  B200_CHECK_CUDA(status);
  TORCH_CHECK(status.scalar_type() == at::kInt && status.numel() >= 1, "status must be an int32 device word");
  return reinterpret_cast<uint32_t*>(status.data_ptr());
}

void gemm_bf16_out(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                   const at::Tensor& status, int64_t splits) {
  B200_CHECK_CUDA(x);
  B200_CHECK_CUDA(w);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(w, at::kBFloat16);
  B200_CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm_bf16: shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm_bf16: inner dims must be contiguous");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == w.size(0), "gemm_bf16: bad out shape");
  if (bias.has_value()) {
    B200_CHECK_DTYPE(*bias, at::kBFloat16);
    TORCH_CHECK(bias->numel() == w.size(0) && bias->is_contiguous(), "gemm_bf16: bad bias");
  }
  c10::cuda::CUDAGuard g(x.device());
  GemmArgs a{};
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.w = w.data_ptr();
  a.ldw = w.stride(0);
  a.bias = bias.has_value() ? bias->data_ptr() : nullptr;
  a.c = out.data_ptr();
  a.ldc = out.stride(0);
  a.M = x.size(0);
  a.N = w.size(0);
  a.K = x.size(1);
  a.status = status_ptr(status);
  a.splits = gemm_bf16_splits(a.M, a.N, a.K, (int)splits);
  at::Tensor partial;
  if (a.splits > 1) {
    partial = at::empty({(int64_t)a.splits * a.M * a.N}, x.options().dtype(at::kFloat));
    a.partial = partial.data_ptr<float>();
    a.partial_cap = partial.numel();
  }
  B200_LAUNCH(gemm_bf16(a, cur_stream()));
}

void rms_norm_out(at::Tensor& out, const at::Tensor& x, const at::Tensor& w, double eps) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(w, at::kBFloat16);
  B200_CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1 && w.is_contiguous(), "rms_norm: layout");
  TORCH_CHECK(out.sizes() == x.sizes() && w.numel() == x.size(1), "rms_norm: shape mismatch");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(rms_norm(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0), w.data_ptr(), x.size(0), x.size(1),
                       (float)eps, cur_stream()));
}

void fused_add_rms_norm_(at::Tensor& x, at::Tensor& residual, const at::Tensor& w, double eps) {
  B200_CHECK_CUDA(x);
  B200_CHECK_DTYPE(x, at::kBFloat16);
  B200_CHECK_DTYPE(residual, at::kBFloat16);
  B200_CHECK_DTYPE(w, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.sizes() == residual.sizes() && x.stride(1) == 1 && residual.stride(1) == 1,
              "fused_add_rms_norm: layout");
  TORCH_CHECK(w.numel() == x.size(1) && w.is_contiguous(), "fused_add_rms_norm: weight");
  c10::cuda::CUDAGuard g(x.device());
  B200_LAUNCH(fused_add_rms_norm(x.data_ptr(), x.stride(0), residual.data_ptr(), residual.stride(0), w.data_ptr(),
                                 x.size(0), x.size(1), (float)eps, cur_stream()));
}

}  // namespace b200
