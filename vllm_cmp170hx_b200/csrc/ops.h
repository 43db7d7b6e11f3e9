// Declarations and schemas of every op in the `_C` extension.
#pragma once
#include <torch/extension.h>

namespace b200 {

// torch_ops.cpp (kernels in the .cu files named beside each)
void gemm_bf16_out(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, at::Tensor& out,
                   const at::Tensor& status, int64_t splits);                       // gemm_bf16.cu
void rms_norm_out(at::Tensor& out, const at::Tensor& x, const at::Tensor& w, double eps);  // norm.cu
void fused_add_rms_norm_(at::Tensor& x, at::Tensor& residual, const at::Tensor& w, double eps);  // norm.cu

// Host (non-op) bindings: C++ runtime pieces exposed through pybind11.
void register_host_bindings(pybind11::module_& m);

}  // namespace b200

// Schema list: one line per op.
#define B200_OP_SCHEMAS(X)                                                                               \
  X("gemm_bf16_out(Tensor x, Tensor w, Tensor? bias, Tensor(a!) out, Tensor(b!) status, int splits) -> ()") \
  X("rms_norm_out(Tensor(a!) out, Tensor x, Tensor w, float eps) -> ()")                                 \
  X("fused_add_rms_norm(Tensor(a!) x, Tensor(b!) residual, Tensor w, float eps) -> ()")

#define B200_OP_IMPLS(X)                   \
  X("gemm_bf16_out", b200::gemm_bf16_out)  \
  X("rms_norm_out", b200::rms_norm_out)    \
  X("fused_add_rms_norm", b200::fused_add_rms_norm_)
