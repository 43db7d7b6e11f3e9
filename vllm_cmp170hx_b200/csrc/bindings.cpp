// Operator registry of the `_C` extension: every sm_100a kernel of the
// package is a `torch.ops.b200.*` op (the role `csrc/exl3/module.cpp:12-85`
// plays for the reference's `_exl3_C`).  Ops are registered for the CUDA
// dispatch key only: on a machine with a GPU there is no silent fallback.
#include <torch/extension.h>
#include <torch/library.h>

#include "ops.h"

namespace {
int64_t build_info() {
  // 100 = sm_100a; bump the low digits when an op's ABI changes.
  return 100 * 1000 + 3;
}
}  // namespace

TORCH_LIBRARY(b200, m) {
  m.def("build_info() -> int", &build_info);
#define B200_OPS_DEF(schema) m.def(schema);
  B200_OP_SCHEMAS(B200_OPS_DEF)
#undef B200_OPS_DEF
}

TORCH_LIBRARY_IMPL(b200, CUDA, m) {
#define B200_OPS_IMPL(name, fn) m.impl(name, &fn);
  B200_OP_IMPLS(B200_OPS_IMPL)
#undef B200_OPS_IMPL
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, mod) {
  mod.def("build_info", &build_info);
  b200::register_host_bindings(mod);
}
