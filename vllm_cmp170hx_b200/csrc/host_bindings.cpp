// pybind11 bindings of the host-side C++ runtime (no device code here).
#include <torch/extension.h>

#include "ops.h"

namespace b200 {

void register_block_pool(pybind11::module_& m);  // block_pool.cpp
void register_row_store(pybind11::module_& m);   // row_store.cpp

void register_host_bindings(pybind11::module_& m) {
  m.attr("ARCH") = "sm_100a";
  register_block_pool(m);
  register_row_store(m);
}

}  // namespace b200
