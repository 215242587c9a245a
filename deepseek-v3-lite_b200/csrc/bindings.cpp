// Python bindings of the sm_100a kernel library (module ops._dsv3_C).  Each
// translation unit registers its own entry points.
#include <torch/extension.h>

#include "status.h"

namespace dsv3 {
void register_gemm(pybind11::module_& m);
void register_elementwise(pybind11::module_& m);
void register_moe(pybind11::module_& m);
void register_attention(pybind11::module_& m);
void register_optim(pybind11::module_& m);
void register_comm(pybind11::module_& m);
void register_ep(pybind11::module_& m);
void register_dp(pybind11::module_& m);
}  // namespace dsv3

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "DeepSeek-V3-Lite sm_100a kernels (tcgen05 GEMM engine, MoE routing, MLA attention, fused optimizer)";
  m.def("status_read", &dsv3::status_read, "Read the device status word (synchronises the current stream)");
  m.def("status_reset", &dsv3::status_reset, "Zero the device status word");
  dsv3::register_gemm(m);
  dsv3::register_elementwise(m);
  dsv3::register_moe(m);
  dsv3::register_attention(m);
  dsv3::register_optim(m);
  dsv3::register_comm(m);
  dsv3::register_ep(m);
  dsv3::register_dp(m);
}
