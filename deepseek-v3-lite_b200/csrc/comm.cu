#include <torch/extension.h>
namespace dsv3 {
void register_comm(pybind11::module_& m) {}
}  // namespace dsv3
