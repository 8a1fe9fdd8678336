// placeholder, filled in below
#include <torch/extension.h>
namespace kb { void register_optim_ops(pybind11::module& m) {} }
