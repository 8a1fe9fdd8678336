// Python bindings of the koochak_b200 native library (module koochak_b200_C).
#include <torch/extension.h>

#include "host_utils.h"

namespace kb {
void gemm_launch(const at::Tensor& a, bool a_mn_major, const at::Tensor& b, bool b_mn_major, at::Tensor& c,
                 const c10::optional<at::Tensor>& d, double alpha, double beta, const c10::optional<at::Tensor>& bias,
                 const c10::optional<at::Tensor>& aux, int64_t act, int64_t block_n, int64_t flags);
void gemm_set_group(int64_t g);
void gemm_set_split(int64_t s);
void gemm_set_profile(const c10::optional<at::Tensor>& buf);
void gemm_set_debug(int64_t mode);
void register_norm_ops(pybind11::module& m);
void register_elementwise_ops(pybind11::module& m);
void register_attention_ops(pybind11::module& m);
void register_optim_ops(pybind11::module& m);
void register_comm_ops(pybind11::module& m);
void register_muon_gather_ops(pybind11::module& m);
}  // namespace kb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "koochak_b200 sm_100a kernels";
  m.def("gemm", &kb::gemm_launch, "tcgen05 GEMM: c = epilogue(alpha * op(a) @ op(b)^T)", pybind11::arg("a"),
        pybind11::arg("a_mn_major"), pybind11::arg("b"), pybind11::arg("b_mn_major"), pybind11::arg("c"),
        pybind11::arg("d") = pybind11::none(), pybind11::arg("alpha") = 1.0, pybind11::arg("beta") = 0.0,
        pybind11::arg("bias") = pybind11::none(), pybind11::arg("aux") = pybind11::none(),
        pybind11::arg("act") = 0, pybind11::arg("block_n") = 0, pybind11::arg("flags") = 0);
  m.def("gemm_set_group", &kb::gemm_set_group,
        "tile-column group width of the GEMM tile order for timing studies (-1: the built-in rule)");
  m.def("gemm_set_split", &kb::gemm_set_split,
        "K-cut of fp32 GEMMs for timing studies: -1 built-in rule, 0 none, 1 stream-K, s >= 2 split-K");
  m.def("gemm_set_profile", &kb::gemm_set_profile,
        "route GEMM pipeline wait counters (int64, >= 4096 entries) to a buffer; None turns it off");
  m.def("gemm_set_debug", &kb::gemm_set_debug,
        "diagnostic GEMM modes for timing studies: bit 0 skips operand loads, bit 1 skips the epilogue (0: off)");
  m.def("read_and_clear_status", &kb::read_and_clear_status, "read and clear the device status word");
  m.def("read_debug_bounds_detail", &kb::read_debug_bounds_detail,
        "(site, index, extent) of the last debug-bounds failure on a device (cleared on read)");
  m.def(
      "debug_bounds_enabled",
      []() {
#ifdef KB_DEBUG_BOUNDS
        return true;
#else
        return false;
#endif
      },
      "whether this library was built with the KB_DEBUG_BOUNDS checks");
  m.def(
      "set_debug_extent_slack", [](int64_t n) { kb::debug_extent_slack().store(n); },
      "elements subtracted from every declared extent (tests use it to make the bounds checks fire)");
  m.def("num_sms", &kb::num_sms, "streaming multiprocessor count of a device");
  m.def("set_sm_reserve", [](int64_t n) { kb::sm_reserve().store((int)std::max<int64_t>(0, n)); },
        "SMs kept free of persistent GEMM / attention grids (for kernels overlapped beside them)");
  m.def("sm_reserve", []() { return kb::sm_reserve().load(); }, "current SM reserve");
  m.def("launch_count", []() { return kb::launch_counter().load(); }, "kernels launched by this library so far");
  m.def(
      "add_launches", [](int64_t n) { kb::launch_counter().fetch_add(n); },
      "count kernels of this library launched by a CUDA-graph replay", pybind11::arg("n"));
  kb::register_norm_ops(m);
  kb::register_elementwise_ops(m);
  kb::register_attention_ops(m);
  kb::register_optim_ops(m);
  kb::register_comm_ops(m);
  kb::register_muon_gather_ops(m);
}
