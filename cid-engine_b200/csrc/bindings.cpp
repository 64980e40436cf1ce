// Python module `cid_engine._C`: build flags (as in the reference's
// csrc/bindings.cpp:3-20) plus the device status word and ABI version.
#include <pybind11/pybind11.h>

#include "cid_engine/ops.hpp"
#include "cid_engine_b200.h"

PYBIND11_MODULE(_C, m) {
  m.doc() = "B200 (sm_100a) native core for cid-engine";
  m.attr("cuda_backend_built") = pybind11::bool_(true);
  m.attr("rocm_backend_built") = pybind11::bool_(false);
  m.attr("cann_backend_built") = pybind11::bool_(false);
  m.def("abi_version", []() { return cid_abi_version(); });
  m.def(
      "device_status",
      [](std::int64_t device, bool reset) { return cid::engine::read_device_status(device, reset); },
      pybind11::arg("device"), pybind11::arg("reset") = false,
      "CID_STATUS_* bits raised by kernels on `device` since the last reset (synchronises).");
  m.def(
      "status_word_ptr",
      [](std::int64_t device) {
        return reinterpret_cast<std::uintptr_t>(
            cid::engine::detail::status_word(at::Device(at::kCUDA, static_cast<int>(device))));
      },
      pybind11::arg("device"),
      "Device address of `device`'s status word, for kernels launched through the C ABI.");
}
