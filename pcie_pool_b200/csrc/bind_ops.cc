// Bindings for the device-local ops and the planner core.  Device arguments
// are raw addresses; `stream` is a cudaStream_t handle as an integer (0 = the
// legacy default stream), e.g. torch.cuda.current_stream().cuda_stream.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>

#include "host_ops.h"
#include "native_ops.h"
#include "planner.h"
#include "ppb_common.h"

namespace py = pybind11;
using namespace ppb;

namespace {

cudaStream_t as_stream(uint64_t s) { return reinterpret_cast<cudaStream_t>(s); }

template <typename T>
std::vector<T> vec(const py::array_t<T, py::array::c_style | py::array::forcecast>& a) {
  std::vector<T> v(static_cast<size_t>(a.size()));
  if (!v.empty()) std::memcpy(v.data(), a.data(), v.size() * sizeof(T));
  return v;
}

}  // namespace

void bind_ops(py::module_& m) {
  py::class_<AdamParams>(m, "AdamParams")
      .def(py::init<>())
      .def_readwrite("lr", &AdamParams::lr)
      .def_readwrite("beta1", &AdamParams::beta1)
      .def_readwrite("beta2", &AdamParams::beta2)
      .def_readwrite("eps", &AdamParams::eps)
      .def_readwrite("weight_decay", &AdamParams::weight_decay)
      .def_readwrite("grad_scale", &AdamParams::grad_scale)
      .def_readwrite("step", &AdamParams::step);

  m.def("fp8_block_quant",
        [](uint64_t src, uint64_t rows, uint64_t cols, uint64_t q, uint64_t scales, uint64_t stream) {
          check_cuda(fp8_block_quant(reinterpret_cast<const void*>(src), rows, cols,
                                     reinterpret_cast<void*>(q), reinterpret_cast<float*>(scales),
                                     as_stream(stream)),
                     "fp8_block_quant");
        });
  m.def("fp8_block_dequant",
        [](uint64_t q, uint64_t scales, uint64_t rows, uint64_t cols, uint64_t out, uint64_t stream) {
          check_cuda(fp8_block_dequant(reinterpret_cast<const void*>(q),
                                       reinterpret_cast<const float*>(scales), rows, cols,
                                       reinterpret_cast<void*>(out), as_stream(stream)),
                     "fp8_block_dequant");
        });
  m.def("gather_units", [](uint64_t addr, uint64_t units, uint32_t unit_bytes, uint64_t dst, uint64_t stream) {
    check_cuda(gather_units(reinterpret_cast<const uint64_t*>(addr), units, unit_bytes,
                            reinterpret_cast<void*>(dst), as_stream(stream)),
               "gather_units");
  });
  m.def("scatter_units", [](uint64_t src, uint64_t addr, uint64_t units, uint32_t unit_bytes, uint64_t stream) {
    check_cuda(scatter_units(reinterpret_cast<const void*>(src), reinterpret_cast<const uint64_t*>(addr),
                             units, unit_bytes, as_stream(stream)),
               "scatter_units");
  });
  m.def("pack_ranges", [](uint64_t addr, uint64_t bytes, uint64_t pos, uint64_t n, uint64_t dst, uint64_t stream) {
    check_cuda(pack_ranges(reinterpret_cast<const uint64_t*>(addr), reinterpret_cast<const uint64_t*>(bytes),
                           reinterpret_cast<const uint64_t*>(pos), n, reinterpret_cast<void*>(dst),
                           as_stream(stream)),
               "pack_ranges");
  });
  m.def("unpack_ranges", [](uint64_t src, uint64_t addr, uint64_t bytes, uint64_t pos, uint64_t n, uint64_t stream) {
    check_cuda(unpack_ranges(reinterpret_cast<const void*>(src), reinterpret_cast<const uint64_t*>(addr),
                             reinterpret_cast<const uint64_t*>(bytes), reinterpret_cast<const uint64_t*>(pos),
                             n, as_stream(stream)),
               "unpack_ranges");
  });
  m.def("fused_adamw",
        [](uint64_t master, uint64_t mm, uint64_t vv, uint64_t grad, uint64_t out, uint64_t n,
           const AdamParams& p, uint64_t stream) {
          check_cuda(fused_adamw(reinterpret_cast<float*>(master), reinterpret_cast<float*>(mm),
                                 reinterpret_cast<float*>(vv), reinterpret_cast<const void*>(grad),
                                 reinterpret_cast<void*>(out), n, p, as_stream(stream)),
                     "fused_adamw");
        });
  m.def("interference", [](uint64_t buf, uint64_t n, int iters, int ctas, uint64_t stream) {
    check_cuda(interference(reinterpret_cast<float*>(buf), n, iters, ctas, as_stream(stream)),
               "interference");
  });
  m.def("checksum_device", [](uint64_t ptr, uint64_t bytes, uint64_t out, uint64_t stream) {
    check_cuda(checksum_device(reinterpret_cast<const void*>(ptr), bytes,
                               reinterpret_cast<unsigned long long*>(out), as_stream(stream)),
               "checksum_device");
  });
  m.def(
      "checksum_host",
      [](uint64_t ptr, uint64_t bytes) { return checksum_host(reinterpret_cast<const void*>(ptr), bytes); },
      py::call_guard<py::gil_scoped_release>());
  m.def(
      "fill_normal_bf16",
      [](uint64_t ptr, uint64_t n, float mean, float stddev, uint64_t seed, int threads) {
        fill_normal_bf16(reinterpret_cast<void*>(ptr), n, mean, stddev, seed, threads);
      },
      py::arg("ptr"), py::arg("n"), py::arg("mean") = 0.0f, py::arg("stddev") = 1.0f, py::arg("seed") = 0,
      py::arg("threads") = 0, py::call_guard<py::gil_scoped_release>());
  m.def(
      "fill_random_bytes",
      [](uint64_t ptr, uint64_t n, uint64_t seed, int threads) {
        fill_random_bytes(reinterpret_cast<void*>(ptr), n, seed, threads);
      },
      py::arg("ptr"), py::arg("n"), py::arg("seed") = 0, py::arg("threads") = 0,
      py::call_guard<py::gil_scoped_release>());
}

void bind_planner(py::module_& m) {
  m.attr("POLICY_LEGACY") = static_cast<int>(kLegacyGreedy);
  m.attr("POLICY_EARLIEST_FINISH") = static_cast<int>(kEarliestFinish);
  m.def(
      "assign_chunks",
      [](py::array_t<uint64_t, py::array::c_style | py::array::forcecast> chunk_bytes,
         std::vector<double> bw, std::vector<double> latency, int policy) {
        auto cb = vec<uint64_t>(chunk_bytes);
        std::vector<int32_t> out;
        {
          py::gil_scoped_release rel;
          out = assign_chunks(cb, bw, latency, policy);
        }
        return py::array_t<int32_t>(static_cast<py::ssize_t>(out.size()), out.data());
      },
      py::arg("chunk_bytes"), py::arg("bw_gibps"), py::arg("latency_s"), py::arg("policy"));
  m.def("concurrent_bandwidth", &concurrent_bandwidth, py::arg("bw_gibps"), py::arg("group"),
        py::arg("group_capacity_gibps"));
  m.def("estimate_makespan", &estimate_makespan, py::arg("total"), py::arg("chunk"),
        py::arg("bw_gibps"), py::arg("latency_s"));
  m.def("choose_chunk_bytes", &choose_chunk_bytes, py::arg("total"), py::arg("candidates"),
        py::arg("bw_gibps"), py::arg("latency_s"));
}
