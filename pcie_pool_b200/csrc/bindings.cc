// Python bindings of the native core (module pcie_pool_b200._C).
//
// Counterpart of the reference's `_turbobus` module (cpp/src/pybind.cpp:64-329):
// host-memory registration, device IPC handles, the data-plane engine and its
// plan/stat records.  Long calls release the GIL.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cuda_runtime.h>

#include <cstring>

#include "engine.h"
#include "vmm.h"
#include "native_ops.h"
#include "planner.h"
#include "ppb_common.h"

namespace py = pybind11;
using namespace ppb;

namespace {

template <typename T>
std::vector<T> to_vec(const py::array_t<T, py::array::c_style | py::array::forcecast>& a) {
  std::vector<T> v(static_cast<size_t>(a.size()));
  if (!v.empty()) std::memcpy(v.data(), a.data(), v.size() * sizeof(T));
  return v;
}

}  // namespace

void bind_ops(py::module_& m);
void bind_planner(py::module_& m);

PYBIND11_MODULE(_C, m) {
  m.doc() = "pcie_pool_b200 native core (sm_100a kernels + PoolEngine)";

  m.attr("OP_COPY") = static_cast<int>(kOpCopy);
  m.attr("OP_SCATTER_UNITS") = static_cast<int>(kOpScatterUnits);
  m.attr("OP_GATHER_UNITS") = static_cast<int>(kOpGatherUnits);
  m.attr("OP_FP8_QUANT") = static_cast<int>(kOpFp8Quant);
  m.attr("OP_SCATTER_RANGES") = static_cast<int>(kOpScatterRanges);
  m.attr("OP_GATHER_RANGES") = static_cast<int>(kOpGatherRanges);
  m.attr("OP_ADAMW") = static_cast<int>(kOpAdamW);
  m.attr("ADAM_TILE_PARAMS") = kAdamTileParams;
  m.attr("ADAM_TILE_BYTES") = kAdamTileBytes;
  m.attr("TILE_BYTES") = kTileBytes;
  m.attr("BUILD_ARCH") = "sm_100a";

  m.def("device_count", [] {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return n;
  });
  m.def("runtime_version", [] {
    int v = 0;
    cudaRuntimeGetVersion(&v);
    return v;
  });
  m.def("set_device", [](int d) { PPB_CUDA(cudaSetDevice(d)); }, py::arg("device"));
  m.def("host_register", &host_register, py::arg("ptr"), py::arg("bytes"),
        py::call_guard<py::gil_scoped_release>());
  m.def("host_unregister", &host_unregister, py::arg("ptr"),
        py::call_guard<py::gil_scoped_release>());
  m.def("is_pinned", [](uint64_t ptr) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, reinterpret_cast<void*>(ptr)) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  });
  m.def("export_ipc_handle", [](uint64_t dptr) {
    cudaIpcMemHandle_t h;
    PPB_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(dptr)));
    return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
  });
  // Base of the device allocation holding `dptr`: an IPC handle names a whole
  // allocation, so a pointer inside a caching-allocator segment travels as
  // handle + (dptr - base) and the receiver adds the offset back.
  m.def("allocation_base", [](uint64_t dptr) {
    using Fn = int (*)(unsigned long long*, size_t*, unsigned long long);
    static Fn fn = [] {
      void* f = nullptr;
      cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
      if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess)
        f = nullptr;
      return reinterpret_cast<Fn>(f);
    }();
    if (fn == nullptr) throw std::runtime_error("CUDA driver does not provide cuMemGetAddressRange");
    unsigned long long base = 0;
    size_t size = 0;
    const int rc = fn(&base, &size, static_cast<unsigned long long>(dptr));
    if (rc != 0) throw std::runtime_error("cuMemGetAddressRange failed with CUresult " + std::to_string(rc));
    return static_cast<uint64_t>(base);
  });
  // VMM shareable device buffers (POSIX file descriptors)
  m.def("vmm_alloc", [](int device, uint64_t bytes) {
    const VmmBuffer b = vmm_alloc(device, bytes);
    return py::make_tuple(b.ptr, b.size, b.fd);
  }, py::arg("device"), py::arg("bytes"));
  m.def("vmm_import", [](int fd, int device, uint64_t size) { return vmm_import(fd, device, size).ptr; },
        py::arg("fd"), py::arg("device"), py::arg("size"));
  m.def("vmm_release", &vmm_release, py::arg("ptr"));
  m.def("vmm_granularity", &vmm_granularity, py::arg("device"));
  // plain cudaMemcpy (either direction, inferred from the pointers)
  m.def("memcpy", [](uint64_t dst, uint64_t src, uint64_t n) {
    PPB_CUDA(cudaMemcpy(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), n, cudaMemcpyDefault));
  }, py::arg("dst"), py::arg("src"), py::arg("bytes"), py::call_guard<py::gil_scoped_release>());
  m.def("open_ipc_handle", [](py::bytes raw, int device) {
    std::string s = raw;
    if (s.size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("IPC handle must be 64 bytes");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, s.data(), sizeof(h));
    DeviceGuard g(device);
    void* p = nullptr;
    PPB_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    return reinterpret_cast<uint64_t>(p);
  });
  m.def("close_ipc_handle", [](uint64_t ptr) {
    PPB_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
  });

  py::class_<EngineOptions>(m, "EngineOptions")
      .def(py::init<>())
      .def_readwrite("slot_bytes", &EngineOptions::slot_bytes)
      .def_readwrite("slots", &EngineOptions::slots)
      .def_readwrite("ctas_per_lane", &EngineOptions::ctas_per_lane)
      .def_readwrite("coalesce_bytes", &EngineOptions::coalesce_bytes)
      .def_readwrite("timeout_s", &EngineOptions::timeout_s)
      .def_readwrite("enable_peer_access", &EngineOptions::enable_peer_access);

  py::class_<ChunkSpec>(m, "ChunkSpec")
      .def(py::init<>())
      .def(py::init([](uint64_t s, uint64_t d, uint64_t b) {
             ChunkSpec c;
             c.src_off = s;
             c.dst_off = d;
             c.bytes = b;
             return c;
           }),
           py::arg("src_off"), py::arg("dst_off"), py::arg("bytes"))
      .def_readwrite("src_off", &ChunkSpec::src_off)
      .def_readwrite("dst_off", &ChunkSpec::dst_off)
      .def_readwrite("bytes", &ChunkSpec::bytes)
      .def_readwrite("unit0", &ChunkSpec::unit0)
      .def_readwrite("tensor", &ChunkSpec::tensor)
      .def_readwrite("count", &ChunkSpec::count);

  py::class_<LaneSpec>(m, "LaneSpec")
      .def(py::init<>())
      .def_readwrite("device", &LaneSpec::device)
      .def_readwrite("chunks", &LaneSpec::chunks)
      .def(
          "set_chunks",
          [](LaneSpec& L, py::array_t<uint64_t, py::array::c_style | py::array::forcecast> src,
             py::array_t<uint64_t, py::array::c_style | py::array::forcecast> dst,
             py::array_t<uint64_t, py::array::c_style | py::array::forcecast> bytes,
             py::object unit0, py::object tensor, py::object count) {
            const auto n = static_cast<size_t>(src.size());
            if (static_cast<size_t>(dst.size()) != n || static_cast<size_t>(bytes.size()) != n)
              throw std::invalid_argument("chunk arrays must have equal lengths");
            auto u = unit0.is_none() ? std::vector<uint32_t>()
                                     : to_vec<uint32_t>(unit0.cast<py::array_t<uint32_t, py::array::c_style | py::array::forcecast>>());
            auto t = tensor.is_none() ? std::vector<uint32_t>()
                                      : to_vec<uint32_t>(tensor.cast<py::array_t<uint32_t, py::array::c_style | py::array::forcecast>>());
            auto c = count.is_none() ? std::vector<uint32_t>()
                                     : to_vec<uint32_t>(count.cast<py::array_t<uint32_t, py::array::c_style | py::array::forcecast>>());
            L.chunks.resize(n);
            const uint64_t* ps = src.data();
            const uint64_t* pd = dst.data();
            const uint64_t* pb = bytes.data();
            for (size_t i = 0; i < n; ++i) {
              L.chunks[i].src_off = ps[i];
              L.chunks[i].dst_off = pd[i];
              L.chunks[i].bytes = pb[i];
              L.chunks[i].unit0 = u.empty() ? 0 : u.at(i);
              L.chunks[i].tensor = t.empty() ? 0 : t.at(i);
              L.chunks[i].count = c.empty() ? 0 : c.at(i);
            }
          },
          py::arg("src_off"), py::arg("dst_off"), py::arg("bytes"), py::arg("unit0") = py::none(),
          py::arg("tensor") = py::none(), py::arg("count") = py::none());

  py::class_<AdamStepSpec>(m, "AdamStepSpec")
      .def(py::init<>())
      .def_readwrite("grads", &AdamStepSpec::grads)
      .def_readwrite("params", &AdamStepSpec::params)
      .def_readwrite("nparams", &AdamStepSpec::nparams)
      .def_readwrite("lr", &AdamStepSpec::lr)
      .def_readwrite("beta1", &AdamStepSpec::beta1)
      .def_readwrite("beta2", &AdamStepSpec::beta2)
      .def_readwrite("eps", &AdamStepSpec::eps)
      .def_readwrite("weight_decay", &AdamStepSpec::weight_decay)
      .def_readwrite("grad_scale", &AdamStepSpec::grad_scale)
      .def_readwrite("step", &AdamStepSpec::step);

  py::class_<QuantTensorSpec>(m, "QuantTensorSpec")
      .def(py::init<>())
      .def_readwrite("q", &QuantTensorSpec::q)
      .def_readwrite("scales", &QuantTensorSpec::scales)
      .def_readwrite("rows", &QuantTensorSpec::rows)
      .def_readwrite("cols", &QuantTensorSpec::cols);

  py::class_<TransferSpec>(m, "TransferSpec")
      .def(py::init<>())
      .def_readwrite("direction", &TransferSpec::direction)
      .def_readwrite("target", &TransferSpec::target)
      .def_readwrite("host_ptr", &TransferSpec::host_ptr)
      .def_readwrite("host_bytes", &TransferSpec::host_bytes)
      .def_readwrite("dev_ptr", &TransferSpec::dev_ptr)
      .def_readwrite("dev_bytes", &TransferSpec::dev_bytes)
      .def_readwrite("lanes", &TransferSpec::lanes)
      .def_readwrite("op", &TransferSpec::op)
      .def_readwrite("checksum", &TransferSpec::checksum)
      .def_readwrite("stage_direct", &TransferSpec::stage_direct)
      .def_readwrite("serialize", &TransferSpec::serialize)
      .def_readwrite("debug_drop_publish", &TransferSpec::debug_drop_publish)
      .def_readwrite("trace", &TransferSpec::trace)
      .def_readwrite("ctas_per_lane", &TransferSpec::ctas_per_lane)
      .def_readwrite("timeout_s", &TransferSpec::timeout_s)
      .def_readwrite("unit_bytes", &TransferSpec::unit_bytes)
      .def_readwrite("tensors", &TransferSpec::tensors)
      .def_readwrite("adam", &TransferSpec::adam)
      .def("set_unit_addrs",
           [](TransferSpec& s, py::array_t<uint64_t, py::array::c_style | py::array::forcecast> a) {
             s.unit_addrs = to_vec<uint64_t>(a);
           })
      .def("set_ranges",
           [](TransferSpec& s, py::array_t<uint64_t, py::array::c_style | py::array::forcecast> addr,
              py::array_t<uint32_t, py::array::c_style | py::array::forcecast> bytes,
              py::array_t<uint64_t, py::array::c_style | py::array::forcecast> pos) {
             s.range_addrs = to_vec<uint64_t>(addr);
             s.range_bytes = to_vec<uint32_t>(bytes);
             s.range_pos = to_vec<uint64_t>(pos);
           })
      .def_property_readonly("num_units", [](const TransferSpec& s) { return s.unit_addrs.size(); });

  py::class_<LaneStats>(m, "LaneStats")
      .def_readonly("device", &LaneStats::device)
      .def_readonly("direct", &LaneStats::direct)
      .def_readonly("bytes", &LaneStats::bytes)
      .def_readonly("chunks", &LaneStats::chunks)
      .def_readonly("cuda_ms", &LaneStats::cuda_ms);

  py::class_<TransferResult>(m, "TransferResult")
      .def_readonly("id", &TransferResult::id)
      .def_readonly("ok", &TransferResult::ok)
      .def_readonly("status_code", &TransferResult::status_code)
      .def_readonly("error_lane", &TransferResult::error_lane)
      .def_readonly("error_chunk", &TransferResult::error_chunk)
      .def_readonly("error_detail", &TransferResult::error_detail)
      .def_readonly("error", &TransferResult::error)
      .def_readonly("bytes", &TransferResult::bytes)
      .def_readonly("cuda_ms", &TransferResult::cuda_ms)
      .def_readonly("submit_to_complete_ms", &TransferResult::submit_to_complete_ms)
      .def_readonly("gib_per_s", &TransferResult::gib_per_s)
      .def_readonly("lanes", &TransferResult::lanes)
      .def_readonly("checksums", &TransferResult::checksums)
      .def_readonly("trace", &TransferResult::trace);

  py::class_<PoolEngine>(m, "PoolEngine")
      .def(py::init<const std::vector<int>&, const EngineOptions&>(), py::arg("devices"),
           py::arg("options") = EngineOptions{})
      .def("submit", &PoolEngine::submit, py::arg("spec"), py::call_guard<py::gil_scoped_release>())
      .def("wait", &PoolEngine::wait, py::arg("id"), py::arg("host_timeout_s") = 0.0,
           py::call_guard<py::gil_scoped_release>())
      .def("query", &PoolEngine::query, py::arg("id"))
      .def("relay_ring", &PoolEngine::relay_ring, py::arg("device"))
      .def("mailbox", &PoolEngine::mailbox, py::arg("device"))
      .def("issued", &PoolEngine::issued, py::arg("device"))
      .def("max_lane_ctas", &PoolEngine::max_lane_ctas, py::arg("device"))
      .def_property_readonly("devices", &PoolEngine::devices)
      .def_property_readonly("options", &PoolEngine::options);

  bind_ops(m);
  bind_planner(m);
}
