// Python bindings of the host-side C++ runtime (module mtorus._C).
#include <pybind11/functional.h>
#include <pybind11/operators.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "core/data_loader.h"
#include "core/precision.h"
#include "core/topology.h"

namespace py = pybind11;
using namespace mtorus;

void bind_comm(py::module_& m);      // comm/bind_comm.cpp
void bind_pipeline(py::module_& m);  // pipeline/bind_pipeline.cpp

static std::string coords_repr(const TorusCoordinates& c) {
  std::string s = "TorusCoordinates(x=" + std::to_string(c.x) + ", y=" + std::to_string(c.y);
  s += c.z ? ", z=" + std::to_string(*c.z) + ")" : ", z=None)";
  return s;
}

static void bind_topology(py::module_& m) {
  py::class_<GPUDevice>(m, "GPUDevice")
      .def(py::init<size_t, std::optional<size_t>, std::string, std::vector<size_t>>(),
           py::arg("id"), py::arg("numa_node"), py::arg("pci_bus_id"), py::arg("nvlink_peers"))
      .def_static("simple", &GPUDevice::simple, py::arg("id"), py::arg("peer_count"))
      .def_readwrite("id", &GPUDevice::id)
      .def_readwrite("numa_node", &GPUDevice::numa_node)
      .def_readwrite("pci_bus_id", &GPUDevice::pci_bus_id)
      .def_readwrite("nvlink_peers", &GPUDevice::nvlink_peers)
      .def("is_nvlink_peer", &GPUDevice::is_nvlink_peer)
      .def("peer_count", &GPUDevice::peer_count)
      .def(py::self == py::self)
      .def("__copy__", [](const GPUDevice& d) { return GPUDevice(d); })
      .def("__repr__", [](const GPUDevice& d) {
        return "GPUDevice(id=" + std::to_string(d.id) + ", pci_bus_id='" + d.pci_bus_id + "', peers=" +
               std::to_string(d.nvlink_peers.size()) + ")";
      });

  py::class_<IntraNodeMesh>(m, "IntraNodeMesh")
      .def(py::init<std::vector<GPUDevice>>(), py::arg("devices"))
      .def_static("full_mesh", &IntraNodeMesh::full_mesh, py::arg("device_count"))
      .def_readonly("devices", &IntraNodeMesh::devices)
      .def("device", [](const IntraNodeMesh& mm, size_t id) -> std::optional<GPUDevice> {
        const GPUDevice* d = mm.device(id);
        if (!d) return std::nullopt;
        return *d;
      })
      .def("device_count", &IntraNodeMesh::device_count)
      .def("are_nvlinked", &IntraNodeMesh::are_nvlinked)
      .def("all_pairs_nvlinked", &IntraNodeMesh::all_pairs_nvlinked)
      .def(py::self == py::self)
      .def("__repr__", [](const IntraNodeMesh& mm) {
        return "IntraNodeMesh(devices=" + std::to_string(mm.device_count()) + ")";
      });

  py::class_<TorusDimensions>(m, "TorusDimensions")
      .def(py::init([](size_t w, size_t h, std::optional<size_t> d) { return TorusDimensions{w, h, d}; }),
           py::arg("width"), py::arg("height"), py::arg("depth") = py::none())
      .def_static("new_2d", &TorusDimensions::new_2d)
      .def_static("new_3d", &TorusDimensions::new_3d)
      .def_readwrite("width", &TorusDimensions::width)
      .def_readwrite("height", &TorusDimensions::height)
      .def_readwrite("depth", &TorusDimensions::depth)
      .def("total_nodes", &TorusDimensions::total_nodes)
      .def("axis_count", &TorusDimensions::axis_count)
      .def("axis_size", &TorusDimensions::axis_size)
      .def(py::self == py::self)
      .def("__repr__", [](const TorusDimensions& d) {
        return "TorusDimensions(" + std::to_string(d.width) + ", " + std::to_string(d.height) +
               (d.depth ? ", " + std::to_string(*d.depth) : std::string()) + ")";
      });

  py::class_<TorusCoordinates>(m, "TorusCoordinates")
      .def(py::init([](size_t x, size_t y, std::optional<size_t> z) { return TorusCoordinates{x, y, z}; }),
           py::arg("x"), py::arg("y"), py::arg("z") = py::none())
      .def_static("new_2d", &TorusCoordinates::new_2d)
      .def_static("new_3d", &TorusCoordinates::new_3d)
      .def_readwrite("x", &TorusCoordinates::x)
      .def_readwrite("y", &TorusCoordinates::y)
      .def_readwrite("z", &TorusCoordinates::z)
      .def("is_3d", &TorusCoordinates::is_3d)
      .def("linear_index", &TorusCoordinates::linear_index)
      .def_static("from_linear", &TorusCoordinates::from_linear)
      .def("neighbors", &TorusCoordinates::neighbors)
      .def("neighbor", &TorusCoordinates::neighbor, py::arg("dims"), py::arg("axis"), py::arg("positive"))
      .def(py::self == py::self)
      .def("__hash__", [](const TorusCoordinates& c) {
        return std::hash<size_t>()(c.x * 1000003u ^ c.y * 10007u ^ (c.z ? *c.z + 1 : 0));
      })
      .def("__repr__", &coords_repr);

  py::class_<MeshTorusHybrid>(m, "MeshTorusHybrid")
      .def_static("new_2d", &MeshTorusHybrid::new_2d, py::arg("width"), py::arg("height"),
                  py::arg("devices_per_node"))
      .def_static("new_3d", &MeshTorusHybrid::new_3d, py::arg("width"), py::arg("height"),
                  py::arg("depth"), py::arg("devices_per_node"))
      .def_readonly("dims", &MeshTorusHybrid::dims)
      .def_readonly("nodes", &MeshTorusHybrid::nodes)
      .def("total_nodes", &MeshTorusHybrid::total_nodes)
      .def("total_devices", &MeshTorusHybrid::total_devices)
      .def("devices_per_node", &MeshTorusHybrid::devices_per_node)
      .def("node_at", [](const MeshTorusHybrid& t, const TorusCoordinates& c) -> std::optional<IntraNodeMesh> {
        const IntraNodeMesh* n = t.node_at(c);
        if (!n) return std::nullopt;
        return *n;
      })
      .def("global_device_id", &MeshTorusHybrid::global_device_id)
      .def("node_neighbors", &MeshTorusHybrid::node_neighbors)
      .def("node_rank", &MeshTorusHybrid::node_rank)
      .def("rank_to_coords", &MeshTorusHybrid::rank_to_coords)
      .def(py::self == py::self)
      .def("__repr__", [](const MeshTorusHybrid& t) {
        return "MeshTorusHybrid(nodes=" + std::to_string(t.total_nodes()) +
               ", devices_per_node=" + std::to_string(t.devices_per_node()) + ")";
      });

  py::class_<DiscoveryConfig>(m, "DiscoveryConfig")
      .def(py::init([](bool full, std::optional<size_t> n) { return DiscoveryConfig{full, n}; }),
           py::arg("assume_full_mesh") = true, py::arg("num_devices_override") = py::none())
      .def_readwrite("assume_full_mesh", &DiscoveryConfig::assume_full_mesh)
      .def_readwrite("num_devices_override", &DiscoveryConfig::num_devices_override);
  m.def("discover_manual", &discover_manual);
  m.def("mesh_from_devices", &mesh_from_devices);
  m.def("topology_aware_placement", [](size_t n, const MeshTorusHybrid& t) {
    std::vector<std::pair<size_t, TorusCoordinates>> out;
    auto c = topology_aware_placement(n, t);
    for (size_t i = 0; i < c.size(); ++i) out.emplace_back(i, c[i]);
    return out;
  });
  m.def("compute_hop_distance", [](const TorusCoordinates& a, const TorusCoordinates& b,
                                   const MeshTorusHybrid& t) { return compute_hop_distance(a, b, t.dims); });
  m.def("torus_distance", [](size_t a, size_t b, size_t size) {
    const size_t d = a > b ? a - b : b - a;
    return std::min(d, size - d);
  });
}

static void bind_precision(py::module_& m) {
  py::enum_<Fp8Format>(m, "Fp8Format").value("E4M3", Fp8Format::E4M3).value("E5M2", Fp8Format::E5M2);
  py::enum_<MasterFormat>(m, "MasterFormat")
      .value("Fp32", MasterFormat::Fp32)
      .value("Bf16", MasterFormat::Bf16);
  py::enum_<LossScaleMode>(m, "LossScaleMode")
      .value("Dynamic", LossScaleMode::Dynamic)
      .value("Static", LossScaleMode::Static);
  m.def("fp8_format_max", &fp8_format_max);
  m.def("fp8_max_finite", &fp8_max_finite);
  m.def("fp8_encode", &fp8_encode);
  m.def("fp8_decode", &fp8_decode);
  m.def("fp8_encode_many", [](const std::vector<float>& v, Fp8Format f) {
    std::vector<uint8_t> o(v.size());
    for (size_t i = 0; i < v.size(); ++i) o[i] = fp8_encode(v[i], f);
    return py::bytes(reinterpret_cast<const char*>(o.data()), o.size());
  });
  m.def("fp8_decode_many", [](py::bytes b, Fp8Format f) {
    std::string s = b;
    std::vector<float> o(s.size());
    for (size_t i = 0; i < s.size(); ++i) o[i] = fp8_decode(static_cast<uint8_t>(s[i]), f);
    return o;
  });

  py::class_<Fp8Tensor>(m, "Fp8Tensor")
      .def(py::init([](std::vector<uint8_t> data, Fp8Format f, float scale) { return Fp8Tensor(std::move(data), f, scale); }),
           py::arg("data"), py::arg("format"), py::arg("scale"))
      .def_readwrite("data", &Fp8Tensor::data)
      .def_readwrite("format", &Fp8Tensor::format)
      .def_readwrite("scale", &Fp8Tensor::scale)
      .def_readwrite("block_scales", &Fp8Tensor::block_scales)
      .def_readwrite("block_size", &Fp8Tensor::block_size)
      .def_readwrite("amax_history", &Fp8Tensor::amax_history)
      .def("with_block_scales", [](Fp8Tensor t, std::vector<float> s) { t.block_scales = std::move(s); return t; })
      .def("with_amax_history", [](Fp8Tensor t, std::vector<float> h) { t.amax_history = std::move(h); return t; })
      .def("len", &Fp8Tensor::len)
      .def("__len__", &Fp8Tensor::len)
      .def("is_empty", &Fp8Tensor::is_empty)
      .def("amax", &Fp8Tensor::amax)
      .def("data_bytes", [](const Fp8Tensor& t) {
        return py::bytes(reinterpret_cast<const char*>(t.data.data()), t.data.size());
      })
      .def("clone", [](const Fp8Tensor& t) { return Fp8Tensor(t); })
      .def(py::self == py::self);

  m.def("to_fp8", &to_fp8);
  m.def("to_fp8_with_scale", &to_fp8_with_scale);
  m.def("to_fp8_per_block", &to_fp8_per_block);
  m.def("from_fp8", &from_fp8);

  py::class_<DelayedScaling>(m, "DelayedScaling")
      .def(py::init<size_t>(), py::arg("history_length"))
      .def("update", &DelayedScaling::update)
      .def("current_amax", &DelayedScaling::current_amax)
      .def("compute_scale", &DelayedScaling::compute_scale)
      .def_property_readonly("amax_history", &DelayedScaling::amax_history)
      .def_property_readonly("history_length", &DelayedScaling::history_length)
      .def_property_readonly("cursor", &DelayedScaling::cursor)
      .def("set_state", &DelayedScaling::set_state)
      .def("clone", [](const DelayedScaling& d) { return DelayedScaling(d); })
      .def(py::self == py::self);

  py::class_<LossScaler>(m, "LossScaler")
      .def_static("new_dynamic", &LossScaler::new_dynamic, py::arg("initial_scale"), py::arg("growth_interval"))
      .def_static("new_static", &LossScaler::new_static, py::arg("scale"))
      .def_readwrite("scale_value", &LossScaler::scale)
      .def_readwrite("mode", &LossScaler::mode)
      .def_readwrite("growth_interval", &LossScaler::growth_interval)
      .def_readwrite("growth_counter", &LossScaler::growth_counter)
      .def("update", &LossScaler::update)
      .def("scale", [](const LossScaler& s) { return s.scale; })
      .def("reset", &LossScaler::reset)
      .def("clone", [](const LossScaler& s) { return LossScaler(s); })
      .def(py::self == py::self);
}

static void bind_data(py::module_& m) {
  m.def("synthetic_token", &synthetic_token, py::arg("seed"), py::arg("batch_index"), py::arg("position"),
        py::arg("per_batch"), py::arg("vocab"));
  py::class_<TokenLoader>(m, "TokenLoader")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, uint64_t, bool, int, int>(), py::arg("batch"),
           py::arg("seq_len"), py::arg("vocab"), py::arg("num_batches"), py::arg("seed"), py::arg("shift"),
           py::arg("depth") = 4, py::arg("workers") = 1)
      // inp / tgt: addresses of int64 [batch, seq_len] host buffers
      .def(
          "next_into",
          [](TokenLoader& l, int64_t inp, int64_t tgt, double timeout_s) {
            return l.next_into(reinterpret_cast<int64_t*>(inp), reinterpret_cast<int64_t*>(tgt), timeout_s);
          },
          py::arg("inp"), py::arg("tgt"), py::arg("timeout_s") = 60.0, py::call_guard<py::gil_scoped_release>())
      .def("seek", &TokenLoader::seek, py::call_guard<py::gil_scoped_release>())
      .def("reset", &TokenLoader::reset, py::call_guard<py::gil_scoped_release>())
      .def("num_batches", &TokenLoader::num_batches)
      .def("current_batch", &TokenLoader::current_batch)
      .def_property_readonly("batch", &TokenLoader::batch)
      .def_property_readonly("seq_len", &TokenLoader::seq_len);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mtorus host runtime (topology, FP8 codec, communicators, pipeline schedules, data loader)";
  m.attr("__version__") = "0.1.0";
  bind_topology(m);
  bind_precision(m);
  bind_comm(m);
  bind_pipeline(m);
  bind_data(m);
}
