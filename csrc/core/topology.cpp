#include "core/topology.h"

#include <algorithm>
#include <cstdio>

namespace mtorus {

GPUDevice GPUDevice::simple(size_t id, size_t peer_count) {
  std::vector<size_t> peers;
  for (size_t p = 0; p < peer_count; ++p)
    if (p != id) peers.push_back(p);
  return GPUDevice(id, std::nullopt, "0000:0" + std::to_string(id) + ":00.0", std::move(peers));
}

bool GPUDevice::is_nvlink_peer(size_t other) const {
  return std::find(nvlink_peers.begin(), nvlink_peers.end(), other) != nvlink_peers.end();
}

IntraNodeMesh::IntraNodeMesh(std::vector<GPUDevice> devs) : devices(std::move(devs)) {
  if (devices.empty()) throw std::invalid_argument("IntraNodeMesh requires at least one device");
  for (const auto& d : devices)
    if (d.id >= devices.size())
      throw std::invalid_argument("Device id " + std::to_string(d.id) + " exceeds device count " +
                                  std::to_string(devices.size()));
}

IntraNodeMesh IntraNodeMesh::full_mesh(size_t n) {
  if (n == 0) throw std::invalid_argument("IntraNodeMesh requires at least one device");
  std::vector<GPUDevice> devs;
  devs.reserve(n);
  for (size_t id = 0; id < n; ++id) {
    std::vector<size_t> peers;
    for (size_t p = 0; p < n; ++p)
      if (p != id) peers.push_back(p);
    devs.emplace_back(id, std::nullopt, "0000:0" + std::to_string(id) + ":00.0", std::move(peers));
  }
  return IntraNodeMesh(std::move(devs));
}

const GPUDevice* IntraNodeMesh::device(size_t id) const {
  for (const auto& d : devices)
    if (d.id == id) return &d;
  return nullptr;
}

bool IntraNodeMesh::are_nvlinked(size_t a, size_t b) const {
  const GPUDevice* d = device(a);
  return d != nullptr && d->is_nvlink_peer(b);
}

bool IntraNodeMesh::all_pairs_nvlinked() const {
  for (size_t i = 0; i < devices.size(); ++i)
    for (size_t j = 0; j < devices.size(); ++j)
      if (i != j && !are_nvlinked(i, j)) return false;
  return true;
}

size_t TorusDimensions::axis_size(size_t axis) const {
  switch (axis) {
    case 0: return width;
    case 1: return height;
    case 2: return depth ? *depth : 1;
    default: throw std::out_of_range("axis out of range: " + std::to_string(axis));
  }
}

size_t TorusCoordinates::linear_index(const TorusDimensions& d) const {
  if (z) return *z * d.width * d.height + y * d.width + x;
  return y * d.width + x;
}

TorusCoordinates TorusCoordinates::from_linear(size_t index, const TorusDimensions& d) {
  if (d.depth) {
    const size_t plane = d.width * d.height;
    const size_t zz = index / plane, rem = index % plane;
    return new_3d(rem % d.width, rem / d.width, zz % *d.depth);
  }
  return new_2d(index % d.width, index / d.width);
}

static size_t wrap(size_t cur, size_t size, bool positive) {
  return positive ? (cur + 1) % size : (cur + size - 1) % size;
}

TorusCoordinates TorusCoordinates::neighbor(const TorusDimensions& d, size_t axis,
                                            bool positive) const {
  TorusCoordinates c = *this;
  switch (axis) {
    case 0: c.x = wrap(x, d.width, positive); break;
    case 1: c.y = wrap(y, d.height, positive); break;
    case 2: c.z = wrap(z ? *z : 0, d.depth ? *d.depth : 1, positive); break;
    default: throw std::out_of_range("axis out of range: " + std::to_string(axis));
  }
  return c;
}

std::vector<std::pair<TorusCoordinates, size_t>> TorusCoordinates::neighbors(
    const TorusDimensions& d) const {
  std::vector<std::pair<TorusCoordinates, size_t>> out;
  const size_t axes = z ? 3 : 2;
  for (size_t a = 0; a < axes; ++a) {
    out.emplace_back(neighbor(d, a, true), a);
    out.emplace_back(neighbor(d, a, false), a);
  }
  return out;
}

MeshTorusHybrid MeshTorusHybrid::new_2d(size_t w, size_t h, size_t dpn) {
  if (w == 0 || h == 0 || dpn == 0)
    throw std::invalid_argument("width, height, and devices_per_node must be > 0");
  MeshTorusHybrid t{TorusDimensions::new_2d(w, h), {}};
  for (size_t i = 0; i < t.dims.total_nodes(); ++i) t.nodes.push_back(IntraNodeMesh::full_mesh(dpn));
  return t;
}

MeshTorusHybrid MeshTorusHybrid::new_3d(size_t w, size_t h, size_t dd, size_t dpn) {
  if (w == 0 || h == 0 || dd == 0 || dpn == 0)
    throw std::invalid_argument("width, height, depth, and devices_per_node must be > 0");
  MeshTorusHybrid t{TorusDimensions::new_3d(w, h, dd), {}};
  for (size_t i = 0; i < t.dims.total_nodes(); ++i) t.nodes.push_back(IntraNodeMesh::full_mesh(dpn));
  return t;
}

size_t MeshTorusHybrid::total_devices() const {
  size_t n = 0;
  for (const auto& m : nodes) n += m.device_count();
  return n;
}

const IntraNodeMesh* MeshTorusHybrid::node_at(const TorusCoordinates& c) const {
  const size_t i = c.linear_index(dims);
  return i < nodes.size() ? &nodes[i] : nullptr;
}

size_t MeshTorusHybrid::global_device_id(const TorusCoordinates& node, size_t local_id) const {
  return node.linear_index(dims) * devices_per_node() + local_id;
}

std::vector<std::pair<TorusCoordinates, IntraNodeMesh>> MeshTorusHybrid::node_neighbors(
    const TorusCoordinates& c) const {
  std::vector<std::pair<TorusCoordinates, IntraNodeMesh>> out;
  for (const auto& nb : c.neighbors(dims)) {
    const IntraNodeMesh* m = node_at(nb.first);
    if (m) out.emplace_back(nb.first, *m);
  }
  return out;
}

std::vector<GPUDevice> discover_manual(const DiscoveryConfig& cfg) {
  const size_t count = cfg.num_devices_override ? *cfg.num_devices_override : 8;
  const size_t half = std::max<size_t>(count / 2, 1);
  std::vector<GPUDevice> devs;
  for (size_t id = 0; id < count; ++id) {
    std::vector<size_t> peers;
    for (size_t p = 0; p < count; ++p)
      if (p != id) peers.push_back(p);
    char bus[32];
    std::snprintf(bus, sizeof(bus), "0000:%02zx:00.0", id + 1);
    devs.emplace_back(id, id / half, bus, std::move(peers));
  }
  return devs;
}

IntraNodeMesh mesh_from_devices(std::vector<GPUDevice> devices, bool assume_full_mesh) {
  if (assume_full_mesh) {
    const size_t n = devices.size();
    for (auto& d : devices) {
      d.nvlink_peers.clear();
      for (size_t p = 0; p < n; ++p)
        if (p != d.id) d.nvlink_peers.push_back(p);
    }
  }
  return IntraNodeMesh(std::move(devices));
}

std::vector<TorusCoordinates> topology_aware_placement(size_t num_stages,
                                                       const MeshTorusHybrid& topo) {
  std::vector<TorusCoordinates> out;
  out.reserve(num_stages);
  for (size_t i = 0; i < num_stages; ++i) out.push_back(topo.rank_to_coords(i));
  return out;
}

size_t compute_hop_distance(const TorusCoordinates& a, const TorusCoordinates& b,
                            const TorusDimensions& dims) {
  auto dist = [](size_t p, size_t q, size_t size) {
    const size_t diff = p > q ? p - q : q - p;
    return std::min(diff, size - diff);
  };
  size_t h = dist(a.x, b.x, dims.width) + dist(a.y, b.y, dims.height);
  if (a.z && b.z && dims.depth) h += dist(*a.z, *b.z, *dims.depth);
  return h;
}

}  // namespace mtorus
