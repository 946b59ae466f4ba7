// Mesh-torus topology model: GPU devices, the NVLink mesh inside a node, torus
// coordinates of nodes, the hybrid (torus of meshes), device discovery,
// stage placement and hop distance.
//
// Semantics follow the reference crate mt-core::topology
// (crates/mt-core/src/topology/{device,mesh,torus,hybrid,discovery}.rs) and
// crates/mt-pipeline/src/placement.rs.  On an 8xB200 NVSwitch box the mesh is
// the physical topology (every GPU pair one switch hop); the torus is a virtual
// overlay used for neighbour exchange and placement.
#pragma once

#include <cstddef>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace mtorus {

struct GPUDevice {
  size_t id = 0;
  std::optional<size_t> numa_node;
  std::string pci_bus_id;
  std::vector<size_t> nvlink_peers;

  GPUDevice() = default;
  GPUDevice(size_t id_, std::optional<size_t> numa, std::string bus, std::vector<size_t> peers)
      : id(id_), numa_node(numa), pci_bus_id(std::move(bus)), nvlink_peers(std::move(peers)) {}
  // peers = every other id in [0, peer_count); bus id "0000:0{id}:00.0"
  static GPUDevice simple(size_t id, size_t peer_count);
  bool is_nvlink_peer(size_t other) const;
  size_t peer_count() const { return nvlink_peers.size(); }
  bool operator==(const GPUDevice& o) const {
    return id == o.id && numa_node == o.numa_node && pci_bus_id == o.pci_bus_id &&
           nvlink_peers == o.nvlink_peers;
  }
};

struct IntraNodeMesh {
  std::vector<GPUDevice> devices;

  // Throws std::invalid_argument when empty or when an id >= device count.
  explicit IntraNodeMesh(std::vector<GPUDevice> devs);
  static IntraNodeMesh full_mesh(size_t device_count);
  const GPUDevice* device(size_t id) const;
  size_t device_count() const { return devices.size(); }
  bool are_nvlinked(size_t a, size_t b) const;
  bool all_pairs_nvlinked() const;
  bool operator==(const IntraNodeMesh& o) const { return devices == o.devices; }
};

struct TorusDimensions {
  size_t width = 1, height = 1;
  std::optional<size_t> depth;
  static TorusDimensions new_2d(size_t w, size_t h) { return {w, h, std::nullopt}; }
  static TorusDimensions new_3d(size_t w, size_t h, size_t d) { return {w, h, d}; }
  size_t total_nodes() const { return width * height * (depth ? *depth : 1); }
  size_t axis_count() const { return depth ? 3 : 2; }
  size_t axis_size(size_t axis) const;
  bool operator==(const TorusDimensions& o) const {
    return width == o.width && height == o.height && depth == o.depth;
  }
};

struct TorusCoordinates {
  size_t x = 0, y = 0;
  std::optional<size_t> z;
  static TorusCoordinates new_2d(size_t x, size_t y) { return {x, y, std::nullopt}; }
  static TorusCoordinates new_3d(size_t x, size_t y, size_t z) { return {x, y, z}; }
  bool is_3d() const { return z.has_value(); }
  // row-major: z*W*H + y*W + x
  size_t linear_index(const TorusDimensions& d) const;
  static TorusCoordinates from_linear(size_t index, const TorusDimensions& d);
  // For each axis: (+ neighbour, axis), (- neighbour, axis); 2 axes for 2-D coords, 3 for 3-D.
  std::vector<std::pair<TorusCoordinates, size_t>> neighbors(const TorusDimensions& d) const;
  // Throws std::out_of_range for axis > 2.  Axis 2 on 2-D coords yields a 3-D coord.
  TorusCoordinates neighbor(const TorusDimensions& d, size_t axis, bool positive) const;
  bool operator==(const TorusCoordinates& o) const { return x == o.x && y == o.y && z == o.z; }
};

struct MeshTorusHybrid {
  TorusDimensions dims;
  std::vector<IntraNodeMesh> nodes;

  static MeshTorusHybrid new_2d(size_t w, size_t h, size_t devices_per_node);
  static MeshTorusHybrid new_3d(size_t w, size_t h, size_t d, size_t devices_per_node);
  size_t total_nodes() const { return nodes.size(); }
  size_t total_devices() const;
  size_t devices_per_node() const { return nodes.empty() ? 0 : nodes[0].device_count(); }
  const IntraNodeMesh* node_at(const TorusCoordinates& c) const;
  size_t global_device_id(const TorusCoordinates& node, size_t local_id) const;
  std::vector<std::pair<TorusCoordinates, IntraNodeMesh>> node_neighbors(
      const TorusCoordinates& c) const;
  size_t node_rank(const TorusCoordinates& c) const { return c.linear_index(dims); }
  TorusCoordinates rank_to_coords(size_t rank) const {
    return TorusCoordinates::from_linear(rank, dims);
  }
  bool operator==(const MeshTorusHybrid& o) const { return dims == o.dims && nodes == o.nodes; }
};

struct DiscoveryConfig {
  bool assume_full_mesh = true;
  std::optional<size_t> num_devices_override;
};

// Manual discovery (no device query): count = override or 8; numa = id / max(count/2, 1);
// bus id "0000:{id+1:02x}:00.0"; full peer lists.
std::vector<GPUDevice> discover_manual(const DiscoveryConfig& cfg);
// Builds the node mesh from a device list, overriding peers with a full mesh when asked.
IntraNodeMesh mesh_from_devices(std::vector<GPUDevice> devices, bool assume_full_mesh);

// Stage i -> torus coordinates of linear rank i (crates/mt-pipeline/src/placement.rs:3-13).
std::vector<TorusCoordinates> topology_aware_placement(size_t num_stages,
                                                       const MeshTorusHybrid& topo);
// Sum over axes of the wrap-around distance min(|a-b|, size-|a-b|) (placement.rs:15-33).
size_t compute_hop_distance(const TorusCoordinates& a, const TorusCoordinates& b,
                            const TorusDimensions& dims);

}  // namespace mtorus
