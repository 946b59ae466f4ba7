#include <algorithm>

#include "comm/comm.h"

namespace mtorus {

const char* collective_op_name(CollectiveOp op) {
  switch (op) {
    case CollectiveOp::AllReduce: return "AllReduce";
    case CollectiveOp::Broadcast: return "Broadcast";
    case CollectiveOp::AllGather: return "AllGather";
    case CollectiveOp::ReduceScatter: return "ReduceScatter";
  }
  return "?";
}

TopologyAwareComm::TopologyAwareComm(std::shared_ptr<Communicator> inner, MeshTorusHybrid topo)
    : inner_(std::move(inner)), topo_(std::move(topo)) {
  if (!inner_) throw CommError("TopologyAwareComm needs a communicator");
}

std::vector<std::pair<size_t, Bytes>> TopologyAwareComm::exchange_with_neighbors(const Bytes& data) {
  const auto nbs = rank_coords().neighbors(topo_.dims);
  std::vector<std::pair<size_t, Bytes>> out;
  out.reserve(nbs.size());
  {
    // a backend with a one-shot exchange (device peer stores) moves all of it at once
    std::vector<size_t> peers;
    for (const auto& nb : nbs) peers.push_back(topo_.node_rank(nb.first));
    std::vector<Bytes> got;
    if (!peers.empty() && inner_->exchange(data, peers, &got)) {
      for (size_t i = 0; i < peers.size(); ++i) out.emplace_back(peers[i], std::move(got[i]));
      return out;
    }
  }
  if (interleaved()) {
    for (const auto& nb : nbs) {
      const size_t r = topo_.node_rank(nb.first);
      inner_->send(data, r);
      out.emplace_back(r, inner_->recv(r));
    }
    return out;
  }
  for (const auto& nb : nbs) inner_->send(data, topo_.node_rank(nb.first));
  for (const auto& nb : nbs) {
    const size_t r = topo_.node_rank(nb.first);
    out.emplace_back(r, inner_->recv(r));
  }
  return out;
}

Bytes TopologyAwareComm::perform_collective(CollectiveOp op, const Bytes& data, DType dt) {
  switch (op) {
    case CollectiveOp::AllReduce: return inner_->all_reduce(data, ReduceOp::Sum, dt);
    case CollectiveOp::Broadcast: return inner_->broadcast(data, 0);
    case CollectiveOp::AllGather: {
      Bytes flat;
      for (const auto& c : inner_->all_gather(data)) flat += c;
      return flat;
    }
    case CollectiveOp::ReduceScatter: {
      const Bytes red = inner_->all_reduce(data, ReduceOp::Sum, dt);
      const size_t chunk = red.size() / std::max<size_t>(inner_->world_size(), 1);
      return red.substr(inner_->rank() * chunk, chunk);
    }
  }
  throw CommError("unknown collective");
}

Bytes TopologyAwareComm::reduce_on_mesh(const Bytes& data, const std::vector<size_t>&, DType dt) {
  return inner_->all_reduce(data, ReduceOp::Sum, dt);
}

Bytes TopologyAwareComm::reduce_on_group(const Bytes& data, const std::vector<size_t>& group, DType dt) {
  if (group.empty()) return data;
  const size_t me = inner_->rank();
  if (std::find(group.begin(), group.end(), me) == group.end())
    throw CommError("rank " + std::to_string(me) + " is not in the group");
  const size_t root = group[0];
  if (me == root) {
    std::vector<Bytes> parts{data};
    for (size_t i = 1; i < group.size(); ++i) parts.push_back(inner_->recv(group[i]));
    Bytes red = reduce_buffers(ReduceOp::Sum, parts, dt);
    for (size_t i = 1; i < group.size(); ++i) inner_->send(red, group[i]);
    return red;
  }
  inner_->send(data, root);
  return inner_->recv(root);
}

std::vector<Bytes> TopologyAwareComm::nearest_neighbor_exchange(const Bytes& data, size_t axis) {
  const TorusCoordinates c = rank_coords();
  const size_t pos = topo_.node_rank(c.neighbor(topo_.dims, axis, true));
  const size_t neg = topo_.node_rank(c.neighbor(topo_.dims, axis, false));
  std::vector<Bytes> out;
  try {
    if (inner_->exchange(data, {pos, neg}, &out)) return out;
  } catch (const CommError&) {
    return {data, data};  // the reference's fallback: the caller's own data per direction
  }
  out.clear();
  auto one = [&](size_t r) {
    try {
      inner_->send(data, r);
    } catch (const CommError&) {
      out.push_back(data);
      return;
    }
    try {
      out.push_back(inner_->recv(r));
    } catch (const CommError&) {
      out.push_back(data);
    }
  };
  if (interleaved()) {
    one(pos);
    one(neg);
    return out;
  }
  bool sent_pos = true, sent_neg = true;
  try { inner_->send(data, pos); } catch (const CommError&) { sent_pos = false; }
  try { inner_->send(data, neg); } catch (const CommError&) { sent_neg = false; }
  for (auto [r, ok] : {std::make_pair(pos, sent_pos), std::make_pair(neg, sent_neg)}) {
    if (!ok) {
      out.push_back(data);
      continue;
    }
    try {
      out.push_back(inner_->recv(r));
    } catch (const CommError&) {
      out.push_back(data);
    }
  }
  return out;
}

Bytes TopologyAwareComm::all_reduce_mesh(const Bytes& data, const std::vector<size_t>& group) {
  try {
    return reduce_on_mesh(data, group);
  } catch (const CommError&) {
    return Bytes();
  }
}

Bytes TopologyAwareComm::pipeline_stage_sendrecv(const Bytes& data, size_t stage_rank) {
  try {
    inner_->send(data, stage_rank);
  } catch (const CommError&) {
    return data;
  }
  try {
    return inner_->recv(stage_rank);
  } catch (const CommError&) {
    return data;
  }
}

Bytes TopologyAwareComm::route_collective(CollectiveOp op, const Bytes& data) {
  try {
    return perform_collective(op, data);
  } catch (const CommError&) {
    return Bytes();
  }
}

}  // namespace mtorus
