// Byte-level communicator interface and its host backends.
//
// Interface and semantics follow crates/mt-comm/src/collective.rs (the
// Communicator trait: send / recv / all_reduce / broadcast / all_gather / rank /
// world_size, ReduceOp {Sum, Product, Min, Max, Mean}).  Errors are thrown as
// CommError instead of anyhow::Result.
//
// Backends here:
//   * MockCommunicator  -- the reference's single-process fake world, bit-exact
//                          (crates/mt-comm/src/mock.rs): shared mailbox, last
//                          write wins, non-consuming non-blocking recv, and
//                          "collectives" over world_size copies of the caller's
//                          own data interpreted as little-endian u64.
//   * LocalWorld        -- a real in-process world for threads: FIFO queues per
//                          (src, dst) pair, blocking recv with a deadline, and
//                          true collectives over every rank's contribution.
//                          Carries a FaultPlan for host-side fault injection.
//   * P2PChannel        -- the reference's in-process point-to-point channel
//                          (crates/mt-comm/src/p2p.rs) with a bounded wait.
//   * TcpCommunicator   -- sockets (tcp.cpp).
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace mtorus {

using Bytes = std::string;

struct CommError : public std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct CommTimeout : public CommError {
  using CommError::CommError;
};

enum class ReduceOp : int { Sum = 0, Product = 1, Min = 2, Max = 3, Mean = 4 };
// Element type used to interpret bytes in reductions.
enum class DType : int { U64 = 0, I64 = 1, F32 = 2, F64 = 3, I32 = 4, U8 = 5 };

const char* reduce_op_name(ReduceOp op);
size_t dtype_size(DType t);

// Element-wise reduction of equally sized byte buffers.
Bytes reduce_buffers(ReduceOp op, const std::vector<Bytes>& chunks, DType dt);
// acc = reduce(acc, x) in place (used by ring algorithms); Mean accumulates a sum.
void reduce_into(ReduceOp op, Bytes& acc, const Bytes& x, DType dt);
void finish_mean(Bytes& acc, size_t n, DType dt);

class Communicator {
 public:
  virtual ~Communicator() = default;
  virtual void send(const Bytes& data, size_t dst) = 0;
  virtual Bytes recv(size_t src) = 0;
  virtual Bytes all_reduce(const Bytes& data, ReduceOp op, DType dt) = 0;
  virtual Bytes broadcast(const Bytes& data, size_t root) = 0;
  virtual std::vector<Bytes> all_gather(const Bytes& data) = 0;
  virtual size_t rank() const = 0;
  virtual size_t world_size() const = 0;
  virtual std::string backend() const { return "abstract"; }
  virtual void barrier();
  // Neighbour exchange in one operation: send `data` to every rank in `peers` and
  // receive one message from each (out[i] from peers[i]).  Backends that move the
  // whole exchange at once (the device communicator's peer-memory kernels) return
  // true; the default returns false and callers fall back to send / recv.
  virtual bool exchange(const Bytes& data, const std::vector<size_t>& peers, std::vector<Bytes>* out) {
    (void)data;
    (void)peers;
    (void)out;
    return false;
  }
};

// ---------------------------------------------------------------- Mock
class MockCommunicator : public Communicator {
 public:
  using Mailboxes = std::vector<std::vector<Bytes>>;
  MockCommunicator(size_t rank, size_t world_size);
  static std::vector<std::shared_ptr<MockCommunicator>> create_world(size_t world_size);
  void send(const Bytes& data, size_t dst) override;
  Bytes recv(size_t src) override;
  Bytes all_reduce(const Bytes& data, ReduceOp op, DType dt) override;
  Bytes broadcast(const Bytes& data, size_t root) override;
  std::vector<Bytes> all_gather(const Bytes& data) override;
  size_t rank() const override { return rank_; }
  size_t world_size() const override { return world_; }
  std::string backend() const override { return "mock"; }
  void barrier() override {}

 private:
  MockCommunicator(size_t rank, size_t world, std::shared_ptr<std::pair<std::mutex, Mailboxes>> mb)
      : rank_(rank), world_(world), mb_(std::move(mb)) {}
  size_t rank_, world_;
  std::shared_ptr<std::pair<std::mutex, Mailboxes>> mb_;
};

// ---------------------------------------------------------------- faults
// Host-side fault injection for the in-process and TCP backends.  An op counter
// runs per rank; when a rule matches (rank, op index, kind) the action fires.
struct FaultRule {
  enum class Action : int { Drop = 0, Delay = 1, Kill = 2, Corrupt = 3 };
  int64_t rank = -1;      // -1: any rank
  int64_t at_op = -1;     // -1: every op; otherwise the op index (0-based, per rank)
  std::string op_kind;    // "" any, or "send", "recv", "all_reduce", ...
  Action action = Action::Drop;
  double delay_s = 0.0;
};

class FaultPlan {
 public:
  void add(const FaultRule& r);
  void clear();
  // Returns the first matching rule for this (rank, op) and advances the counter.
  std::optional<FaultRule> check(size_t rank, const std::string& kind);
  int64_t ops_seen(size_t rank) const;

 private:
  mutable std::mutex mu_;
  std::vector<FaultRule> rules_;
  std::map<size_t, int64_t> counters_;
};

// ---------------------------------------------------------------- LocalWorld
class LocalHub;

class LocalCommunicator : public Communicator {
 public:
  LocalCommunicator(size_t rank, std::shared_ptr<LocalHub> hub);
  void send(const Bytes& data, size_t dst) override;
  Bytes recv(size_t src) override;
  // Non-blocking probe: the next message from src if one is queued.
  std::optional<Bytes> try_recv(size_t src);
  Bytes all_reduce(const Bytes& data, ReduceOp op, DType dt) override;
  Bytes broadcast(const Bytes& data, size_t root) override;
  std::vector<Bytes> all_gather(const Bytes& data) override;
  void barrier() override;
  size_t rank() const override { return rank_; }
  size_t world_size() const override;
  std::string backend() const override { return "local"; }
  double timeout_s() const;

 private:
  void maybe_fault(const std::string& kind, bool* drop);
  size_t rank_;
  std::shared_ptr<LocalHub> hub_;
};

// A world of `n` ranks meant to be driven by n threads (one per rank).
class LocalWorld {
 public:
  static std::vector<std::shared_ptr<LocalCommunicator>> create(size_t n, double timeout_s,
                                                                std::shared_ptr<FaultPlan> faults);
};

// ---------------------------------------------------------------- P2P
class P2PHandle {
 public:
  P2PHandle();
  void set_result(const Bytes& data);
  // Waits up to timeout_s (< 0: the reference's unbounded wait, polled) for the result.
  Bytes wait(double timeout_s = 30.0);
  std::optional<Bytes> try_get() const;

 private:
  struct State {
    std::mutex mu;
    std::condition_variable cv;
    std::optional<Bytes> value;
  };
  std::shared_ptr<State> st_;
};

class P2PChannel {
 public:
  P2PChannel(size_t rank, size_t world_size);
  static std::vector<std::shared_ptr<P2PChannel>> create_group(size_t world_size);
  P2PHandle isend(const Bytes& data, size_t dst);
  // Snapshots the buffer slot (src -> this rank) at call time, as the reference does.
  P2PHandle irecv(size_t src);
  std::pair<P2PHandle, P2PHandle> sendrecv(const Bytes& data, size_t dst, size_t src);
  size_t rank() const { return rank_; }
  size_t world_size() const { return world_; }

 private:
  using Buffers = std::vector<std::vector<Bytes>>;
  P2PChannel(size_t r, size_t w, std::shared_ptr<std::pair<std::mutex, Buffers>> b)
      : rank_(r), world_(w), buf_(std::move(b)) {}
  size_t rank_, world_;
  std::shared_ptr<std::pair<std::mutex, Buffers>> buf_;
};

// ---------------------------------------------------------------- TCP (tcp.cpp)
// Frame: u64 little-endian length, then the payload.
void tcp_send_frame(int fd, const Bytes& data);
Bytes tcp_recv_frame(int fd, double timeout_s);

class TcpCommunicator : public Communicator {
 public:
  // Binds addresses[rank] ("host:port"; port 0 = ephemeral), accepts from lower
  // ranks in a background thread and dials every higher rank, retrying until
  // connect_timeout_s.  Unreachable peers are left unconnected (sends to them
  // raise), like the reference.
  TcpCommunicator(size_t rank, std::vector<std::string> addresses, double connect_timeout_s,
                  double op_timeout_s, bool dial = true);
  ~TcpCommunicator() override;
  uint16_t port() const { return port_; }
  // Dial `dst` at `addr` explicitly (reference connect_to).
  void connect_to(size_t dst, const std::string& addr, double timeout_s);
  // Block until every peer is connected or the deadline passes; returns the missing ranks.
  std::vector<size_t> wait_connected(double timeout_s);
  std::vector<size_t> connected_peers() const;
  void send(const Bytes& data, size_t dst) override;
  Bytes recv(size_t src) override;
  Bytes all_reduce(const Bytes& data, ReduceOp op, DType dt) override;
  Bytes broadcast(const Bytes& data, size_t root) override;
  std::vector<Bytes> all_gather(const Bytes& data) override;
  size_t rank() const override { return rank_; }
  size_t world_size() const override { return addrs_.size(); }
  std::string backend() const override { return "tcp"; }
  void set_fault_plan(std::shared_ptr<FaultPlan> f) { faults_ = std::move(f); }
  void close();

 private:
  struct Peer {
    std::atomic<int> fd{-1};
    std::mutex send_mu, recv_mu;  // one sender / one receiver per socket at a time
  };
  Peer* peer(size_t r);
  void accept_loop();
  void sendrecv(const Bytes& out, size_t dst, Bytes& in, size_t src);

  size_t rank_;
  std::vector<std::string> addrs_;
  double op_timeout_;
  int listen_fd_ = -1;
  uint16_t port_ = 0;
  std::vector<std::unique_ptr<Peer>> peers_;
  mutable std::mutex conn_mu_;
  std::condition_variable conn_cv_;
  std::unique_ptr<std::thread> acceptor_;
  std::shared_ptr<FaultPlan> faults_;
  bool closing_ = false;
};

// ---------------------------------------------------------------- topology aware
class MeshTorusHybrid;

}  // namespace mtorus

#include "core/topology.h"

namespace mtorus {

enum class CollectiveOp : int { AllReduce = 0, Broadcast = 1, AllGather = 2, ReduceScatter = 3 };
const char* collective_op_name(CollectiveOp op);

// Communicator wrapper that knows the mesh-torus topology
// (crates/mt-comm/src/topology_aware.rs).  The inner communicator's rank is a
// torus *node* rank.  With the Mock backend the exchanges interleave send/recv
// per neighbour exactly like the reference; with blocking backends all sends are
// posted before the receives, which is required to avoid a cyclic wait around
// the ring.
class TopologyAwareComm {
 public:
  TopologyAwareComm(std::shared_ptr<Communicator> inner, MeshTorusHybrid topo);
  size_t rank() const { return inner_->rank(); }
  size_t world_size() const { return inner_->world_size(); }
  std::shared_ptr<Communicator> inner() const { return inner_; }
  const MeshTorusHybrid& topology() const { return topo_; }
  TorusCoordinates rank_coords() const { return topo_.rank_to_coords(inner_->rank()); }

  std::vector<std::pair<size_t, Bytes>> exchange_with_neighbors(const Bytes& data);
  // AllReduce = Sum all_reduce (u64 elements like the reference); Broadcast from 0;
  // AllGather flattened; ReduceScatter = all_reduce then this rank's slice.
  Bytes perform_collective(CollectiveOp op, const Bytes& data, DType dt = DType::U64);
  // Reference semantics: the group is ignored and the whole world reduces.
  Bytes reduce_on_mesh(const Bytes& data, const std::vector<size_t>& group, DType dt = DType::U64);
  // Group-restricted sum over the listed ranks (gather to group[0], reduce, scatter back).
  Bytes reduce_on_group(const Bytes& data, const std::vector<size_t>& group, DType dt);

  // TopologyAwareCommunicator (crates/mt-core/src/topology/coordinator.rs:22-27)
  std::vector<Bytes> nearest_neighbor_exchange(const Bytes& data, size_t axis);
  Bytes all_reduce_mesh(const Bytes& data, const std::vector<size_t>& group);
  Bytes pipeline_stage_sendrecv(const Bytes& data, size_t stage_rank);
  Bytes route_collective(CollectiveOp op, const Bytes& data);

 private:
  bool interleaved() const { return inner_->backend() == "mock"; }
  std::shared_ptr<Communicator> inner_;
  MeshTorusHybrid topo_;
};

}  // namespace mtorus
