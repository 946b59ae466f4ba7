#include "comm/comm.h"

#include <algorithm>
#include <cstring>

namespace mtorus {

const char* reduce_op_name(ReduceOp op) {
  switch (op) {
    case ReduceOp::Sum: return "Sum";
    case ReduceOp::Product: return "Product";
    case ReduceOp::Min: return "Min";
    case ReduceOp::Max: return "Max";
    case ReduceOp::Mean: return "Mean";
  }
  return "?";
}

size_t dtype_size(DType t) {
  switch (t) {
    case DType::U64: case DType::I64: case DType::F64: return 8;
    case DType::F32: case DType::I32: return 4;
    case DType::U8: return 1;
  }
  return 1;
}

template <typename T>
static void reduce_typed(ReduceOp op, T* acc, const T* x, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    switch (op) {
      case ReduceOp::Sum: case ReduceOp::Mean: acc[i] = acc[i] + x[i]; break;
      case ReduceOp::Product: acc[i] = acc[i] * x[i]; break;
      case ReduceOp::Min: acc[i] = std::min(acc[i], x[i]); break;
      case ReduceOp::Max: acc[i] = std::max(acc[i], x[i]); break;
    }
  }
}

template <typename T>
static void mean_typed(T* acc, size_t n, size_t count) {
  for (size_t i = 0; i < n; ++i) acc[i] = static_cast<T>(acc[i] / static_cast<T>(count));
}

void reduce_into(ReduceOp op, Bytes& acc, const Bytes& x, DType dt) {
  const size_t es = dtype_size(dt);
  const size_t n = std::min(acc.size(), x.size()) / es;
  void* a = acc.data();
  const void* b = x.data();
  switch (dt) {
    case DType::U64: reduce_typed(op, static_cast<uint64_t*>(a), static_cast<const uint64_t*>(b), n); break;
    case DType::I64: reduce_typed(op, static_cast<int64_t*>(a), static_cast<const int64_t*>(b), n); break;
    case DType::F32: reduce_typed(op, static_cast<float*>(a), static_cast<const float*>(b), n); break;
    case DType::F64: reduce_typed(op, static_cast<double*>(a), static_cast<const double*>(b), n); break;
    case DType::I32: reduce_typed(op, static_cast<int32_t*>(a), static_cast<const int32_t*>(b), n); break;
    case DType::U8: reduce_typed(op, reinterpret_cast<uint8_t*>(a), reinterpret_cast<const uint8_t*>(b), n); break;
  }
}

void finish_mean(Bytes& acc, size_t count, DType dt) {
  const size_t n = acc.size() / dtype_size(dt);
  void* a = acc.data();
  switch (dt) {
    case DType::U64: mean_typed(static_cast<uint64_t*>(a), n, count); break;
    case DType::I64: mean_typed(static_cast<int64_t*>(a), n, count); break;
    case DType::F32: mean_typed(static_cast<float*>(a), n, count); break;
    case DType::F64: mean_typed(static_cast<double*>(a), n, count); break;
    case DType::I32: mean_typed(static_cast<int32_t*>(a), n, count); break;
    case DType::U8: mean_typed(reinterpret_cast<uint8_t*>(a), n, count); break;
  }
}

// Reference semantics (mock.rs:34-64): element count from the first chunk,
// trailing bytes that do not fill an element are dropped.
Bytes reduce_buffers(ReduceOp op, const std::vector<Bytes>& chunks, DType dt) {
  if (chunks.empty()) return Bytes();
  const size_t es = dtype_size(dt);
  const size_t n = chunks[0].size() / es;
  if (n == 0) return Bytes();
  Bytes acc = chunks[0].substr(0, n * es);
  for (size_t c = 1; c < chunks.size(); ++c) {
    Bytes x = chunks[c];
    if (x.size() < n * es) x.resize(n * es, '\0');
    reduce_into(op, acc, x, dt);
  }
  if (op == ReduceOp::Mean) finish_mean(acc, chunks.size(), dt);
  return acc;
}

void Communicator::barrier() {
  Bytes one(8, '\0');
  all_reduce(one, ReduceOp::Sum, DType::U64);
}

// ---------------------------------------------------------------- Mock
MockCommunicator::MockCommunicator(size_t rank, size_t world)
    : rank_(rank), world_(world), mb_(std::make_shared<std::pair<std::mutex, Mailboxes>>()) {
  mb_->second.assign(world, std::vector<Bytes>(world));
}

std::vector<std::shared_ptr<MockCommunicator>> MockCommunicator::create_world(size_t world) {
  auto mb = std::make_shared<std::pair<std::mutex, Mailboxes>>();
  mb->second.assign(world, std::vector<Bytes>(world));
  std::vector<std::shared_ptr<MockCommunicator>> out;
  for (size_t r = 0; r < world; ++r)
    out.push_back(std::shared_ptr<MockCommunicator>(new MockCommunicator(r, world, mb)));
  return out;
}

void MockCommunicator::send(const Bytes& data, size_t dst) {
  if (dst >= world_)
    throw CommError("destination " + std::to_string(dst) + " >= world_size " + std::to_string(world_));
  std::lock_guard<std::mutex> lk(mb_->first);
  mb_->second[rank_][dst] = data;
}

Bytes MockCommunicator::recv(size_t src) {
  if (src >= world_)
    throw CommError("source " + std::to_string(src) + " >= world_size " + std::to_string(world_));
  std::lock_guard<std::mutex> lk(mb_->first);
  return mb_->second[src][rank_];
}

Bytes MockCommunicator::all_reduce(const Bytes& data, ReduceOp op, DType dt) {
  return reduce_buffers(op, std::vector<Bytes>(world_, data), dt);
}

Bytes MockCommunicator::broadcast(const Bytes& data, size_t root) {
  if (root >= world_)
    throw CommError("root " + std::to_string(root) + " >= world_size " + std::to_string(world_));
  return data;
}

std::vector<Bytes> MockCommunicator::all_gather(const Bytes& data) {
  return std::vector<Bytes>(world_, data);
}

// ---------------------------------------------------------------- FaultPlan
void FaultPlan::add(const FaultRule& r) {
  std::lock_guard<std::mutex> lk(mu_);
  rules_.push_back(r);
}
void FaultPlan::clear() {
  std::lock_guard<std::mutex> lk(mu_);
  rules_.clear();
  counters_.clear();
}
std::optional<FaultRule> FaultPlan::check(size_t rank, const std::string& kind) {
  std::lock_guard<std::mutex> lk(mu_);
  const int64_t idx = counters_[rank]++;
  for (const auto& r : rules_) {
    if (r.rank >= 0 && static_cast<size_t>(r.rank) != rank) continue;
    if (r.at_op >= 0 && r.at_op != idx) continue;
    if (!r.op_kind.empty() && r.op_kind != kind) continue;
    return r;
  }
  return std::nullopt;
}
int64_t FaultPlan::ops_seen(size_t rank) const {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = counters_.find(rank);
  return it == counters_.end() ? 0 : it->second;
}

// ---------------------------------------------------------------- LocalWorld
class LocalHub {
 public:
  LocalHub(size_t n, double timeout_s, std::shared_ptr<FaultPlan> f)
      : n_(n), timeout_(timeout_s), faults(std::move(f)), queues_(n * n), dead_(n, false) {}

  size_t n_;
  double timeout_;
  std::shared_ptr<FaultPlan> faults;

  std::mutex mu;
  std::condition_variable cv;
  std::vector<std::deque<Bytes>> queues_;  // [src * n + dst]
  std::vector<bool> dead_;
  // collective rendezvous
  uint64_t gen = 0;
  size_t arrived = 0;
  std::vector<Bytes> slots;
  std::vector<Bytes> result_all;
  Bytes result;
  uint64_t done_gen = 0;
  std::string coll_kind;

  std::chrono::steady_clock::time_point deadline() const {
    return std::chrono::steady_clock::now() +
           std::chrono::microseconds(static_cast<int64_t>(timeout_ * 1e6));
  }
  void check_dead(size_t who) {
    for (size_t r = 0; r < n_; ++r)
      if (dead_[r] && r != who) throw CommError("rank " + std::to_string(r) + " has left the world");
  }
};

LocalCommunicator::LocalCommunicator(size_t rank, std::shared_ptr<LocalHub> hub)
    : rank_(rank), hub_(std::move(hub)) {}

size_t LocalCommunicator::world_size() const { return hub_->n_; }
double LocalCommunicator::timeout_s() const { return hub_->timeout_; }

void LocalCommunicator::maybe_fault(const std::string& kind, bool* drop) {
  if (!hub_->faults) return;
  auto r = hub_->faults->check(rank_, kind);
  if (!r) return;
  switch (r->action) {
    case FaultRule::Action::Drop:
      if (drop) *drop = true;
      break;
    case FaultRule::Action::Delay:
      std::this_thread::sleep_for(std::chrono::microseconds(static_cast<int64_t>(r->delay_s * 1e6)));
      break;
    case FaultRule::Action::Kill: {
      std::lock_guard<std::mutex> lk(hub_->mu);
      hub_->dead_[rank_] = true;
      hub_->cv.notify_all();
      throw CommError("rank " + std::to_string(rank_) + " killed by fault plan at " + kind);
    }
    case FaultRule::Action::Corrupt:
      break;
  }
}

void LocalCommunicator::send(const Bytes& data, size_t dst) {
  if (dst >= hub_->n_) throw CommError("destination " + std::to_string(dst) + " out of range");
  bool drop = false;
  maybe_fault("send", &drop);
  std::lock_guard<std::mutex> lk(hub_->mu);
  if (hub_->dead_[rank_]) throw CommError("rank " + std::to_string(rank_) + " has left the world");
  if (!drop) hub_->queues_[rank_ * hub_->n_ + dst].push_back(data);
  hub_->cv.notify_all();
}

Bytes LocalCommunicator::recv(size_t src) {
  if (src >= hub_->n_) throw CommError("source " + std::to_string(src) + " out of range");
  maybe_fault("recv", nullptr);
  std::unique_lock<std::mutex> lk(hub_->mu);
  auto& q = hub_->queues_[src * hub_->n_ + rank_];
  const auto dl = hub_->deadline();
  while (q.empty()) {
    if (hub_->dead_[src]) throw CommError("rank " + std::to_string(src) + " has left the world");
    if (hub_->cv.wait_until(lk, dl) == std::cv_status::timeout && q.empty())
      throw CommTimeout("recv from rank " + std::to_string(src) + " timed out");
  }
  Bytes out = std::move(q.front());
  q.pop_front();
  return out;
}

std::optional<Bytes> LocalCommunicator::try_recv(size_t src) {
  std::lock_guard<std::mutex> lk(hub_->mu);
  auto& q = hub_->queues_[src * hub_->n_ + rank_];
  if (q.empty()) return std::nullopt;
  Bytes out = std::move(q.front());
  q.pop_front();
  return out;
}

// Generation-counted rendezvous: every rank deposits, the last arrival computes,
// everyone reads the result of that generation.
template <typename Fn>
static void rendezvous(LocalHub& h, size_t rank, const std::string& kind, const Bytes& in, Fn compute,
                       Bytes* out, std::vector<Bytes>* out_all) {
  std::unique_lock<std::mutex> lk(h.mu);
  h.check_dead(rank);
  if (h.arrived == 0) {
    h.slots.assign(h.n_, Bytes());
    h.coll_kind = kind;
  } else if (h.coll_kind != kind) {
    throw CommError("collective mismatch: rank " + std::to_string(rank) + " called " + kind +
                    " while others are in " + h.coll_kind);
  }
  const uint64_t my_gen = h.gen;
  h.slots[rank] = in;
  if (++h.arrived == h.n_) {
    compute(h);
    h.arrived = 0;
    h.done_gen = ++h.gen;
    h.cv.notify_all();
  } else {
    const auto dl = h.deadline();
    while (h.done_gen <= my_gen) {
      for (size_t r = 0; r < h.n_; ++r)
        if (h.dead_[r]) {
          h.arrived = 0;
          throw CommError("rank " + std::to_string(r) + " has left the world during " + kind);
        }
      if (h.cv.wait_until(lk, dl) == std::cv_status::timeout && h.done_gen <= my_gen) {
        throw CommTimeout(kind + " timed out waiting for peers");
      }
    }
  }
  if (out) *out = h.result;
  if (out_all) *out_all = h.result_all;
}

Bytes LocalCommunicator::all_reduce(const Bytes& data, ReduceOp op, DType dt) {
  maybe_fault("all_reduce", nullptr);
  Bytes out;
  rendezvous(*hub_, rank_, "all_reduce", data,
             [&](LocalHub& h) { h.result = reduce_buffers(op, h.slots, dt); }, &out, nullptr);
  return out;
}

Bytes LocalCommunicator::broadcast(const Bytes& data, size_t root) {
  if (root >= hub_->n_) throw CommError("root " + std::to_string(root) + " out of range");
  maybe_fault("broadcast", nullptr);
  Bytes out;
  rendezvous(*hub_, rank_, "broadcast", data, [&](LocalHub& h) { h.result = h.slots[root]; }, &out,
             nullptr);
  return out;
}

std::vector<Bytes> LocalCommunicator::all_gather(const Bytes& data) {
  maybe_fault("all_gather", nullptr);
  std::vector<Bytes> out;
  rendezvous(*hub_, rank_, "all_gather", data, [&](LocalHub& h) { h.result_all = h.slots; }, nullptr,
             &out);
  return out;
}

void LocalCommunicator::barrier() {
  maybe_fault("barrier", nullptr);
  rendezvous(*hub_, rank_, "barrier", Bytes(), [](LocalHub&) {}, nullptr, nullptr);
}

std::vector<std::shared_ptr<LocalCommunicator>> LocalWorld::create(size_t n, double timeout_s,
                                                                   std::shared_ptr<FaultPlan> faults) {
  if (n == 0) throw CommError("world size must be > 0");
  auto hub = std::make_shared<LocalHub>(n, timeout_s, std::move(faults));
  std::vector<std::shared_ptr<LocalCommunicator>> out;
  for (size_t r = 0; r < n; ++r) out.push_back(std::make_shared<LocalCommunicator>(r, hub));
  return out;
}

// ---------------------------------------------------------------- P2P
P2PHandle::P2PHandle() : st_(std::make_shared<State>()) {}

void P2PHandle::set_result(const Bytes& data) {
  {
    std::lock_guard<std::mutex> lk(st_->mu);
    st_->value = data;
  }
  st_->cv.notify_all();
}

Bytes P2PHandle::wait(double timeout_s) {
  std::unique_lock<std::mutex> lk(st_->mu);
  if (timeout_s < 0) {
    st_->cv.wait(lk, [&] { return st_->value.has_value(); });
  } else if (!st_->cv.wait_for(lk, std::chrono::microseconds(static_cast<int64_t>(timeout_s * 1e6)),
                               [&] { return st_->value.has_value(); })) {
    throw CommTimeout("P2PHandle::wait timed out");
  }
  return *st_->value;
}

std::optional<Bytes> P2PHandle::try_get() const {
  std::lock_guard<std::mutex> lk(st_->mu);
  return st_->value;
}

P2PChannel::P2PChannel(size_t rank, size_t world)
    : rank_(rank), world_(world), buf_(std::make_shared<std::pair<std::mutex, Buffers>>()) {
  buf_->second.assign(world, std::vector<Bytes>(world));
}

std::vector<std::shared_ptr<P2PChannel>> P2PChannel::create_group(size_t world) {
  auto b = std::make_shared<std::pair<std::mutex, Buffers>>();
  b->second.assign(world, std::vector<Bytes>(world));
  std::vector<std::shared_ptr<P2PChannel>> out;
  for (size_t r = 0; r < world; ++r) out.push_back(std::shared_ptr<P2PChannel>(new P2PChannel(r, world, b)));
  return out;
}

P2PHandle P2PChannel::isend(const Bytes& data, size_t dst) {
  if (dst >= world_) throw CommError("destination " + std::to_string(dst) + " out of range");
  {
    std::lock_guard<std::mutex> lk(buf_->first);
    buf_->second[rank_][dst] = data;
  }
  P2PHandle h;
  h.set_result(data);
  return h;
}

P2PHandle P2PChannel::irecv(size_t src) {
  if (src >= world_) throw CommError("source " + std::to_string(src) + " out of range");
  Bytes snap;
  {
    std::lock_guard<std::mutex> lk(buf_->first);
    snap = buf_->second[src][rank_];
  }
  P2PHandle h;
  h.set_result(snap);
  return h;
}

std::pair<P2PHandle, P2PHandle> P2PChannel::sendrecv(const Bytes& data, size_t dst, size_t src) {
  P2PHandle s = isend(data, dst);
  P2PHandle r = irecv(src);
  return {s, r};
}

}  // namespace mtorus
