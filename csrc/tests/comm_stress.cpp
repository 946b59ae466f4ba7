// Multi-threaded stress driver for the host communication library, built with
// ThreadSanitizer or AddressSanitizer + UndefinedBehaviorSanitizer
// (mtorus/utils/sanitize.py compiles it together with the library sources).
//
// The reference has no race detection at all (its only concurrency is the
// parking_lot locks around the mock mailboxes, crates/mt-comm/src/mock.rs:6-32,
// and the tokio mutex of the TCP backend, crates/mt-comm/src/tcp.rs:12-20).  This
// driver runs every thread-shared part of the C++ runtime from one thread per rank
// and checks each result, so a sanitizer report points at a real interleaving:
//
//   * LocalWorld: collectives of every ReduceOp / dtype, broadcast, all_gather,
//     barrier, ring send/recv and try_recv polling, from 4 rank threads;
//   * a FaultPlan shared by the rank threads (delay rules on the hot path);
//   * TopologyAwareComm neighbour exchange and collectives on a 2x2 torus;
//   * P2PChannel isend / irecv / sendrecv and P2PHandle waits across threads;
//   * TcpCommunicator over 127.0.0.1: ring all_reduce / all_gather / broadcast from
//     3 rank threads, then two threads per rank sending concurrently to one peer,
//     and a ring in which one rank's fault plan kills it mid-collective;
//   * the prefetching TokenLoader: 3 worker threads, a consumer that seeks back and
//     forth while fills are in flight, every batch checked against synthetic_token;
//   * single-threaded, for the undefined-behaviour checker: the FP8 codec over all
//     256 codes and over special / extreme floats, the scaling and loss-scale state
//     machines, the pipeline op lists, simulator and stage-data frames.
//
// Exit status 0 when every check passed; a sanitizer that finds an error makes
// the process exit non-zero (halt_on_error / exitcode options set by the runner).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <string>
#include <thread>
#include <vector>

#include "comm/comm.h"
#include "core/data_loader.h"
#include "core/precision.h"
#include "core/topology.h"
#include "pipeline/schedule.h"

using namespace mtorus;

namespace {

std::atomic<int> g_failures{0};

void check(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "CHECK FAILED: %s\n", what);
    g_failures.fetch_add(1);
  }
}

template <class T>
Bytes pack(const std::vector<T>& v) {
  return Bytes(reinterpret_cast<const char*>(v.data()), v.size() * sizeof(T));
}
template <class T>
std::vector<T> unpack(const Bytes& b) {
  std::vector<T> v(b.size() / sizeof(T));
  std::memcpy(v.data(), b.data(), v.size() * sizeof(T));
  return v;
}

void run_threads(size_t n, const std::function<void(size_t)>& body) {
  std::vector<std::thread> ts;
  for (size_t r = 0; r < n; ++r)
    ts.emplace_back([&, r] {
      try {
        body(r);
      } catch (const std::exception& e) {
        std::fprintf(stderr, "rank %zu raised: %s\n", r, e.what());
        g_failures.fetch_add(1);
      }
    });
  for (auto& t : ts) t.join();
}

void local_world(int rounds) {
  const size_t n = 4;
  auto faults = std::make_shared<FaultPlan>();
  FaultRule slow;
  slow.op_kind = "all_reduce";
  slow.action = FaultRule::Action::Delay;
  slow.delay_s = 0.0005;
  slow.rank = 2;
  faults->add(slow);
  auto world = LocalWorld::create(n, 20.0, faults);
  run_threads(n, [&](size_t r) {
    auto& c = *world[r];
    for (int it = 0; it < rounds; ++it) {
      std::vector<float> x(64 + it % 7);
      for (size_t i = 0; i < x.size(); ++i) x[i] = float(r + 1) * float(i + 1);
      auto s = unpack<float>(c.all_reduce(pack(x), ReduceOp::Sum, DType::F32));
      check(s.size() == x.size() && s[3] == 10.f * 4.f, "local all_reduce sum");
      auto m = unpack<float>(c.all_reduce(pack(x), ReduceOp::Max, DType::F32));
      check(m[0] == 4.f, "local all_reduce max");
      std::vector<uint64_t> u(5, r + 1);
      auto p = unpack<uint64_t>(c.all_reduce(pack(u), ReduceOp::Product, DType::U64));
      check(p[4] == 24, "local all_reduce product");
      auto b = c.broadcast(r == size_t(it) % n ? Bytes("root" + std::to_string(it)) : Bytes(), size_t(it) % n);
      check(b == "root" + std::to_string(it), "local broadcast");
      auto g = c.all_gather(Bytes(1 + r, char('a' + r)));
      check(g.size() == n && g[3] == "dddd", "local all_gather");
      // ring: send right, then receive from the left (queues make this deadlock-free)
      c.send(std::to_string(r) + ":" + std::to_string(it), (r + 1) % n);
      auto in = c.recv((r + n - 1) % n);
      check(in == std::to_string((r + n - 1) % n) + ":" + std::to_string(it), "local ring");
      c.barrier();
      check(!c.try_recv((r + 1) % n).has_value(), "local try_recv empty after barrier");
    }
  });
  check(faults->ops_seen(2) >= rounds, "fault plan counted rank 2's ops");
}

void torus(int rounds) {
  auto world = LocalWorld::create(4, 20.0, nullptr);
  run_threads(4, [&](size_t r) {
    TopologyAwareComm tc(world[r], MeshTorusHybrid::new_2d(2, 2, 1));
    for (int it = 0; it < rounds; ++it) {
      auto got = tc.exchange_with_neighbors(Bytes(8, char('0' + r)));
      check(!got.empty(), "torus exchange");
      std::vector<uint64_t> v(3, r);
      auto s = unpack<uint64_t>(tc.perform_collective(CollectiveOp::AllReduce, pack(v)));
      check(s[0] == 6, "torus all_reduce");
    }
  });
}

void p2p(int rounds) {
  const size_t n = 4;
  auto group = P2PChannel::create_group(n);
  run_threads(n, [&](size_t r) {
    auto& ch = *group[r];
    for (int it = 0; it < rounds; ++it) {
      auto [s, rv] = ch.sendrecv(Bytes(16, char(r)), (r + 1) % n, (r + n - 1) % n);
      check(s.wait(5.0).size() == 16, "p2p send handle");
      const Bytes in = rv.wait(5.0);  // a snapshot: empty or a full 16-byte message
      check(in.empty() || in.size() == 16, "p2p irecv snapshot");
    }
  });
  // a handle completed by one thread and awaited by others
  P2PHandle h;
  std::vector<std::thread> waiters;
  std::atomic<int> ok{0};
  for (int i = 0; i < 3; ++i)
    waiters.emplace_back([&] {
      if (h.wait(10.0) == "done") ok.fetch_add(1);
    });
  std::thread setter([&] { h.set_result("done"); });
  setter.join();
  for (auto& t : waiters) t.join();
  check(ok.load() == 3, "p2p handle cross-thread wait");
}

void tcp(int rounds) {
  const size_t n = 3;
  std::vector<std::string> addrs(n, "127.0.0.1:0");
  std::vector<std::unique_ptr<TcpCommunicator>> cs;
  for (size_t r = 0; r < n; ++r) cs.emplace_back(new TcpCommunicator(r, addrs, 5.0, 20.0, false));
  for (size_t r = 0; r < n; ++r)
    for (size_t d = r + 1; d < n; ++d) cs[r]->connect_to(d, "127.0.0.1:" + std::to_string(cs[d]->port()), 5.0);
  for (size_t r = 0; r < n; ++r) check(cs[r]->wait_connected(5.0).empty(), "tcp connected");
  run_threads(n, [&](size_t r) {
    auto& c = *cs[r];
    for (int it = 0; it < rounds; ++it) {
      std::vector<double> x(37, double(r + 1));
      auto s = unpack<double>(c.all_reduce(pack(x), ReduceOp::Sum, DType::F64));
      check(s.size() == 37 && s[36] == 6.0, "tcp all_reduce");
      auto g = c.all_gather(std::to_string(r));
      check(g.size() == n && g[2] == "2", "tcp all_gather");
      auto b = c.broadcast(r == 1 ? Bytes(1000, 'x') : Bytes(), 1);
      check(b.size() == 1000, "tcp broadcast");
    }
  });
  // two sender threads per rank into the same peer socket, one receiver thread per source
  run_threads(n, [&](size_t r) {
    auto& c = *cs[r];
    const size_t dst = (r + 1) % n, src = (r + n - 1) % n;
    std::thread a([&] {
      for (int i = 0; i < rounds; ++i) c.send(Bytes(64, 'a'), dst);
    });
    std::thread b([&] {
      for (int i = 0; i < rounds; ++i) c.send(Bytes(96, 'b'), dst);
    });
    int na = 0, nb = 0;
    for (int i = 0; i < 2 * rounds; ++i) {
      const Bytes m = c.recv(src);
      if (m == Bytes(64, 'a')) ++na;
      else if (m == Bytes(96, 'b')) ++nb;
    }
    a.join();
    b.join();
    check(na == rounds && nb == rounds, "tcp concurrent senders keep frames whole");
  });
  for (auto& c : cs) c->close();
}

void codec_and_schedules() {
  for (Fp8Format f : {Fp8Format::E4M3, Fp8Format::E5M2}) {
    for (int b = 0; b < 256; ++b) {
      const float v = fp8_decode(uint8_t(b), f);
      if (std::isfinite(v)) check(fp8_decode(fp8_encode(v, f), f) == v, "fp8 code round trip");
    }
    const float specials[] = {0.f, -0.f, 1e-45f, -1e-45f, 1e-30f, 3.4e38f, -3.4e38f,
                              std::numeric_limits<float>::infinity(), -std::numeric_limits<float>::infinity(),
                              std::numeric_limits<float>::quiet_NaN(), 448.f, 57344.f, 1e6f};
    for (float x : specials) (void)fp8_decode(fp8_encode(x, f), f);
    std::vector<float> v(1000);
    for (size_t i = 0; i < v.size(); ++i) v[i] = std::ldexp(float(i % 17) - 8.f, int(i % 40) - 20);
    auto t = to_fp8(v, f);
    check(from_fp8(t).size() == v.size(), "to_fp8 / from_fp8");
    auto tb = to_fp8_per_block(v, f, 33);
    check(from_fp8(tb).size() == v.size(), "per-block round trip");
    (void)to_fp8(std::vector<float>(5, 0.f), f);
  }
  DelayedScaling ds(16);
  for (int i = 0; i < 100; ++i) ds.update(float(i % 13));
  check(ds.current_amax() == 12.f, "delayed scaling amax");
  (void)ds.compute_scale(Fp8Format::E4M3);
  auto ls = LossScaler::new_dynamic(65536.f, 3);
  for (int i = 0; i < 200; ++i) ls.update(i % 7 == 0);
  for (ScheduleType t : {ScheduleType::Gpipe, ScheduleType::OneF1B})
    for (size_t s = 1; s <= 8; ++s)
      for (size_t m = 1; m <= 16; m += 3) {
        auto ops = build_schedule(t, s, m);
        check(ops.size() == s, "schedule has one op list per stage");
        auto tl = simulate_schedule(t, s, m, 1.0, 2.0, 0.1);
        (void)tl;
        (void)ideal_bubble_fraction(s, m);
      }
  std::vector<float> vals(6 * 5);
  for (size_t i = 0; i < vals.size(); ++i) vals[i] = float(i) - 7.5f;
  std::vector<float> back;
  uint64_t rows = 0, cols = 0;
  stage_data_from_bytes(stage_data_to_bytes(vals, 6, 5), back, rows, cols);
  check(back == vals && rows == 6 && cols == 5, "stage data frame");
  decompress_stage_data(compress_stage_data(vals, 6, 5, Fp8Format::E4M3), back, rows, cols);
  check(back.size() == vals.size(), "fp8 stage frame");
}

void token_loader(int rounds) {
  const int64_t B = 3, S = 17, V = 1000, N = 40;
  TokenLoader l(B, S, V, N, 9, true, 3, 3);
  std::vector<int64_t> inp(B * S), tgt(B * S);
  for (int it = 0; it < rounds; ++it) {
    const int64_t start = (it * 7) % N;
    l.seek(start);
    for (int64_t i = start; i < std::min<int64_t>(N, start + 5); ++i) {
      check(l.next_into(inp.data(), tgt.data(), 10.0), "loader batch available");
      const uint64_t per = (uint64_t)(B * (S + 1));
      check(inp[0] == synthetic_token(9, (uint64_t)i, 0, per, V), "loader batch content");
      check(tgt[0] == synthetic_token(9, (uint64_t)i, 1, per, V), "loader shifted target");
    }
  }
  l.seek(N - 1);
  check(l.next_into(inp.data(), tgt.data(), 10.0) && !l.next_into(inp.data(), tgt.data(), 10.0),
        "loader ends after num_batches");
}

// A rank killed by its fault plan in the middle of a ring all_reduce: its send
// thread closes every socket while its receiving thread is inside recv.  Every
// rank must leave with a CommError (EOF or timeout), none may hang.
void tcp_kill() {
  const size_t n = 3;
  std::vector<std::string> addrs(n, "127.0.0.1:0");
  auto faults = std::make_shared<FaultPlan>();
  FaultRule kill;
  kill.rank = 1;
  kill.at_op = 5;
  kill.op_kind = "send";
  kill.action = FaultRule::Action::Kill;
  faults->add(kill);
  std::vector<std::unique_ptr<TcpCommunicator>> cs;
  for (size_t r = 0; r < n; ++r) cs.emplace_back(new TcpCommunicator(r, addrs, 5.0, 2.0, false));
  for (size_t r = 0; r < n; ++r)
    for (size_t d = r + 1; d < n; ++d) cs[r]->connect_to(d, "127.0.0.1:" + std::to_string(cs[d]->port()), 5.0);
  for (size_t r = 0; r < n; ++r) check(cs[r]->wait_connected(5.0).empty(), "tcp connected");
  cs[1]->set_fault_plan(faults);
  std::atomic<int> errors{0};
  std::vector<std::thread> ts;
  for (size_t r = 0; r < n; ++r)
    ts.emplace_back([&, r] {
      try {
        for (int it = 0; it < 20; ++it) cs[r]->all_reduce(pack(std::vector<float>(300, 1.f)), ReduceOp::Sum, DType::F32);
      } catch (const CommError&) {
        errors.fetch_add(1);
      }
    });
  for (auto& t : ts) t.join();
  check(errors.load() == int(n), "every rank leaves the killed ring with a CommError");
  for (auto& c : cs) c->close();
}

}  // namespace

int main(int argc, char** argv) {
  const int rounds = argc > 1 ? std::atoi(argv[1]) : 50;
  codec_and_schedules();
  token_loader(rounds);
  local_world(rounds);
  torus(rounds / 5 + 1);
  p2p(rounds);
  tcp(rounds / 5 + 1);
  tcp_kill();
  const int f = g_failures.load();
  std::printf("comm_stress: %d rounds, %d failed checks\n", rounds, f);
  return f == 0 ? 0 : 1;
}
