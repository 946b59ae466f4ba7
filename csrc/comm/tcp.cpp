// TCP communicator over POSIX sockets.
//
// Reference: crates/mt-comm/src/tcp.rs.  Kept: the frame format (u64 LE length
// + payload, LEN_PREFIX_SIZE = 8) and the handshake (the dialling rank sends its
// rank as u64 LE; lower ranks dial higher ranks).  Changed: the listener binds
// addresses[rank] instead of an arbitrary ephemeral port, each peer connection
// has separate send and receive locks (a concurrent send and recv cannot
// deadlock), connects retry until a deadline, every blocking read has a
// timeout, and the Communicator methods work: collectives are ring algorithms
// built on send/recv (the reference's sync methods all bail).
#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

#include "comm/comm.h"

namespace mtorus {

namespace {

std::pair<std::string, uint16_t> split_addr(const std::string& a) {
  const auto p = a.rfind(':');
  if (p == std::string::npos) throw CommError("bad address '" + a + "' (want host:port)");
  return {a.substr(0, p), static_cast<uint16_t>(std::stoi(a.substr(p + 1)))};
}

sockaddr_in resolve(const std::string& host, uint16_t port) {
  sockaddr_in sa{};
  sa.sin_family = AF_INET;
  sa.sin_port = htons(port);
  if (inet_pton(AF_INET, host.c_str(), &sa.sin_addr) == 1) return sa;
  addrinfo hints{}, *res = nullptr;
  hints.ai_family = AF_INET;
  if (getaddrinfo(host.c_str(), nullptr, &hints, &res) != 0 || !res)
    throw CommError("cannot resolve host '" + host + "'");
  sa.sin_addr = reinterpret_cast<sockaddr_in*>(res->ai_addr)->sin_addr;
  freeaddrinfo(res);
  return sa;
}

void write_all(int fd, const char* p, size_t n) {
  while (n > 0) {
    const ssize_t w = ::send(fd, p, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      throw CommError(std::string("socket write failed: ") + std::strerror(errno));
    }
    p += w;
    n -= static_cast<size_t>(w);
  }
}

void read_all(int fd, char* p, size_t n, double timeout_s) {
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::microseconds(static_cast<int64_t>(timeout_s * 1e6));
  while (n > 0) {
    const auto left = std::chrono::duration_cast<std::chrono::milliseconds>(
        deadline - std::chrono::steady_clock::now()).count();
    if (left <= 0) throw CommTimeout("socket read timed out");
    pollfd pfd{fd, POLLIN, 0};
    const int pr = ::poll(&pfd, 1, static_cast<int>(std::min<int64_t>(left, 1000)));
    if (pr < 0) {
      if (errno == EINTR) continue;
      throw CommError(std::string("poll failed: ") + std::strerror(errno));
    }
    if (pr == 0) continue;
    const ssize_t r = ::recv(fd, p, n, 0);
    if (r == 0) throw CommError("peer closed the connection");
    if (r < 0) {
      if (errno == EINTR || errno == EAGAIN) continue;
      throw CommError(std::string("socket read failed: ") + std::strerror(errno));
    }
    p += r;
    n -= static_cast<size_t>(r);
  }
}

uint64_t le64(const char* b) {
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | static_cast<uint8_t>(b[i]);
  return v;
}
void put_le64(char* b, uint64_t v) {
  for (int i = 0; i < 8; ++i) b[i] = static_cast<char>((v >> (8 * i)) & 0xFF);
}

int dial(const std::string& addr, double timeout_s) {
  auto [host, port] = split_addr(addr);
  const sockaddr_in sa = resolve(host, port);
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::microseconds(static_cast<int64_t>(timeout_s * 1e6));
  while (true) {
    const int fd = ::socket(AF_INET, SOCK_STREAM, 0);
    if (fd < 0) throw CommError("socket() failed");
    if (port != 0 && ::connect(fd, reinterpret_cast<const sockaddr*>(&sa), sizeof(sa)) == 0) {
      int one = 1;
      setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
      return fd;
    }
    ::close(fd);
    if (std::chrono::steady_clock::now() >= deadline) return -1;
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
}

}  // namespace

void tcp_send_frame(int fd, const Bytes& data) {
  char hdr[8];
  put_le64(hdr, data.size());
  write_all(fd, hdr, 8);
  if (!data.empty()) write_all(fd, data.data(), data.size());
}

Bytes tcp_recv_frame(int fd, double timeout_s) {
  char hdr[8];
  read_all(fd, hdr, 8, timeout_s);
  const uint64_t len = le64(hdr);
  Bytes out(len, '\0');
  if (len) read_all(fd, out.data(), len, timeout_s);
  return out;
}

TcpCommunicator::TcpCommunicator(size_t rank, std::vector<std::string> addresses,
                                 double connect_timeout_s, double op_timeout_s, bool dial_peers)
    : rank_(rank), addrs_(std::move(addresses)), op_timeout_(op_timeout_s) {
  if (rank_ >= addrs_.size()) throw CommError("rank out of range of the address list");
  for (size_t i = 0; i < addrs_.size(); ++i) peers_.push_back(std::make_unique<Peer>());
  auto [host, port] = split_addr(addrs_[rank_]);
  listen_fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
  if (listen_fd_ < 0) throw CommError("socket() failed");
  int one = 1;
  setsockopt(listen_fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in sa = resolve(host, port);
  if (::bind(listen_fd_, reinterpret_cast<sockaddr*>(&sa), sizeof(sa)) != 0) {
    ::close(listen_fd_);
    throw CommError("bind(" + addrs_[rank_] + ") failed: " + std::strerror(errno));
  }
  ::listen(listen_fd_, 128);
  socklen_t sl = sizeof(sa);
  getsockname(listen_fd_, reinterpret_cast<sockaddr*>(&sa), &sl);
  port_ = ntohs(sa.sin_port);
  acceptor_ = std::make_unique<std::thread>([this] { accept_loop(); });
  if (dial_peers) {
    for (size_t dst = rank_ + 1; dst < addrs_.size(); ++dst) {
      try {
        connect_to(dst, addrs_[dst], connect_timeout_s);
      } catch (const CommError&) {
        // unreachable peers stay unconnected; a later send to them raises
      }
    }
  }
}

TcpCommunicator::~TcpCommunicator() { close(); }

void TcpCommunicator::close() {
  {
    std::lock_guard<std::mutex> lk(conn_mu_);
    if (closing_) return;
    closing_ = true;
  }
  if (acceptor_ && acceptor_->joinable()) acceptor_->join();
  if (listen_fd_ >= 0) ::close(listen_fd_);
  listen_fd_ = -1;
  // Shut every socket down first: that wakes a thread of this rank blocked in
  // send / recv on it (EOF or EPIPE).  Close the descriptor only once no thread is
  // inside send / recv on it, so that no call can reach a reused descriptor.
  for (auto& p : peers_) {
    const int fd = p->fd.load();
    if (fd >= 0) ::shutdown(fd, SHUT_RDWR);
  }
  for (auto& p : peers_) {
    std::scoped_lock lk(p->send_mu, p->recv_mu);
    const int fd = p->fd.exchange(-1);
    if (fd >= 0) ::close(fd);
  }
}

void TcpCommunicator::accept_loop() {
  while (true) {
    {
      std::lock_guard<std::mutex> lk(conn_mu_);
      if (closing_) return;
    }
    pollfd pfd{listen_fd_, POLLIN, 0};
    if (::poll(&pfd, 1, 100) <= 0) continue;
    const int fd = ::accept(listen_fd_, nullptr, nullptr);
    if (fd < 0) continue;
    char hdr[8];
    try {
      read_all(fd, hdr, 8, 5.0);
    } catch (const CommError&) {
      ::close(fd);
      continue;
    }
    const uint64_t src = le64(hdr);
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    std::lock_guard<std::mutex> lk(conn_mu_);
    if (src >= peers_.size() || peers_[src]->fd >= 0) {
      ::close(fd);
      continue;
    }
    peers_[src]->fd = fd;
    conn_cv_.notify_all();
  }
}

void TcpCommunicator::connect_to(size_t dst, const std::string& addr, double timeout_s) {
  if (dst >= peers_.size()) throw CommError("destination out of range");
  const int fd = dial(addr, timeout_s);
  if (fd < 0) throw CommError("cannot connect to rank " + std::to_string(dst) + " at " + addr);
  char hdr[8];
  put_le64(hdr, rank_);
  write_all(fd, hdr, 8);
  std::lock_guard<std::mutex> lk(conn_mu_);
  if (peers_[dst]->fd >= 0) ::close(peers_[dst]->fd);
  peers_[dst]->fd = fd;
  conn_cv_.notify_all();
}

std::vector<size_t> TcpCommunicator::wait_connected(double timeout_s) {
  std::unique_lock<std::mutex> lk(conn_mu_);
  auto missing = [&] {
    std::vector<size_t> m;
    for (size_t r = 0; r < peers_.size(); ++r)
      if (r != rank_ && peers_[r]->fd < 0) m.push_back(r);
    return m;
  };
  conn_cv_.wait_for(lk, std::chrono::microseconds(static_cast<int64_t>(timeout_s * 1e6)),
                    [&] { return missing().empty(); });
  return missing();
}

std::vector<size_t> TcpCommunicator::connected_peers() const {
  std::lock_guard<std::mutex> lk(conn_mu_);
  std::vector<size_t> out;
  for (size_t r = 0; r < peers_.size(); ++r)
    if (peers_[r]->fd >= 0) out.push_back(r);
  return out;
}

TcpCommunicator::Peer* TcpCommunicator::peer(size_t r) {
  if (r >= peers_.size() || r == rank_) throw CommError("invalid peer rank " + std::to_string(r));
  std::lock_guard<std::mutex> lk(conn_mu_);
  if (peers_[r]->fd < 0) throw CommError("no connection to rank " + std::to_string(r));
  return peers_[r].get();
}

void TcpCommunicator::send(const Bytes& data, size_t dst) {
  if (faults_) {
    auto f = faults_->check(rank_, "send");
    if (f && f->action == FaultRule::Action::Drop) return;
    if (f && f->action == FaultRule::Action::Delay)
      std::this_thread::sleep_for(std::chrono::microseconds(static_cast<int64_t>(f->delay_s * 1e6)));
    if (f && f->action == FaultRule::Action::Kill) {
      close();
      throw CommError("rank " + std::to_string(rank_) + " killed by fault plan");
    }
  }
  Peer* p = peer(dst);
  std::lock_guard<std::mutex> lk(p->send_mu);
  tcp_send_frame(p->fd, data);
}

Bytes TcpCommunicator::recv(size_t src) {
  Peer* p = peer(src);
  std::lock_guard<std::mutex> lk(p->recv_mu);
  return tcp_recv_frame(p->fd, op_timeout_);
}

void TcpCommunicator::sendrecv(const Bytes& out, size_t dst, Bytes& in, size_t src) {
  std::exception_ptr err;
  std::thread t([&] {
    try {
      send(out, dst);
    } catch (...) {
      err = std::current_exception();
    }
  });
  try {
    in = recv(src);
  } catch (...) {
    t.join();
    throw;
  }
  t.join();
  if (err) std::rethrow_exception(err);
}

Bytes TcpCommunicator::all_reduce(const Bytes& data, ReduceOp op, DType dt) {
  const size_t n = world_size();
  const size_t es = dtype_size(dt);
  const size_t ne = data.size() / es;
  Bytes acc = data.substr(0, ne * es);
  if (n == 1) {
    if (op == ReduceOp::Mean) finish_mean(acc, 1, dt);
    return acc;
  }
  // chunk c covers elements [c*ne/n, (c+1)*ne/n)
  auto lo = [&](size_t c) { return (c * ne / n) * es; };
  auto len = [&](size_t c) { return lo(c + 1) - lo(c); };
  const size_t right = (rank_ + 1) % n, left = (rank_ + n - 1) % n;
  for (size_t s = 0; s + 1 < n; ++s) {  // reduce-scatter
    const size_t cs = (rank_ + n - s) % n, cr = (rank_ + n - s - 1) % n;
    Bytes in;
    sendrecv(acc.substr(lo(cs), len(cs)), right, in, left);
    Bytes mine = acc.substr(lo(cr), len(cr));
    reduce_into(op, mine, in, dt);
    acc.replace(lo(cr), len(cr), mine);
  }
  for (size_t s = 0; s + 1 < n; ++s) {  // all-gather of the reduced chunks
    const size_t cs = (rank_ + 1 + n - s) % n, cr = (rank_ + n - s) % n;
    Bytes in;
    sendrecv(acc.substr(lo(cs), len(cs)), right, in, left);
    acc.replace(lo(cr), len(cr), in);
  }
  if (op == ReduceOp::Mean) finish_mean(acc, n, dt);
  return acc;
}

Bytes TcpCommunicator::broadcast(const Bytes& data, size_t root) {
  if (root >= world_size()) throw CommError("root " + std::to_string(root) + " out of range");
  if (rank_ == root) {
    for (size_t r = 0; r < world_size(); ++r)
      if (r != root) send(data, r);
    return data;
  }
  return recv(root);
}

std::vector<Bytes> TcpCommunicator::all_gather(const Bytes& data) {
  const size_t n = world_size();
  std::vector<Bytes> out(n);
  out[rank_] = data;
  const size_t right = (rank_ + 1) % n, left = (rank_ + n - 1) % n;
  for (size_t s = 0; s + 1 < n; ++s) {
    const size_t cs = (rank_ + n - s) % n, cr = (rank_ + n - s - 1) % n;
    sendrecv(out[cs], right, out[cr], left);
  }
  return out;
}

}  // namespace mtorus
