// pybind11 bindings of the communicator layer.
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "comm/comm.h"

namespace py = pybind11;
using namespace mtorus;

namespace {

// Lets Python subclasses (for example the NCCL communicator) implement the
// interface and be used by the C++ TopologyAwareComm.
class PyCommunicator : public Communicator {
 public:
  using Communicator::Communicator;
  void send(const Bytes& data, size_t dst) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const Communicator*>(this), "send");
    if (!f) throw CommError("send not implemented");
    f(py::bytes(data), dst);
  }
  Bytes recv(size_t src) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const Communicator*>(this), "recv");
    if (!f) throw CommError("recv not implemented");
    return f(src).cast<std::string>();
  }
  Bytes all_reduce(const Bytes& data, ReduceOp op, DType dt) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const Communicator*>(this), "all_reduce");
    if (!f) throw CommError("all_reduce not implemented");
    return f(py::bytes(data), op, dt).cast<std::string>();
  }
  Bytes broadcast(const Bytes& data, size_t root) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const Communicator*>(this), "broadcast");
    if (!f) throw CommError("broadcast not implemented");
    return f(py::bytes(data), root).cast<std::string>();
  }
  std::vector<Bytes> all_gather(const Bytes& data) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const Communicator*>(this), "all_gather");
    if (!f) throw CommError("all_gather not implemented");
    std::vector<Bytes> out;
    for (auto item : f(py::bytes(data))) out.push_back(item.cast<std::string>());
    return out;
  }
  size_t rank() const override { PYBIND11_OVERRIDE_PURE(size_t, Communicator, rank, ); }
  size_t world_size() const override { PYBIND11_OVERRIDE_PURE(size_t, Communicator, world_size, ); }
  std::string backend() const override { PYBIND11_OVERRIDE(std::string, Communicator, backend, ); }
  void barrier() override { PYBIND11_OVERRIDE(void, Communicator, barrier, ); }
  bool exchange(const Bytes& data, const std::vector<size_t>& peers, std::vector<Bytes>* out) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const Communicator*>(this), "exchange");
    if (!f) return false;
    py::object r = f(py::bytes(data), peers);
    if (r.is_none()) return false;
    out->clear();
    for (auto item : r) out->push_back(item.cast<std::string>());
    if (out->size() != peers.size()) throw CommError("exchange returned the wrong number of messages");
    return true;
  }
};

py::bytes B(const Bytes& b) { return py::bytes(b); }
py::list BL(const std::vector<Bytes>& v) {
  py::list l;
  for (const auto& b : v) l.append(py::bytes(b));
  return l;
}

}  // namespace

void bind_comm(py::module_& m) {
  static py::exception<CommError> comm_error(m, "CommError", PyExc_RuntimeError);
  static py::exception<CommTimeout> comm_timeout(m, "CommTimeout", comm_error.ptr());
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const CommTimeout& e) {
      PyErr_SetString(comm_timeout.ptr(), e.what());
    } catch (const CommError& e) {
      PyErr_SetString(comm_error.ptr(), e.what());
    }
  });

  py::enum_<ReduceOp>(m, "ReduceOp")
      .value("Sum", ReduceOp::Sum)
      .value("Product", ReduceOp::Product)
      .value("Min", ReduceOp::Min)
      .value("Max", ReduceOp::Max)
      .value("Mean", ReduceOp::Mean)
      .def("to_string", [](ReduceOp o) { return std::string(reduce_op_name(o)); });
  py::enum_<DType>(m, "DType")
      .value("U64", DType::U64)
      .value("I64", DType::I64)
      .value("F32", DType::F32)
      .value("F64", DType::F64)
      .value("I32", DType::I32)
      .value("U8", DType::U8);
  py::enum_<CollectiveOp>(m, "CollectiveOp")
      .value("AllReduce", CollectiveOp::AllReduce)
      .value("Broadcast", CollectiveOp::Broadcast)
      .value("AllGather", CollectiveOp::AllGather)
      .value("ReduceScatter", CollectiveOp::ReduceScatter)
      .def("to_string", [](CollectiveOp o) { return std::string(collective_op_name(o)); });
  m.def("reduce_buffers", [](ReduceOp op, const std::vector<std::string>& chunks, DType dt) {
    return B(reduce_buffers(op, chunks, dt));
  });

  py::class_<Communicator, PyCommunicator, std::shared_ptr<Communicator>>(m, "Communicator")
      .def(py::init<>())
      .def("send", [](Communicator& c, const std::string& d, size_t dst) {
        py::gil_scoped_release r;
        c.send(d, dst);
      }, py::arg("data"), py::arg("dst"))
      .def("recv", [](Communicator& c, size_t src) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = c.recv(src);
        }
        return B(out);
      }, py::arg("src"))
      .def("all_reduce", [](Communicator& c, const std::string& d, ReduceOp op, DType dt) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = c.all_reduce(d, op, dt);
        }
        return B(out);
      }, py::arg("data"), py::arg("op"), py::arg("dtype") = DType::U64)
      .def("broadcast", [](Communicator& c, const std::string& d, size_t root) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = c.broadcast(d, root);
        }
        return B(out);
      }, py::arg("data"), py::arg("root"))
      .def("all_gather", [](Communicator& c, const std::string& d) {
        std::vector<Bytes> out;
        {
          py::gil_scoped_release r;
          out = c.all_gather(d);
        }
        return BL(out);
      }, py::arg("data"))
      .def("barrier", [](Communicator& c) {
        py::gil_scoped_release r;
        c.barrier();
      })
      .def("rank", &Communicator::rank)
      .def("world_size", &Communicator::world_size)
      .def("backend", &Communicator::backend);

  py::class_<MockCommunicator, Communicator, std::shared_ptr<MockCommunicator>>(m, "MockCommunicator")
      .def(py::init<size_t, size_t>(), py::arg("rank"), py::arg("world_size"))
      .def_static("create_world", &MockCommunicator::create_world, py::arg("world_size"));

  py::class_<FaultRule> fr(m, "FaultRule");
  py::enum_<FaultRule::Action>(fr, "Action")
      .value("Drop", FaultRule::Action::Drop)
      .value("Delay", FaultRule::Action::Delay)
      .value("Kill", FaultRule::Action::Kill)
      .value("Corrupt", FaultRule::Action::Corrupt);
  fr.def(py::init([](int64_t rank, int64_t at_op, std::string kind, FaultRule::Action a, double delay) {
         return FaultRule{rank, at_op, std::move(kind), a, delay};
       }),
       py::arg("rank") = -1, py::arg("at_op") = -1, py::arg("op_kind") = "",
       py::arg("action") = FaultRule::Action::Drop, py::arg("delay_s") = 0.0)
      .def_readwrite("rank", &FaultRule::rank)
      .def_readwrite("at_op", &FaultRule::at_op)
      .def_readwrite("op_kind", &FaultRule::op_kind)
      .def_readwrite("action", &FaultRule::action)
      .def_readwrite("delay_s", &FaultRule::delay_s);
  py::class_<FaultPlan, std::shared_ptr<FaultPlan>>(m, "FaultPlan")
      .def(py::init<>())
      .def("add", &FaultPlan::add)
      .def("clear", &FaultPlan::clear)
      .def("ops_seen", &FaultPlan::ops_seen);

  py::class_<LocalCommunicator, Communicator, std::shared_ptr<LocalCommunicator>>(m, "LocalCommunicator")
      .def("try_recv", [](LocalCommunicator& c, size_t src) -> py::object {
        auto v = c.try_recv(src);
        if (!v) return py::none();
        return py::bytes(*v);
      })
      .def("timeout_s", &LocalCommunicator::timeout_s);
  m.def("local_world", &LocalWorld::create, py::arg("n"), py::arg("timeout_s") = 30.0,
        py::arg("faults") = nullptr);

  py::class_<P2PHandle>(m, "P2PHandle")
      .def(py::init<>())
      .def("set_result", [](P2PHandle& h, const std::string& d) { h.set_result(d); })
      .def("wait", [](P2PHandle& h, double t) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = h.wait(t);
        }
        return B(out);
      }, py::arg("timeout_s") = 30.0)
      .def("try_get", [](const P2PHandle& h) -> py::object {
        auto v = h.try_get();
        if (!v) return py::none();
        return py::bytes(*v);
      });
  py::class_<P2PChannel, std::shared_ptr<P2PChannel>>(m, "P2PChannel")
      .def(py::init<size_t, size_t>(), py::arg("rank"), py::arg("world_size"))
      .def_static("create_group", &P2PChannel::create_group)
      .def("isend", [](P2PChannel& c, const std::string& d, size_t dst) { return c.isend(d, dst); })
      .def("irecv", &P2PChannel::irecv)
      .def("sendrecv", [](P2PChannel& c, const std::string& d, size_t dst, size_t src) {
        return c.sendrecv(d, dst, src);
      })
      .def("rank", &P2PChannel::rank)
      .def("world_size", &P2PChannel::world_size);

  py::class_<TcpCommunicator, Communicator, std::shared_ptr<TcpCommunicator>>(m, "TcpCommunicator")
      .def(py::init([](size_t rank, std::vector<std::string> addrs, double ct, double ot, bool dial) {
             py::gil_scoped_release r;
             return std::make_shared<TcpCommunicator>(rank, std::move(addrs), ct, ot, dial);
           }),
           py::arg("rank"), py::arg("addresses"), py::arg("connect_timeout_s") = 5.0,
           py::arg("op_timeout_s") = 60.0, py::arg("dial") = true)
      .def("port", &TcpCommunicator::port)
      .def("connect_to", [](TcpCommunicator& c, size_t dst, const std::string& addr, double t) {
        py::gil_scoped_release r;
        c.connect_to(dst, addr, t);
      }, py::arg("dst"), py::arg("addr"), py::arg("timeout_s") = 5.0)
      .def("wait_connected", [](TcpCommunicator& c, double t) {
        py::gil_scoped_release r;
        return c.wait_connected(t);
      }, py::arg("timeout_s") = 10.0)
      .def("connected_peers", &TcpCommunicator::connected_peers)
      .def("set_fault_plan", &TcpCommunicator::set_fault_plan)
      .def("close", [](TcpCommunicator& c) {
        py::gil_scoped_release r;
        c.close();
      });

  m.def("tcp_send_frame", [](int fd, const std::string& d) {
    py::gil_scoped_release r;
    tcp_send_frame(fd, d);
  }, py::arg("fd"), py::arg("data"));
  m.def("tcp_recv_frame", [](int fd, double t) {
    Bytes out;
    {
      py::gil_scoped_release r;
      out = tcp_recv_frame(fd, t);
    }
    return B(out);
  }, py::arg("fd"), py::arg("timeout_s") = 30.0);

  py::class_<TopologyAwareComm, std::shared_ptr<TopologyAwareComm>>(m, "TopologyAwareComm")
      .def(py::init<std::shared_ptr<Communicator>, MeshTorusHybrid>(), py::arg("inner"), py::arg("topology"),
           py::keep_alive<1, 2>())
      .def("rank", &TopologyAwareComm::rank)
      .def("world_size", &TopologyAwareComm::world_size)
      .def("inner", &TopologyAwareComm::inner)
      .def("topology", &TopologyAwareComm::topology)
      .def("rank_coords", &TopologyAwareComm::rank_coords)
      .def("exchange_with_neighbors", [](TopologyAwareComm& t, const std::string& d) {
        std::vector<std::pair<size_t, Bytes>> out;
        {
          py::gil_scoped_release r;
          out = t.exchange_with_neighbors(d);
        }
        py::list l;
        for (auto& p : out) l.append(py::make_tuple(p.first, py::bytes(p.second)));
        return l;
      })
      .def("perform_collective", [](TopologyAwareComm& t, CollectiveOp op, const std::string& d, DType dt) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = t.perform_collective(op, d, dt);
        }
        return B(out);
      }, py::arg("op"), py::arg("data"), py::arg("dtype") = DType::U64)
      .def("reduce_on_mesh", [](TopologyAwareComm& t, const std::string& d, std::vector<size_t> g, DType dt) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = t.reduce_on_mesh(d, g, dt);
        }
        return B(out);
      }, py::arg("data"), py::arg("group"), py::arg("dtype") = DType::U64)
      .def("reduce_on_group", [](TopologyAwareComm& t, const std::string& d, std::vector<size_t> g, DType dt) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = t.reduce_on_group(d, g, dt);
        }
        return B(out);
      }, py::arg("data"), py::arg("group"), py::arg("dtype") = DType::U64)
      .def("nearest_neighbor_exchange", [](TopologyAwareComm& t, const std::string& d, size_t axis) {
        std::vector<Bytes> out;
        {
          py::gil_scoped_release r;
          out = t.nearest_neighbor_exchange(d, axis);
        }
        return BL(out);
      })
      .def("all_reduce_mesh", [](TopologyAwareComm& t, const std::string& d, std::vector<size_t> g) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = t.all_reduce_mesh(d, g);
        }
        return B(out);
      })
      .def("pipeline_stage_sendrecv", [](TopologyAwareComm& t, const std::string& d, size_t s) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = t.pipeline_stage_sendrecv(d, s);
        }
        return B(out);
      })
      .def("route_collective", [](TopologyAwareComm& t, CollectiveOp op, const std::string& d) {
        Bytes out;
        {
          py::gil_scoped_release r;
          out = t.route_collective(op, d);
        }
        return B(out);
      });
}
