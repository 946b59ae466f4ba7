// pybind11 bindings of the pipeline schedule builder and wire formats.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "pipeline/schedule.h"

namespace py = pybind11;
using namespace mtorus;

void bind_pipeline(py::module_& m) {
  py::enum_<ScheduleType>(m, "ScheduleType")
      .value("Gpipe", ScheduleType::Gpipe)
      .value("OneF1B", ScheduleType::OneF1B);
  py::class_<PipeOp> op(m, "PipeOp");
  py::enum_<PipeOp::Kind>(op, "Kind")
      .value("Forward", PipeOp::Kind::Forward)
      .value("Backward", PipeOp::Kind::Backward)
      .value("RecvAct", PipeOp::Kind::RecvAct)
      .value("SendAct", PipeOp::Kind::SendAct)
      .value("RecvGrad", PipeOp::Kind::RecvGrad)
      .value("SendGrad", PipeOp::Kind::SendGrad);
  op.def_readonly("kind", &PipeOp::kind)
      .def_readonly("microbatch", &PipeOp::microbatch)
      .def_readonly("peer", &PipeOp::peer)
      .def("__eq__", [](const PipeOp& a, const PipeOp& b) { return a == b; })
      .def("__repr__", [](const PipeOp& o) {
        static const char* names[] = {"F", "B", "RecvAct", "SendAct", "RecvGrad", "SendGrad"};
        std::string s = std::string(names[(int)o.kind]) + "(" + std::to_string(o.microbatch);
        if (o.peer >= 0) s += ", peer=" + std::to_string(o.peer);
        return s + ")";
      });
  m.def("build_schedule", &build_schedule, py::arg("schedule_type"), py::arg("num_stages"),
        py::arg("num_microbatches"));
  m.def("rank_program", &rank_program, py::arg("schedule_type"), py::arg("stage"), py::arg("num_stages"),
        py::arg("num_microbatches"));
  py::class_<TimelineResult>(m, "TimelineResult")
      .def_readonly("makespan", &TimelineResult::makespan)
      .def_readonly("bubble_fraction", &TimelineResult::bubble_fraction)
      .def_readonly("stage_busy", &TimelineResult::stage_busy)
      .def_readonly("peak_inflight", &TimelineResult::peak_inflight)
      .def_readonly("stage_peak_inflight", &TimelineResult::stage_peak_inflight);
  m.def("simulate_schedule", &simulate_schedule, py::arg("schedule_type"), py::arg("num_stages"),
        py::arg("num_microbatches"), py::arg("t_fwd") = 1.0, py::arg("t_bwd") = 2.0, py::arg("t_comm") = 0.0);
  m.def("ideal_bubble_fraction", &ideal_bubble_fraction);
  m.def("stage_data_to_bytes", [](const std::vector<float>& v, uint64_t r, uint64_t c) {
    return py::bytes(stage_data_to_bytes(v, r, c));
  });
  m.def("stage_data_from_bytes", [](const std::string& b) {
    std::vector<float> v;
    uint64_t r, c;
    stage_data_from_bytes(b, v, r, c);
    return py::make_tuple(v, r, c);
  });
  m.def("compress_stage_data", [](const std::vector<float>& v, uint64_t r, uint64_t c, Fp8Format f) {
    return py::bytes(compress_stage_data(v, r, c, f));
  });
  m.def("decompress_stage_data", [](const std::string& b) {
    std::vector<float> v;
    uint64_t r, c;
    decompress_stage_data(b, v, r, c);
    return py::make_tuple(v, r, c);
  });
}
