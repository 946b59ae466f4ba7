// Pipeline schedules (GPipe, 1F1B) as per-stage op lists, the per-rank
// communication program derived from them, a timeline simulator for bubble
// accounting, and the stage wire formats.
//
// Op lists follow crates/mt-pipeline/src/schedule/{gpipe,onef1b}.rs: 1F1B stage s
// runs warmup = min(S-s-1, M) forwards, then (F, B) pairs for the remaining
// micro-batches, then the cooldown backwards.  GPipe runs all forwards then all
// backwards.  The wire formats follow crates/mt-pipeline/src/stage.rs:37-58
// (StageData: rows u64 | cols u64 | f32 values, little endian) and
// crates/mt-pipeline/src/communicator.rs:44-73 (FP8 frame: rows u64 | cols u64 |
// format u8 | scale f32 | len u64 | fp8 bytes = 29-byte header).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "core/precision.h"

namespace mtorus {

enum class ScheduleType : int { Gpipe = 0, OneF1B = 1 };

struct PipeOp {
  enum class Kind : int { Forward = 0, Backward = 1, RecvAct = 2, SendAct = 3, RecvGrad = 4, SendGrad = 5 };
  Kind kind;
  int64_t microbatch;
  int64_t peer;  // stage on the other end for send/recv ops, -1 otherwise
  bool operator==(const PipeOp& o) const {
    return kind == o.kind && microbatch == o.microbatch && peer == o.peer;
  }
};

// Compute-only op lists (Forward / Backward) per stage.
std::vector<std::vector<PipeOp>> build_schedule(ScheduleType t, size_t num_stages, size_t num_microbatches);
// Full per-rank program with the receives / sends around each compute op, in an
// order that cannot deadlock with blocking point-to-point transport when all
// stages run it concurrently.
std::vector<PipeOp> rank_program(ScheduleType t, size_t stage, size_t num_stages, size_t num_microbatches);

struct TimelineResult {
  double makespan = 0;
  double bubble_fraction = 0;      // idle compute time / (stages * makespan)
  std::vector<double> stage_busy;  // per stage compute time
  size_t peak_inflight = 0;        // max activations stashed on any stage
  std::vector<size_t> stage_peak_inflight;
};
// Event-driven simulation of the op lists with fixed per-op costs and a
// point-to-point latency between adjacent stages.
TimelineResult simulate_schedule(ScheduleType t, size_t num_stages, size_t num_microbatches,
                                 double t_fwd, double t_bwd, double t_comm);
double ideal_bubble_fraction(size_t num_stages, size_t num_microbatches);

// Wire formats.
std::string stage_data_to_bytes(const std::vector<float>& values, uint64_t rows, uint64_t cols);
void stage_data_from_bytes(const std::string& b, std::vector<float>& values, uint64_t& rows, uint64_t& cols);
std::string compress_stage_data(const std::vector<float>& values, uint64_t rows, uint64_t cols, Fp8Format fmt);
void decompress_stage_data(const std::string& b, std::vector<float>& values, uint64_t& rows, uint64_t& cols);

}  // namespace mtorus
