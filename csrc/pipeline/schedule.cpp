#include "pipeline/schedule.h"

#include <algorithm>
#include <cstring>
#include <deque>
#include <stdexcept>

namespace mtorus {

using K = PipeOp::Kind;

std::vector<std::vector<PipeOp>> build_schedule(ScheduleType t, size_t S, size_t M) {
  std::vector<std::vector<PipeOp>> out(S);
  for (size_t s = 0; s < S; ++s) {
    auto& ops = out[s];
    if (t == ScheduleType::Gpipe) {
      for (size_t m = 0; m < M; ++m) ops.push_back({K::Forward, (int64_t)m, -1});
      for (size_t m = 0; m < M; ++m) ops.push_back({K::Backward, (int64_t)m, -1});
      continue;
    }
    const size_t warmup = std::min(S - s - 1, M);
    const size_t steady = M > warmup ? M - warmup : 0;
    size_t f = 0, b = 0;
    for (size_t i = 0; i < warmup; ++i) ops.push_back({K::Forward, (int64_t)f++, -1});
    for (size_t i = 0; i < steady; ++i) {
      ops.push_back({K::Forward, (int64_t)f++, -1});
      ops.push_back({K::Backward, (int64_t)b++, -1});
    }
    for (size_t i = 0; i < warmup; ++i) ops.push_back({K::Backward, (int64_t)b++, -1});
  }
  return out;
}

std::vector<PipeOp> rank_program(ScheduleType t, size_t s, size_t S, size_t M) {
  if (s >= S) throw std::invalid_argument("stage out of range");
  const auto ops = build_schedule(t, S, M)[s];
  std::vector<PipeOp> prog;
  const int64_t prev = (int64_t)s - 1, next = s + 1 < S ? (int64_t)s + 1 : -1;
  for (const auto& op : ops) {
    if (op.kind == K::Forward) {
      if (prev >= 0) prog.push_back({K::RecvAct, op.microbatch, prev});
      prog.push_back(op);
      if (next >= 0) prog.push_back({K::SendAct, op.microbatch, next});
    } else {
      if (next >= 0) prog.push_back({K::RecvGrad, op.microbatch, next});
      prog.push_back(op);
      if (prev >= 0) prog.push_back({K::SendGrad, op.microbatch, prev});
    }
  }
  return prog;
}

double ideal_bubble_fraction(size_t S, size_t M) {
  if (S == 0 || M == 0) return 0.0;
  return double(S - 1) / double(M + S - 1);
}

TimelineResult simulate_schedule(ScheduleType t, size_t S, size_t M, double tf, double tb, double tc) {
  TimelineResult r;
  if (S == 0 || M == 0) return r;
  const auto sched = build_schedule(t, S, M);
  // ready times of activations arriving at stage s for microbatch m, grads likewise
  std::vector<std::vector<double>> act_ready(S, std::vector<double>(M, -1.0));
  std::vector<std::vector<double>> grad_ready(S, std::vector<double>(M, -1.0));
  for (size_t m = 0; m < M; ++m) act_ready[0][m] = 0.0;
  for (size_t m = 0; m < M; ++m) grad_ready[S - 1][m] = -2.0;  // set when the forward finishes
  std::vector<size_t> idx(S, 0);
  std::vector<double> clock(S, 0.0);
  r.stage_busy.assign(S, 0.0);
  r.stage_peak_inflight.assign(S, 0);
  std::vector<size_t> inflight(S, 0);
  size_t remaining = 0;
  for (auto& v : sched) remaining += v.size();
  while (remaining > 0) {
    bool progressed = false;
    for (size_t s = 0; s < S; ++s) {
      if (idx[s] >= sched[s].size()) continue;
      const PipeOp& op = sched[s][idx[s]];
      const size_t m = (size_t)op.microbatch;
      double ready;
      if (op.kind == K::Forward) {
        ready = act_ready[s][m];
      } else {
        ready = grad_ready[s][m];
      }
      if (ready < 0) continue;  // dependency not produced yet
      const double start = std::max(clock[s], ready);
      const double dur = op.kind == K::Forward ? tf : tb;
      const double end = start + dur;
      clock[s] = end;
      r.stage_busy[s] += dur;
      if (op.kind == K::Forward) {
        inflight[s]++;
        r.stage_peak_inflight[s] = std::max(r.stage_peak_inflight[s], inflight[s]);
        if (s + 1 < S) act_ready[s + 1][m] = end + tc;
        else grad_ready[s][m] = end;  // loss gradient available at the last stage
      } else {
        inflight[s]--;
        if (s > 0) grad_ready[s - 1][m] = end + tc;
      }
      idx[s]++;
      remaining--;
      progressed = true;
    }
    if (!progressed) throw std::runtime_error("schedule deadlocks");
  }
  r.makespan = *std::max_element(clock.begin(), clock.end());
  double busy = 0;
  for (double b : r.stage_busy) busy += b;
  r.bubble_fraction = 1.0 - busy / (r.makespan * S);
  r.peak_inflight = *std::max_element(r.stage_peak_inflight.begin(), r.stage_peak_inflight.end());
  return r;
}

static void put_u64(std::string& b, uint64_t v) {
  for (int i = 0; i < 8; ++i) b.push_back(static_cast<char>((v >> (8 * i)) & 0xFF));
}
static uint64_t get_u64(const std::string& b, size_t off) {
  if (off + 8 > b.size()) throw std::invalid_argument("truncated frame");
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | static_cast<uint8_t>(b[off + i]);
  return v;
}

std::string stage_data_to_bytes(const std::vector<float>& v, uint64_t rows, uint64_t cols) {
  if (v.size() != rows * cols) throw std::invalid_argument("data length mismatch");
  std::string b;
  b.reserve(16 + v.size() * 4);
  put_u64(b, rows);
  put_u64(b, cols);
  const size_t off = b.size();
  b.resize(off + v.size() * 4);
  std::memcpy(&b[off], v.data(), v.size() * 4);  // little-endian host
  return b;
}

void stage_data_from_bytes(const std::string& b, std::vector<float>& v, uint64_t& rows, uint64_t& cols) {
  rows = get_u64(b, 0);
  cols = get_u64(b, 8);
  const size_t n = rows * cols;
  if (b.size() < 16 + n * 4) throw std::invalid_argument("truncated StageData");
  v.resize(n);
  std::memcpy(v.data(), b.data() + 16, n * 4);
}

std::string compress_stage_data(const std::vector<float>& v, uint64_t rows, uint64_t cols, Fp8Format fmt) {
  const Fp8Tensor t = to_fp8(v, fmt);
  std::string b;
  b.reserve(29 + t.data.size());
  put_u64(b, rows);
  put_u64(b, cols);
  b.push_back(static_cast<char>(fmt == Fp8Format::E5M2 ? 1 : 0));
  char sc[4];
  std::memcpy(sc, &t.scale, 4);
  b.append(sc, 4);
  put_u64(b, t.data.size());
  b.append(reinterpret_cast<const char*>(t.data.data()), t.data.size());
  return b;
}

void decompress_stage_data(const std::string& b, std::vector<float>& v, uint64_t& rows, uint64_t& cols) {
  if (b.size() < 29) throw std::invalid_argument("truncated FP8 frame");
  rows = get_u64(b, 0);
  cols = get_u64(b, 8);
  const Fp8Format fmt = static_cast<uint8_t>(b[16]) == 1 ? Fp8Format::E5M2 : Fp8Format::E4M3;
  float scale;
  std::memcpy(&scale, b.data() + 17, 4);
  const uint64_t len = get_u64(b, 21);
  if (b.size() < 29 + len) throw std::invalid_argument("truncated FP8 payload");
  Fp8Tensor t(std::vector<uint8_t>(b.begin() + 29, b.begin() + 29 + len), fmt, scale);
  v = from_fp8(t);
}

}  // namespace mtorus
