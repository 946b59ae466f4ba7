// Prefetching synthetic token source: the native counterpart of the reference's
// SyntheticDataLoader (examples/gpt-1b/src/synthetic_data.rs: an iterator of
// uniform-random [B, S] token batches with num_batches / current_batch / reset).
//
// Batch i is a pure function of (seed, i): token j of the batch's B * n stream
// (n = S, or S + 1 for next-token targets) is
//     mix(key(seed) ^ mix(i * B * n + j))  mapped onto [0, vocab) by a 64x64 -> 128-bit
// multiply-high, where mix is the SplitMix64 finaliser (S. Vigna, "splitmix64.c",
// 2015; constants from that published method).  So any batch can be regenerated
// (seek() after a checkpoint restore) and the Python reference can recompute it.
// `workers` threads fill a ring of `depth` slots ahead of the consumer; next_into()
// waits (bounded) for the next batch and copies it into caller-owned host memory
// (pinned buffers for an asynchronous host-to-device copy).
#pragma once

#include <condition_variable>
#include <cstdint>
#include <mutex>
#include <thread>
#include <vector>

namespace mtorus {

uint64_t splitmix64_mix(uint64_t z);
// Token j of batch i (the stream before the input / target split).
int64_t synthetic_token(uint64_t seed, uint64_t i, uint64_t j, uint64_t per_batch, uint64_t vocab);

class TokenLoader {
 public:
  TokenLoader(int64_t batch, int64_t seq_len, int64_t vocab, int64_t num_batches, uint64_t seed, bool shift,
              int depth = 4, int workers = 1);
  ~TokenLoader();
  TokenLoader(const TokenLoader&) = delete;
  TokenLoader& operator=(const TokenLoader&) = delete;

  // Copies the next batch into inp / tgt (int64 [B, S] each, row-major) and returns
  // true; false once num_batches batches were handed out.  Throws std::runtime_error
  // if no batch becomes ready within timeout_s.
  bool next_into(int64_t* inp, int64_t* tgt, double timeout_s = 60.0);
  // Restart at batch `index` (reset() == seek(0)); drops prefetched batches.
  void seek(int64_t index);
  void reset() { seek(0); }
  int64_t num_batches() const { return num_batches_; }
  int64_t current_batch() const;
  int64_t batch() const { return batch_; }
  int64_t seq_len() const { return seq_; }

 private:
  struct Slot {
    int64_t index = -1;  // batch held (-1: none); -2: being filled
    std::vector<int64_t> tokens;
  };
  void worker_loop();
  void fill(Slot& s, int64_t index) const;

  const int64_t batch_, seq_, vocab_, num_batches_, per_batch_;
  const uint64_t seed_;
  const bool shift_;
  std::vector<Slot> slots_;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  int64_t next_fill_ = 0;     // next batch index a worker should produce
  int64_t next_out_ = 0;      // next batch index the consumer takes
  uint64_t generation_ = 0;   // bumped by seek(): fills of an older generation are dropped
  bool stop_ = false;
  std::vector<std::thread> workers_;
};

}  // namespace mtorus
