#include "core/data_loader.h"

#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>

namespace mtorus {

uint64_t splitmix64_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

int64_t synthetic_token(uint64_t seed, uint64_t i, uint64_t j, uint64_t per_batch, uint64_t vocab) {
  const uint64_t key = splitmix64_mix(seed + 0x9E3779B97F4A7C15ull);
  const uint64_t r = splitmix64_mix(key ^ splitmix64_mix(i * per_batch + j));
  return (int64_t)(((unsigned __int128)r * vocab) >> 64);
}

TokenLoader::TokenLoader(int64_t batch, int64_t seq_len, int64_t vocab, int64_t num_batches, uint64_t seed,
                         bool shift, int depth, int workers)
    : batch_(batch),
      seq_(seq_len),
      vocab_(vocab),
      num_batches_(num_batches),
      per_batch_(batch * (seq_len + (shift ? 1 : 0))),
      seed_(seed),
      shift_(shift) {
  if (batch <= 0 || seq_len <= 0 || vocab <= 0 || num_batches < 0 || depth <= 0 || workers <= 0)
    throw std::invalid_argument("TokenLoader: positive batch, seq_len, vocab, depth, workers and num_batches >= 0");
  slots_.resize((size_t)depth);
  for (int w = 0; w < workers; ++w) workers_.emplace_back([this] { worker_loop(); });
}

TokenLoader::~TokenLoader() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& t : workers_) t.join();
}

void TokenLoader::fill(Slot& s, int64_t index) const {
  s.tokens.resize((size_t)per_batch_);
  for (int64_t j = 0; j < per_batch_; ++j)
    s.tokens[(size_t)j] = synthetic_token(seed_, (uint64_t)index, (uint64_t)j, (uint64_t)per_batch_, (uint64_t)vocab_);
}

void TokenLoader::worker_loop() {
  std::unique_lock<std::mutex> lk(mu_);
  while (true) {
    // a free slot and a batch left to produce, within `depth` of the consumer
    Slot* free_slot = nullptr;
    const int64_t depth = (int64_t)slots_.size();
    if (!stop_ && next_fill_ < num_batches_ && next_fill_ < next_out_ + depth) {
      for (auto& s : slots_)
        if (s.index == -1) {
          free_slot = &s;
          break;
        }
    }
    if (stop_) return;
    if (!free_slot) {
      cv_.wait(lk);
      continue;
    }
    const int64_t index = next_fill_++;
    const uint64_t gen = generation_;
    free_slot->index = -2;
    Slot local;
    local.tokens.swap(free_slot->tokens);
    lk.unlock();
    fill(local, index);
    lk.lock();
    free_slot->tokens.swap(local.tokens);
    free_slot->index = (gen == generation_) ? index : -1;
    cv_.notify_all();
  }
}

bool TokenLoader::next_into(int64_t* inp, int64_t* tgt, double timeout_s) {
  std::unique_lock<std::mutex> lk(mu_);
  if (next_out_ >= num_batches_) return false;
  const int64_t want = next_out_;
  Slot* ready = nullptr;
  const auto deadline =
      std::chrono::steady_clock::now() + std::chrono::microseconds((int64_t)(timeout_s * 1e6));
  while (true) {
    for (auto& s : slots_)
      if (s.index == want) ready = &s;
    if (ready) break;
    if (cv_.wait_until(lk, deadline) == std::cv_status::timeout) {
      for (auto& s : slots_)
        if (s.index == want) ready = &s;
      if (ready) break;
      throw std::runtime_error("TokenLoader: batch " + std::to_string(want) + " not ready within the timeout");
    }
  }
  const int64_t n = seq_ + (shift_ ? 1 : 0);
  const int64_t* t = ready->tokens.data();
  for (int64_t b = 0; b < batch_; ++b) {
    std::memcpy(inp + b * seq_, t + b * n, (size_t)seq_ * sizeof(int64_t));
    std::memcpy(tgt + b * seq_, t + b * n + (shift_ ? 1 : 0), (size_t)seq_ * sizeof(int64_t));
  }
  ready->index = -1;
  ++next_out_;
  cv_.notify_all();
  return true;
}

void TokenLoader::seek(int64_t index) {
  std::lock_guard<std::mutex> lk(mu_);
  if (index < 0 || index > num_batches_) throw std::out_of_range("TokenLoader::seek: index out of range");
  ++generation_;
  for (auto& s : slots_)
    if (s.index >= 0) s.index = -1;  // slots being filled (-2) are dropped when their fill lands
  next_fill_ = next_out_ = index;
  cv_.notify_all();
}

int64_t TokenLoader::current_batch() const {
  std::lock_guard<std::mutex> lk(mu_);
  return next_out_;
}

}  // namespace mtorus
