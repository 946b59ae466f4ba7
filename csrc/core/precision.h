// FP8 precision primitives: formats, a bit-exact software FP8 codec, the host
// Fp8Tensor container, per-tensor / per-block quantisation, delayed amax
// scaling and the loss scaler.
//
// Semantics follow crates/mt-core/src/precision/{config,fp8_tensor,quantize,
// scaling,loss_scale}.rs.  Scale = format_max / amax (1 when amax == 0),
// stored = fp8(x * scale), dequantised = fp8 / scale.  format_max is the
// reference's constant (416 for E4M3, 49152 for E5M2: the MAX of the Rust
// `float8` crate, one code below the OCP maxima); the codec itself is OCP
// E4M3FN / E5M2 with round-to-nearest-even and saturation to the largest
// finite value, the same rounding the device's cvt.rn.satfinite uses.
#pragma once

#include <cstdint>
#include <optional>
#include <vector>

namespace mtorus {

enum class Fp8Format : int { E4M3 = 0, E5M2 = 1 };
enum class MasterFormat : int { Fp32 = 0, Bf16 = 1 };

float fp8_format_max(Fp8Format f);     // reference constant: 416 / 49152
float fp8_max_finite(Fp8Format f);     // OCP: 448 / 57344
uint8_t fp8_encode(float x, Fp8Format f);
float fp8_decode(uint8_t b, Fp8Format f);

struct Fp8Tensor {
  std::vector<uint8_t> data;
  Fp8Format format = Fp8Format::E4M3;
  float scale = 1.f;
  std::optional<std::vector<float>> block_scales;
  // Explicit block size of block-scaled tensors (the reference infers it as
  // ceil(len / num_blocks), which is wrong for ragged tails; we keep it).
  std::optional<size_t> block_size;
  std::vector<float> amax_history;

  Fp8Tensor() = default;
  Fp8Tensor(std::vector<uint8_t> d, Fp8Format f, float s) : data(std::move(d)), format(f), scale(s) {}
  size_t len() const { return data.size(); }
  bool is_empty() const { return data.empty(); }
  // last history entry; else format_max / scale when scale > 0; else 0
  float amax() const;
  bool operator==(const Fp8Tensor& o) const {
    return data == o.data && format == o.format && scale == o.scale &&
           block_scales == o.block_scales && amax_history == o.amax_history;
  }
};

float abs_max(const float* v, size_t n);
Fp8Tensor to_fp8(const std::vector<float>& v, Fp8Format f);
Fp8Tensor to_fp8_with_scale(const std::vector<float>& v, Fp8Format f, float scale);
Fp8Tensor to_fp8_per_block(const std::vector<float>& v, Fp8Format f, size_t block_size);
std::vector<float> from_fp8(const Fp8Tensor& t);

class DelayedScaling {
 public:
  explicit DelayedScaling(size_t history_length);
  void update(float amax);
  float current_amax() const;  // max over the whole ring (unwritten slots are 0)
  float compute_scale(Fp8Format f) const;
  const std::vector<float>& amax_history() const { return hist_; }
  size_t history_length() const { return hist_.size(); }
  size_t cursor() const { return cursor_; }
  void set_state(std::vector<float> hist, size_t cursor);
  bool operator==(const DelayedScaling& o) const { return hist_ == o.hist_ && cursor_ == o.cursor_; }

 private:
  std::vector<float> hist_;
  size_t cursor_ = 0;
};

enum class LossScaleMode : int { Dynamic = 0, Static = 1 };

struct LossScaler {
  float scale = 1.f;
  LossScaleMode mode = LossScaleMode::Static;
  size_t growth_interval = 0;
  size_t growth_counter = 0;

  static LossScaler new_dynamic(float initial_scale, size_t growth_interval);
  static LossScaler new_static(float scale);
  void update(bool overflow);
  void reset(float initial_scale) {
    scale = initial_scale;
    growth_counter = 0;
  }
  bool operator==(const LossScaler& o) const {
    return scale == o.scale && mode == o.mode && growth_interval == o.growth_interval &&
           growth_counter == o.growth_counter;
  }
};

}  // namespace mtorus
