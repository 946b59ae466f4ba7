#include "core/precision.h"

#include <cmath>
#include <stdexcept>

namespace mtorus {

float fp8_format_max(Fp8Format f) { return f == Fp8Format::E4M3 ? 416.f : 49152.f; }
float fp8_max_finite(Fp8Format f) { return f == Fp8Format::E4M3 ? 448.f : 57344.f; }

// Generic minifloat encoder: `mbits` mantissa bits, exponent bias `bias`,
// smallest normal exponent emin, largest finite code `max_code`.
static uint8_t encode_minifloat(float x, int mbits, int bias, uint8_t max_code, uint8_t nan_code) {
  const uint8_t sign = std::signbit(x) ? 0x80 : 0x00;
  if (std::isnan(x)) return sign | nan_code;
  const float a = std::fabs(x);
  const int emin = 1 - bias;
  const float mscale = static_cast<float>(1 << mbits);
  uint32_t code;
  if (a < std::ldexp(1.f, emin)) {
    // subnormal: a = q * 2^(emin - mbits); q == 2^mbits rolls into the first normal
    const float q = std::nearbyint(std::ldexp(a, mbits - emin));
    code = static_cast<uint32_t>(q);
  } else {
    int k;
    const float fr = std::frexp(a, &k);  // a = fr * 2^k, fr in [0.5, 1)
    int e = k - 1;
    float q = std::nearbyint((fr * 2.f - 1.f) * mscale);
    if (q >= mscale) {
      q = 0.f;
      ++e;
    }
    const long field = static_cast<long>(e + bias);
    if (field > 0xFF) return sign | max_code;
    code = static_cast<uint32_t>(field << mbits) | static_cast<uint32_t>(q);
  }
  if (code > max_code || std::isinf(a)) return sign | max_code;  // saturate to finite
  return sign | static_cast<uint8_t>(code);
}

uint8_t fp8_encode(float x, Fp8Format f) {
  if (f == Fp8Format::E4M3) return encode_minifloat(x, 3, 7, 0x7E, 0x7F);
  return encode_minifloat(x, 2, 15, 0x7B, 0x7F);
}

float fp8_decode(uint8_t b, Fp8Format f) {
  const float sign = (b & 0x80) ? -1.f : 1.f;
  if (f == Fp8Format::E4M3) {
    const int e = (b >> 3) & 0xF, m = b & 0x7;
    if (e == 15 && m == 7) return std::nanf("");
    if (e == 0) return sign * std::ldexp(static_cast<float>(m), -9);
    return sign * std::ldexp(1.f + m / 8.f, e - 7);
  }
  const int e = (b >> 2) & 0x1F, m = b & 0x3;
  if (e == 31) return m == 0 ? sign * INFINITY : std::nanf("");
  if (e == 0) return sign * std::ldexp(static_cast<float>(m), -16);
  return sign * std::ldexp(1.f + m / 4.f, e - 15);
}

float Fp8Tensor::amax() const {
  if (!amax_history.empty()) return amax_history.back();
  if (scale > 0.f) return fp8_format_max(format) / scale;
  return 0.f;
}

float abs_max(const float* v, size_t n) {
  float m = 0.f;
  for (size_t i = 0; i < n; ++i) m = std::fmax(m, std::fabs(v[i]));
  return m;
}

static std::vector<uint8_t> quantize_bytes(const float* v, size_t n, Fp8Format f, float scale) {
  std::vector<uint8_t> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = fp8_encode(v[i] * scale, f);
  return out;
}

Fp8Tensor to_fp8(const std::vector<float>& v, Fp8Format f) {
  const float amax = abs_max(v.data(), v.size());
  const float scale = amax == 0.f ? 1.f : fp8_format_max(f) / amax;
  Fp8Tensor t(quantize_bytes(v.data(), v.size(), f, scale), f, scale);
  t.amax_history = {amax};
  return t;
}

Fp8Tensor to_fp8_with_scale(const std::vector<float>& v, Fp8Format f, float scale) {
  Fp8Tensor t(quantize_bytes(v.data(), v.size(), f, scale), f, scale);
  t.amax_history = {abs_max(v.data(), v.size())};
  return t;
}

Fp8Tensor to_fp8_per_block(const std::vector<float>& v, Fp8Format f, size_t block_size) {
  if (block_size == 0) throw std::invalid_argument("block_size must be > 0");
  const size_t nb = (v.size() + block_size - 1) / block_size;
  std::vector<uint8_t> data;
  data.reserve(v.size());
  std::vector<float> scales;
  scales.reserve(nb);
  for (size_t b = 0; b < nb; ++b) {
    const size_t s = b * block_size, e = std::min(v.size(), s + block_size);
    const float amax = abs_max(v.data() + s, e - s);
    const float sc = amax == 0.f ? 1.f : fp8_format_max(f) / amax;
    scales.push_back(sc);
    for (size_t i = s; i < e; ++i) data.push_back(fp8_encode(v[i] * sc, f));
  }
  Fp8Tensor t(std::move(data), f, scales.empty() ? 1.f : scales[0]);
  t.block_scales = std::move(scales);
  t.block_size = block_size;
  t.amax_history = {abs_max(v.data(), v.size())};
  return t;
}

std::vector<float> from_fp8(const Fp8Tensor& t) {
  std::vector<float> out(t.data.size());
  if (t.block_scales) {
    const auto& bs = *t.block_scales;
    size_t block = t.block_size ? *t.block_size
                                : (bs.empty() ? t.data.size()
                                              : (t.data.size() + bs.size() - 1) / bs.size());
    if (block == 0) block = 1;
    for (size_t i = 0; i < t.data.size(); ++i) {
      const size_t b = i / block;
      const float sc = b < bs.size() ? bs[b] : 1.f;
      out[i] = fp8_decode(t.data[i], t.format) / sc;
    }
  } else {
    for (size_t i = 0; i < t.data.size(); ++i) out[i] = fp8_decode(t.data[i], t.format) / t.scale;
  }
  return out;
}

DelayedScaling::DelayedScaling(size_t h) : hist_(h, 0.f) {
  if (h == 0) throw std::invalid_argument("history_length must be > 0");
}

void DelayedScaling::update(float amax) {
  hist_[cursor_] = amax;
  cursor_ = (cursor_ + 1) % hist_.size();
}

float DelayedScaling::current_amax() const {
  float m = 0.f;
  for (float a : hist_) m = std::fmax(m, a);
  return m;
}

float DelayedScaling::compute_scale(Fp8Format f) const {
  const float a = current_amax();
  return a == 0.f ? 1.f : fp8_format_max(f) / a;
}

void DelayedScaling::set_state(std::vector<float> hist, size_t cursor) {
  if (hist.empty()) throw std::invalid_argument("history must be non-empty");
  if (cursor >= hist.size()) throw std::invalid_argument("cursor out of range");
  hist_ = std::move(hist);
  cursor_ = cursor;
}

LossScaler LossScaler::new_dynamic(float s, size_t gi) {
  return LossScaler{s, LossScaleMode::Dynamic, gi, 0};
}
LossScaler LossScaler::new_static(float s) { return LossScaler{s, LossScaleMode::Static, 0, 0}; }

void LossScaler::update(bool overflow) {
  if (mode == LossScaleMode::Static) return;
  if (overflow) {
    scale /= 2.f;
    if (scale < 1.f) scale = 1.f;
    growth_counter = 0;
  } else {
    ++growth_counter;
    if (growth_counter >= growth_interval) {
      scale *= 2.f;
      growth_counter = 0;
    }
  }
}

}  // namespace mtorus
