// TEST INFRASTRUCTURE (oracle side) — never linked into the product library.
//
// Seeded synthetic-weight generator and 4-bit affine g64 quantizer, restated on
// the CPU so the oracle can rebuild the exact bytes the CUDA generator writes.
// Every step uses only integer arithmetic and single IEEE-rounded float
// operations (int->float conversion, one multiply, one subtract, one divide,
// rint, round-to-nearest-even bf16 narrowing), so the CPU and GPU produce
// bit-identical packed nibbles, scales and biases.
//
// Layout produced (the reference's canonical packing, native/projection_reference.h:16
// and src/serving/qwen_tests.rs:81-82): element (row, col) of a 4-bit matrix is
// nibble col%8 of uint32 word col/8 of the row (LSB first); one bf16 scale and
// bias per 64 consecutive columns; dequantized value = scale*q + bias with scale
// and bias widened to float (native/projection_reference.h:8-22).
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>

namespace synth {

inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// FNV-1a over the tensor's reference name.
inline uint64_t tensor_id(const std::string& name) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (unsigned char c : name) { h ^= c; h *= 0x100000001b3ull; }
  return h;
}

inline uint64_t tensor_key(uint64_t seed, uint64_t tid) {
  return mix64(seed * 0x632BE59BD9B4E019ull ^ mix64(tid));
}

// Irwin-Hall(4) approximation of N(0, 1) scaled by `stddev`:
// s = sum of four 16-bit uniforms, w = float(s - 131070) * (stddev / 37837.2265).
inline float normal(uint64_t key, uint64_t index, float stddev) {
  uint64_t h = mix64(key ^ (index * 0xD1B54A32D192ED03ull));
  int32_t s = int32_t(h & 0xFFFF) + int32_t((h >> 16) & 0xFFFF) + int32_t((h >> 32) & 0xFFFF) +
              int32_t(h >> 48);
  const float k = stddev / 37837.2265f;
  return float(s - 131070) * k;
}

inline uint16_t bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return uint16_t((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
inline float bf16_to_float(uint16_t b) {
  uint32_t u = uint32_t(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// Quantize one group of 64 values: scale = (max-min)/15, bias = min, both
// narrowed to bf16; q = clamp(rint((w - bias) / scale), 0, 15).
inline void quantize_group(const float* w, uint8_t* q, uint16_t* scale_bits, uint16_t* bias_bits) {
  float lo = w[0], hi = w[0];
  for (int i = 1; i < 64; ++i) { lo = w[i] < lo ? w[i] : lo; hi = w[i] > hi ? w[i] : hi; }
  float scale = (hi - lo) / 15.0f;
  *scale_bits = bf16_rne(scale);
  *bias_bits = bf16_rne(lo);
  const float s = bf16_to_float(*scale_bits), b = bf16_to_float(*bias_bits);
  for (int i = 0; i < 64; ++i) {
    float v = s > 0.0f ? rintf((w[i] - b) / s) : 0.0f;
    v = v < 0.0f ? 0.0f : (v > 15.0f ? 15.0f : v);
    q[i] = uint8_t(v);
  }
}

}  // namespace synth
