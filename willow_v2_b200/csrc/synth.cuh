// Device side of the seeded synthetic-weight generator; bit-identical to willow_v2_b200/synth.py.
// splitmix64 (Steele, Lea, Flood 2014; public domain) over a key derived from (seed, layer, expert, tensor):
// word k of super-block b is finalize(key + (32 b + k + 1) * gamma). fp16 scales are
// fp16_rne(1e-3 + (word >> 40) * (3e-3 / 2^24)) with one correctly rounded float64 multiply and add.
#pragma once

#include <stdint.h>

namespace wmoe {
namespace synth {

constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
constexpr int kWordsPerBlock = 32;
constexpr int kTensorGateUp = 0;
constexpr int kTensorDown = 1;

__host__ __device__ __forceinline__ uint64_t finalize(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t mix(uint64_t z) { return finalize(z + kGamma); }

__host__ __device__ __forceinline__ uint64_t tensor_key(uint64_t seed, uint64_t layer, uint64_t expert,
                                                        uint64_t tensor) {
  uint64_t k = mix(seed);
  k = mix(k + layer);
  return mix(k + 2 * expert + tensor);
}

__host__ __device__ __forceinline__ uint64_t word(uint64_t key, uint64_t block, uint64_t k) {
  return finalize(key + (block * kWordsPerBlock + k + 1) * kGamma);
}

// float64 -> fp16 bits, round to nearest even, for positive values in fp16's normal range (the generator's
// scales lie in [1e-3, 4e-3]).
__host__ __device__ __forceinline__ uint16_t f64_to_f16_rne_normal(double v) {
#ifdef __CUDA_ARCH__
  const uint64_t b = static_cast<uint64_t>(__double_as_longlong(v));
#else
  uint64_t b;
  __builtin_memcpy(&b, &v, 8);
#endif
  const int e = static_cast<int>((b >> 52) & 0x7FF) - 1023;
  const uint64_t m = b & ((1ull << 52) - 1);
  uint32_t h = (static_cast<uint32_t>(e + 15) << 10) | static_cast<uint32_t>(m >> 42);
  const uint64_t rem = m & ((1ull << 42) - 1), half = 1ull << 41;
  if (rem > half || (rem == half && (h & 1u))) h += 1;  // a carry into the exponent is the correct result
  return static_cast<uint16_t>(h);
}

__host__ __device__ __forceinline__ uint16_t scale_f16(uint64_t w) {
  const double step = 3e-3 / 16777216.0;
#ifdef __CUDA_ARCH__
  const double v = __dadd_rn(__dmul_rn(static_cast<double>(w >> 40), step), 1e-3);
#else
  volatile double prod = static_cast<double>(w >> 40) * step;  // no contraction into a fused multiply-add
  const double v = prod + 1e-3;
#endif
  return f64_to_f16_rne_normal(v);
}

}  // namespace synth
}  // namespace wmoe
