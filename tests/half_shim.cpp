// Test-only C wrapper over the host fp16 / bf16 conversions
// (aicompiler-test_b200/csrc/half_convert.hpp), compiled with g++ by
// tests/test_half_convert.py.
#include <cstddef>
#include <cstdint>

#include "half_convert.hpp"

extern "C" {
void to_half(const float *in, std::uint16_t *out, std::size_t n) {
  for (std::size_t i = 0; i < n; ++i) out[i] = tensor::cuda::floatToHalfBits(in[i]);
}
void from_half(const std::uint16_t *in, float *out, std::size_t n) {
  for (std::size_t i = 0; i < n; ++i) out[i] = tensor::cuda::halfBitsToFloat(in[i]);
}
void to_bf16(const float *in, std::uint16_t *out, std::size_t n) {
  for (std::size_t i = 0; i < n; ++i) out[i] = tensor::cuda::floatToBFloat16Bits(in[i]);
}
void from_bf16(const std::uint16_t *in, float *out, std::size_t n) {
  for (std::size_t i = 0; i < n; ++i) out[i] = tensor::cuda::bfloat16BitsToFloat(in[i]);
}
}
