// Host-side IEEE binary16 / bfloat16 conversion (round to nearest, ties to
// even), used wherever host floats become fp16/bf16 device storage. The
// reference converts logical host floats to fp16/bf16 when it creates Metal
// buffers (MetalRuntime.mm:42-104, 537-556); this is an independent
// implementation of the same IEEE rounding.
#pragma once

#include <cstdint>
#include <cstring>

namespace tensor::cuda {

inline std::uint16_t floatToHalfBits(float value) {
  std::uint32_t f;
  std::memcpy(&f, &value, 4);
  const std::uint32_t sign = (f >> 16) & 0x8000u;
  const std::uint32_t absf = f & 0x7fffffffu;
  if (absf >= 0x7f800000u) {  // inf or NaN
    return static_cast<std::uint16_t>(sign | 0x7c00u | (absf > 0x7f800000u ? 0x0200u : 0u));
  }
  if (absf >= 0x477ff000u) {  // rounds to >= 65520 -> inf
    return static_cast<std::uint16_t>(sign | 0x7c00u);
  }
  const int exp = static_cast<int>(absf >> 23);  // biased fp32 exponent
  if (exp < 113) {
    // Result is subnormal (or zero) in fp16: value = m * 2^-24.
    if (exp < 102) return static_cast<std::uint16_t>(sign);  // < 2^-25: rounds to 0
    const std::uint32_t mant = (absf & 0x7fffffu) | 0x800000u;
    const int shift = 126 - exp;  // 14..24
    std::uint32_t half = mant >> shift;
    const std::uint32_t rem = mant & ((1u << shift) - 1u);
    const std::uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) ++half;
    return static_cast<std::uint16_t>(sign | half);
  }
  // Normal fp16: rebias exponent, round 13 dropped mantissa bits.
  std::uint32_t half = ((static_cast<std::uint32_t>(exp - 112)) << 10) | ((absf >> 13) & 0x3ffu);
  const std::uint32_t rem = absf & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) ++half;  // carry may bump exponent
  return static_cast<std::uint16_t>(sign | half);
}

inline float halfBitsToFloat(std::uint16_t h) {
  const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
  const std::uint32_t exp = (h >> 10) & 0x1fu;
  const std::uint32_t mant = h & 0x3ffu;
  std::uint32_t f;
  if (exp == 0) {
    if (mant == 0) {
      f = sign;
    } else {
      // subnormal: value = mant * 2^-24
      float v = static_cast<float>(mant) * (1.0f / 16777216.0f);
      std::memcpy(&f, &v, 4);
      f |= sign;
    }
  } else if (exp == 31) {
    f = sign | 0x7f800000u | (mant << 13);
  } else {
    f = sign | ((exp + 112) << 23) | (mant << 13);
  }
  float out;
  std::memcpy(&out, &f, 4);
  return out;
}

inline std::uint16_t floatToBFloat16Bits(float value) {
  std::uint32_t f;
  std::memcpy(&f, &value, 4);
  if ((f & 0x7fffffffu) > 0x7f800000u) return static_cast<std::uint16_t>((f >> 16) | 0x40u);
  const std::uint32_t lsb = (f >> 16) & 1u;
  f += 0x7fffu + lsb;
  return static_cast<std::uint16_t>(f >> 16);
}

inline float bfloat16BitsToFloat(std::uint16_t b) {
  const std::uint32_t f = static_cast<std::uint32_t>(b) << 16;
  float out;
  std::memcpy(&out, &f, 4);
  return out;
}

}  // namespace tensor::cuda
