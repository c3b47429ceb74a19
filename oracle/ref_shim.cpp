// TEST INFRASTRUCTURE ONLY (oracle). Never linked into the product library.
//
// Compile shim for building the reference's own fp32 CPU decode path from its
// unmodified sources. The reference's CPU build breaks in
// src/csrc/models/minimind/ascend_matmul.cpp (uses `cpu_matvec` before any
// declaration at :627 and :690 in the non-Ascend branches). Instead of editing
// that file we leave it out of the build and provide the handful of symbols the
// CPU path links against, with the behaviour the non-Ascend build gives them:
//   cube_matvec_available()  -> false   (ascend_matmul.cpp:376-382)
//   cube_matmul_available()  -> false   (ascend_matmul.cpp:505-511)
// With both false, LanguageModel::forward_next_token takes the CPU
// fall-through (language_model.cpp:317-332) and never calls the cube_* math.
#include "ascend_matmul.h"

#include <cmath>
#include <cstring>
#include <stdexcept>

namespace minimind::model {

bool cube_matvec_available() { return false; }
bool cube_matmul_available() { return false; }

std::vector<float> cube_matvec(const std::vector<float>&, int64_t, int64_t, const std::vector<float>&) {
  throw std::runtime_error("cube_matvec is unavailable in the CPU oracle build");
}

std::vector<float> cube_matmul(const std::vector<float>&, int64_t, int64_t, const std::vector<float>&, int64_t) {
  throw std::runtime_error("cube_matmul is unavailable in the CPU oracle build");
}

int32_t cube_matvec_argmax(const std::vector<float>&, int64_t, int64_t, const std::vector<float>&) {
  throw std::runtime_error("cube_matvec_argmax is unavailable in the CPU oracle build");
}

// IEEE binary16 conversions (round to nearest even); only present so that the
// custom-op translation unit links. The CPU decode path does not call them.
uint16_t float_to_half(float value) {
  uint32_t bits = 0;
  std::memcpy(&bits, &value, sizeof(bits));
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int32_t exponent = static_cast<int32_t>((bits >> 23) & 0xFF) - 127 + 15;
  uint32_t mantissa = bits & 0x7FFFFFu;
  if (((bits >> 23) & 0xFF) == 0xFF) {
    return static_cast<uint16_t>(sign | 0x7C00u | (mantissa ? 0x200u : 0u));
  }
  if (exponent >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
  if (exponent <= 0) {
    if (exponent < -10) return static_cast<uint16_t>(sign);
    mantissa |= 0x800000u;
    const int shift = 14 - exponent;
    uint32_t half = mantissa >> shift;
    const uint32_t rem = mantissa & ((1u << shift) - 1u);
    const uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) ++half;
    return static_cast<uint16_t>(sign | half);
  }
  uint32_t half = sign | (static_cast<uint32_t>(exponent) << 10) | (mantissa >> 13);
  const uint32_t rem = mantissa & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) ++half;
  return static_cast<uint16_t>(half);
}

float half_to_float(uint16_t value) {
  const float sign = (value & 0x8000u) ? -1.0F : 1.0F;
  const int exponent = (value >> 10) & 0x1F;
  const int mantissa = value & 0x3FF;
  if (exponent == 0) return sign * std::ldexp(static_cast<float>(mantissa), -24);
  if (exponent == 31) return mantissa ? NAN : sign * INFINITY;
  return sign * std::ldexp(static_cast<float>(mantissa | 0x400), exponent - 25);
}

}  // namespace minimind::model
