// bf16 <-> float8_e4m3fn conversions of FP8Codec (ashkv/codecs/fp8.py:32-79),
// shared by the tensor codec (fp8_codec.cu) and the page transcoder (migrate.cu).
#pragma once

#include "common.cuh"

namespace ashkv {
namespace {

constexpr uint32_t kBf16Fp8Limit = 0x43E8u;  // bf16 bits of 464.0

// Two bf16 (one 32-bit word, element 0 in the low half) -> two e4m3fn bytes
// (element 0 in the low byte).
__device__ __forceinline__ uint32_t fp8x2_from_bf16x2(uint32_t w) {
  uint16_t d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(bf16hi(w)), "f"(bf16lo(w)));
  uint32_t r = d;
  const uint32_t mag = w & 0x7FFF7FFFu;
  const uint32_t over = __vcmpgtu2(mag, kBf16Fp8Limit * 0x10001u);  // 0xFFFF per element above 464 / inf / NaN
  if (over) {
    const uint32_t nan2 = 0x7F7Fu | ((w >> 8) & 0x80u) | ((w >> 16) & 0x8000u);
    const uint32_t m = (over & 0xFFu) | ((over >> 16) & 0xFF00u);
    r = (r & ~m) | (nan2 & m);
  }
  return r;
}

// Two e4m3fn bytes (low byte = element 0) -> two bf16 (element 0 low).
__device__ __forceinline__ uint32_t bf16x2_from_fp8x2(uint32_t c16) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(static_cast<uint16_t>(c16)));
  float lo, hi;
  asm("{.reg .b16 l, u;\n\tmov.b32 {l, u}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, u;}"
      : "=f"(lo), "=f"(hi) : "r"(h));
  return f32x2_to_bf16x2(lo, hi);
}

}  // namespace
}  // namespace ashkv
