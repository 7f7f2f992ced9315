// Per-group arithmetic of the INT4 codec (ashkv/codecs/int4.py:38-112),
// shared by the tensor codec (int4_codec.cu) and the page transcoder
// (migrate.cu): numpy's rounding and int8 cast, the bf16 scale as torch's CPU
// cast writes it, and the packing of eight values into eight nibbles.
#pragma once

#include "common.cuh"

namespace ashkv {
namespace {

constexpr uint16_t kCpuNanBf16 = 0xFFFFu;

// torch CPU fp32 -> bf16.
__device__ __forceinline__ uint32_t bf16_cpu(float f) {
  return f != f ? kCpuNanBf16 : f32_to_bf16(f);
}

// numpy: clip(int8(round_half_even(v)), -8, 7) + 8.
__device__ __forceinline__ uint32_t nibble_np(float v) {
  int32_t r;
  asm("cvt.rni.sat.s32.f32 %0, %1;" : "=r"(r) : "f"(v));  // NaN -> 0
  if (!(fabsf(v) < 2147483648.0f)) r = INT32_MIN;         // numpy's cvttss2si result
  int32_t q = static_cast<int8_t>(static_cast<uint8_t>(r));
  q = q < -8 ? -8 : (q > 7 ? 7 : q);
  return static_cast<uint32_t>(q + 8);
}

// Quotient RN(RN(7x) / am) for the fast path (am finite, am in [2^-100, 2^100]).
struct GroupDiv {
  float am;
  Recip y;
  int mode;  // 0: Markstein, 1: __fdiv_rn, 2: am not finite -> every code is 0
};
__device__ __forceinline__ GroupDiv group_div(float am) {
  GroupDiv d;
  d.am = am;
  d.y = make_recip(am);
  d.mode = !(fabsf(am) <= 3.4028235e38f) ? 2 : (recip_ok(am) ? 0 : 1);
  return d;
}
__device__ __forceinline__ uint32_t nibble_of(float x, const GroupDiv& d) {
  if (d.mode == 2) return 8u;
  const float p = __fmul_rn(x, 7.0f);
  const float v = d.mode == 0 ? div_rn(p, d.am, d.y) : __fdiv_rn(p, d.am);
  return nibble_np(v);
}

__device__ __forceinline__ float group_max_finish(float m) {
  return max_nan(m, 1e-8f);
}

__device__ __forceinline__ void unpack_chunk(uint4 v, float (&x)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) { x[2 * k] = bf16lo(w[k]); x[2 * k + 1] = bf16hi(w[k]); }
}

__device__ __forceinline__ float chunk_max(float m, const float (&x)[8]) {
  m = max3_abs_nan(m, x[0], x[1]);
  m = max3_abs_nan(m, x[2], x[3]);
  m = max3_abs_nan(m, x[4], x[5]);
  return max3_abs_nan(m, x[6], x[7]);
}

// Eight values of a group with divisor d -> eight nibbles (element 0 in the
// high nibble of the low byte).
__device__ __forceinline__ uint32_t pack_chunk(const float (&x)[8], const GroupDiv& d) {
  uint32_t out = 0;
  if (d.mode == 0) {
    // am finite and in Markstein's range: every x is finite and |x| <= am, so
    // v = RN(RN(7x)/am) lies in [-7, 7] and numpy's cast and clip are the
    // identity; RN(v + 1.5*2^23 + 8) leaves rint(v) + 8 (ties to even, 8 being
    // even) in the low 4 bits.  When am is a bf16 absmax (not the 1e-8 floor)
    // the quotient of the 11-bit product 7x by it needs no correction step.
    const f2 yhi = pk2(d.y.hi, d.y.hi), ylo = pk2(d.y.lo, d.y.lo), nb = pk2(-d.am, -d.am);
    const f2 seven = pk2(7.0f, 7.0f), magic = pk2(12582920.0f, 12582920.0f);
    const bool shortq = short_significand(d.am);
    uint32_t t[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const f2 p = mul2(pk2(x[2 * k], x[2 * k + 1]), seven);
      float v0, v1;
      upk2(add2(shortq ? div2_short(p, yhi, ylo) : div2_rn(p, yhi, ylo, nb), magic), v0, v1);
      t[2 * k] = __float_as_uint(v0);
      t[2 * k + 1] = __float_as_uint(v1);
    }
    // bytes m0..m3 and m4..m7 (each t's low byte is its nibble value, < 16)
    const uint32_t X = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
    const uint32_t Y = __byte_perm(__byte_perm(t[4], t[5], 0x0040), __byte_perm(t[6], t[7], 0x0040), 0x5410);
    // byte j of X*16 + (X >> 8) is (m_j << 4) + m_{j+1}: keep bytes 0 and 2 of each
    out = __byte_perm(X * 16u + (X >> 8), Y * 16u + (Y >> 8), 0x6420);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      out |= ((nibble_of(x[2 * k], d) << 4) | nibble_of(x[2 * k + 1], d)) << (8 * k);
  }
  return out;
}

// Eight nibbles (element 0 in the high nibble of the low byte) with scale s ->
// eight bf16 values out = bf16(RN(RN(float(q - 8) * s) / 7)) (torch CPU NaN
// encoding), packed two per word.
__device__ __forceinline__ void unpack_nibbles8(uint32_t code, float s, uint32_t (&o)[4]) {
  const bool fast = s >= 0x1p-90f && s <= 0x1p+90f;
  if (fast) {
    const Recip y7 = make_recip(7.0f);
    const f2 yhi = pk2(y7.hi, y7.hi), ylo = pk2(y7.lo, y7.lo), bias = pk2(-8388616.0f, -8388616.0f);
    const f2 ss = pk2(s, s);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (code >> (8 * b)) & 0xFFu;
      const f2 q = add2(pk2(__uint_as_float(0x4B000000u | (byte >> 4)), __uint_as_float(0x4B000000u | (byte & 15u))),
                        bias);
      float v0, v1;
      upk2(div2_short(mul2(q, ss), yhi, ylo), v0, v1);
      o[b] = f32x2_to_bf16x2(v0, v1);
    }
  } else {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (code >> (8 * b)) & 0xFFu;
      const float v0 = __fdiv_rn(__fmul_rn(float(int(byte >> 4) - 8), s), 7.0f);
      const float v1 = __fdiv_rn(__fmul_rn(float(int(byte & 15u) - 8), s), 7.0f);
      o[b] = bf16_cpu(v0) | (bf16_cpu(v1) << 16);
    }
  }
}

}  // namespace
}  // namespace ashkv
