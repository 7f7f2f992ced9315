// Shared device/host helpers for libashkv_cuda (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ashkv.h"

namespace ashkv {

// ---------------------------------------------------------------- host side
// Records the last CUDA error (thread-local) and maps it to a status code.
ashkv_status_t check_launch(const char* what);
void set_error(const char* what, cudaError_t err);
void set_message(const char* text);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

int sm_count();

// cuTensorMapEncodeTiled fetched once through the runtime's driver entry point
// (no -lcuda); nullptr when unavailable.  Cast to PFN_cuTensorMapEncodeTiled_v12000.
void* tensor_map_encoder();

// ---------------------------------------------------------------- bf16/fp16
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// Two bf16 products in one instruction, each the exact product rounded once to
// bf16 (round to nearest even).
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Per-half unsigned maximum of two 16-bit pairs.
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Running max of |x| over bf16 pairs as 16-bit patterns: for non-NaN values the
// order of |x| is the order of its bit pattern (sign cleared); NaN patterns lie
// above 0x7F80 (infinity).
__device__ __forceinline__ uint32_t absmax_bits_bf16x2(uint32_t m, uint32_t w) { return max_u16x2(m, w & 0x7FFF7FFFu); }

// max |x| over the N words (2N bf16 values) a lane holds of a row, reduced over
// the team of TEAM consecutive lanes, ignoring NaN (fmaxf semantics).  Called by
// every lane of the warp; inactive lanes pass zeros.  A row holding a NaN (bit
// maximum above 0x7F80) is redone with fmaxf.
template <int TEAM, int N>
__device__ __forceinline__ float team_absmax_bf16(const uint32_t (&w)[N]) {
  uint32_t mb = 0;
#pragma unroll
  for (int k = 0; k < N; ++k) mb = absmax_bits_bf16x2(mb, w[k]);
  uint32_t m = max(mb & 0xFFFFu, mb >> 16);
#pragma unroll
  for (int off = TEAM / 2; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
  if (!__any_sync(0xFFFFFFFFu, m > 0x7F80u)) return __uint_as_float(m << 16);
  float am = 0.0f;
#pragma unroll
  for (int k = 0; k < N; ++k) am = fmaxf(am, fmaxf(fabsf(bf16lo(w[k])), fabsf(bf16hi(w[k]))));
#pragma unroll
  for (int off = TEAM / 2; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, off));
  return am;
}
__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }

// fp32 -> bf16, round to nearest even; NaN becomes 0x7FFF.
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
// Two fp32 -> packed bf16x2 (lo in bits 0..15), round to nearest even.
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint16_t f32_to_f16(float f) {
  return __half_as_ushort(__float2half_rn(f));
}
__device__ __forceinline__ float f16_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// Streaming 16-byte load through the non-coherent path (data read once).
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ float4 ld_nc_f4(const void* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}
// Streaming 16-byte store (evict-first: written once, not re-read soon).
__device__ __forceinline__ void st_cs_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// NaN-propagating max (PTX max.NaN): NaN if either input is NaN.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Round-half-even of a value already clamped to [0, 2^22) via the 1.5*2^23
// magic constant; returns the integer in the low mantissa bits.
__device__ __forceinline__ uint32_t rint_small(float v) {
  return __float_as_uint(__fadd_rn(v, 12582912.0f)) & 0x3FFFFFu;
}

// ---------------------------------------------------------------- Philox
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
// as 1, 2, 3", SC'11): 10 rounds of two 32x32->64 multiplies with the round
// key bumped by the Weyl constants between rounds.
struct Philox4 { uint32_t v[4]; };

__device__ __host__ __forceinline__ void mulhilo32(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  uint64_t p = uint64_t(a) * uint64_t(b);
  hi = uint32_t(p >> 32);
  lo = uint32_t(p);
}

__device__ __host__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                          uint32_t k0, uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  constexpr uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, c0, hi0, lo0);
    mulhilo32(M1, c2, hi1, lo1);
    uint32_t n0 = hi1 ^ c1 ^ k0;
    uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += W0; k1 += W1;
  }
  Philox4 out;
  out.v[0] = c0; out.v[1] = c1; out.v[2] = c2; out.v[3] = c3;
  return out;
}

// The same generator with the ten round keys precomputed by
// philox_round_keys(): rk[2r], rk[2r+1] = key + r * (W0, W1).
__device__ __forceinline__ Philox4 philox4x32_10_rk(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                    const uint32_t (&rk)[20]) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, c0, hi0, lo0);
    mulhilo32(M1, c2, hi1, lo1);
    const uint32_t n0 = hi1 ^ c1 ^ rk[2 * r];
    const uint32_t n2 = hi0 ^ c3 ^ rk[2 * r + 1];
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
  }
  Philox4 out;
  out.v[0] = c0; out.v[1] = c1; out.v[2] = c2; out.v[3] = c3;
  return out;
}

inline void philox_round_keys(uint64_t seed, uint32_t (&rk)[20]) {
  uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    rk[2 * r] = k0; rk[2 * r + 1] = k1;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
}


// ---------------------------------------------------------------- sm_100 vector ops
// 256-bit streaming load / store (one full 32-byte sector per thread).
struct U8 { uint32_t v[8]; };
__device__ __forceinline__ U8 ld_nc_v8(const void* p) {
  U8 r;
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]),
                 "=r"(r.v[6]), "=r"(r.v[7])
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_cs_v8(void* p, const U8& r) {
  asm volatile("st.global.cs.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
               :: "l"(p), "r"(r.v[0]), "r"(r.v[1]), "r"(r.v[2]), "r"(r.v[3]), "r"(r.v[4]), "r"(r.v[5]),
                  "r"(r.v[6]), "r"(r.v[7]) : "memory");
}

// Packed fp32 pairs (lo, hi) in a 64-bit register; f32x2 arithmetic rounds
// each lane exactly like the scalar .rn instruction.  One exception was
// measured: mul.rn.f32x2 feeding add.rn.f32x2 came out as one fused
// multiply-add (single rounding), so a product that must be rounded before a
// sum is added with scalar add.rn, which is never contracted.
typedef unsigned long long f2;
__device__ __forceinline__ f2 pk2(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(f2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// max(|a|, |b|, |c|), NaN if any input is NaN.
__device__ __forceinline__ float max3_abs_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// fp32 pair -> packed bf16x2, round to nearest even (NaN -> 0x7FFF).
__device__ __forceinline__ uint32_t f32x2_to_bf16x2_pk(f2 v) {
  float lo, hi;
  upk2(v, lo, hi);
  return f32x2_to_bf16x2(lo, hi);
}

// Correctly rounded division by a divisor shared by many dividends.
// Per divisor b: y_hi = RN(1/b), y_lo = RN((1 - b*y_hi) * y_hi), so that
// y_hi + y_lo approximates 1/b to ~2^-47.  Per dividend a:
//   q0 = RN(a*y_hi + RN(a*y_lo))   -- within one ulp of a/b
//   r  = a - q0*b                  -- exact (fused multiply-add)
//   q1 = RN(q0 + r*y_hi)           -- = RN(a/b)
// The last step is Markstein's correction (P. Markstein, IBM J. Res. Dev.
// 34(1), 1990): with y within half an ulp of 1/b and q0 within one ulp of
// a/b it yields the correctly rounded quotient, barring overflow/underflow,
// which recip_ok() excludes by keeping b inside [2^-100, 2^100].
struct Recip { float hi, lo; };
__device__ __forceinline__ Recip make_recip(float b) {
  Recip r;
  r.hi = __frcp_rn(b);
  const float e = __fmaf_rn(-b, r.hi, 1.0f);
  r.lo = __fmul_rn(e, r.hi);
  return r;
}
__device__ __forceinline__ bool recip_ok(float b) { return fabsf(b) >= 0x1p-100f && fabsf(b) <= 0x1p+100f; }
__device__ __forceinline__ float div_rn(float a, float b, Recip y) {
  const float q0 = __fmaf_rn(a, y.hi, __fmul_rn(a, y.lo));
  const float r = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(r, y.hi, q0);
}
// The same on fp32 pairs: Y_HI/Y_LO/NB = (y.hi, y.hi), (y.lo, y.lo), (-b, -b).
__device__ __forceinline__ f2 div2_rn(f2 a, f2 yhi, f2 ylo, f2 nb) {
  const f2 q0 = fma2(a, yhi, mul2(a, ylo));
  const f2 r = fma2(q0, nb, a);
  return fma2(r, yhi, q0);
}

// The first step alone is already RN(a/b) when b's significand has at most 11
// bits and a's at most 19 (products of bf16/fp16 values and small integers).
// Write a = S*2^s, b = A*2^t with S, A odd integers, S < 2^19, A < 2^11.  A
// rounding boundary of the binade [2^E, 2^(E+1)) is (2m+1)*2^(E-24), and
// S*2^(s-t) - A*(2m+1)*2^(E-24) is a nonzero multiple of 2^(E-24) (it could only
// vanish with S >= 2^24), so a/b lies more than 2^-36*|a/b| from every
// boundary, while a*y_hi + RN(a*y_lo) differs from a/b by less than 2^-46*|a/b|
// (y_hi + y_lo errs by < 2^-47/|b|).  Holds while a*y_lo is a normal number,
// i.e. for |a/b| >= 2^-100.
__device__ __forceinline__ bool short_significand(float b) { return (__float_as_uint(b) & 0x1FFFu) == 0u; }
__device__ __forceinline__ float div_short(float a, Recip y) { return __fmaf_rn(a, y.hi, __fmul_rn(a, y.lo)); }
__device__ __forceinline__ f2 div2_short(f2 a, f2 yhi, f2 ylo) { return fma2(a, yhi, mul2(a, ylo)); }


// ---------------------------------------------------------------- INT8 codec arithmetic
// Shared by the row kernels (int8_codec.cu) and the page kernels (pages.cu);
// restates ashkv/codecs/int8.py:70-80 (encode) and :110-115 (decode) as the
// reference's Triton kernel executes them on the GPU:
//   q    = s / am, s = x * 127 rounded to the input dtype.  Triton lowers an
//          fp32 division to PTX div.full.f32 (an approximation within 2 ulp,
//          not IEEE division); for divisors below 2^126 that instruction equals
//          RN(s * rcp.approx(am)) bit for bit (checked on a B200 over every bf16
//          and every fp16 dividend/divisor pair), so rows with am < 2^126 take
//          one reciprocal per row and one multiply per element, and larger
//          divisors take div.full.f32 itself.
//   code = low byte of int32(trunc(RN(q + (q > 0 ? 0.5 : -0.5))))
//          (Triton's fp32 -> int8 cast: convert to int32, saturating, NaN -> 0,
//          then keep the low byte; only an infinite product leaves [-128, 127]:
//          +inf gives -1 and -inf gives 0, as the reference does).
__device__ __forceinline__ float rcp_approx(float b) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(b));
  return r;
}
__device__ __forceinline__ float div_full(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
struct Int8Div {
  float am;
  float r;    // rcp.approx(am)
  bool full;  // am >= 2^126 (or not finite): div.full.f32 per element
};
__device__ __forceinline__ Int8Div int8_div(float am) {
  Int8Div d;
  d.am = am;
  d.full = !(am < 0x1p126f);
  d.r = rcp_approx(am);
  return d;
}
__device__ __forceinline__ float int8_quot(float s, const Int8Div& d) {
  return d.full ? div_full(s, d.am) : __fmul_rn(s, d.r);
}
// int32 whose low byte is the code.  The half is copysign(0.5, q), one logic op
// instead of a compare and a select: it equals q > 0 ? 0.5 : -0.5 for every q
// but the zeros (+0 takes +0.5 here), where both sums truncate to 0, and a NaN
// q gives NaN either way.
__device__ __forceinline__ int32_t int8_round(float q) {
  const float h = __uint_as_float((__float_as_uint(q) & 0x80000000u) | 0x3F000000u);
  const float r = __fadd_rn(q, h);
  int32_t c;
  asm("cvt.rzi.s32.f32 %0, %1;" : "=r"(c) : "f"(r));  // saturating; NaN -> 0
  return c;
}
__device__ __forceinline__ int32_t int8_code(float s, const Int8Div& d) { return int8_round(int8_quot(s, d)); }
// Four bf16 inputs (two words, element 0 in the low half of w0) -> four
// codes packed little-endian: s = bf16(x * 127) (exact product, one rounding).
__device__ __forceinline__ uint32_t int8_codes4_bf16(uint32_t w0, uint32_t w1, const Int8Div& d) {
  const uint32_t s01 = bf16x2_mul(w0, 0x42FE42FEu);  // bf16 127.0 in both halves
  const uint32_t s23 = bf16x2_mul(w1, 0x42FE42FEu);
  float q[4];
  if (!d.full) {
    const f2 R = pk2(d.r, d.r);
    upk2(mul2(pk2(bf16lo(s01), bf16hi(s01)), R), q[0], q[1]);
    upk2(mul2(pk2(bf16lo(s23), bf16hi(s23)), R), q[2], q[3]);
  } else {
    q[0] = div_full(bf16lo(s01), d.am);
    q[1] = div_full(bf16hi(s01), d.am);
    q[2] = div_full(bf16lo(s23), d.am);
    q[3] = div_full(bf16hi(s23), d.am);
  }
  const uint32_t c0 = uint32_t(int8_round(q[0])), c1 = uint32_t(int8_round(q[1]));
  const uint32_t c2 = uint32_t(int8_round(q[2])), c3 = uint32_t(int8_round(q[3]));
  return __byte_perm(__byte_perm(c0, c1, 0x0040), __byte_perm(c2, c3, 0x0040), 0x5410);
}
// Decode: v = RN(RN(float(code) * scale) / 127).  `fast` when the scale is
// finite and in [2^-90, 2^90] (products are 0 or at least 2^-90, and code *
// scale is exact with at most 8 + 11 significant bits, so div_short applies to
// the division by 127; scale > 0 keeps the sign of zero products).
__device__ __forceinline__ bool int8_dec_fast(float scale) { return scale >= 0x1p-90f && scale <= 0x1p+90f; }
__device__ __forceinline__ float int8_dequant(int32_t c, float scale, bool fast) {
  const float p = __fmul_rn(float(c), scale);
  return fast ? div_short(p, make_recip(127.0f)) : __fdiv_rn(p, 127.0f);
}
// Four int8 codes (one word, code 0 in the low byte) -> float(code) exactly,
// without an int->float conversion: 0x4B400000 | (byte ^ 0x80) is the float
// 1.5*2^23 + 128 + code.
__device__ __forceinline__ void int8x4_to_f2(uint32_t w, f2& lo, f2& hi) {
  const uint32_t b = w ^ 0x80808080u;
  const f2 nbias = pk2(-12583040.0f, -12583040.0f);  // -(1.5*2^23 + 128)
  lo = add2(pk2(__uint_as_float(__byte_perm(b, 0x4B400000u, 0x7640)),
                __uint_as_float(__byte_perm(b, 0x4B400000u, 0x7641))), nbias);
  hi = add2(pk2(__uint_as_float(__byte_perm(b, 0x4B400000u, 0x7642)),
                __uint_as_float(__byte_perm(b, 0x4B400000u, 0x7643))), nbias);
}

// ---------------------------------------------------------------- TMA / mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `max_polls` polls (each poll may suspend briefly).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t max_polls) {
  for (uint32_t i = 0; i < max_polls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// 2-D tiled TMA load (coordinates: x = innermost element index, y = row).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      :: "r"(smem_u32(smem_dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}

}  // namespace ashkv
