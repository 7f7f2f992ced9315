// Per-group arithmetic of the dithered N-bit codec, shared by the tensor
// codec (nbit_codec.cu) and the page transcoder (migrate.cu).
//
// Restates DitheredNBitCodec.encode/decode (ashkv/codecs/nbit_dithered.py:
// 57-104, 140-167) for one group of 32 elements: mean, standard deviation,
// sigma-rule outliers, inlier absmax, delta, dithered quantisation and
// MSB-first packing; and the inverse dequantisation.
#pragma once

#include "common.cuh"

namespace ashkv {
namespace {

struct NbitEncParams {
  const uint16_t* src;
  int64_t n_groups;
  const float* dither;
  uint32_t round_keys[20];  // Philox key schedule: (k0 + r*W0, k1 + r*W1) for r = 0..9
  uint64_t seed;
  uint64_t dither_offset;
  float sigma;
  float half_states;
  uint16_t* scales;
  uint8_t* codes;
  uint32_t* bucket_counts;
  uint32_t* bucket_entries;
  int32_t bucket_cap;
  uint32_t* status;
};

// One thread per 32-element group, one warp (32 groups) per outlier bucket.
//
// Outlier decisions are made against the reference threshold without
// computing its fp64 variance in the common case: fp32 sums of the values and
// of their squares, with rigorous error bounds, give thr_lo <= thr <= thr_hi.  If every |x - mu| of
// the group is <= thr_lo the group has no outliers (the usual case).
// Otherwise per-element masks against thr_lo and thr_hi are built; if they
// agree, that is the exact mask, and only if some |x - mu| falls between the
// two bounds is the exact fp64 threshold computed.
// A group's 32 bf16 values as 4 chunks of 8 (16 bytes each), plus access to
// element e of the group owned by another lane of the warp.
struct RegGroup {  // held in registers; other groups read back from global memory
  const uint32_t* w;
  const uint16_t* src;  // the kernel's source (group g at src + 32 g)
  int64_t g0;           // group of lane 0 of the warp
  __device__ __forceinline__ uint4 chunk(int c) const { return make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]); }
  __device__ __forceinline__ uint32_t elem(int owner_lane, int e) const { return src[(g0 + owner_lane) * 32 + e]; }
};
struct SmemGroup {  // rows of a 64-byte-swizzled shared-memory tile (the warp's bucket), one per lane
  uint32_t tile, row, sw;
  __device__ __forceinline__ uint4 chunk(int c) const { return lds128(row + 16u * (uint32_t(c) ^ sw)); }
  __device__ __forceinline__ uint32_t elem(int owner_lane, int e) const {
    const uint32_t osw = uint32_t(owner_lane >> 1) & 3u;
    const uint32_t a = tile + uint32_t(owner_lane) * 64u + 16u * ((uint32_t(e) >> 3) ^ osw) + 2u * (uint32_t(e) & 7u);
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
  }
};

// Hardware square-root approximation (relative error below 2^-21).
__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Two signed 16-bit integers clamped to [0, hi]: max(min(v, hi), 0) per half.
__device__ __forceinline__ uint32_t clamp_codes_s16x2(uint32_t v, uint32_t hi) {
  uint32_t r;
  asm("min.relu.s16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(hi | (hi << 16)));
  return r;
}

__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float min3_nan(float a, float b, float c) {
  float r;
  asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float min_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// (RN(bf16lo(w) + a), RN(bf16hi(w) + b)): sm_100 mixed-precision adds, one rounding each.
__device__ __forceinline__ f2 add_bf16x2_f32(uint32_t w, float a, float b) {
  float lo, hi;
  asm("{ .reg .b16 l, h; mov.b32 {l, h}, %2; add.rn.f32.bf16 %0, l, %3; add.rn.f32.bf16 %1, h, %4; }"
      : "=f"(lo), "=f"(hi) : "r"(w), "f"(a), "f"(b));
  return pk2(lo, hi);
}

__device__ __forceinline__ double warp_sum_f64(double v) {  // pairwise (butterfly) order, same in every lane
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) v = __dadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  return v;
}
// max |v| over the warp, NaN if any lane holds NaN: the bit patterns of non-negative floats
// order like unsigned integers (NaNs above +inf), so one redux.sync max does it.
__device__ __forceinline__ float warp_max_abs_nan(float v) {
  return __uint_as_float(__reduce_max_sync(0xFFFFFFFFu, __float_as_uint(v) & 0x7FFFFFFFu));
}

template <typename Src>
__device__ __forceinline__ void chunk_pairs(const Src& src, int c, f2 (&P)[4]) {
  const uint4 q = src.chunk(c);
  P[0] = pk2(bf16lo(q.x), bf16hi(q.x));
  P[1] = pk2(bf16lo(q.y), bf16hi(q.y));
  P[2] = pk2(bf16lo(q.z), bf16hi(q.z));
  P[3] = pk2(bf16lo(q.w), bf16hi(q.w));
}

// Encodes one group (writes its packed codes and bf16 delta) and returns the
// outlier bit mask.  The group is read from `src` twice (statistics, then
// quantisation) so only one 8-element chunk is live in registers at a time.
template <int BITS, int DMODE, typename Src>
__device__ __forceinline__ uint32_t encode_group(const Src& src, const NbitEncParams& p, int64_t g, bool active) {
  constexpr uint32_t kMaxCode = (1u << BITS) - 1u;
  // ---- one pass over the group: the sum in the reference's order, acc[i] =
  //      ((x_i + x_{8+i}) + x_{16+i}) + x_{24+i}, then acc[0] + ... + acc[7] in
  //      order (PyTorch's CPU reduction order for a 32-wide inner dimension);
  //      the sum of squares; the signed maximum and minimum (NaN-propagating).
  // the group's two Philox draws do not depend on its values: computing them first gives
  // the scheduler independent work beside the statistics' dependency chains
  Philox4 rd[2];
  if constexpr (DMODE == ASHKV_DITHER_PHILOX) {
    const uint64_t ctr = (p.dither_offset + uint64_t(g) * 32) >> 4;
    rd[0] = philox4x32_10_rk(uint32_t(ctr), uint32_t(ctr >> 32), 0u, 0u, p.round_keys);
    rd[1] = philox4x32_10_rk(uint32_t(ctr + 1), uint32_t((ctr + 1) >> 32), 0u, 0u, p.round_keys);
  }
  f2 A[4];
  chunk_pairs(src, 0, A);
  f2 SQ0 = mul2(A[0], A[0]), SQ1 = mul2(A[1], A[1]);
  SQ0 = fma2(A[2], A[2], SQ0);
  SQ1 = fma2(A[3], A[3], SQ1);
  float mx, mn;
  {
    float a0, a1, b0, b1, c0, c1, d0, d1;
    upk2(A[0], a0, a1); upk2(A[1], b0, b1); upk2(A[2], c0, c1); upk2(A[3], d0, d1);
    mx = max3_nan(max3_nan(a0, a1, b0), max3_nan(b1, c0, c1), max_nan(d0, d1));
    mn = min3_nan(min3_nan(a0, a1, b0), min3_nan(b1, c0, c1), min_nan(d0, d1));
  }
#pragma unroll
  for (int c = 1; c < 4; ++c) {
    f2 P[4];
    chunk_pairs(src, c, P);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      A[i] = add2(A[i], P[i]);
      if (i & 1) SQ1 = fma2(P[i], P[i], SQ1);
      else SQ0 = fma2(P[i], P[i], SQ0);
      float x0, x1;
      upk2(P[i], x0, x1);
      mx = max3_nan(mx, x0, x1);
      mn = min3_nan(mn, x0, x1);
    }
  }
  float acc[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) upk2(A[i], acc[2 * i], acc[2 * i + 1]);
  float s = acc[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) s = __fadd_rn(s, acc[i]);
  const float mu = __fmul_rn(s, 0.03125f);
  // max |x - mu| = max(RN(max x - mu), RN(mu - min x)) (rounding is monotone and odd).
  const float dmax = max_nan(__fadd_rn(mx, -mu), __fadd_rn(mu, -mn));
  const float xmax = max_nan(fabsf(mx), fabsf(mn));
  float q2a, q2b;
  upk2(add2(SQ0, SQ1), q2a, q2b);
  const float q2 = __fadd_rn(q2a, q2b);

  // Bounds on the reference threshold from M2 = sum (x - m)^2 = q2_exact - 32 m^2
  // (m the exact mean).  q2 is within 10u of q2_exact (u = 2^-24: at most ten
  // roundings deep), and |m - mu| <= 31 u max|x| =: emu, so with mlo = max(|mu| - emu, 0)
  // and mhi = |mu| + emu,
  //   RN(RN(q2 (1 - 2^-17)) - RN(RN(32 mhi^2) (1 + 2^-17))) <= M2
  //   RN(RN(q2 (1 + 2^-17)) - RN(RN(32 mlo^2) (1 - 2^-17))) >= M2,
  // the 2^-17 = 128u margins covering every rounding on the way.  The bounds
  // only choose between the fast and the exact outlier path; the threshold
  // arithmetic below (sqrt.approx and the product by RN(1/31), each within
  // 2^-21 relative, the fp32 rounding of sd, + 1e-8 and * sigma in the
  // reference) is covered by the 2^-12 margin on the threshold.
  const float sigma = p.sigma;
  const bool bounds_ok = sigma > 0.0f && isfinite(q2) && isfinite(xmax);
  float thr_lo = 0.0f, thr_hi = 0.0f;
  if (bounds_ok) {
    const float emu = 31.0001f * 0x1p-24f * xmax;
    const float amu = fabsf(mu);
    const float mlo = fmaxf(amu - emu, 0.0f), mhi = amu + emu;
    const float m2_hi = q2 * (1.0f + 0x1p-17f) - (32.0f * (mlo * mlo)) * (1.0f - 0x1p-17f);
    const float m2_lo = fmaxf(q2 * (1.0f - 0x1p-17f) - (32.0f * (mhi * mhi)) * (1.0f + 0x1p-17f), 0.0f);
    constexpr float kInv31 = 1.0f / 31.0f;
    thr_hi = sigma * (sqrt_approx(m2_hi * kInv31) + 1e-8f) * (1.0f + 0x1p-12f);
    thr_lo = sigma * (sqrt_approx(m2_lo * kInv31) + 1e-8f) * (1.0f - 0x1p-12f);
  }
  // Groups whose max |x - mu| exceeds thr_lo are resolved by the whole warp,
  // one group at a time: lane e takes element e, masks come from ballots, and
  // if an |x - mu| lies between the bounds the exact threshold is computed
  // (fp64, pairwise order over the 32 elements).
  uint32_t omask = 0;
  float am = xmax;
  const int lane = threadIdx.x & 31;
  uint32_t todo = __ballot_sync(0xFFFFFFFFu, active && !(bounds_ok && dmax <= thr_lo));
  while (todo) {
    const int owner = __ffs(todo) - 1;
    todo &= todo - 1;
    const float mu_o = __shfl_sync(0xFFFFFFFFu, mu, owner);
    const float lo_o = __shfl_sync(0xFFFFFFFFu, thr_lo, owner);
    const float hi_o = __shfl_sync(0xFFFFFFFFu, thr_hi, owner);
    const bool ok_o = __shfl_sync(0xFFFFFFFFu, int(bounds_ok), owner) != 0;
    const float x = bf16_to_f32(uint16_t(src.elem(owner, lane)));
    const float d = fabsf(__fadd_rn(x, -mu_o));
    const uint32_t mlo = __ballot_sync(0xFFFFFFFFu, d > lo_o);
    uint32_t m = __ballot_sync(0xFFFFFFFFu, d > hi_o);
    if (!ok_o || mlo != m) {
      const double s64 = warp_sum_f64(double(x));
      const double e = __dadd_rn(double(x), -__dmul_rn(s64, 0.03125));
      const double m2e = warp_sum_f64(__dmul_rn(e, e));
      const float sd = __double2float_rn(__dsqrt_rn(__ddiv_rn(m2e, 31.0)));
      const float thr = __fmul_rn(sigma, __fadd_rn(sd, 1e-8f));
      m = __ballot_sync(0xFFFFFFFFu, d > thr);
    }
    const float amv = warp_max_abs_nan((m >> lane) & 1u ? mu_o : x);
    if (lane == owner) {
      omask = m;
      am = amv;
    }
  }
  if (!active) omask = 0;
  if (!(am >= 1e-8f) && am == am) am = 1e-8f;  // clamp(min=1e-8); NaN propagates
  // delta = RN(am / half) by Markstein's correction with the compile-time reciprocal pair of
  // half: exact for every finite am >= 1e-8 (checked exhaustively for the three halves; no
  // step can underflow or overflow there), NaN stays NaN, and +inf is passed through.
  constexpr float kHalf = float(kMaxCode) * 0.5f;
  constexpr float kHy = 1.0f / kHalf;
  constexpr float kHlo = float(double(float(1.0 - double(kHalf) * double(kHy))) * double(kHy));
  const float dq = div_rn(am, kHalf, Recip{kHy, kHlo});
  const float delta = am == INFINITY ? am : dq;

  // ---- dither, quantise (x' + (U-0.5)*delta) / delta + half, pack
  const Recip y = make_recip(delta);
  const bool fast_div = recip_ok(delta);
  const f2 DELTA = pk2(delta, delta), YHI = pk2(y.hi, y.hi), YLO = pk2(y.lo, y.lo), NDELTA = pk2(-delta, -delta);
  const float half = p.half_states;
  const f2 HALF = pk2(half, half), MAGIC = pk2(12582912.0f, 12582912.0f);
  uint32_t o[BITS];  // packed codes: 32 * BITS bits, MSB-first within each byte
#pragma unroll
  for (int k = 0; k < BITS; ++k) o[k] = 0u;
#pragma unroll
  for (int c = 0; c < 4; ++c) {  // 8 elements per chunk, 16 per Philox draw
    const uint4 raw = src.chunk(c);
    const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
    f2 DZ[4];
    if constexpr (DMODE == ASHKV_DITHER_TENSOR) {
      U8 u;
      if (active) u = ld_nc_v8(p.dither + g * 32 + 8 * c);
      else {
#pragma unroll
        for (int k = 0; k < 8; ++k) u.v[k] = 0x3F000000u;  // 0.5 -> zero dither
      }
#pragma unroll
      for (int h = 0; h < 4; ++h)
        DZ[h] = add2(pk2(__uint_as_float(u.v[2 * h]), __uint_as_float(u.v[2 * h + 1])), pk2(-0.5f, -0.5f));
    } else {
      const Philox4& rr = rd[c >> 1];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // U = (b + 0.5) / 256 from byte b = e & 15 of the draw for counter e >> 4:
        // f = 1 + (2b + 1) * 2^-16, so U - 0.5 = 128 f - 128.5 exactly
        const uint32_t wv = rr.v[2 * (c & 1) + (h >> 1)];
        const float flo = __uint_as_float(__byte_perm(wv, 0x3F808080u, (h & 1) ? 0x7624 : 0x7604));
        const float fhi = __uint_as_float(__byte_perm(wv, 0x3F808080u, (h & 1) ? 0x7634 : 0x7614));
        DZ[h] = fma2(pk2(flo, fhi), pk2(128.0f, 128.0f), pk2(-128.5f, -128.5f));
      }
    }
    // v = RN(RN(a / delta) + half), a = x' + noise; code = clamp(rint(v), 0, 2^bits - 1).
    // rint: RN(v + 1.5 * 2^23) leaves rint(v) in the low mantissa bits (|v| < 2^22).
    // With delta in Markstein's range every a is finite and |a / delta| <= half + 1,
    // so the clamp runs on the integers (two codes per s16x2 word); otherwise the
    // float clamp comes first (NaN -> 0), as in the reference.
    f2 Q[4];
    // a = RN(x' + RN((U - 0.5) * delta)), x' = mu at outliers.  The sum is a scalar add (a
    // packed add.rn.f32x2 fed by a packed multiply was measured to come out single-rounded, a
    // fused multiply-add, which flips codes one ulp from a rounding tie): every element takes
    // the bf16 operand directly (add.rn.f32.bf16: exact widening, one rounding), and only the
    // chunks holding outliers then redo those elements with mu (one divergent path, not two).
    float NZ[8];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      upk2(mul2(DZ[h], DELTA), NZ[2 * h], NZ[2 * h + 1]);
      Q[h] = add_bf16x2_f32(rw[h], NZ[2 * h], NZ[2 * h + 1]);
    }
    if (omask & (0xFFu << (8 * c))) {  // outliers of this chunk take x' = mu
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int e = 8 * c + 2 * h;
        float q0, q1;
        upk2(Q[h], q0, q1);
        if ((omask >> e) & 1u) q0 = __fadd_rn(mu, NZ[2 * h]);
        if ((omask >> (e + 1)) & 1u) q1 = __fadd_rn(mu, NZ[2 * h + 1]);
        Q[h] = pk2(q0, q1);
      }
    }
    if (fast_div) {
#pragma unroll
      for (int h = 0; h < 4; ++h) Q[h] = add2(add2(div2_rn(Q[h], YHI, YLO, NDELTA), HALF), MAGIC);
    } else {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float a0, a1;
        upk2(Q[h], a0, a1);
        const float v0 = fminf(fmaxf(__fadd_rn(__fdiv_rn(a0, delta), half), 0.0f), float(kMaxCode));
        const float v1 = fminf(fmaxf(__fadd_rn(__fdiv_rn(a1, delta), half), 0.0f), float(kMaxCode));
        Q[h] = add2(pk2(v0, v1), MAGIC);
      }
    }
    if constexpr (DMODE == ASHKV_DITHER_PHILOX) {
      // No clamp is needed: |U - 0.5| <= 127.5/256 and |x'| <= am = delta * half (1 + 2^-23),
      // so |a / delta| < half + 0.4982, and v = RN(RN(a / delta) + half) lies in
      // (-0.5, 2 half + 0.5) = (-0.5, 2^BITS - 0.5): its rint is already a code, and
      // byte 0 of each float above (1.5 * 2^23 + code) holds it.  The slow path
      // clamps in float first.
      uint32_t u[8];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float t0, t1;
        upk2(Q[h], t0, t1);
        u[2 * h] = __float_as_uint(t0);
        u[2 * h + 1] = __float_as_uint(t1);
      }
      if constexpr (BITS == 8) {
        o[2 * c] = __byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410);
        o[2 * c + 1] = __byte_perm(__byte_perm(u[4], u[5], 0x0040), __byte_perm(u[6], u[7], 0x0040), 0x5410);
      } else if constexpr (BITS == 4) {
        // byte 0 of u0 * 16 + u1 is (c0 << 4) | c1; the bits above byte 0 never carry into it.
        const uint32_t b0 = u[0] * 16u + u[1], b1 = u[2] * 16u + u[3], b2 = u[4] * 16u + u[5], b3 = u[6] * 16u + u[7];
        o[c] = __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
      } else {
        const uint32_t b0 = (u[0] * 4u + u[1]) * 16u + (u[2] * 4u + u[3]);
        const uint32_t b1 = (u[4] * 4u + u[5]) * 16u + (u[6] * 4u + u[7]);
        const uint32_t half16 = __byte_perm(b0, b1, 0x0040);
        if ((c & 1) == 0) o[c >> 1] = half16;
        else o[c >> 1] = __byte_perm(o[c >> 1], half16, 0x5410);
      }
    } else {
      uint32_t W[4];  // codes of elements 2h (low half) and 2h + 1 (high half)
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float t0, t1;
        upk2(Q[h], t0, t1);
        W[h] = clamp_codes_s16x2(__byte_perm(__float_as_uint(t0), __float_as_uint(t1), 0x5410), kMaxCode);
      }
      // bytes c0..c3 of elements 8c..8c+3, and c4..c7
      const uint32_t X = __byte_perm(W[0], W[1], 0x6420), Y = __byte_perm(W[2], W[3], 0x6420);
      if constexpr (BITS == 8) {
        o[2 * c] = X;
        o[2 * c + 1] = Y;
      } else if constexpr (BITS == 4) {
        // byte j of X*16 + (X >> 8) is (c_j << 4) + c_{j+1}: keep bytes 0 and 2 of each half.
        o[c] = __byte_perm(X * 16u + (X >> 8), Y * 16u + (Y >> 8), 0x6420);
      } else {
        const uint32_t tx = X * 4u + (X >> 8), ty = Y * 4u + (Y >> 8);   // bytes 0, 2: c0c1, c2c3
        const uint32_t ux = tx * 16u + (tx >> 16), uy = ty * 16u + (ty >> 16);  // byte 0: c0c1c2c3
        o[c >> 1] |= (__byte_perm(ux, uy, 0x0040) & 0xFFFFu) << (16 * (c & 1));
      }
    }
  }

  if (active) {
    p.scales[g] = f32_to_bf16(delta);
    if constexpr (BITS == 4) {
      st_cs_v4(p.codes + g * 16, make_uint4(o[0], o[1], o[2], o[3]));
    } else if constexpr (BITS == 2) {
      *reinterpret_cast<uint2*>(p.codes + g * 8) = make_uint2(o[0], o[1]);
    } else {
      U8 ov;
#pragma unroll
      for (int k = 0; k < 8; ++k) ov.v[k] = o[k];
      st_cs_v8(p.codes + g * 32, ov);
    }
  }
  return omask;
}

// One group's packed codes (32 * BITS bits, MSB-first within each byte) and its delta.
template <int BITS>
struct GroupCodes {
  uint32_t w[BITS];
  float delta;
};
template <int BITS>
__device__ __forceinline__ void load_group(const uint16_t* scales, const uint8_t* codes, int64_t g,
                                           GroupCodes<BITS>& gc) {
  gc.delta = bf16_to_f32(scales[g]);
  if constexpr (BITS == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(codes + g * 16);
    gc.w[0] = v.x; gc.w[1] = v.y; gc.w[2] = v.z; gc.w[3] = v.w;
  } else if constexpr (BITS == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(codes + g * 8);
    gc.w[0] = v.x; gc.w[1] = v.y;
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(codes + g * 32);
    const uint4 b = *reinterpret_cast<const uint4*>(codes + g * 32 + 16);
    gc.w[0] = a.x; gc.w[1] = a.y; gc.w[2] = a.z; gc.w[3] = a.w;
    gc.w[4] = b.x; gc.w[5] = b.y; gc.w[6] = b.z; gc.w[7] = b.w;
  }
}

// Byte j of m (a code < 256) as the float 2^23 + code.
__device__ __forceinline__ float code_plus_2p23(uint32_t m, int j) {
  return __uint_as_float(__byte_perm(m, 0x4B000000u, 0x7540u + uint32_t(j)));
}

// out = bf16((code - half) * delta) for the 32 elements of a group:
// float(code) = (2^23 + code) - 2^23 exactly, then the reference's two roundings.
template <int BITS>
__device__ __forceinline__ void group_bf16(const GroupCodes<BITS>& gc, float half, uint32_t (&o)[16]) {
  const f2 DEL = pk2(gc.delta, gc.delta), NH = pk2(-half, -half), N23 = pk2(-8388608.0f, -8388608.0f);
  auto pair = [&](float a, float b) { return f32x2_to_bf16x2_pk(mul2(add2(add2(pk2(a, b), N23), NH), DEL)); };
  if constexpr (BITS == 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // word k: elements 8k .. 8k+7, byte j = (elem 8k+2j) << 4 | elem 8k+2j+1
      const uint32_t hi = (gc.w[k] >> 4) & 0x0F0F0F0Fu, lo = gc.w[k] & 0x0F0F0F0Fu;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[4 * k + j] = pair(code_plus_2p23(hi, j), code_plus_2p23(lo, j));
    }
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {  // word k: elements 16k .. 16k+15, four per byte
      const uint32_t c0 = (gc.w[k] >> 6) & 0x03030303u, c1 = (gc.w[k] >> 4) & 0x03030303u;
      const uint32_t c2 = (gc.w[k] >> 2) & 0x03030303u, c3 = gc.w[k] & 0x03030303u;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[8 * k + 2 * j] = pair(code_plus_2p23(c0, j), code_plus_2p23(c1, j));
        o[8 * k + 2 * j + 1] = pair(code_plus_2p23(c2, j), code_plus_2p23(c3, j));
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) {  // word k: elements 4k .. 4k+3, one per byte
      o[2 * k] = pair(code_plus_2p23(gc.w[k], 0), code_plus_2p23(gc.w[k], 1));
      o[2 * k + 1] = pair(code_plus_2p23(gc.w[k], 2), code_plus_2p23(gc.w[k], 3));
    }
  }
}
template <int BITS>
__device__ __forceinline__ void store_group(const GroupCodes<BITS>& gc, float half, uint16_t* out) {
  uint32_t o[16];
  group_bf16<BITS>(gc, half, o);
  U8 lo, hi;
#pragma unroll
  for (int k = 0; k < 8; ++k) { lo.v[k] = o[k]; hi.v[k] = o[8 + k]; }
  st_cs_v8(out, lo);
  st_cs_v8(out + 16, hi);
}

}  // namespace
}  // namespace ashkv
