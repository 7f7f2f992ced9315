// Dithered N-bit group codec with 3-sigma outlier isolation (sm_100a).
//
// Restates DitheredNBitCodec (ashkv/codecs/nbit_dithered.py:43-167) and
// DitheredINT2Codec (ashkv/codecs/int2_dithered.py:36-147).  The reference
// runs ~10 op-by-op tensor passes plus a nonzero()/host sync per call; here a
// single pass does everything per 32-element group in one thread:
//   load (16-byte streaming loads) -> mean -> fp64 variance -> outlier mask
//   -> inlier absmax -> delta -> dithered quantise -> MSB-first pack ->
//   one vector store of the codes + one bf16 delta store.
// Outliers are ranked with a CTA-wide scan of per-group popcounts, so each
// CTA (256 groups = one "bucket" of 8192 elements) writes its ascending
// outlier list with no global synchronisation.
//
// Arithmetic follows the reference exactly as PyTorch evaluates it on the
// host: every fp32 operation is a separate IEEE operation (no contraction),
// the group mean uses PyTorch's 8-lane partial-sum order, the standard
// deviation is PyTorch's fp64 computation rounded once to fp32, divisions
// are true divisions and rounding is half-to-even.
#include "common.cuh"

namespace ashkv {
namespace {

constexpr int kThreads = ASHKV_NBIT_BUCKET_GROUPS;  // one group per thread, one bucket per CTA

struct NbitEncParams {
  const uint16_t* src;
  int64_t n_groups;
  const float* dither;
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

struct NbitDecParams {
  const uint16_t* scales;
  const uint8_t* codes;
  int64_t n_groups;
  float half_states;
  const uint32_t* bucket_counts;
  const uint32_t* bucket_entries;
  int32_t bucket_cap;
  uint16_t* dst;
  uint32_t* status;
};

// Inclusive scan across the CTA of one uint32 per thread; returns the
// exclusive prefix and writes the CTA total to *total.
__device__ __forceinline__ uint32_t cta_exclusive_scan(uint32_t v, uint32_t* smem_warp, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, inc, off);
    if (lane >= off) inc += n;
  }
  if (lane == 31) smem_warp[warp] = inc;
  __syncthreads();
  uint32_t warp_base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    const uint32_t t = smem_warp[w];
    if (w < warp) warp_base += t;
    tot += t;
  }
  total = tot;
  return warp_base + inc - v;
}

// Exact reference threshold sigma * (sd + 1e-8), sd = fp32(sqrt(M2 / 31)) with
// M2 accumulated in fp64 (two-pass).  Used only when the fast bound below
// cannot decide every element of a group.
__device__ __forceinline__ float exact_threshold(const f2 (&X)[16], float sigma) {
  double s64 = 0.0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    float x0, x1;
    upk2(X[k], x0, x1);
    s64 = __dadd_rn(__dadd_rn(s64, double(x0)), double(x1));
  }
  const double mu64 = __dmul_rn(s64, 0.03125);
  double m2 = 0.0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    float x0, x1;
    upk2(X[k], x0, x1);
    const double d0 = __dadd_rn(double(x0), -mu64);
    m2 = __dadd_rn(m2, __dmul_rn(d0, d0));
    const double d1 = __dadd_rn(double(x1), -mu64);
    m2 = __dadd_rn(m2, __dmul_rn(d1, d1));
  }
  const float sd = __double2float_rn(__dsqrt_rn(__ddiv_rn(m2, 31.0)));
  return __fmul_rn(sigma, __fadd_rn(sd, 1e-8f));
}

// One thread per 32-element group, one CTA (256 groups) per outlier bucket.
//
// Outlier decisions are made against the reference threshold without
// computing its fp64 variance in the common case: an fp32 variance with a
// rigorous error bound gives thr_lo <= thr <= thr_hi.  If every |x - mu| of
// the group is <= thr_lo the group has no outliers (the usual case).
// Otherwise per-element masks against thr_lo and thr_hi are built; if they
// agree, that is the exact mask, and only if some |x - mu| falls between the
// two bounds is the exact fp64 threshold computed.
template <int BITS, int DMODE>
__global__ void __launch_bounds__(kThreads, 2) nbit_encode_kernel(const NbitEncParams p) {
  constexpr uint32_t kMaxCode = (1u << BITS) - 1u;
  __shared__ uint32_t s_warp[kThreads / 32];

  const int64_t g = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = g < p.n_groups;

  // ---- load 32 bf16 as two full 32-byte sectors
  f2 X[16];
  {
    U8 a, b;
    if (active) {
      a = ld_nc_v8(p.src + g * 32);
      b = ld_nc_v8(p.src + g * 32 + 16);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) a.v[k] = b.v[k] = 0u;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      X[k] = pk2(bf16lo(a.v[k]), bf16hi(a.v[k]));
      X[8 + k] = pk2(bf16lo(b.v[k]), bf16hi(b.v[k]));
    }
  }

  // ---- mean: lane accumulators acc[i] = ((x_i + x_{8+i}) + x_{16+i}) + x_{24+i},
  //      then acc[0] + acc[1] + ... + acc[7] in order (PyTorch's CPU order).
  f2 A[4] = {X[0], X[1], X[2], X[3]};
#pragma unroll
  for (int j = 1; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] = add2(A[i], X[4 * j + i]);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) upk2(A[i], acc[2 * i], acc[2 * i + 1]);
  float s = acc[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) s = __fadd_rn(s, acc[i]);
  const float mu = __fmul_rn(s, 0.03125f);

  // ---- fp32 variance estimate, max|x - mu|, max|x| (NaN-propagating)
  const f2 NMU = pk2(-mu, -mu);
  f2 M2 = pk2(0.0f, 0.0f);
  float dmax = 0.0f, xmax = 0.0f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const f2 D = add2(X[k], NMU);
    M2 = fma2(D, D, M2);
    float d0, d1, x0, x1;
    upk2(D, d0, d1);
    upk2(X[k], x0, x1);
    dmax = max3_abs_nan(dmax, d0, d1);
    xmax = max3_abs_nan(xmax, x0, x1);
  }
  float m2a, m2b;
  upk2(M2, m2a, m2b);
  const float m2 = __fadd_rn(m2a, m2b);

  // Bounds on the reference threshold.  m2 has relative error < 2^-19 w.r.t.
  // sum (x - mu32)^2, which exceeds the exact M2 by 32 (mu - mu32)^2 with
  // |mu - mu32| <= 31 * 2^-24 * max|x|.  Margins of 2^-16 / 2^-14 cover the
  // remaining roundings (fp32 bound arithmetic, the fp32 rounding of sd,
  // + 1e-8 and * sigma in the reference).
  const float sigma = p.sigma;
  const bool bounds_ok = sigma > 0.0f && isfinite(m2) && isfinite(xmax);
  float thr_lo = 0.0f, thr_hi = 0.0f;
  if (bounds_ok) {
    const float emu = 31.0001f * 0x1p-24f * xmax;
    const float m2_hi = m2 * (1.0f + 0x1p-16f);
    const float m2_lo = fmaxf(m2 * (1.0f - 0x1p-16f) - 32.0f * emu * emu * (1.0f + 0x1p-16f), 0.0f);
    thr_hi = sigma * (sqrtf(m2_hi / 31.0f) + 1e-8f) * (1.0f + 0x1p-14f);
    thr_lo = sigma * (sqrtf(m2_lo / 31.0f) + 1e-8f) * (1.0f - 0x1p-14f);
  }
  uint32_t omask = 0;
  float am = xmax;
  if (!(bounds_ok && dmax <= thr_lo)) {
    uint32_t mlo = 0, mhi = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      float x0, x1;
      upk2(X[k], x0, x1);
      const float d0 = fabsf(__fadd_rn(x0, -mu)), d1 = fabsf(__fadd_rn(x1, -mu));
      mlo |= (uint32_t(d0 > thr_lo) << (2 * k)) | (uint32_t(d1 > thr_lo) << (2 * k + 1));
      mhi |= (uint32_t(d0 > thr_hi) << (2 * k)) | (uint32_t(d1 > thr_hi) << (2 * k + 1));
    }
    omask = mhi;
    if (!bounds_ok || mlo != mhi) {
      const float thr = exact_threshold(X, sigma);
      omask = 0;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        float x0, x1;
        upk2(X[k], x0, x1);
        omask |= (uint32_t(fabsf(__fadd_rn(x0, -mu)) > thr) << (2 * k)) |
                 (uint32_t(fabsf(__fadd_rn(x1, -mu)) > thr) << (2 * k + 1));
      }
    }
    if (omask) {
      am = 0.0f;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        float x0, x1;
        upk2(X[k], x0, x1);
        x0 = (omask >> (2 * k)) & 1u ? mu : x0;
        x1 = (omask >> (2 * k + 1)) & 1u ? mu : x1;
        X[k] = pk2(x0, x1);
        am = max3_abs_nan(am, x0, x1);
      }
    }
  }
  if (!active) omask = 0;
  if (!(am >= 1e-8f) && am == am) am = 1e-8f;  // clamp(min=1e-8); NaN propagates
  const float delta = __fdiv_rn(am, p.half_states);

  // ---- dither, quantise (x' + (U-0.5)*delta) / delta + half, pack
  const Recip y = make_recip(delta);
  const bool fast_div = recip_ok(delta);
  const f2 DELTA = pk2(delta, delta), YHI = pk2(y.hi, y.hi), YLO = pk2(y.lo, y.lo), NDELTA = pk2(-delta, -delta);
  const f2 HALF = pk2(p.half_states, p.half_states);
  const f2 MAGIC = pk2(12582912.0f, 12582912.0f);
  const f2 C128 = pk2(128.0f, 128.0f), CM = pk2(-128.5f, -128.5f), NHALF = pk2(-0.5f, -0.5f);
  // packed codes: 32 * BITS / 32 words (MSB-first within each byte)
  uint32_t o[BITS];
#pragma unroll
  for (int k = 0; k < BITS; ++k) o[k] = 0u;
#pragma unroll
  for (int c = 0; c < 4; ++c) {  // 8 elements per Philox draw
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
        DZ[h] = add2(pk2(__uint_as_float(u.v[2 * h]), __uint_as_float(u.v[2 * h + 1])), NHALF);
    } else {
      const uint64_t ctr = ((p.dither_offset + uint64_t(g) * 32) >> 3) + c;
      const Philox4 r = philox4x32_10(uint32_t(ctr), uint32_t(ctr >> 32), 0u, 0u, uint32_t(p.seed),
                                      uint32_t(p.seed >> 32));
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // f = 1 + h16 * 2^-23; U - 0.5 = 128 f - 128.5 exactly
        const float flo = __uint_as_float(__byte_perm(r.v[h], 0x3F800000u, 0x7610));
        const float fhi = __uint_as_float(__byte_perm(r.v[h], 0x3F800000u, 0x7632));
        DZ[h] = fma2(pk2(flo, fhi), C128, CM);
      }
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int k = 4 * c + h;
      const f2 A2 = add2(X[k], mul2(DZ[h], DELTA));
      f2 Q;
      if (fast_div) {
        Q = div2_rn(A2, YHI, YLO, NDELTA);
      } else {
        float a0, a1;
        upk2(A2, a0, a1);
        Q = pk2(__fdiv_rn(a0, delta), __fdiv_rn(a1, delta));
      }
      float v0, v1;
      upk2(add2(Q, HALF), v0, v1);
      v0 = fminf(fmaxf(v0, 0.0f), float(kMaxCode));  // NaN -> 0
      v1 = fminf(fmaxf(v1, 0.0f), float(kMaxCode));
      float t0, t1;
      upk2(add2(pk2(v0, v1), MAGIC), t0, t1);
      const uint32_t c0 = __float_as_uint(t0) & kMaxCode, c1 = __float_as_uint(t1) & kMaxCode;
      // element e = 2k (+1) sits in byte e*BITS/8, MSB first within the byte
      if constexpr (BITS == 4) {
        o[k >> 2] |= ((c0 << 4) | c1) << (8 * (k & 3));
      } else if constexpr (BITS == 2) {
        const int e = 2 * k;  // even: the pair shares a byte
        o[e >> 4] |= ((c0 << (6 - 2 * (e & 3))) | (c1 << (4 - 2 * (e & 3)))) << (8 * ((e >> 2) & 3));
      } else {
        o[k >> 1] |= (c0 | (c1 << 8)) << (16 * (k & 1));
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

  // ---- outlier list of this bucket, ascending element order.
  const uint32_t cnt = uint32_t(__popc(omask));
  uint32_t total = 0;
  uint32_t pos = cta_exclusive_scan(cnt, s_warp, total);
  if (threadIdx.x == 0) {
    p.bucket_counts[blockIdx.x] = total;
    if (total > uint32_t(p.bucket_cap)) atomicOr(p.status, ASHKV_FLAG_OUTLIER_OVERFLOW);
  }
  if (cnt) {
    uint32_t* out = p.bucket_entries + int64_t(blockIdx.x) * p.bucket_cap;
    uint32_t m = omask;
    while (m) {
      const int i = __ffs(m) - 1;
      m &= m - 1;
      if (pos < uint32_t(p.bucket_cap)) {
        const uint32_t local = uint32_t(threadIdx.x) * 32u + uint32_t(i);
        out[pos] = (local << 16) | uint32_t(p.src[g * 32 + i]);  // original bits (rare path)
      }
      ++pos;
    }
  }
}

template <int BITS>
__device__ __forceinline__ void unpack_codes(const uint8_t* codes, int64_t g, uint32_t (&code)[32]) {
  if constexpr (BITS == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(codes + g * 16);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b = (w[k] >> (8 * j)) & 0xFFu;
        code[8 * k + 2 * j] = b >> 4;
        code[8 * k + 2 * j + 1] = b & 0xFu;
      }
  } else if constexpr (BITS == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(codes + g * 8);
    const uint32_t w[2] = {v.x, v.y};
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b = (w[k] >> (8 * j)) & 0xFFu;
        const int i = 16 * k + 4 * j;
        code[i] = b >> 6; code[i + 1] = (b >> 4) & 3u; code[i + 2] = (b >> 2) & 3u; code[i + 3] = b & 3u;
      }
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(codes + g * 32);
    const uint4 b = *reinterpret_cast<const uint4*>(codes + g * 32 + 16);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) code[4 * k + j] = (w[k] >> (8 * j)) & 0xFFu;
  }
}

template <int BITS>
__device__ __forceinline__ void dequant_group(const uint16_t* scales, const uint8_t* codes, int64_t g,
                                              float half, uint16_t* dst) {
  uint32_t code[32];
  unpack_codes<BITS>(codes, g, code);
  const float delta = bf16_to_f32(scales[g]);
  uint32_t o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float a = __fmul_rn(__fadd_rn(float(code[2 * i]), -half), delta);
    const float b = __fmul_rn(__fadd_rn(float(code[2 * i + 1]), -half), delta);
    o[i] = f32x2_to_bf16x2(a, b);
  }
  uint16_t* out = dst + g * 32;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    st_cs_v4(out + 8 * k, make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]));
}

template <int BITS>
__global__ void __launch_bounds__(kThreads) nbit_decode_kernel(const NbitDecParams p) {
  const int64_t g = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (g < p.n_groups) dequant_group<BITS>(p.scales, p.codes, g, p.half_states, p.dst);
  if (!p.bucket_counts) return;
  __syncthreads();  // the bucket's dense values are stored before its outliers overwrite them
  const uint32_t n = min(p.bucket_counts[blockIdx.x], uint32_t(p.bucket_cap));
  const uint32_t* ent = p.bucket_entries + int64_t(blockIdx.x) * p.bucket_cap;
  const int64_t base = int64_t(blockIdx.x) * ASHKV_NBIT_BUCKET_ELEMS;
  const int64_t n_elems = p.n_groups * 32;
  for (uint32_t j = threadIdx.x; j < n; j += kThreads) {
    const uint32_t e = ent[j];
    const int64_t idx = base + (e >> 16);
    if (idx < n_elems) p.dst[idx] = uint16_t(e & 0xFFFFu);
    else atomicOr(p.status, ASHKV_FLAG_INDEX_RANGE);
  }
}

template <int BITS>
__global__ void __launch_bounds__(kThreads) nbit_dequant_kernel(const uint16_t* scales, const uint8_t* codes,
                                                                int64_t n_groups, float half, uint16_t* dst) {
  const int64_t g = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (g < n_groups) dequant_group<BITS>(scales, codes, g, half, dst);
}

__global__ void __launch_bounds__(256) scatter_outliers_kernel(const int32_t* idx, const uint16_t* val, int64_t n,
                                                               int64_t n_elems, uint16_t* dst, uint32_t* status) {
  for (int64_t k = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; k < n; k += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = idx[k];
    if (i >= 0 && i < n_elems) dst[i] = val[k];
    else atomicOr(status, ASHKV_FLAG_INDEX_RANGE);
  }
}

// Single-CTA exclusive scan over bucket counts (clamped to the capacity).
__global__ void __launch_bounds__(1024) bucket_scan_kernel(const uint32_t* counts, int32_t cap, int64_t n,
                                                           uint32_t* offsets, uint32_t* total) {
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < n; base += 1024) {
    const int64_t i = base + threadIdx.x;
    const uint32_t v = i < n ? min(counts[i], uint32_t(cap)) : 0u;
    uint32_t inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, off);
      if (lane >= off) inc += t;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    uint32_t wbase = 0, tile = 0;
    for (int w = 0; w < 32; ++w) {
      const uint32_t t = s_warp[w];
      if (w < warp) wbase += t;
      tile += t;
    }
    const uint32_t carry = s_carry;
    if (i < n) offsets[i] = carry + wbase + inc - v;
    __syncthreads();
    if (threadIdx.x == 0) s_carry = carry + tile;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    offsets[n] = s_carry;
    *total = s_carry;
  }
}

__global__ void __launch_bounds__(256) bucket_flatten_kernel(const uint32_t* counts, const uint32_t* entries,
                                                             int32_t cap, const uint32_t* offsets,
                                                             int32_t* out_idx, uint16_t* out_val) {
  const int64_t b = blockIdx.x;
  const uint32_t n = min(counts[b], uint32_t(cap));
  const uint32_t off = offsets[b];
  const uint32_t* ent = entries + b * cap;
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
    const uint32_t e = ent[j];
    out_idx[off + j] = int32_t(b * ASHKV_NBIT_BUCKET_ELEMS + (e >> 16));
    out_val[off + j] = uint16_t(e & 0xFFFFu);
  }
}

float half_states_for(int bits) { return float((1 << bits) - 1) / 2.0f; }

}  // namespace
}  // namespace ashkv

using namespace ashkv;

extern "C" ashkv_status_t ashkv_nbit_encode(
    const void* d_src, int64_t n_groups, int32_t bits, float sigma,
    int32_t dither_mode, const float* d_dither, uint64_t seed, uint64_t dither_elem_offset,
    void* d_scales, void* d_codes,
    uint32_t* d_bucket_counts, uint32_t* d_bucket_entries, int32_t bucket_cap,
    uint32_t* d_status, void* stream) {
  if (n_groups < 0 || bucket_cap < 0) return ASHKV_BAD_ARGUMENT;
  if (bits != 2 && bits != 4 && bits != 8) return ASHKV_BAD_ARGUMENT;
  if (dither_mode != ASHKV_DITHER_TENSOR && dither_mode != ASHKV_DITHER_PHILOX) return ASHKV_BAD_ARGUMENT;
  if (n_groups == 0) return ASHKV_OK;
  if (!d_src || !d_scales || !d_codes || !d_bucket_counts || !d_status) return ASHKV_BAD_ARGUMENT;
  if (bucket_cap > 0 && !d_bucket_entries) return ASHKV_BAD_ARGUMENT;
  if (dither_mode == ASHKV_DITHER_TENSOR && !d_dither) return ASHKV_BAD_ARGUMENT;
  if (dither_mode == ASHKV_DITHER_PHILOX && (dither_elem_offset % 8)) return ASHKV_BAD_ARGUMENT;
  // 16-byte vector accesses; the 2-bit codes use 8-byte stores.
  // 32-byte vector loads of the source and dither; 8/16/32-byte code stores.
  if (!aligned(d_src, 32) || !aligned(d_scales, 2) || !aligned(d_codes, bits == 2 ? 8 : bits == 4 ? 16 : 32))
    return ASHKV_BAD_ARGUMENT;
  if (dither_mode == ASHKV_DITHER_TENSOR && !aligned(d_dither, 32)) return ASHKV_BAD_ARGUMENT;
  const int64_t n_buckets = (n_groups + kThreads - 1) / kThreads;
  if (n_buckets > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;

  NbitEncParams p;
  p.src = static_cast<const uint16_t*>(d_src); p.n_groups = n_groups;
  p.dither = d_dither; p.seed = seed; p.dither_offset = dither_elem_offset;
  p.sigma = sigma; p.half_states = half_states_for(bits);
  p.scales = static_cast<uint16_t*>(d_scales); p.codes = static_cast<uint8_t*>(d_codes);
  p.bucket_counts = d_bucket_counts; p.bucket_entries = d_bucket_entries; p.bucket_cap = bucket_cap;
  p.status = d_status;

  cudaStream_t st = as_stream(stream);
  const dim3 grid{unsigned(n_buckets)}, block{unsigned(kThreads)};
  if (dither_mode == ASHKV_DITHER_TENSOR) {
    if (bits == 2) nbit_encode_kernel<2, ASHKV_DITHER_TENSOR><<<grid, block, 0, st>>>(p);
    else if (bits == 4) nbit_encode_kernel<4, ASHKV_DITHER_TENSOR><<<grid, block, 0, st>>>(p);
    else nbit_encode_kernel<8, ASHKV_DITHER_TENSOR><<<grid, block, 0, st>>>(p);
  } else {
    if (bits == 2) nbit_encode_kernel<2, ASHKV_DITHER_PHILOX><<<grid, block, 0, st>>>(p);
    else if (bits == 4) nbit_encode_kernel<4, ASHKV_DITHER_PHILOX><<<grid, block, 0, st>>>(p);
    else nbit_encode_kernel<8, ASHKV_DITHER_PHILOX><<<grid, block, 0, st>>>(p);
  }
  return check_launch("nbit_encode");
}

extern "C" ashkv_status_t ashkv_nbit_decode(
    const void* d_scales, const void* d_codes, int64_t n_groups, int32_t bits,
    const uint32_t* d_bucket_counts, const uint32_t* d_bucket_entries, int32_t bucket_cap,
    void* d_dst, uint32_t* d_status, void* stream) {
  if (n_groups < 0 || bucket_cap < 0) return ASHKV_BAD_ARGUMENT;
  if (bits != 2 && bits != 4 && bits != 8) return ASHKV_BAD_ARGUMENT;
  if (n_groups == 0) return ASHKV_OK;
  if (!d_scales || !d_codes || !d_dst) return ASHKV_BAD_ARGUMENT;
  if (d_bucket_counts && (!d_status || (bucket_cap > 0 && !d_bucket_entries))) return ASHKV_BAD_ARGUMENT;
  if (!aligned(d_dst, 16) || !aligned(d_scales, 2) || !aligned(d_codes, bits == 2 ? 8 : 16))
    return ASHKV_BAD_ARGUMENT;
  const int64_t n_buckets = (n_groups + kThreads - 1) / kThreads;
  if (n_buckets > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;

  NbitDecParams p;
  p.scales = static_cast<const uint16_t*>(d_scales); p.codes = static_cast<const uint8_t*>(d_codes);
  p.n_groups = n_groups; p.half_states = half_states_for(bits);
  p.bucket_counts = d_bucket_counts; p.bucket_entries = d_bucket_entries; p.bucket_cap = bucket_cap;
  p.dst = static_cast<uint16_t*>(d_dst); p.status = d_status;
  cudaStream_t st = as_stream(stream);
  const dim3 grid{unsigned(n_buckets)}, block{unsigned(kThreads)};
  if (bits == 2) nbit_decode_kernel<2><<<grid, block, 0, st>>>(p);
  else if (bits == 4) nbit_decode_kernel<4><<<grid, block, 0, st>>>(p);
  else nbit_decode_kernel<8><<<grid, block, 0, st>>>(p);
  return check_launch("nbit_decode");
}

extern "C" ashkv_status_t ashkv_nbit_outliers_flatten(
    const uint32_t* d_bucket_counts, const uint32_t* d_bucket_entries, int32_t bucket_cap,
    int64_t n_buckets, uint32_t* d_offsets,
    int32_t* d_out_index, uint16_t* d_out_value, uint32_t* d_total, void* stream) {
  if (n_buckets < 0 || bucket_cap < 0) return ASHKV_BAD_ARGUMENT;
  if (!d_offsets || !d_total) return ASHKV_BAD_ARGUMENT;
  if (n_buckets > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  if (n_buckets == 0) {
    if (cudaMemsetAsync(d_total, 0, sizeof(uint32_t), st) != cudaSuccess ||
        cudaMemsetAsync(d_offsets, 0, sizeof(uint32_t), st) != cudaSuccess)
      return check_launch("nbit_flatten_memset");
    return ASHKV_OK;
  }
  if (!d_bucket_counts || (bucket_cap > 0 && (!d_bucket_entries || !d_out_index || !d_out_value)))
    return ASHKV_BAD_ARGUMENT;
  bucket_scan_kernel<<<1, 1024, 0, st>>>(d_bucket_counts, bucket_cap, n_buckets, d_offsets, d_total);
  ashkv_status_t s = check_launch("nbit_bucket_scan");
  if (s != ASHKV_OK || bucket_cap == 0) return s;
  bucket_flatten_kernel<<<unsigned(n_buckets), 256, 0, st>>>(d_bucket_counts, d_bucket_entries, bucket_cap,
                                                             d_offsets, d_out_index, d_out_value);
  return check_launch("nbit_bucket_flatten");
}

extern "C" ashkv_status_t ashkv_nbit_decode_flat(
    const void* d_scales, const void* d_codes, int64_t n_groups, int32_t bits,
    const int32_t* d_out_index, const uint16_t* d_out_value, int64_t n_outliers,
    void* d_dst, uint32_t* d_status, void* stream) {
  if (n_groups < 0 || n_outliers < 0) return ASHKV_BAD_ARGUMENT;
  if (bits != 2 && bits != 4 && bits != 8) return ASHKV_BAD_ARGUMENT;
  if (n_groups == 0) return ASHKV_OK;
  if (!d_scales || !d_codes || !d_dst) return ASHKV_BAD_ARGUMENT;
  if (n_outliers > 0 && (!d_out_index || !d_out_value || !d_status)) return ASHKV_BAD_ARGUMENT;
  if (!aligned(d_dst, 16) || !aligned(d_scales, 2) || !aligned(d_codes, bits == 2 ? 8 : 16))
    return ASHKV_BAD_ARGUMENT;
  const int64_t n_blocks = (n_groups + kThreads - 1) / kThreads;
  if (n_blocks > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  const float half = half_states_for(bits);
  const auto* sc = static_cast<const uint16_t*>(d_scales);
  const auto* cd = static_cast<const uint8_t*>(d_codes);
  auto* dst = static_cast<uint16_t*>(d_dst);
  if (bits == 2) nbit_dequant_kernel<2><<<unsigned(n_blocks), kThreads, 0, st>>>(sc, cd, n_groups, half, dst);
  else if (bits == 4) nbit_dequant_kernel<4><<<unsigned(n_blocks), kThreads, 0, st>>>(sc, cd, n_groups, half, dst);
  else nbit_dequant_kernel<8><<<unsigned(n_blocks), kThreads, 0, st>>>(sc, cd, n_groups, half, dst);
  ashkv_status_t s = check_launch("nbit_dequant");
  if (s != ASHKV_OK || n_outliers == 0) return s;
  const int64_t want = (n_outliers + 255) / 256;
  const unsigned blocks = unsigned(want < 4096 ? want : 4096);
  scatter_outliers_kernel<<<blocks, 256, 0, st>>>(d_out_index, d_out_value, n_outliers, n_groups * 32, dst, d_status);
  return check_launch("nbit_scatter_outliers");
}
