// Dithered N-bit group codec with 3-sigma outlier isolation (sm_100a).
//
// Restates DitheredNBitCodec (ashkv/codecs/nbit_dithered.py:43-167) and
// DitheredINT2Codec (ashkv/codecs/int2_dithered.py:36-147).  The reference
// runs ~10 op-by-op tensor passes plus a nonzero()/host sync per call; here a
// single pass does everything per 32-element group in one thread:
//   load (16-byte streaming loads) -> mean -> fp64 variance -> outlier mask
//   -> inlier absmax -> delta -> dithered quantise -> MSB-first pack ->
//   one vector store of the codes + one bf16 delta store.
// Outliers are ranked with a warp scan of per-group popcounts: each warp's
// 32 groups form one "bucket" of 1024 elements whose ascending outlier list
// the warp writes with no CTA or global synchronisation.
//
// Arithmetic follows the reference exactly as PyTorch evaluates it on the
// host: every fp32 operation is a separate IEEE operation (no contraction),
// the group mean uses PyTorch's 8-lane partial-sum order, the standard
// deviation is PyTorch's fp64 computation rounded once to fp32, divisions
// are true divisions and rounding is half-to-even.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace ashkv {
namespace {

constexpr int kThreads = 256;                     // 8 warps per CTA
constexpr int kWarps = kThreads / 32;
static_assert(ASHKV_NBIT_BUCKET_GROUPS == 32, "one bucket per warp, one group per lane");

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

// One thread per 32-element group, one warp (32 groups) per outlier bucket.
//
// Outlier decisions are made against the reference threshold without
// computing its fp64 variance in the common case: an fp32 variance with a
// rigorous error bound gives thr_lo <= thr <= thr_hi.  If every |x - mu| of
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

__device__ __forceinline__ double warp_sum_f64(double v) {  // pairwise (butterfly) order, same in every lane
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) v = __dadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  return v;
}
__device__ __forceinline__ float warp_max_abs_nan(float v) {
  v = fabsf(v);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = max_nan(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  return v;
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
// outlier bit mask.  The group is re-read from `src` for each pass so only
// one 8-element chunk is live in registers at a time.
template <int BITS, int DMODE, typename Src>
__device__ __forceinline__ uint32_t encode_group(const Src& src, const NbitEncParams& p, int64_t g, bool active) {
  constexpr uint32_t kMaxCode = (1u << BITS) - 1u;
  // ---- mean: acc[i] = ((x_i + x_{8+i}) + x_{16+i}) + x_{24+i}, then acc[0] + ... + acc[7]
  //      in order (PyTorch's CPU reduction order for a 32-wide inner dimension).
  f2 A[4];
  chunk_pairs(src, 0, A);
#pragma unroll
  for (int c = 1; c < 4; ++c) {
    f2 P[4];
    chunk_pairs(src, c, P);
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] = add2(A[i], P[i]);
  }
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
  for (int c = 0; c < 4; ++c) {
    f2 P[4];
    chunk_pairs(src, c, P);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const f2 D = add2(P[i], NMU);
      M2 = fma2(D, D, M2);
      float d0, d1, x0, x1;
      upk2(D, d0, d1);
      upk2(P[i], x0, x1);
      dmax = max3_abs_nan(dmax, d0, d1);
      xmax = max3_abs_nan(xmax, x0, x1);
    }
  }
  float m2a, m2b;
  upk2(M2, m2a, m2b);
  const float m2 = __fadd_rn(m2a, m2b);

  // Bounds on the reference threshold.  m2 has relative error < 2^-19 w.r.t.
  // sum (x - mu32)^2, which exceeds the exact M2 by 32 (mu - mu32)^2 with
  // |mu - mu32| <= 31 * 2^-24 * max|x|.  The bounds only choose between the
  // fast and the exact outlier path, so they are evaluated with approximate
  // operations: the product by RN(1/31) and sqrt.approx each err by less than
  // 2^-21 relative (a flushed subnormal only lowers a bound by far less than
  // the 1e-8 term's margin), and margins of 2^-16 on m2 and 2^-12 on the
  // threshold cover them together with the other roundings (fp32 bound
  // arithmetic, the fp32 rounding of sd, + 1e-8 and * sigma in the reference).
  const float sigma = p.sigma;
  const bool bounds_ok = sigma > 0.0f && isfinite(m2) && isfinite(xmax);
  float thr_lo = 0.0f, thr_hi = 0.0f;
  if (bounds_ok) {
    const float emu = 31.0001f * 0x1p-24f * xmax;
    const float m2_hi = m2 * (1.0f + 0x1p-16f);
    const float m2_lo = fmaxf(m2 * (1.0f - 0x1p-16f) - 32.0f * emu * emu * (1.0f + 0x1p-16f), 0.0f);
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
  const float delta = __fdiv_rn(am, p.half_states);

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
  for (int c = 0; c < 4; ++c) {  // 8 elements per chunk / Philox draw
    f2 P[4];
    chunk_pairs(src, c, P);
    if (omask & (0xFFu << (8 * c))) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float x0, x1;
        upk2(P[i], x0, x1);
        const int e = 8 * c + 2 * i;
        P[i] = pk2((omask >> e) & 1u ? mu : x0, (omask >> (e + 1)) & 1u ? mu : x1);
      }
    }
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
      const uint64_t ctr = ((p.dither_offset + uint64_t(g) * 32) >> 3) + c;
      const Philox4 r = philox4x32_10_rk(uint32_t(ctr), uint32_t(ctr >> 32), 0u, 0u, p.round_keys);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // f = 1 + h16 * 2^-23, so U - 0.5 = 128 f - 128.5 exactly
        const float flo = __uint_as_float(__byte_perm(r.v[h], 0x3F800000u, 0x7610));
        const float fhi = __uint_as_float(__byte_perm(r.v[h], 0x3F800000u, 0x7632));
        DZ[h] = fma2(pk2(flo, fhi), pk2(128.0f, 128.0f), pk2(-128.5f, -128.5f));
      }
    }
    // v = RN(RN(a / delta) + half), a = x' + noise; code = clamp(rint(v), 0, 2^bits - 1).
    // rint: RN(v + 1.5 * 2^23) leaves rint(v) in the low mantissa bits (|v| < 2^22).
    // With delta in Markstein's range every a is finite and |a / delta| <= half + 1,
    // so the clamp runs on the integers (two codes per s16x2 word); otherwise the
    // float clamp comes first (NaN -> 0), as in the reference.
    f2 Q[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) Q[h] = add2(P[h], mul2(DZ[h], DELTA));  // a = x' + noise
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

// Append this lane's outliers (bits of omask) to the warp's bucket; the
// ranks come from a warp scan, so the list is in ascending element order.
// Called by all 32 lanes; inactive lanes pass omask = 0.
__device__ __forceinline__ void write_outliers(const NbitEncParams& p, int64_t bucket, int64_t g, uint32_t omask) {
  const int lane = threadIdx.x & 31;
  if (!__any_sync(0xFFFFFFFFu, omask != 0)) {  // the common case: no outliers in the bucket
    if (lane == 0) p.bucket_counts[bucket] = 0;
    return;
  }
  const uint32_t cnt = uint32_t(__popc(omask));
  uint32_t inc = cnt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, off);
    if (lane >= off) inc += t;
  }
  const uint32_t total = __shfl_sync(0xFFFFFFFFu, inc, 31);
  uint32_t pos = inc - cnt;
  if (lane == 0) {
    p.bucket_counts[bucket] = total;
    if (total > uint32_t(p.bucket_cap)) atomicOr(p.status, ASHKV_FLAG_OUTLIER_OVERFLOW);
  }
  if (cnt) {
    uint32_t* out = p.bucket_entries + bucket * p.bucket_cap;
    uint32_t m = omask;
    while (m) {
      const int i = __ffs(m) - 1;
      m &= m - 1;
      if (pos < uint32_t(p.bucket_cap)) {
        const uint32_t local = uint32_t(lane) * 32u + uint32_t(i);
        out[pos] = (local << 16) | uint32_t(p.src[g * 32 + i]);  // original bits (rare path)
      }
      ++pos;
    }
  }
}

// Direct-load variant: each warp encodes one bucket, each lane loads its
// 64-byte group with two 256-bit loads.  Used when a tensor map cannot be built.
template <int BITS, int DMODE>
__global__ void __launch_bounds__(kThreads, 2) nbit_encode_kernel(const NbitEncParams p) {
  const int64_t g = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = g < p.n_groups;
  uint32_t w[16];
  if (active) {
    const U8 a = ld_nc_v8(p.src + g * 32);
    const U8 b = ld_nc_v8(p.src + g * 32 + 16);
#pragma unroll
    for (int k = 0; k < 8; ++k) { w[k] = a.v[k]; w[8 + k] = b.v[k]; }
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) w[k] = 0u;
  }
  const int64_t g0 = g - (threadIdx.x & 31);
  if (g0 >= p.n_groups) return;  // whole warp past the end
  const uint32_t omask = encode_group<BITS, DMODE>(RegGroup{w, p.src, g0}, p, g, active);
  write_outliers(p, g0 / 32, g, omask);
}

constexpr int kTileBytes = 32 * 64;            // one bucket of bf16 = 2 KiB
constexpr uint32_t kMaxPolls = 1u << 24;       // bounded mbarrier waits

// Persistent TMA variant with one pipeline per warp: warp w of CTA c walks
// buckets b = (c * kWarps + w) + i * (gridDim.x * kWarps).  A 2-D tensor map
// views the source as [n_groups, 32] bf16; one TMA copy brings a bucket
// (32 rows of 64 bytes) into one of the warp's STAGES shared-memory stages
// with the 64-byte swizzle (16-byte chunk k of row r stored at chunk
// k ^ ((r >> 1) & 3)), so the 8 lanes of each shared-memory phase hit 8
// distinct bank groups when they read their own row.  Lane 0 refills a stage
// once the warp has encoded its bucket; warps never wait for one another.
template <int BITS, int DMODE, int STAGES>
__global__ void __launch_bounds__(kThreads, 4) nbit_encode_tma_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                       const NbitEncParams p, int64_t n_buckets) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kWarps][STAGES];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t* my_tiles = tiles + warp * (STAGES * kTileBytes);
  uint64_t* bar = full[warp];
  const int64_t first = int64_t(blockIdx.x) * kWarps + warp, step = int64_t(gridDim.x) * kWarps;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(&bar[s], 1);
    mbar_init_fence();
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      const int64_t b = first + int64_t(s) * step;
      if (b < n_buckets) {
        mbar_arrive_expect_tx(&bar[s], kTileBytes);
        tma_load_2d(my_tiles + s * kTileBytes, &tmap, &bar[s], 0, int32_t(b * 32));
      }
    }
  }
  __syncwarp();
  const uint32_t sw = uint32_t(lane >> 1) & 3u;
  for (int64_t it = 0;; ++it) {
    const int64_t b = first + it * step;
    if (b >= n_buckets) break;
    const int s = int(it % STAGES);
    const uint32_t parity = uint32_t(it / STAGES) & 1u;
    const bool ok = mbar_wait_bounded(&bar[s], parity, kMaxPolls);
    if (!__all_sync(0xFFFFFFFFu, ok)) {
      // Give up: flag it, let this warp's copies already issued land, and leave.
      if (lane == 0) {
        atomicOr(p.status, ASHKV_FLAG_TIMEOUT);
        for (int k = 0; k < STAGES; ++k) {
          const int64_t i2 = it + k;
          if (first + i2 * step < n_buckets)
            mbar_wait_bounded(&bar[i2 % STAGES], uint32_t(i2 / STAGES) & 1u, kMaxPolls);
        }
      }
      return;
    }
    const int64_t g = b * 32 + lane;
    const bool active = g < p.n_groups;
    const uint32_t tile = smem_u32(my_tiles + s * kTileBytes);
    const SmemGroup src{tile, tile + uint32_t(lane) * 64u, sw};
    const uint32_t omask = encode_group<BITS, DMODE>(src, p, g, active);
    write_outliers(p, b, g, omask);
    __syncwarp();  // every lane is done with stage s
    if (lane == 0) {
      const int64_t nb = b + int64_t(STAGES) * step;
      if (nb < n_buckets) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&bar[s], kTileBytes);
        tma_load_2d(my_tiles + s * kTileBytes, &tmap, &bar[s], 0, int32_t(nb * 32));
      }
    }
  }
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
__device__ __forceinline__ void store_group(const GroupCodes<BITS>& gc, float half, uint16_t* out) {
  const f2 DEL = pk2(gc.delta, gc.delta), NH = pk2(-half, -half), N23 = pk2(-8388608.0f, -8388608.0f);
  uint32_t o[16];
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
  U8 lo, hi;
#pragma unroll
  for (int k = 0; k < 8; ++k) { lo.v[k] = o[k]; hi.v[k] = o[8 + k]; }
  st_cs_v8(out, lo);
  st_cs_v8(out + 16, hi);
}

template <int BITS>
__device__ __forceinline__ void dequant_group(const uint16_t* scales, const uint8_t* codes, int64_t g,
                                              float half, uint16_t* dst) {
  GroupCodes<BITS> gc;
  load_group<BITS>(scales, codes, g, gc);
  store_group<BITS>(gc, half, dst + g * 32);
}

// Overwrite bucket b's outliers (after its dense values are stored); one warp.
__device__ __forceinline__ void scatter_bucket(const NbitDecParams& p, int64_t bucket, uint32_t count) {
  const uint32_t n = min(count, uint32_t(p.bucket_cap));
  const uint32_t* ent = p.bucket_entries + bucket * p.bucket_cap;
  const int64_t base = bucket * ASHKV_NBIT_BUCKET_ELEMS;
  const int64_t n_elems = p.n_groups * 32;
  for (uint32_t j = threadIdx.x & 31; j < n; j += 32) {
    const uint32_t e = ent[j];
    const int64_t idx = base + (e >> 16);
    if (idx < n_elems) p.dst[idx] = uint16_t(e & 0xFFFFu);
    else atomicOr(p.status, ASHKV_FLAG_INDEX_RANGE);
  }
}

// Two groups per lane (g and g + kThreads; both loads issued before either is
// converted), so each warp covers buckets w and w + kWarps of its CTA's 16;
// after a warp barrier it overwrites those buckets' outliers.
template <int BITS>
__global__ void __launch_bounds__(kThreads) nbit_decode_kernel(const NbitDecParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t ga = int64_t(blockIdx.x) * (2 * kThreads) + threadIdx.x, gb = ga + kThreads;
  const int64_t bucket_a = (ga - lane) / 32, bucket_b = (gb - lane) / 32;
  const bool has_a = bucket_a * 32 < p.n_groups, has_b = bucket_b * 32 < p.n_groups;  // warp-uniform
  // the buckets' counts are fetched first so their latency overlaps the dequantisation
  const uint32_t count_a = (p.bucket_counts && has_a) ? p.bucket_counts[bucket_a] : 0u;
  const uint32_t count_b = (p.bucket_counts && has_b) ? p.bucket_counts[bucket_b] : 0u;
  GroupCodes<BITS> a, b;
  if (ga < p.n_groups) load_group<BITS>(p.scales, p.codes, ga, a);
  if (gb < p.n_groups) load_group<BITS>(p.scales, p.codes, gb, b);
  if (ga < p.n_groups) store_group<BITS>(a, p.half_states, p.dst + ga * 32);
  if (gb < p.n_groups) store_group<BITS>(b, p.half_states, p.dst + gb * 32);
  if (!p.bucket_counts) return;
  __syncwarp();  // the buckets' dense values are stored before their outliers overwrite them
  if (has_a) scatter_bucket(p, bucket_a, count_a);
  if (has_b) scatter_bucket(p, bucket_b, count_b);
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

// Outlier-list scan in three phases: each CTA scans a tile of kScanTile
// bucket counts (clamped to the capacity) into tile-relative offsets and a
// tile total; one CTA scans the tile totals; the flatten kernel adds the
// tile's base.  Tile totals live after the n_buckets + 1 offsets.
constexpr int kScanTile = 4096;  // 1024 threads x 4 buckets

__device__ __forceinline__ uint32_t block_exclusive_scan_1024(uint32_t v, uint32_t* s_warp, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, off);
    if (lane >= off) inc += t;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = s_warp[lane];
    uint32_t wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, wi, off);
      if (lane >= off) wi += t;
    }
    s_warp[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) s_warp[32] = wi;
  }
  __syncthreads();
  total = s_warp[32];
  return s_warp[warp] + inc - v;
}

__global__ void __launch_bounds__(1024) bucket_scan_tiles_kernel(const uint32_t* counts, int32_t cap, int64_t n,
                                                                 uint32_t* offsets, uint32_t* tile_totals) {
  __shared__ uint32_t s_warp[33];
  const int64_t base = int64_t(blockIdx.x) * kScanTile + int64_t(threadIdx.x) * 4;
  uint32_t v[4], local = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = base + k < n ? min(counts[base + k], uint32_t(cap)) : 0u;
    local += v[k];
  }
  uint32_t total;
  uint32_t run = block_exclusive_scan_1024(local, s_warp, total);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (base + k < n) offsets[base + k] = run;
    run += v[k];
  }
  if (threadIdx.x == 0) tile_totals[blockIdx.x] = total;
}

// Exclusive scan of the tile totals in place (one CTA); writes the grand total.
__global__ void __launch_bounds__(1024) tile_scan_kernel(uint32_t* tile_totals, int64_t n_tiles, uint32_t* end,
                                                         uint32_t* total_out) {
  __shared__ uint32_t s_warp[33];
  uint32_t carry = 0;
  for (int64_t b0 = 0; b0 < n_tiles; b0 += 1024) {
    const int64_t i = b0 + threadIdx.x;
    const uint32_t v = i < n_tiles ? tile_totals[i] : 0u;
    uint32_t chunk;
    const uint32_t ex = block_exclusive_scan_1024(v, s_warp, chunk);
    if (i < n_tiles) tile_totals[i] = carry + ex;
    carry += chunk;
    __syncthreads();  // s_warp is reused by the next chunk
  }
  if (threadIdx.x == 0) {
    *end = carry;
    *total_out = carry;
  }
}

// One warp per bucket; turns offsets[b] into the bucket's absolute position.
__global__ void __launch_bounds__(256) bucket_flatten_kernel(const uint32_t* counts, const uint32_t* entries,
                                                             int32_t cap, int64_t n_buckets, uint32_t* offsets,
                                                             const uint32_t* tile_base, int32_t* out_idx,
                                                             uint16_t* out_val) {
  const int64_t b = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (b >= n_buckets) return;
  const uint32_t n = min(counts[b], uint32_t(cap));
  const uint32_t off = offsets[b] + tile_base[b / kScanTile];
  __syncwarp();
  if ((threadIdx.x & 31) == 0) offsets[b] = off;
  const uint32_t* ent = entries + b * cap;
  for (uint32_t j = threadIdx.x & 31; j < n; j += 32) {
    const uint32_t e = ent[j];
    out_idx[off + j] = int32_t(b * ASHKV_NBIT_BUCKET_ELEMS + (e >> 16));
    out_val[off + j] = uint16_t(e & 0xFFFFu);
  }
}

float half_states_for(int bits) { return float((1 << bits) - 1) / 2.0f; }

constexpr int kStages = 3;      // 3 buckets in flight per warp: 48 KiB of tiles per CTA
constexpr int kCtasPerSm = 4;   // 32 warps per SM

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    else
      cudaGetLastError();
  });
  return fn;
}

// [n_groups, 32] bf16 rows of 64 bytes, box = one bucket (32 rows), 64-byte swizzle.
bool make_group_tmap(CUtensorMap* map, const void* src, int64_t n_groups) {
  auto fn = tmap_encode_fn();
  if (!fn || n_groups <= 0 || n_groups > 0x7FFFFF00LL || !aligned(src, 16)) return false;
  cuuint64_t dims[2] = {32, cuuint64_t(n_groups)};
  cuuint64_t strides[1] = {64};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(src), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BITS, int DMODE>
ashkv_status_t launch_tma(const CUtensorMap& tmap, const NbitEncParams& p, int64_t n_buckets, unsigned grid,
                          cudaStream_t st) {
  constexpr int smem = kWarps * kStages * kTileBytes + 1024;
  auto kern = nbit_encode_tma_kernel<BITS, DMODE, kStages>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] { attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); });
  if (attr_err != cudaSuccess) {
    set_error("nbit_encode_tma smem attribute", attr_err);
    return ASHKV_LAUNCH_ERROR;
  }
  kern<<<grid, kThreads, smem, st>>>(tmap, p, n_buckets);
  return check_launch("nbit_encode_tma");
}

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
  const int64_t n_buckets = (n_groups + 31) / 32;
  if (n_groups > 0x7FFFFF00LL) return ASHKV_BAD_ARGUMENT;

  NbitEncParams p;
  p.src = static_cast<const uint16_t*>(d_src); p.n_groups = n_groups;
  p.dither = d_dither; p.seed = seed; p.dither_offset = dither_elem_offset;
  philox_round_keys(seed, p.round_keys);
  p.sigma = sigma; p.half_states = half_states_for(bits);
  p.scales = static_cast<uint16_t*>(d_scales); p.codes = static_cast<uint8_t*>(d_codes);
  p.bucket_counts = d_bucket_counts; p.bucket_entries = d_bucket_entries; p.bucket_cap = bucket_cap;
  p.status = d_status;

  cudaStream_t st = as_stream(stream);
  CUtensorMap tmap;
  if (make_group_tmap(&tmap, d_src, n_groups)) {
    const int sms = sm_count() > 0 ? sm_count() : 148;
    const int64_t want = int64_t(sms) * kCtasPerSm, need = (n_buckets + kWarps - 1) / kWarps;
    const unsigned grid = unsigned(need < want ? need : want);
    const bool tensor = dither_mode == ASHKV_DITHER_TENSOR;
    ashkv_status_t s = ASHKV_OK;
    if (bits == 2) s = tensor ? launch_tma<2, ASHKV_DITHER_TENSOR>(tmap, p, n_buckets, grid, st)
                              : launch_tma<2, ASHKV_DITHER_PHILOX>(tmap, p, n_buckets, grid, st);
    else if (bits == 4) s = tensor ? launch_tma<4, ASHKV_DITHER_TENSOR>(tmap, p, n_buckets, grid, st)
                                   : launch_tma<4, ASHKV_DITHER_PHILOX>(tmap, p, n_buckets, grid, st);
    else s = tensor ? launch_tma<8, ASHKV_DITHER_TENSOR>(tmap, p, n_buckets, grid, st)
                    : launch_tma<8, ASHKV_DITHER_PHILOX>(tmap, p, n_buckets, grid, st);
    return s;
  }
  const dim3 grid{unsigned((n_groups + kThreads - 1) / kThreads)}, block{unsigned(kThreads)};
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
  if (!aligned(d_dst, 32) || !aligned(d_scales, 2) || !aligned(d_codes, bits == 2 ? 8 : 16))
    return ASHKV_BAD_ARGUMENT;
  const int64_t n_ctas = (n_groups + 2 * kThreads - 1) / (2 * kThreads);  // 16 buckets per CTA
  if (n_ctas > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;

  NbitDecParams p;
  p.scales = static_cast<const uint16_t*>(d_scales); p.codes = static_cast<const uint8_t*>(d_codes);
  p.n_groups = n_groups; p.half_states = half_states_for(bits);
  p.bucket_counts = d_bucket_counts; p.bucket_entries = d_bucket_entries; p.bucket_cap = bucket_cap;
  p.dst = static_cast<uint16_t*>(d_dst); p.status = d_status;
  cudaStream_t st = as_stream(stream);
  const dim3 grid{unsigned(n_ctas)}, block{unsigned(kThreads)};
  if (bits == 2) nbit_decode_kernel<2><<<grid, block, 0, st>>>(p);
  else if (bits == 4) nbit_decode_kernel<4><<<grid, block, 0, st>>>(p);
  else nbit_decode_kernel<8><<<grid, block, 0, st>>>(p);
  return check_launch("nbit_decode");
}

extern "C" int64_t ashkv_nbit_flatten_scratch_ints(int64_t n_buckets) {
  if (n_buckets < 0) return -1;
  return n_buckets + 1 + (n_buckets + kScanTile - 1) / kScanTile;
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
  const int64_t n_tiles = (n_buckets + kScanTile - 1) / kScanTile;
  uint32_t* tile_totals = d_offsets + n_buckets + 1;
  bucket_scan_tiles_kernel<<<unsigned(n_tiles), 1024, 0, st>>>(d_bucket_counts, bucket_cap, n_buckets, d_offsets,
                                                               tile_totals);
  tile_scan_kernel<<<1, 1024, 0, st>>>(tile_totals, n_tiles, d_offsets + n_buckets, d_total);
  ashkv_status_t s = check_launch("nbit_bucket_scan");
  if (s != ASHKV_OK) return s;
  bucket_flatten_kernel<<<unsigned((n_buckets + 7) / 8), 256, 0, st>>>(d_bucket_counts, d_bucket_entries,
                                                                       bucket_cap, n_buckets, d_offsets, tile_totals,
                                                                       d_out_index, d_out_value);
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
  if (!aligned(d_dst, 32) || !aligned(d_scales, 2) || !aligned(d_codes, bits == 2 ? 8 : 16))
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
