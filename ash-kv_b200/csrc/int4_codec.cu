// INT4 group codec: per-group absmax scale, two signed 4-bit codes per byte.
//
// Replaces INT4Codec (ashkv/codecs/int4.py:38-112 of the reference), which
// runs in numpy on the host.  Per group of G values (the input zero-padded
// to a multiple of G):
//   am    = maximum(max|x|, 1e-8)              NaN propagates (np.max, np.maximum)
//   q     = clip(int8(round_half_even(RN(x*7) / am)), -8, 7)
//           int8() is numpy's x86 cast: truncate to int32 (NaN, inf and
//           out-of-range give INT32_MIN) and keep the low byte
//   byte  = (q[2j] + 8) << 4 | (q[2j+1] + 8)   even element in the high nibble
//   scale = bf16(am)                           torch CPU cast: RNE, NaN -> 0xFFFF
// Decode: out = bf16(RN(RN(float(nibble - 8) * float(scale)) / 7)), with the
// same CPU NaN encoding.
//
// Divisions are correctly rounded: the per-group reciprocal pair plus
// Markstein's correction (common.cuh) where its range conditions hold, the
// reciprocal pair alone where dividend and divisor have short significands
// (div2_short: 7x by a bf16 absmax, q*s by 7), __fdiv_rn elsewhere.
// Groups whose G is a power of two in [8, 256] take the fast kernels (G/32
// threads per group with 32 values each, or G/8 threads for G = 8, 16; 16-byte
// loads); any other G takes a warp-per-group kernel.
#include "common.cuh"
#include "int4_group.cuh"

namespace ashkv {
namespace {


// ---------------------------------------------------------------- fast encode
// TPG = G/8 threads per group, 8 values per thread (one 16-byte load) -> one
// 32-bit store of 8 nibbles.  Values at index >= n are the zero padding.
__device__ __forceinline__ uint4 load_chunk(const uint16_t* __restrict__ src, int64_t n, int64_t c, bool active) {
  const int64_t e0 = c * 8;
  if (!active) return make_uint4(0u, 0u, 0u, 0u);
  if (e0 + 8 <= n) return ld_nc_v4(src + e0);
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = e0 + 2 * k < n ? src[e0 + 2 * k] : 0u;
    const uint32_t hi = e0 + 2 * k + 1 < n ? src[e0 + 2 * k + 1] : 0u;
    w[k] = lo | (hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}


// Called by every lane of the warp (the group maximum is a shuffle reduction).
template <int TPG>
__device__ __forceinline__ void encode_chunk(uint4 v, int64_t c, bool active, uint16_t* __restrict__ scales,
                                             uint32_t* __restrict__ packed) {
  float x[8];
  unpack_chunk(v, x);
  float m = chunk_max(0.0f, x);
#pragma unroll
  for (int off = 1; off < TPG; off <<= 1) m = max_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
  const float am = group_max_finish(m);
  if (!active) return;
  if ((c % TPG) == 0) scales[c / TPG] = static_cast<uint16_t>(bf16_cpu(am));
  packed[c] = pack_chunk(x, group_div(am));
}

// Two chunks per lane per iteration (c and c + stride), both loaded before
// either is encoded.  The loop runs per warp (c0 = the warp's first chunk) so
// that every lane takes part in the shuffles; n_chunks is a multiple of TPG,
// so the lanes of one group are all active or all idle.  Used for G = 8, 16.
template <int TPG>
__global__ void __launch_bounds__(256) int4_encode_fast(const uint16_t* __restrict__ src, int64_t n,
                                                        int64_t n_chunks, uint16_t* __restrict__ scales,
                                                        uint32_t* __restrict__ packed) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int lane = threadIdx.x & 31;
  for (int64_t c0 = int64_t(blockIdx.x) * blockDim.x + (threadIdx.x & ~31); c0 < n_chunks; c0 += 2 * stride) {
    const int64_t ca = c0 + lane, cb = ca + stride;
    const bool act_a = ca < n_chunks, act_b = cb < n_chunks;
    const uint4 va = load_chunk(src, n, ca, act_a);
    const uint4 vb = load_chunk(src, n, cb, act_b);
    encode_chunk<TPG>(va, ca, act_a, scales, packed);
    encode_chunk<TPG>(vb, cb, act_b, scales, packed);
  }
}

// G = 32 * TEAM (32..256): TEAM lanes per group, 4 chunks of 8 values per lane
// (chunk k * TEAM + lane-in-team of the group, so each load and store of a warp
// is contiguous), so the group's shuffles, divisor and scale are spread over 32
// values per lane.  Warps walk tiles of 32 / TEAM groups.
template <int TEAM>
__global__ void __launch_bounds__(256) int4_encode_team(const uint16_t* __restrict__ src, int64_t n,
                                                        int64_t n_groups, uint16_t* __restrict__ scales,
                                                        uint32_t* __restrict__ packed) {
  constexpr int GPW = 32 / TEAM;
  const int lane = threadIdx.x & 31, lin = lane % TEAM;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  for (int64_t g0 = (int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5)) * GPW; g0 < n_groups;
       g0 += warps * GPW) {
    const int64_t g = g0 + lane / TEAM;
    const bool active = g < n_groups;
    const int64_t c0 = g * (4 * TEAM) + lin;
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = load_chunk(src, n, c0 + k * TEAM, active);
    float x[4][8];
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      unpack_chunk(v[k], x[k]);
      m = chunk_max(m, x[k]);
    }
#pragma unroll
    for (int off = 1; off < TEAM; off <<= 1) m = max_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    const float am = group_max_finish(m);
    if (!active) continue;
    if (lin == 0) scales[g] = static_cast<uint16_t>(bf16_cpu(am));
    const GroupDiv d = group_div(am);
#pragma unroll
    for (int k = 0; k < 4; ++k) packed[c0 + k * TEAM] = pack_chunk(x[k], d);
  }
}

// ---------------------------------------------------------------- generic encode
// One warp per group, any G.  For odd G a byte can hold the last value of
// group g and the first of group g + 1; the warp of group g writes it, so it
// also reduces group g + 1's maximum.
__device__ float warp_group_max(const uint16_t* src, int64_t n, int64_t g, int32_t G, int lane) {
  float m = 0.0f;
  for (int32_t k = lane; k < G; k += 32) {
    const int64_t i = g * G + k;
    const float x = i < n ? bf16_to_f32(src[i]) : 0.0f;
    m = max3_abs_nan(m, x, x);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
  return group_max_finish(m);
}

__global__ void int4_encode_generic(const uint16_t* __restrict__ src, int64_t n, int32_t G, int64_t n_groups,
                                    uint16_t* __restrict__ scales, uint8_t* __restrict__ packed) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  for (int64_t g = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); g < n_groups; g += warps) {
    const float am = warp_group_max(src, n, g, G, lane);
    const bool odd = (G & 1) != 0;
    const float am_next = (odd && g + 1 < n_groups) ? warp_group_max(src, n, g + 1, G, lane) : am;
    if (lane == 0) scales[g] = static_cast<uint16_t>(bf16_cpu(am));
    const GroupDiv d = group_div(am), dn = group_div(am_next);
    const int64_t first = g * G, end = first + G;
    // bytes whose even element lies in this group
    for (int64_t j = (first + 1) / 2 + lane; 2 * j < end; j += 32) {
      const int64_t i = 2 * j;
      const float x0 = i < n ? bf16_to_f32(src[i]) : 0.0f;
      const float x1 = i + 1 < n ? bf16_to_f32(src[i + 1]) : 0.0f;
      const uint32_t hi = nibble_of(x0, d);
      const uint32_t lo = nibble_of(x1, i + 1 < end ? d : dn);
      packed[j] = static_cast<uint8_t>((hi << 4) | lo);
    }
  }
}

// ---------------------------------------------------------------- decode
// out = bf16(RN(q * s) / 7).  Fast when s is finite and in [2^-90, 2^90]
// (then q*s is 0 or at least 2^-90, and exact with at most 12 significant bits,
// so the division by 7 takes div2_short; s > 0 keeps the sign of 0).

template <int EPT>
__global__ void __launch_bounds__(256) int4_decode_fast(const uint16_t* __restrict__ scales,
                                                        const uint8_t* __restrict__ packed, int64_t n_chunks,
                                                        int32_t chunks_per_group, uint16_t* __restrict__ dst) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const Recip y7 = make_recip(7.0f);
  const f2 yhi = pk2(y7.hi, y7.hi), ylo = pk2(y7.lo, y7.lo), bias = pk2(-8388616.0f, -8388616.0f);
  for (int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; c < n_chunks; c += stride) {
    const float s = bf16_to_f32(scales[c / chunks_per_group]);
    const bool fast = s >= 0x1p-90f && s <= 0x1p+90f;
    uint32_t code[EPT / 8];
    if constexpr (EPT == 16) {
      const uint2 v = *reinterpret_cast<const uint2*>(packed + c * 8);
      code[0] = v.x; code[1] = v.y;
    } else {
      code[0] = *reinterpret_cast<const uint32_t*>(packed + c * 4);
    }
    uint32_t o[EPT / 2];
    if (fast) {
      const f2 ss = pk2(s, s);
#pragma unroll
      for (int b = 0; b < EPT / 2; ++b) {
        const uint32_t byte = (code[b / 4] >> (8 * (b % 4))) & 0xFFu;
        // q - 8 = (2^23 + q) - (2^23 + 8) exactly; q * s has at most 4 + 8 bits,
        // so the division by 7 needs no correction step (div2_short)
        const f2 q = add2(pk2(__uint_as_float(0x4B000000u | (byte >> 4)), __uint_as_float(0x4B000000u | (byte & 15u))),
                          bias);
        float v0, v1;
        upk2(div2_short(mul2(q, ss), yhi, ylo), v0, v1);
        o[b] = f32x2_to_bf16x2(v0, v1);
      }
    } else {
#pragma unroll
      for (int b = 0; b < EPT / 2; ++b) {
        const uint32_t byte = (code[b / 4] >> (8 * (b % 4))) & 0xFFu;
        const float v0 = __fdiv_rn(__fmul_rn(float(int(byte >> 4) - 8), s), 7.0f);
        const float v1 = __fdiv_rn(__fmul_rn(float(int(byte & 15u) - 8), s), 7.0f);
        o[b] = bf16_cpu(v0) | (bf16_cpu(v1) << 16);
      }
    }
    if constexpr (EPT == 16) {
      U8 r;
#pragma unroll
      for (int k = 0; k < 8; ++k) r.v[k] = o[k];
      st_cs_v8(dst + c * 16, r);
    } else {
      st_cs_v4(dst + c * 8, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

__global__ void int4_decode_generic(const uint16_t* __restrict__ scales, const uint8_t* __restrict__ packed,
                                    int64_t total, int32_t G, uint16_t* __restrict__ dst) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t byte = packed[i >> 1];
    const int q = int((i & 1) == 0 ? (byte >> 4) : (byte & 15u)) - 8;
    const float s = bf16_to_f32(scales[i / G]);
    const float p = __fmul_rn(float(q), s);
    dst[i] = static_cast<uint16_t>(bf16_cpu(__fdiv_rn(p, 7.0f)));
  }
}

unsigned grid_for(int64_t items, int threads) {
  const int64_t need = (items + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count() > 0 ? sm_count() : 148) * 8;
  return unsigned(need < cap ? (need > 0 ? need : 1) : cap);
}

bool fast_group(int32_t G) { return G >= 8 && G <= 256 && (G & (G - 1)) == 0; }

}  // namespace
}  // namespace ashkv

using namespace ashkv;

extern "C" int64_t ashkv_int4_group_count(int64_t n, int32_t group_size) {
  if (n < 0 || group_size <= 0) return -1;
  return (n + group_size - 1) / group_size;
}

extern "C" ashkv_status_t ashkv_int4_encode(const void* src_bf16, int64_t n, int32_t group_size,
                                            void* scales_bf16, void* packed, void* stream) {
  if (n < 0 || group_size <= 0) return ASHKV_BAD_ARGUMENT;
  const int64_t n_groups = (n + group_size - 1) / group_size;
  if ((n_groups * group_size) & 1) {
    set_message("ashkv_int4_encode: padded value count is odd");
    return ASHKV_BAD_ARGUMENT;
  }
  if (n == 0) return ASHKV_OK;
  if (!src_bf16 || !scales_bf16 || !packed) return ASHKV_BAD_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  const auto* src = static_cast<const uint16_t*>(src_bf16);
  auto* sc = static_cast<uint16_t*>(scales_bf16);
  if (fast_group(group_size) && aligned(src, 16) && aligned(packed, 4) && n_groups * group_size < (int64_t(1) << 40)) {
    const int64_t n_chunks = n_groups * (group_size / 8);
    auto* pk = static_cast<uint32_t*>(packed);
    const unsigned grid = grid_for(group_size >= 32 ? n_groups * (group_size / 32) : n_chunks, 256);
    switch (group_size / 8) {
      case 1: int4_encode_fast<1><<<grid, 256, 0, s>>>(src, n, n_chunks, sc, pk); break;
      case 2: int4_encode_fast<2><<<grid, 256, 0, s>>>(src, n, n_chunks, sc, pk); break;
      case 4: int4_encode_team<1><<<grid, 256, 0, s>>>(src, n, n_groups, sc, pk); break;
      case 8: int4_encode_team<2><<<grid, 256, 0, s>>>(src, n, n_groups, sc, pk); break;
      case 16: int4_encode_team<4><<<grid, 256, 0, s>>>(src, n, n_groups, sc, pk); break;
      default: int4_encode_team<8><<<grid, 256, 0, s>>>(src, n, n_groups, sc, pk); break;
    }
  } else {
    int4_encode_generic<<<grid_for(n_groups * 32, 256), 256, 0, s>>>(src, n, group_size, n_groups, sc,
                                                                     static_cast<uint8_t*>(packed));
  }
  return check_launch("ashkv_int4_encode");
}

extern "C" ashkv_status_t ashkv_int4_decode(const void* scales_bf16, const void* packed, int64_t n_groups,
                                            int32_t group_size, void* dst_bf16, void* stream) {
  if (n_groups < 0 || group_size <= 0) return ASHKV_BAD_ARGUMENT;
  const int64_t total = n_groups * group_size;
  if (total & 1) {
    set_message("ashkv_int4_decode: value count is odd");
    return ASHKV_BAD_ARGUMENT;
  }
  if (total == 0) return ASHKV_OK;
  if (!scales_bf16 || !packed || !dst_bf16) return ASHKV_BAD_ARGUMENT;
  cudaStream_t s = as_stream(stream);
  const auto* sc = static_cast<const uint16_t*>(scales_bf16);
  const auto* pk = static_cast<const uint8_t*>(packed);
  auto* dst = static_cast<uint16_t*>(dst_bf16);
  if (group_size % 16 == 0 && aligned(pk, 8) && aligned(dst, 32)) {
    const int64_t n_chunks = total / 16;
    int4_decode_fast<16><<<grid_for(n_chunks, 256), 256, 0, s>>>(sc, pk, n_chunks, group_size / 16, dst);
  } else if (group_size % 8 == 0 && aligned(pk, 4) && aligned(dst, 16)) {
    const int64_t n_chunks = total / 8;
    int4_decode_fast<8><<<grid_for(n_chunks, 256), 256, 0, s>>>(sc, pk, n_chunks, group_size / 8, dst);
  } else {
    int4_decode_generic<<<grid_for(total, 256), 256, 0, s>>>(sc, pk, total, group_size, dst);
  }
  return check_launch("ashkv_int4_decode");
}
