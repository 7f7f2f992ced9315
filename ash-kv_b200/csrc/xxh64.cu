// XXH64 over many equal-sized items (KV pages), one digest per item.
//
// Produces the same 64-bit value as xxhash.xxh64(page_bytes, seed).intdigest(),
// which the reference's checksum() returns (ashkv/codecs/checksum.py:26-37).
// The algorithm is the public XXH64 specification (Collet): four 64-bit lane
// accumulators consume 32-byte stripes, are merged, the <32-byte tail is
// folded in and the result avalanched.  On the GPU each item is hashed by a
// quad of threads, one per lane accumulator; each thread keeps 8 stripes of
// loads in flight ahead of its serial multiply chain so the kernel streams
// at memory rate, then the quad merges through warp shuffles.
#include "common.cuh"

namespace ashkv {
namespace {

constexpr uint64_t P1 = 0x9E3779B185EBCA87ull;
constexpr uint64_t P2 = 0xC2B2AE3D27D4EB4Full;
constexpr uint64_t P3 = 0x165667B19E3779F9ull;
constexpr uint64_t P4 = 0x85EBCA77C2B2AE63ull;
constexpr uint64_t P5 = 0x27D4EB2F165667C5ull;

__device__ __forceinline__ uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
__device__ __forceinline__ uint64_t xxround(uint64_t acc, uint64_t in) {
  acc += in * P2;
  acc = rotl64(acc, 31);
  return acc * P1;
}
__device__ __forceinline__ uint64_t xxmerge(uint64_t h, uint64_t v) {
  h ^= xxround(0, v);
  return h * P1 + P4;
}

template <bool ALIGNED8>
__device__ __forceinline__ uint64_t rd64(const uint8_t* p) {
  if constexpr (ALIGNED8) {
    return __ldg(reinterpret_cast<const unsigned long long*>(p));
  } else {
    uint64_t v = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) v |= uint64_t(p[i]) << (8 * i);
    return v;
  }
}
__device__ __forceinline__ uint32_t rd32(const uint8_t* p) {
  return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

constexpr int kPrefetch = 8;

template <bool ALIGNED8>
__global__ void __launch_bounds__(256) xxh64_items_kernel(const uint8_t* data, int64_t n_items, int64_t len,
                                                          int64_t stride, uint64_t seed, uint64_t* out) {
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t item = t >> 2;
  const int lane = int(threadIdx.x & 3);
  const bool active = item < n_items;
  const uint8_t* base = data + (active ? item : 0) * stride;

  uint64_t v;
  switch (lane) {
    case 0: v = seed + P1 + P2; break;
    case 1: v = seed + P2; break;
    case 2: v = seed; break;
    default: v = seed - P1; break;
  }
  const int64_t n_stripes = len / 32;
  if (active) {
    const uint8_t* p = base + 8 * lane;
    int64_t s = 0;
    for (; s + kPrefetch <= n_stripes; s += kPrefetch) {
      uint64_t w[kPrefetch];
#pragma unroll
      for (int k = 0; k < kPrefetch; ++k) w[k] = rd64<ALIGNED8>(p + (s + k) * 32);
#pragma unroll
      for (int k = 0; k < kPrefetch; ++k) v = xxround(v, w[k]);
    }
    for (; s < n_stripes; ++s) v = xxround(v, rd64<ALIGNED8>(p + s * 32));
  }
  // Gather the quad's lane accumulators (the quad is 4 consecutive lanes).
  const unsigned qbase = (threadIdx.x & 31u) & ~3u;
  const uint64_t v1 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 0));
  const uint64_t v2 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 1));
  const uint64_t v3 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 2));
  const uint64_t v4 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 3));
  if (!active || lane != 0) return;

  uint64_t h;
  if (len >= 32) {
    h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
    h = xxmerge(h, v1); h = xxmerge(h, v2); h = xxmerge(h, v3); h = xxmerge(h, v4);
  } else {
    h = seed + P5;
  }
  h += uint64_t(len);
  const uint8_t* q = base + n_stripes * 32;
  int64_t rem = len - n_stripes * 32;
  while (rem >= 8) {
    h ^= xxround(0, rd64<ALIGNED8>(q));
    h = rotl64(h, 27) * P1 + P4;
    q += 8; rem -= 8;
  }
  if (rem >= 4) {
    h ^= uint64_t(rd32(q)) * P1;
    h = rotl64(h, 23) * P2 + P3;
    q += 4; rem -= 4;
  }
  while (rem > 0) {
    h ^= uint64_t(*q) * P5;
    h = rotl64(h, 11) * P1;
    ++q; --rem;
  }
  h ^= h >> 33; h *= P2;
  h ^= h >> 29; h *= P3;
  h ^= h >> 32;
  out[item] = h;
}

}  // namespace
}  // namespace ashkv

using namespace ashkv;

extern "C" ashkv_status_t ashkv_xxh64_items(
    const void* d_data, int64_t n_items, int64_t item_bytes, int64_t item_stride,
    uint64_t seed, uint64_t* d_out, void* stream) {
  if (n_items < 0 || item_bytes < 0 || item_stride < 0) return ASHKV_BAD_ARGUMENT;
  if (n_items == 0) return ASHKV_OK;
  if (!d_out || (item_bytes > 0 && !d_data)) return ASHKV_BAD_ARGUMENT;
  if (n_items > 1 && item_stride < item_bytes) return ASHKV_BAD_ARGUMENT;
  const int64_t threads = n_items * 4;
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;
  const auto* data = static_cast<const uint8_t*>(d_data);
  cudaStream_t st = as_stream(stream);
  const bool a8 = aligned(d_data, 8) && (item_stride % 8 == 0);
  if (a8) xxh64_items_kernel<true><<<unsigned(blocks), 256, 0, st>>>(data, n_items, item_bytes, item_stride, seed, d_out);
  else xxh64_items_kernel<false><<<unsigned(blocks), 256, 0, st>>>(data, n_items, item_bytes, item_stride, seed, d_out);
  return check_launch("xxh64_items");
}
