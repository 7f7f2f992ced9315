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
// One lane step written around the chain's critical path.  With the lane state
// kept as a = acc + in * P2 (the sum before the rotation), the next state is
// rotl(a, 31) * P1 + in' * P2: the 64-bit addend rides in the wide multiply-add
// of the low product, and the two cross products go to the high word, so the
// 64-bit add no longer follows the multiply (in' * P2 is off the chain).
__device__ __forceinline__ uint64_t rot_mul_add(uint64_t a, uint64_t m) {
  const uint32_t al = uint32_t(a), ah = uint32_t(a >> 32);
  const uint32_t rl = __funnelshift_l(ah, al, 31), rh = __funnelshift_l(al, ah, 31);  // rotl(a, 31)
  const uint64_t w = uint64_t(rl) * uint32_t(P1) + m;
  const uint32_t t = rl * uint32_t(P1 >> 32) + rh * uint32_t(P1);
  return w + (uint64_t(t) << 32);
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

// ---------------------------------------------------------------------------
// Page-sized items: the four lane chains of an item are serial (a 64-bit
// multiply chain per 8-byte word), so the parallelism is 4 threads per item;
// the register prefetch above keeps only 64 bytes per thread in flight, which
// leaves a few thousand pages far from HBM rate.  Here a CTA hashes 32 items at
// a time and streams them through shared memory in chunks of kChunk bytes per
// item, kStages chunks deep, with cp.async copies (hardware-completed: no spin
// waits), so each SM keeps about 128 KiB of page data in flight while its
// quads run the multiply chains out of shared memory.
constexpr int kItemsPerCta = 32;           // 128 threads: a quad per item
constexpr int kChunk = 2048;               // bytes of an item per stage
constexpr int kRow = kChunk + 16;          // padded: the 8 quads of a warp read 8 rows in 2 wavefronts
constexpr int kStages = 3;
constexpr int kStagedSmem = kStages * kItemsPerCta * kRow;  // 198,144 bytes
constexpr int64_t kStagedMinBytes = 1024;  // items shorter than this take xxh64_items_kernel
// Above about 80 items per SM the register-prefetch kernel has enough warps to
// hide its latency and is faster (measured on 32 KiB pages: staged 80 / 151 us,
// register prefetch 108 / 125 us at 8192 / 16384 pages).
constexpr int64_t kStagedMaxItemsPerSm = 80;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }
__device__ __forceinline__ uint64_t lds64(const uint8_t* p) {
  uint64_t v;
  asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ uint64_t lane_init(int lane, uint64_t seed) {
  switch (lane) {
    case 0: return seed + P1 + P2;
    case 1: return seed + P2;
    case 2: return seed;
    default: return seed - P1;
  }
}

// Requires: data 16-byte aligned, stride a multiple of 16, len >= kStagedMinBytes.
// The CTA walks the sequence of (item group, chunk) entries of its groups
// (blockIdx.x, + gridDim.x, ...); entry q lands in stage q % kStages.
__global__ void __launch_bounds__(kItemsPerCta * 4, 1) xxh64_items_staged_kernel(
    const uint8_t* data, int64_t n_items, int64_t len, int64_t stride, uint64_t seed, uint64_t* out) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int kPieces = kChunk / 16;                 // 16-byte copies per item chunk
  constexpr int kItemStep = kItemsPerCta * 4 / kPieces;  // items one pass of the CTA's copies covers
  const int tid = threadIdx.x, slot = tid >> 2, lane = tid & 3;
  const int piece = tid % kPieces, it0 = tid / kPieces;
  const int64_t n_stripes = len / 32, sbytes = n_stripes * 32;
  const int64_t n_chunks = (sbytes + kChunk - 1) / kChunk;
  const int64_t n_groups = (n_items + kItemsPerCta - 1) / kItemsPerCta;
  const int64_t my_groups = n_groups > blockIdx.x ? (n_groups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t total = my_groups * n_chunks;

  // issue position (group, chunk, stage) and consume position
  int64_t ig = blockIdx.x, ic = 0;
  int istage = 0;
  auto issue = [&]() {
    const int64_t cb = sbytes - ic * kChunk;
    const bool full = cb >= kChunk;
    const int pieces = full ? kPieces : int(cb / 16);
    uint8_t* stage = sm + istage * (kItemsPerCta * kRow);
    if (piece < pieces) {
      const uint8_t* src = data + (ig * kItemsPerCta + it0) * stride + ic * kChunk + piece * 16;
      uint8_t* dst = stage + it0 * kRow + piece * 16;
#pragma unroll 4
      for (int it = it0; it < kItemsPerCta; it += kItemStep) {
        if (ig * kItemsPerCta + it < n_items) cp_async16(dst, src);
        src += kItemStep * stride;
        dst += kItemStep * kRow;
      }
    }
    if (++ic == n_chunks) { ic = 0; ig += gridDim.x; }
    if (++istage == kStages) istage = 0;
  };
#pragma unroll
  for (int q = 0; q < kStages - 1; ++q) {
    if (q < total) issue();
    cp_async_commit();
  }
  int64_t cg = blockIdx.x, cc = 0;
  int cstage = 0;
  uint64_t v = lane_init(lane, seed);
  for (int64_t q = 0; q < total; ++q) {
    if (q + kStages - 1 < total) issue();
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // entry q has landed (this thread's copies)
    __syncthreads();               // ... and every other thread's
    const int64_t item = cg * kItemsPerCta + slot;
    const int64_t cb = sbytes - cc * kChunk;
    const int rows = int((cb < kChunk ? cb : kChunk) / 32);
    const uint8_t* row = sm + cstage * (kItemsPerCta * kRow) + slot * kRow + 8 * lane;
    if (rows == kChunk / 32) {  // full chunk: a fixed trip count, loads hoisted ahead of the chain
      uint64_t a = v + lds64(row) * P2;
#pragma unroll 16
      for (int r = 1; r < kChunk / 32; ++r) a = rot_mul_add(a, lds64(row + r * 32) * P2);
      v = rot_mul_add(a, 0);  // = xxround applied to all kChunk / 32 words
    } else {
#pragma unroll 8
      for (int r = 0; r < rows; ++r) v = xxround(v, lds64(row + r * 32));
    }
    if (cc == n_chunks - 1) {  // the group's items are complete: merge, tail, avalanche
      const unsigned qbase = (tid & 31u) & ~3u;
      const uint64_t v1 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 0));
      const uint64_t v2 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 1));
      const uint64_t v3 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 2));
      const uint64_t v4 = __shfl_sync(0xFFFFFFFFu, v, int(qbase + 3));
      if (lane == 0 && item < n_items) {
        uint64_t h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
        h = xxmerge(h, v1); h = xxmerge(h, v2); h = xxmerge(h, v3); h = xxmerge(h, v4);
        h += uint64_t(len);
        const uint8_t* q8 = data + item * stride + sbytes;
        int64_t rem = len - sbytes;
        while (rem >= 8) {
          h ^= xxround(0, rd64<true>(q8));
          h = rotl64(h, 27) * P1 + P4;
          q8 += 8; rem -= 8;
        }
        if (rem >= 4) {
          h ^= uint64_t(rd32(q8)) * P1;
          h = rotl64(h, 23) * P2 + P3;
          q8 += 4; rem -= 4;
        }
        while (rem > 0) {
          h ^= uint64_t(*q8) * P5;
          h = rotl64(h, 11) * P1;
          ++q8; --rem;
        }
        h ^= h >> 33; h *= P2;
        h ^= h >> 29; h *= P3;
        h ^= h >> 32;
        out[item] = h;
      }
      v = lane_init(lane, seed);
    }
    if (++cc == n_chunks) { cc = 0; cg += gridDim.x; }
    if (++cstage == kStages) cstage = 0;
    __syncthreads();  // this stage is refilled by the next iteration's issue
  }
  cp_async_wait<0>();
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
  const int64_t sms = sm_count() > 0 ? sm_count() : 148;
  if (item_bytes >= kStagedMinBytes && n_items <= sms * kStagedMaxItemsPerSm && aligned(d_data, 16) &&
      (n_items == 1 || item_stride % 16 == 0)) {
    if (cudaFuncSetAttribute(xxh64_items_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStagedSmem) !=
        cudaSuccess)
      return check_launch("xxh64_items smem attribute");
    const int64_t groups = (n_items + kItemsPerCta - 1) / kItemsPerCta;
    const unsigned grid = unsigned(groups < sms ? groups : sms);
    xxh64_items_staged_kernel<<<grid, kItemsPerCta * 4, kStagedSmem, st>>>(data, n_items, item_bytes,
                                                                            n_items == 1 ? 0 : item_stride, seed,
                                                                            d_out);
    return check_launch("xxh64_items");
  }
  const bool a8 = aligned(d_data, 8) && (item_stride % 8 == 0);
  if (a8) xxh64_items_kernel<true><<<unsigned(blocks), 256, 0, st>>>(data, n_items, item_bytes, item_stride, seed, d_out);
  else xxh64_items_kernel<false><<<unsigned(blocks), 256, 0, st>>>(data, n_items, item_bytes, item_stride, seed, d_out);
  return check_launch("xxh64_items");
}
