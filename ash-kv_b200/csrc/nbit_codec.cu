// Dithered N-bit group codec with 3-sigma outlier isolation (sm_100a).
//
// Restates DitheredNBitCodec (ashkv/codecs/nbit_dithered.py:43-167) and
// DitheredINT2Codec (ashkv/codecs/int2_dithered.py:36-147).  The reference
// runs ~10 op-by-op tensor passes plus a nonzero()/host sync per call; here a
// single pass does everything per 32-element group in one thread:
//   load -> mean, sum of squares, min/max (one read) -> outlier mask (fp64
//   variance only near the threshold) -> inlier absmax -> delta -> dithered
//   quantise (second read) -> MSB-first pack -> one vector store of the codes
//   + one bf16 delta store.
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
#include "nbit_group.cuh"

namespace ashkv {
namespace {

constexpr int kThreads = 256;                     // 8 warps per CTA
constexpr int kWarps = kThreads / 32;
static_assert(ASHKV_NBIT_BUCKET_GROUPS == 32, "one bucket per warp, one group per lane");


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
  if (dither_mode == ASHKV_DITHER_PHILOX && (dither_elem_offset % 16)) return ASHKV_BAD_ARGUMENT;
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
