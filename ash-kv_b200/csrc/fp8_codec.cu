// FP8 (E4M3FN) codec: bf16 <-> float8_e4m3fn, one byte per element.
//
// Replaces the casts of FP8Codec (ashkv/codecs/fp8.py:32-79 of the reference):
//   encode: tensor.to(torch.float8_e4m3fn)   -- round to nearest even, no
//           saturation: |x| > 464 (rounds past 448), inf and NaN -> 0x7F|sign
//   decode: view(float8_e4m3fn).to(bfloat16) -- exact; NaN -> 0x7FFF (the
//           bf16 NaN torch's CUDA cast writes)
//
// Both directions are pure streams (2 B in / 1 B out, and back).  The fast
// kernels move 16 elements per thread with 256-bit bf16 accesses and 128-bit
// fp8 accesses and convert with the hardware e4m3x2 instructions; the one
// difference from torch's rule (cvt .satfinite clamps to 448 where torch
// writes NaN) is patched with an integer compare on the bf16 bits.
#include "common.cuh"
#include "fp8_conv.cuh"

namespace ashkv {
namespace {


// 16 elements per thread; src 32-byte aligned, dst 16-byte aligned.
__global__ void __launch_bounds__(256) fp8_encode_v16(const uint16_t* __restrict__ src, int64_t n16,
                                                      uint8_t* __restrict__ dst) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const U8 x = ld_nc_v8(src + i * 16);
    uint4 o;
    o.x = fp8x2_from_bf16x2(x.v[0]) | (fp8x2_from_bf16x2(x.v[1]) << 16);
    o.y = fp8x2_from_bf16x2(x.v[2]) | (fp8x2_from_bf16x2(x.v[3]) << 16);
    o.z = fp8x2_from_bf16x2(x.v[4]) | (fp8x2_from_bf16x2(x.v[5]) << 16);
    o.w = fp8x2_from_bf16x2(x.v[6]) | (fp8x2_from_bf16x2(x.v[7]) << 16);
    st_cs_v4(dst + i * 16, o);
  }
}

// One element per thread: unaligned buffers and the ragged tail.
__global__ void fp8_encode_scalar(const uint16_t* __restrict__ src, int64_t begin, int64_t n,
                                  uint8_t* __restrict__ dst) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = begin + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = static_cast<uint8_t>(fp8x2_from_bf16x2(src[i]));
}

// 16 elements per thread; src 16-byte aligned, dst 32-byte aligned.
__global__ void __launch_bounds__(256) fp8_decode_v16(const uint8_t* __restrict__ src, int64_t n16,
                                                      uint16_t* __restrict__ dst) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 c = ld_nc_v4(src + i * 16);
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
    U8 o;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o.v[2 * k] = bf16x2_from_fp8x2(w[k] & 0xFFFFu);
      o.v[2 * k + 1] = bf16x2_from_fp8x2(w[k] >> 16);
    }
    st_cs_v8(dst + i * 16, o);
  }
}

__global__ void fp8_decode_scalar(const uint8_t* __restrict__ src, int64_t begin, int64_t n,
                                  uint16_t* __restrict__ dst) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = begin + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = static_cast<uint16_t>(bf16x2_from_fp8x2(src[i]));
}

unsigned grid_for(int64_t items, int threads) {
  const int64_t need = (items + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count() > 0 ? sm_count() : 148) * 8;
  return unsigned(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace
}  // namespace ashkv

using namespace ashkv;

extern "C" ashkv_status_t ashkv_fp8_encode(const void* src_bf16, int64_t n, void* dst_fp8, void* stream) {
  if (n < 0 || (n > 0 && (!src_bf16 || !dst_fp8))) return ASHKV_BAD_ARGUMENT;
  if (n == 0) return ASHKV_OK;
  cudaStream_t s = as_stream(stream);
  const auto* src = static_cast<const uint16_t*>(src_bf16);
  auto* dst = static_cast<uint8_t*>(dst_fp8);
  int64_t done = 0;
  if (aligned(src, 32) && aligned(dst, 16)) {
    const int64_t n16 = n / 16;
    if (n16) fp8_encode_v16<<<grid_for(n16, 256), 256, 0, s>>>(src, n16, dst);
    done = n16 * 16;
  }
  if (done < n) fp8_encode_scalar<<<grid_for(n - done, 256), 256, 0, s>>>(src, done, n, dst);
  return check_launch("ashkv_fp8_encode");
}

extern "C" ashkv_status_t ashkv_fp8_decode(const void* src_fp8, int64_t n, void* dst_bf16, void* stream) {
  if (n < 0 || (n > 0 && (!src_fp8 || !dst_bf16))) return ASHKV_BAD_ARGUMENT;
  if (n == 0) return ASHKV_OK;
  cudaStream_t s = as_stream(stream);
  const auto* src = static_cast<const uint8_t*>(src_fp8);
  auto* dst = static_cast<uint16_t*>(dst_bf16);
  int64_t done = 0;
  if (aligned(src, 16) && aligned(dst, 32)) {
    const int64_t n16 = n / 16;
    if (n16) fp8_decode_v16<<<grid_for(n16, 256), 256, 0, s>>>(src, n16, dst);
    done = n16 * 16;
  }
  if (done < n) fp8_decode_scalar<<<grid_for(n - done, 256), 256, 0, s>>>(src, done, n, dst);
  return check_launch("ashkv_fp8_decode");
}
