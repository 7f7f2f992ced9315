// Strided host<->device / device<->device copy entry point.
//
// The SGLang host pool keeps one 2*head_num*head_dim-byte slot per
// (token, layer); a compressed slot only uses its first 2*head_num +
// head_num*head_dim bytes.  A pitched copy moves just those bytes for many
// slots in one DMA operation instead of gathering whole slots on the host.
#include <algorithm>

#include "common.cuh"

extern "C" ashkv_status_t ashkv_memcpy2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                                         int64_t width, int64_t height, void* stream) {
  if (width < 0 || height < 0 || dst_pitch < width || src_pitch < width) return ASHKV_BAD_ARGUMENT;
  if (width == 0 || height == 0) return ASHKV_OK;
  if (!dst || !src) return ASHKV_BAD_ARGUMENT;
  const cudaError_t e = cudaMemcpy2DAsync(dst, size_t(dst_pitch), src, size_t(src_pitch), size_t(width),
                                          size_t(height), cudaMemcpyDefault, ashkv::as_stream(stream));
  if (e != cudaSuccess) {
    ashkv::set_error("memcpy2d", e);
    cudaGetLastError();
    return ASHKV_LAUNCH_ERROR;
  }
  return ASHKV_OK;
}

// ---------------------------------------------------------------- indexed row copies
// Gather/scatter of row slices between device memory and page-locked host
// memory by a device index list, in one kernel: the SGLang hooks move the
// slots of arbitrary (non-contiguous) host pool rows without a host-side
// gather.  Host memory is read and written through its device mapping
// (zero-copy over the host link); a pointer that is neither device memory nor
// mapped page-locked host memory is refused before any launch.
namespace ashkv {
namespace {

struct RowCopyParams {
  uint8_t* dst;
  const uint8_t* src;
  int64_t dst_row_stride, dst_sub_stride, src_row_stride, src_sub_stride;
  const int64_t* dst_index;
  const int64_t* src_index;
  int64_t dst_rows, src_rows;  // rows the buffers hold (index bound)
  int64_t chunks;              // width / 16
  int64_t n_sub, n_rows;
  uint32_t* status;
};

// One warp per (row, sub-row) item, lanes over 16-byte chunks, 4 chunks in flight per lane.
__global__ void __launch_bounds__(256) copy_rows_kernel(const RowCopyParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  const int64_t items = p.n_rows * p.n_sub;
  for (int64_t it = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); it < items; it += warps) {
    const int64_t r = it / p.n_sub, s = it - r * p.n_sub;
    const int64_t dr = p.dst_index ? p.dst_index[r] : r;
    const int64_t sr = p.src_index ? p.src_index[r] : r;
    if (dr < 0 || dr >= p.dst_rows || sr < 0 || sr >= p.src_rows) {
      if (lane == 0 && p.status) atomicOr(p.status, ASHKV_FLAG_INDEX_RANGE);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(p.src + sr * p.src_row_stride + s * p.src_sub_stride);
    uint4* dst = reinterpret_cast<uint4*>(p.dst + dr * p.dst_row_stride + s * p.dst_sub_stride);
    for (int64_t c0 = lane; c0 < p.chunks; c0 += 4 * 32) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + u * 32 < p.chunks) v[u] = src[c0 + u * 32];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + u * 32 < p.chunks) dst[c0 + u * 32] = v[u];
    }
  }
}

// The device address of p (device memory, or mapped page-locked host memory), else nullptr.
const void* device_view(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return p;
  if (a.type == cudaMemoryTypeHost) return a.devicePointer;
  return nullptr;
}

}  // namespace
}  // namespace ashkv

extern "C" ashkv_status_t ashkv_copy_rows_indexed(
    void* dst, int64_t dst_row_stride, int64_t dst_sub_stride, const int64_t* d_dst_index, int64_t dst_rows,
    const void* src, int64_t src_row_stride, int64_t src_sub_stride, const int64_t* d_src_index, int64_t src_rows,
    int64_t width, int64_t n_sub, int64_t n_rows, uint32_t* d_status, void* stream) {
  using namespace ashkv;
  if (width < 0 || n_sub < 0 || n_rows < 0 || dst_rows < 0 || src_rows < 0) return ASHKV_BAD_ARGUMENT;
  if (width == 0 || n_sub == 0 || n_rows == 0) return ASHKV_OK;
  if (!dst || !src) return ASHKV_BAD_ARGUMENT;
  if ((width | dst_row_stride | dst_sub_stride | src_row_stride | src_sub_stride) % 16 || !aligned(dst, 16) ||
      !aligned(src, 16)) {
    set_message("ashkv_copy_rows_indexed: addresses, strides and width must be multiples of 16 bytes");
    return ASHKV_BAD_ARGUMENT;
  }
  RowCopyParams p{};
  p.dst = static_cast<uint8_t*>(const_cast<void*>(device_view(dst)));
  p.src = static_cast<const uint8_t*>(device_view(src));
  const bool idx_ok = (!d_dst_index || device_view(d_dst_index)) && (!d_src_index || device_view(d_src_index));
  if (!p.dst || !p.src || !idx_ok) {
    set_message("ashkv_copy_rows_indexed: every pointer must be device memory or page-locked host memory "
                "mapped for this device (index lists: device memory)");
    return ASHKV_BAD_ARGUMENT;
  }
  p.dst_row_stride = dst_row_stride; p.dst_sub_stride = dst_sub_stride; p.dst_index = d_dst_index;
  p.src_row_stride = src_row_stride; p.src_sub_stride = src_sub_stride; p.src_index = d_src_index;
  p.dst_rows = dst_rows; p.src_rows = src_rows;
  p.chunks = width / 16; p.n_sub = n_sub; p.n_rows = n_rows; p.status = d_status;
  const int64_t items = n_rows * n_sub;
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t g = std::min<int64_t>((items + 7) / 8, int64_t(sms) * 8);
  copy_rows_kernel<<<unsigned(g > 0 ? g : 1), 256, 0, as_stream(stream)>>>(p);
  return check_launch("copy_rows_indexed");
}

// ---------------------------------------------------------------- fill
// A 32-bit pattern over `bytes` of device memory: 32-byte streaming stores for
// the 32-byte-aligned body, 4-byte stores for the head and tail, grid-stride
// over 16 CTAs of 128 threads per SM.  Clears staging buffers and slot tails,
// and is the plain write stream the write-dominated decoders are compared with.
namespace ashkv {
namespace {
__global__ void __launch_bounds__(128) fill32_kernel(uint32_t* head, int64_t n_head, uint32_t* body, int64_t n_body,
                                                     uint32_t* tail, int64_t n_tail, uint32_t v) {
  const int64_t i0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x, step = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = i0; i < n_body; i += step)
    asm volatile("st.global.cs.v8.u32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" :: "l"(body + 8 * i), "r"(v) : "memory");
  if (i0 < n_head) head[i0] = v;
  if (i0 < n_tail) tail[i0] = v;
}
}  // namespace
}  // namespace ashkv

extern "C" ashkv_status_t ashkv_fill32(void* d_dst, int64_t bytes, uint32_t value, void* stream) {
  using namespace ashkv;
  if (bytes < 0 || (bytes & 3)) return ASHKV_BAD_ARGUMENT;
  if (bytes == 0) return ASHKV_OK;
  if (!d_dst || !aligned(d_dst, 4)) return ASHKV_BAD_ARGUMENT;
  const uintptr_t a = reinterpret_cast<uintptr_t>(d_dst), end = a + uintptr_t(bytes);
  uintptr_t b0 = (a + 31) & ~uintptr_t(31), b1 = end & ~uintptr_t(31);
  if (b1 < b0) b0 = b1 = end;  // shorter than one aligned 32-byte block: all head
  const int64_t n_head = int64_t(b0 - a) / 4, n_body = int64_t(b1 - b0) / 32, n_tail = int64_t(end - b1) / 4;
  const int64_t need = (std::max<int64_t>(n_body, 8) + 127) / 128;
  const int64_t cap = int64_t(sm_count() > 0 ? sm_count() : 148) * 16;
  const unsigned grid = unsigned(std::max<int64_t>(1, std::min(need, cap)));
  fill32_kernel<<<grid, 128, 0, as_stream(stream)>>>(reinterpret_cast<uint32_t*>(a), n_head,
                                                     reinterpret_cast<uint32_t*>(b0), n_body,
                                                     reinterpret_cast<uint32_t*>(b1), n_tail, value);
  return check_launch("fill32");
}
