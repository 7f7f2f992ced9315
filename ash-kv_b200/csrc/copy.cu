// Strided host<->device / device<->device copy entry point.
//
// The SGLang host pool keeps one 2*head_num*head_dim-byte slot per
// (token, layer); a compressed slot only uses its first 2*head_num +
// head_num*head_dim bytes.  A pitched copy moves just those bytes for many
// slots in one DMA operation instead of gathering whole slots on the host.
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
