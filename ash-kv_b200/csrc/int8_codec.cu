// INT8 per-row absmax codec (sm_100a).
//
// Restates the arithmetic of the reference's Triton kernels
// (ashkv/codecs/int8.py:50-81 encode, :98-116 decode) as a single-pass CUDA
// kernel: a "team" of threads owns one row, keeps the row in registers
// between the absmax reduction and the quantisation, and issues 16-byte
// loads/stores.  Short rows (INT8Codec, 128 elements) take row_len / 32
// threads with 32 elements each, packing several rows per warp; long rows (the
// SGLang hooks, head_num * head_dim elements) spread over a full warp.
#include "common.cuh"

namespace ashkv {
namespace {

struct Int8EncParams {
  const uint16_t* src;      // bf16 or fp16 bits
  int64_t n_rows;
  int32_t row_len;
  int64_t src_stride;       // elements
  const int64_t* row_index; // optional gather
  uint8_t* codes;
  int64_t codes_stride;     // bytes
  uint8_t* scales;          // byte-addressed
  int32_t scales_per_slot;
  int32_t sps_shift;        // log2(scales_per_slot) when it is a power of two, else -1
  int64_t scale_slot_stride;
  int32_t scale_fp16;
  int32_t fp32_product;
  // several layers in one launch (blockIdx.y = layer): source rows from
  // layer_src[layer], codes and scales shifted by layer * layer_*_offset bytes
  const uint64_t* layer_src;
  int32_t n_layers;
  int64_t layer_codes_offset;
  int64_t layer_scales_offset;
};

__device__ __forceinline__ Int8EncParams for_layer(const Int8EncParams& p0) {
  Int8EncParams p = p0;
  if (p0.layer_src) {
    const int64_t l = blockIdx.y;
    p.src = reinterpret_cast<const uint16_t*>(p0.layer_src[l]);
    p.codes += l * p0.layer_codes_offset;
    p.scales += l * p0.layer_scales_offset;
  }
  return p;
}

struct Int8DecParams {
  const uint8_t* codes;
  int64_t codes_stride;
  const uint8_t* scales;
  int32_t scales_per_slot;
  int32_t sps_shift;        // log2(scales_per_slot) when it is a power of two, else -1
  int64_t scale_slot_stride;
  int32_t scale_fp16;
  int64_t n_rows;
  int32_t row_len;
  uint16_t* dst;
  int32_t dst_fp16;
  int64_t dst_stride;
  const int64_t* row_index;
};

template <bool FP16>
__device__ __forceinline__ float in_lo(uint32_t w) {
  if constexpr (FP16) return __half2float(__ushort_as_half(uint16_t(w & 0xFFFFu)));
  else return bf16lo(w);
}
template <bool FP16>
__device__ __forceinline__ float in_hi(uint32_t w) {
  if constexpr (FP16) return __half2float(__ushort_as_half(uint16_t(w >> 16)));
  else return bf16hi(w);
}

// s = x * 127 rounded to the input dtype (Triton >= 3 keeps the bf16/fp16
// product of a tensor and a weakly-typed Python float in the tensor's dtype).
template <bool FP16>
__device__ __forceinline__ float scaled127(float x, bool fp32_product) {
  float p = __fmul_rn(x, 127.0f);  // exact for bf16 inputs (8+7 bits); fp16 needs <= 18 bits
  if (fp32_product) return p;
  if constexpr (FP16) return __half2float(__float2half_rn(p));
  else return __bfloat162float(__float2bfloat16_rn(p));
}

// Byte offset of row r's scale: (r / sps) * slot_stride + (r % sps) * 2, with
// shifts when sps is a power of two (the plain array and the hooks' head counts).
__device__ __forceinline__ int64_t scale_offset(int64_t r, int32_t sps, int32_t sps_shift, int64_t slot_stride) {
  if (sps_shift >= 0) return (r >> sps_shift) * slot_stride + (r & ((int64_t(1) << sps_shift) - 1)) * 2;
  return (r / sps) * slot_stride + (r % sps) * 2;
}

// Each thread owns NCH chunks of 8 consecutive elements of its row.
// bf16 rows of up to 2 chunks per lane take two rows per team, both loaded
// before either is encoded (more bytes in flight per thread).
template <bool FP16, int NCH>
__host__ __device__ constexpr int enc_rows_per_team() { return (!FP16 && NCH <= 2) ? 2 : 1; }

template <int NCH>
struct LoadedRow {
  uint4 chunk[NCH];
  float am;
};

template <bool FP16, int NCH, int TEAM>
__device__ __forceinline__ void load_row(const Int8EncParams& p, int64_t r, bool active, int lane_in_team,
                                         LoadedRow<NCH>& L) {
  L.am = 0.0f;
  if (!active) return;
  const int64_t src_row = p.row_index ? p.row_index[r] : r;
  const uint16_t* row = p.src + src_row * p.src_stride;
#pragma unroll
  for (int c = 0; c < NCH; ++c) L.chunk[c] = ld_nc_v4(row + (int64_t(c) * TEAM + lane_in_team) * 8);
}

// Called by every lane of the warp (the row maximum is a shuffle reduction).
template <bool FP16, int NCH, int TEAM>
__device__ __forceinline__ void encode_loaded_row(const Int8EncParams& p, int64_t r, bool active, int lane_in_team,
                                                  LoadedRow<NCH>& L) {
  float am = 0.0f;
  if constexpr (!FP16) {
    uint32_t words[4 * NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const bool a = active;
      words[4 * c] = a ? L.chunk[c].x : 0u; words[4 * c + 1] = a ? L.chunk[c].y : 0u;
      words[4 * c + 2] = a ? L.chunk[c].z : 0u; words[4 * c + 3] = a ? L.chunk[c].w : 0u;
    }
    am = team_absmax_bf16<TEAM>(words);  // NaN ignored, like tl.maximum
  } else {
    if (active) {
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const uint32_t w[4] = {L.chunk[c].x, L.chunk[c].y, L.chunk[c].z, L.chunk[c].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          am = fmaxf(am, fabsf(in_lo<FP16>(w[k])));  // fmaxf ignores NaN, like tl.maximum
          am = fmaxf(am, fabsf(in_hi<FP16>(w[k])));
        }
      }
    }
#pragma unroll
    for (int off = TEAM / 2; off > 0; off >>= 1)
      am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, off, TEAM));
  }
  if (!active) return;
  am = fmaxf(am, 1e-8f);

  if (lane_in_team == 0) {
    uint8_t* sp = p.scales + scale_offset(r, p.scales_per_slot, p.sps_shift, p.scale_slot_stride);
    uint16_t sv = p.scale_fp16 ? f32_to_f16(am) : f32_to_bf16(am);
    *reinterpret_cast<uint16_t*>(sp) = sv;
  }

  uint8_t* out = p.codes + r * p.codes_stride;
  const bool f32p = p.fp32_product != 0;
  const Int8Div d = int8_div(am);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const uint32_t w[4] = {L.chunk[c].x, L.chunk[c].y, L.chunk[c].z, L.chunk[c].w};
    uint32_t packed[2];
    if (!FP16 && !f32p) {
      packed[0] = int8_codes4_bf16(w[0], w[1], d);
      packed[1] = int8_codes4_bf16(w[2], w[3], d);
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t b = 0;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint32_t word = w[h * 2 + k];
          const int32_t c0 = int8_code(scaled127<FP16>(in_lo<FP16>(word), f32p), d);
          const int32_t c1 = int8_code(scaled127<FP16>(in_hi<FP16>(word), f32p), d);
          b |= (uint32_t(c0) & 0xFFu) << (16 * k);
          b |= (uint32_t(c1) & 0xFFu) << (16 * k + 8);
        }
        packed[h] = b;
      }
    }
    *reinterpret_cast<uint2*>(out + (int64_t(c) * TEAM + lane_in_team) * 8) = make_uint2(packed[0], packed[1]);
  }
}

// Each thread owns NCH chunks of 8 consecutive elements of its row(s).
template <bool FP16, int NCH, int TEAM>
__global__ void __launch_bounds__(256) int8_encode_kernel(const Int8EncParams p0) {
  const Int8EncParams p = for_layer(p0);
  constexpr int ROWS_PER_PASS = 256 / TEAM;
  constexpr int RPT = enc_rows_per_team<FP16, NCH>();
  const int lane_in_team = threadIdx.x % TEAM;
  const int64_t r0 = int64_t(blockIdx.x) * (ROWS_PER_PASS * RPT) + threadIdx.x / TEAM;
  LoadedRow<NCH> L[RPT];
#pragma unroll
  for (int u = 0; u < RPT; ++u) {
    const int64_t r = r0 + int64_t(u) * ROWS_PER_PASS;
    load_row<FP16, NCH, TEAM>(p, r, r < p.n_rows, lane_in_team, L[u]);
  }
#pragma unroll
  for (int u = 0; u < RPT; ++u) {
    const int64_t r = r0 + int64_t(u) * ROWS_PER_PASS;
    encode_loaded_row<FP16, NCH, TEAM>(p, r, r < p.n_rows, lane_in_team, L[u]);
  }
}

// Generic path: any row length / alignment, one element per thread step.
template <bool FP16>
__global__ void __launch_bounds__(256) int8_encode_generic_kernel(const Int8EncParams p0) {
  const Int8EncParams p = for_layer(p0);
  const int64_t r = int64_t(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= p.n_rows) return;
  const int64_t src_row = p.row_index ? p.row_index[r] : r;
  const uint16_t* row = p.src + src_row * p.src_stride;
  float am = 0.0f;
  for (int i = lane; i < p.row_len; i += 32) {
    const uint32_t w = row[i];
    am = fmaxf(am, fabsf(in_lo<FP16>(w)));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, off));
  am = fmaxf(am, 1e-8f);
  if (lane == 0) {
    uint8_t* sp = p.scales + scale_offset(r, p.scales_per_slot, p.sps_shift, p.scale_slot_stride);
    *reinterpret_cast<uint16_t*>(sp) = p.scale_fp16 ? f32_to_f16(am) : f32_to_bf16(am);
  }
  uint8_t* out = p.codes + r * p.codes_stride;
  const Int8Div d = int8_div(am);
  for (int i = lane; i < p.row_len; i += 32) {
    const uint32_t w = row[i];
    out[i] = uint8_t(int8_code(scaled127<FP16>(in_lo<FP16>(w), p.fp32_product != 0), d) & 0xFF);
  }
}


__device__ __forceinline__ uint16_t out_bits(float v, bool fp16) {
  // Triton casts to bf16 first, then the store converts to the pointer's type.
  const float b = __bfloat162float(__float2bfloat16_rn(v));
  return fp16 ? f32_to_f16(b) : f32_to_bf16(v);
}

template <int NCH, int TEAM>
__global__ void __launch_bounds__(256) int8_decode_kernel(const Int8DecParams p) {
  constexpr int ROWS_PER_CTA = 256 / TEAM;
  const int lane_in_team = threadIdx.x % TEAM;
  const int64_t r = int64_t(blockIdx.x) * ROWS_PER_CTA + threadIdx.x / TEAM;
  if (r >= p.n_rows) return;
  const uint16_t sbits = *reinterpret_cast<const uint16_t*>(
      p.scales + scale_offset(r, p.scales_per_slot, p.sps_shift, p.scale_slot_stride));
  const float scale = p.scale_fp16 ? f16_to_f32(sbits) : bf16_to_f32(sbits);
  const uint8_t* in = p.codes + r * p.codes_stride;
  const int64_t dst_row = p.row_index ? p.row_index[r] : r;
  uint16_t* out = p.dst + dst_row * p.dst_stride;
  const bool f16 = p.dst_fp16 != 0;
  const bool fast = int8_dec_fast(scale);
  const Recip y = make_recip(127.0f);
  const f2 S = pk2(scale, scale), YHI = pk2(y.hi, y.hi), YLO = pk2(y.lo, y.lo);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t e0 = (int64_t(c) * TEAM + lane_in_team) * 8;
    const uint2 w = *reinterpret_cast<const uint2*>(in + e0);
    const uint32_t ww[2] = {w.x, w.y};
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      f2 F[2];  // float(code) of bytes 0,1 and 2,3 of ww[h]
      int8x4_to_f2(ww[h], F[0], F[1]);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float a, b;
        if (fast) {
          upk2(div2_short(mul2(F[k], S), YHI, YLO), a, b);
        } else {
          upk2(F[k], a, b);
          a = __fdiv_rn(__fmul_rn(a, scale), 127.0f);
          b = __fdiv_rn(__fmul_rn(b, scale), 127.0f);
        }
        o[h * 2 + k] = f16 ? (uint32_t(out_bits(a, true)) | (uint32_t(out_bits(b, true)) << 16))
                           : f32x2_to_bf16x2(a, b);
      }
    }
    *reinterpret_cast<uint4*>(out + e0) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(256) int8_decode_generic_kernel(const Int8DecParams p) {
  const int64_t r = int64_t(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= p.n_rows) return;
  const uint16_t sbits = *reinterpret_cast<const uint16_t*>(
      p.scales + scale_offset(r, p.scales_per_slot, p.sps_shift, p.scale_slot_stride));
  const float scale = p.scale_fp16 ? f16_to_f32(sbits) : bf16_to_f32(sbits);
  const uint8_t* in = p.codes + r * p.codes_stride;
  const int64_t dst_row = p.row_index ? p.row_index[r] : r;
  uint16_t* out = p.dst + dst_row * p.dst_stride;
  const bool fast = int8_dec_fast(scale);
  for (int i = lane; i < p.row_len; i += 32)
    out[i] = out_bits(int8_dequant(int32_t(int8_t(in[i])), scale, fast), p.dst_fp16 != 0);
}

int32_t pow2_shift(int32_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int32_t k = 0;
  while ((1 << k) < v) ++k;
  return k;
}

// Threads per row and 8-element chunks per thread.  Rows of 32..1016 elements
// whose chunk count is 4 x a power of two take 4 chunks per thread (team =
// chunks / 4), so the per-row work -- the shuffle reduction, the divisor, the
// scale -- is spread over 32 elements per thread; longer rows take a full warp.
template <typename P, typename KFast>
bool pick_team(int32_t row_len, int& team, int& nch) {
  if (row_len % 8 != 0) return false;
  const int chunks = row_len / 8;
  if (chunks >= 4 && chunks < 128 && chunks % 4 == 0 && !((chunks / 4) & (chunks / 4 - 1))) {
    team = chunks / 4;
    nch = 4;
    return true;
  }
  team = chunks >= 32 ? 32 : chunks;
  if (team & (team - 1)) return false;  // team must be a power of two
  if (chunks % team) return false;
  nch = chunks / team;
  return nch == 1 || nch == 2 || nch == 4 || nch == 8 || nch == 16;
}

}  // namespace

#define ASHKV_ENC_CASE(FP, NC, TM)                                                        \
  if (nch == NC && team == TM) {                                                          \
    int8_encode_kernel<FP, NC, TM><<<dim3(unsigned((p.n_rows + (256 / TM) * enc_rows_per_team<FP, NC>() - 1) / \
                                             ((256 / TM) * enc_rows_per_team<FP, NC>())), unsigned(p.n_layers)), \
                                      256, 0, st>>>(p);                                   \
    return check_launch("int8_encode");                                                  \
  }

template <bool FP16>
static ashkv_status_t launch_encode(const Int8EncParams& p, int team, int nch, bool fast, cudaStream_t st) {
  if (fast) {
    ASHKV_ENC_CASE(FP16, 1, 1) ASHKV_ENC_CASE(FP16, 1, 2) ASHKV_ENC_CASE(FP16, 1, 4)
    ASHKV_ENC_CASE(FP16, 1, 8) ASHKV_ENC_CASE(FP16, 1, 16) ASHKV_ENC_CASE(FP16, 1, 32)
    ASHKV_ENC_CASE(FP16, 2, 1) ASHKV_ENC_CASE(FP16, 2, 32) ASHKV_ENC_CASE(FP16, 4, 1)
    ASHKV_ENC_CASE(FP16, 4, 2) ASHKV_ENC_CASE(FP16, 4, 4) ASHKV_ENC_CASE(FP16, 4, 8)
    ASHKV_ENC_CASE(FP16, 4, 16) ASHKV_ENC_CASE(FP16, 4, 32) ASHKV_ENC_CASE(FP16, 8, 32)
    ASHKV_ENC_CASE(FP16, 16, 32)
  }
  int8_encode_generic_kernel<FP16><<<dim3(unsigned((p.n_rows + 7) / 8), unsigned(p.n_layers)), 256, 0, st>>>(p);
  return check_launch("int8_encode_generic");
}
#undef ASHKV_ENC_CASE

}  // namespace ashkv

using namespace ashkv;

extern "C" ashkv_status_t ashkv_int8_encode_rows(
    const void* d_src, int32_t src_dtype, int64_t n_rows, int32_t row_len,
    int64_t src_row_stride, const int64_t* d_row_index,
    void* d_codes, int64_t codes_row_stride,
    void* d_scales, int32_t scale_dtype, int32_t scales_per_slot, int64_t scale_slot_stride,
    uint32_t flags, void* stream) {
  if (n_rows < 0 || row_len <= 0 || scales_per_slot <= 0) return ASHKV_BAD_ARGUMENT;
  if (src_dtype != ASHKV_DTYPE_BF16 && src_dtype != ASHKV_DTYPE_FP16) return ASHKV_BAD_ARGUMENT;
  if (scale_dtype != ASHKV_DTYPE_BF16 && scale_dtype != ASHKV_DTYPE_FP16) return ASHKV_BAD_ARGUMENT;
  if (n_rows == 0) return ASHKV_OK;
  if (!d_src || !d_codes || !d_scales) return ASHKV_BAD_ARGUMENT;
  if (n_rows > (int64_t(1) << 40)) return ASHKV_BAD_ARGUMENT;
  if (!aligned(d_scales, 2) || (scale_slot_stride % 2)) return ASHKV_BAD_ARGUMENT;

  Int8EncParams p{};
  p.n_layers = 1;
  p.src = static_cast<const uint16_t*>(d_src);
  p.n_rows = n_rows; p.row_len = row_len; p.src_stride = src_row_stride; p.row_index = d_row_index;
  p.codes = static_cast<uint8_t*>(d_codes); p.codes_stride = codes_row_stride;
  p.scales = static_cast<uint8_t*>(d_scales); p.scales_per_slot = scales_per_slot;
  p.sps_shift = pow2_shift(scales_per_slot);
  p.scale_slot_stride = scale_slot_stride; p.scale_fp16 = scale_dtype == ASHKV_DTYPE_FP16;
  p.fp32_product = (flags & ASHKV_INT8_FP32_PRODUCT) ? 1 : 0;

  int team = 0, nch = 0;
  bool fast = pick_team<void, void>(row_len, team, nch);
  // 16-byte loads need 16-byte aligned rows; 8-byte stores need 8-byte aligned code rows.
  fast = fast && aligned(d_src, 16) && ((src_row_stride * 2) % 16 == 0) &&
         aligned(d_codes, 8) && (codes_row_stride % 8 == 0);
  cudaStream_t st = as_stream(stream);
  return src_dtype == ASHKV_DTYPE_FP16 ? launch_encode<true>(p, team, nch, fast, st)
                                       : launch_encode<false>(p, team, nch, fast, st);
}

extern "C" ashkv_status_t ashkv_int8_encode_rows_layers(
    const uint64_t* d_layer_src, int32_t n_layers, int32_t src_dtype, int64_t n_rows, int32_t row_len,
    int64_t src_row_stride, const int64_t* d_row_index,
    void* d_codes, int64_t codes_row_stride, int64_t layer_codes_offset,
    void* d_scales, int32_t scale_dtype, int32_t scales_per_slot, int64_t scale_slot_stride,
    int64_t layer_scales_offset, uint32_t flags, void* stream) {
  if (n_rows < 0 || row_len <= 0 || scales_per_slot <= 0 || n_layers < 0 || n_layers > 65535)
    return ASHKV_BAD_ARGUMENT;
  if (src_dtype != ASHKV_DTYPE_BF16 && src_dtype != ASHKV_DTYPE_FP16) return ASHKV_BAD_ARGUMENT;
  if (scale_dtype != ASHKV_DTYPE_BF16 && scale_dtype != ASHKV_DTYPE_FP16) return ASHKV_BAD_ARGUMENT;
  if (n_rows == 0 || n_layers == 0) return ASHKV_OK;
  if (!d_layer_src || !d_codes || !d_scales) return ASHKV_BAD_ARGUMENT;
  if (n_rows > (int64_t(1) << 40)) return ASHKV_BAD_ARGUMENT;
  if (!aligned(d_scales, 2) || (scale_slot_stride % 2) || (layer_scales_offset % 2)) return ASHKV_BAD_ARGUMENT;

  Int8EncParams p{};
  p.n_layers = n_layers;
  p.layer_src = d_layer_src;
  p.src = nullptr;
  p.n_rows = n_rows; p.row_len = row_len; p.src_stride = src_row_stride; p.row_index = d_row_index;
  p.codes = static_cast<uint8_t*>(d_codes); p.codes_stride = codes_row_stride;
  p.layer_codes_offset = layer_codes_offset;
  p.scales = static_cast<uint8_t*>(d_scales); p.scales_per_slot = scales_per_slot;
  p.sps_shift = pow2_shift(scales_per_slot);
  p.scale_slot_stride = scale_slot_stride; p.scale_fp16 = scale_dtype == ASHKV_DTYPE_FP16;
  p.layer_scales_offset = layer_scales_offset;
  p.fp32_product = (flags & ASHKV_INT8_FP32_PRODUCT) ? 1 : 0;

  int team = 0, nch = 0;
  bool fast = pick_team<void, void>(row_len, team, nch);
  // every layer's rows must meet the fast kernel's alignment: the caller guarantees
  // 16-byte aligned layer bases (checked on the host side of the binding)
  fast = fast && ((src_row_stride * 2) % 16 == 0) && aligned(d_codes, 8) && (codes_row_stride % 8 == 0) &&
         (layer_codes_offset % 8 == 0);
  cudaStream_t st = as_stream(stream);
  return src_dtype == ASHKV_DTYPE_FP16 ? launch_encode<true>(p, team, nch, fast, st)
                                       : launch_encode<false>(p, team, nch, fast, st);
}

#define ASHKV_DEC_CASE(NC, TM)                                                             \
  if (nch == NC && team == TM) {                                                           \
    int8_decode_kernel<NC, TM><<<unsigned((p.n_rows + 256 / TM - 1) / (256 / TM)), 256, 0, st>>>(p); \
    return check_launch("int8_decode");                                                   \
  }

extern "C" ashkv_status_t ashkv_int8_decode_rows(
    const void* d_codes, int64_t codes_row_stride,
    const void* d_scales, int32_t scale_dtype, int32_t scales_per_slot, int64_t scale_slot_stride,
    int64_t n_rows, int32_t row_len,
    void* d_dst, int32_t dst_dtype, int64_t dst_row_stride, const int64_t* d_row_index,
    void* stream) {
  if (n_rows < 0 || row_len <= 0 || scales_per_slot <= 0) return ASHKV_BAD_ARGUMENT;
  if (scale_dtype != ASHKV_DTYPE_BF16 && scale_dtype != ASHKV_DTYPE_FP16) return ASHKV_BAD_ARGUMENT;
  if (dst_dtype != ASHKV_DTYPE_BF16 && dst_dtype != ASHKV_DTYPE_FP16) return ASHKV_BAD_ARGUMENT;
  if (n_rows == 0) return ASHKV_OK;
  if (!d_codes || !d_scales || !d_dst) return ASHKV_BAD_ARGUMENT;
  if (!aligned(d_scales, 2) || (scale_slot_stride % 2)) return ASHKV_BAD_ARGUMENT;

  Int8DecParams p;
  p.codes = static_cast<const uint8_t*>(d_codes); p.codes_stride = codes_row_stride;
  p.scales = static_cast<const uint8_t*>(d_scales); p.scales_per_slot = scales_per_slot;
  p.sps_shift = pow2_shift(scales_per_slot);
  p.scale_slot_stride = scale_slot_stride; p.scale_fp16 = scale_dtype == ASHKV_DTYPE_FP16;
  p.n_rows = n_rows; p.row_len = row_len;
  p.dst = static_cast<uint16_t*>(d_dst); p.dst_fp16 = dst_dtype == ASHKV_DTYPE_FP16;
  p.dst_stride = dst_row_stride; p.row_index = d_row_index;

  int team = 0, nch = 0;
  bool fast = pick_team<void, void>(row_len, team, nch);
  fast = fast && aligned(d_codes, 8) && (codes_row_stride % 8 == 0) &&
         aligned(d_dst, 16) && ((dst_row_stride * 2) % 16 == 0);
  cudaStream_t st = as_stream(stream);
  if (fast) {
    ASHKV_DEC_CASE(1, 1) ASHKV_DEC_CASE(1, 2) ASHKV_DEC_CASE(1, 4) ASHKV_DEC_CASE(1, 8)
    ASHKV_DEC_CASE(1, 16) ASHKV_DEC_CASE(1, 32) ASHKV_DEC_CASE(2, 1) ASHKV_DEC_CASE(2, 32)
    ASHKV_DEC_CASE(4, 1) ASHKV_DEC_CASE(4, 2) ASHKV_DEC_CASE(4, 4) ASHKV_DEC_CASE(4, 8) ASHKV_DEC_CASE(4, 16)
    ASHKV_DEC_CASE(4, 32) ASHKV_DEC_CASE(8, 32) ASHKV_DEC_CASE(16, 32)
  }
  int8_decode_generic_kernel<<<unsigned((n_rows + 7) / 8), 256, 0, st>>>(p);
  return check_launch("int8_decode_generic");
}
#undef ASHKV_DEC_CASE
