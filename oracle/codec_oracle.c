/*
 * codec_oracle.c — TEST INFRASTRUCTURE ONLY.
 *
 * A scalar CPU restatement of the reference ASH-KV codec arithmetic, used by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker for the CUDA kernels in libashkv_cuda.so.  Nothing in the product
 * links or calls this file.
 *
 * Build: see oracle/build.py (gcc -O2 -ffp-contract=off, so every float
 * operation below is one IEEE-754 operation, as in the reference's PyTorch
 * evaluation on the host).
 *
 * Reference functions restated (paths relative to the ASH-KV source tree):
 *   oracle_int8_encode / _decode   ashkv/codecs/int8.py:50-81, :98-116
 *   oracle_nbit_encode / _decode   ashkv/codecs/nbit_dithered.py:43-167
 *                                  ashkv/codecs/int2_dithered.py:36-147 (bits = 2)
 *   oracle_xxh64                   ashkv/codecs/checksum.py:26-37 (xxhash.xxh64,
 *                                  public XXH64 specification)
 *   oracle_philox4x32_10           Salmon et al., SC'11 (the production dither source)
 *   oracle_fp8_encode / _decode    ashkv/codecs/fp8.py:32-79 (torch float8_e4m3fn casts)
 *   oracle_int4_encode / _decode   ashkv/codecs/int4.py:38-112
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ------------------------------------------------------------ conversions */
static float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

/* fp32 -> bf16, round to nearest even, NaN -> 0x7FFF (CUDA's encoding). */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u = f32_to_bits(f);
  if (isnan(f)) return 0x7FFF;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* fp32 -> fp16, round to nearest even, overflow -> inf, NaN -> 0x7FFF. */
uint16_t oracle_f32_to_f16(float f) {
  uint32_t u = f32_to_bits(f);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  if (isnan(f)) return 0x7FFF;
  uint32_t a = u & 0x7FFFFFFFu;
  if (a >= 0x47800000u) return sign | 0x7C00u; /* >= 65536 -> inf (also catches inf) */
  if (a < 0x33000000u) return sign;            /* < 2^-25 -> +-0 */
  int32_t e = (int32_t)(a >> 23) - 127;
  uint32_t m = (a & 0x7FFFFFu) | 0x800000u;    /* 24-bit significand */
  if (e < -14) {                               /* subnormal result */
    int shift = -14 - e + 13;                  /* bits to drop */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return sign | (uint16_t)q;
  }
  uint32_t q = m >> 13, rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  uint32_t h = ((uint32_t)(e + 15) << 10) + (q - 0x400u);  /* carry into exponent is fine */
  if (h >= 0x7C00u) return sign | 0x7C00u;
  return sign | (uint16_t)h;
}

float oracle_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  if (e == 0) {
    float v = ldexpf((float)m, -24);
    return sign ? -v : v;
  }
  if (e == 31) return bits_to_f32(sign | 0x7F800000u | (m << 13));
  return bits_to_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* ------------------------------------------------------------ INT8 codec */
static float in_val(const uint16_t* src, int64_t i, int fp16) {
  return fp16 ? oracle_f16_to_f32(src[i]) : bf16_to_f32(src[i]);
}

/* Triton's fp32 -> int8 cast on the GPU: truncate to int32 (saturating, NaN
 * -> 0), keep the low byte.  Only an infinite product leaves [-128, 127]:
 * +inf gives -1 and -inf gives 0 (pinned by the B200 reference fixtures). */
static int8_t triton_cast_s8(float r) {
  int32_t v;
  if (isnan(r)) v = 0;
  else if (r >= 2147483648.0f) v = INT32_MAX;
  else if (r <= -2147483648.0f) v = INT32_MIN;
  else v = (int32_t)r; /* C cast truncates toward zero */
  return (int8_t)(uint8_t)((uint32_t)v & 0xFFu);
}

/* Per row: am = max(max|x| (NaN ignored), 1e-8); s = x*127 rounded to the
 * input dtype (fp32 if fp32_product); code = cast(trunc(s/am +- 0.5)).
 *
 * The reference's Triton kernel divides with PTX div.full.f32, an
 * approximation within 2 ulp whose exact results this CPU restatement cannot
 * reproduce; it divides exactly and, when `tie` is given, sets tie[i] = 1 for
 * every element whose exact quotient lies within 2^-20 * max(|q|, 1) of a
 * half-integer.  Only there can the two divisions give codes one apart. */
void oracle_int8_encode(const uint16_t* src, int src_fp16, int64_t n_rows, int32_t row_len,
                        int fp32_product, int8_t* codes, uint16_t* scales, int scale_fp16, uint8_t* tie) {
  for (int64_t r = 0; r < n_rows; ++r) {
    const uint16_t* row = src + r * row_len;
    float am = 0.0f;
    for (int32_t i = 0; i < row_len; ++i) {
      /* every NaN is skipped, signalling ones too (the GPU max instruction's
         rule; C library fmaxf may return a NaN for a signalling operand) */
      const float a = fabsf(in_val(row, i, src_fp16));
      if (a > am) am = a;
    }
    am = fmaxf(am, 1e-8f);
    scales[r] = scale_fp16 ? oracle_f32_to_f16(am) : oracle_f32_to_bf16(am);
    for (int32_t i = 0; i < row_len; ++i) {
      float p = in_val(row, i, src_fp16) * 127.0f;
      float s;
      if (fp32_product) s = p;
      else if (src_fp16) s = oracle_f16_to_f32(oracle_f32_to_f16(p));
      else s = bf16_to_f32(oracle_f32_to_bf16(p));
      float q = s / am;
      float rr = q + (q > 0.0f ? 0.5f : -0.5f);
      codes[r * row_len + i] = triton_cast_s8(rr);
      if (tie) {
        const double aq = fabs((double)s / (double)am);
        const double f = aq - floor(aq);
        tie[r * row_len + i] = (uint8_t)(isfinite(aq) && fabs(f - 0.5) <= ldexp(1.0, -20) * fmax(aq, 1.0));
      }
    }
  }
}

/* out = bf16(float(code) * float(scale) / 127), then (dst_fp16) converted to fp16. */
void oracle_int8_decode(const int8_t* codes, const uint16_t* scales, int scale_fp16, int64_t n_rows,
                        int32_t row_len, uint16_t* dst, int dst_fp16) {
  for (int64_t r = 0; r < n_rows; ++r) {
    float sc = scale_fp16 ? oracle_f16_to_f32(scales[r]) : bf16_to_f32(scales[r]);
    for (int32_t i = 0; i < row_len; ++i) {
      float v = ((float)codes[r * row_len + i] * sc) / 127.0f;
      uint16_t b = oracle_f32_to_bf16(v);
      dst[r * row_len + i] = dst_fp16 ? oracle_f32_to_f16(bf16_to_f32(b)) : b;
    }
  }
}

/* ------------------------------------------------------------ N-bit codec */
static float max_nan(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}

/* Pairwise sum of 32 doubles: level k adds elements i and i ^ 2^k. */
static double pairwise_sum32(const double* v) {
  double a[32];
  for (int i = 0; i < 32; ++i) a[i] = v[i];
  for (int w = 1; w < 32; w <<= 1)
    for (int i = 0; i < 32; i += 2 * w) a[i] = a[i] + a[i + w];
  return a[0];
}

/* Groups of 32 elements; `dither` holds U in [0, 1) per element (the
 * reference's torch.rand draw), noise = (U - 0.5) * delta. */
void oracle_nbit_encode(const uint16_t* src, int64_t n_groups, int bits, float sigma,
                        const float* dither, uint16_t* scales, uint8_t* codes, uint32_t* omask_out) {
  const float half = (float)((1 << bits) - 1) / 2.0f;
  const float maxc = (float)((1 << bits) - 1);
  for (int64_t g = 0; g < n_groups; ++g) {
    float x[32];
    for (int i = 0; i < 32; ++i) x[i] = bf16_to_f32(src[g * 32 + i]);
    /* mean: PyTorch's CPU reduction order for a 32-wide inner dimension. */
    float acc[8];
    for (int i = 0; i < 8; ++i) acc[i] = x[i];
    for (int j = 1; j < 4; ++j)
      for (int i = 0; i < 8; ++i) acc[i] = acc[i] + x[8 * j + i];
    float s = acc[0];
    for (int i = 1; i < 8; ++i) s = s + acc[i];
    const float mu = s / 32.0f;
    /* unbiased std in fp64 (two-pass, pairwise sums), rounded once to fp32;
     * PyTorch computes the same quantity in fp64 (Welford), the fp32 result
     * agrees except when it sits within ~1e-16 of a rounding boundary. */
    double t[32];
    for (int i = 0; i < 32; ++i) t[i] = (double)x[i];
    const double mu64 = pairwise_sum32(t) * 0.03125;
    for (int i = 0; i < 32; ++i) {
      const double d = (double)x[i] - mu64;
      t[i] = d * d;
    }
    const double m2 = pairwise_sum32(t);
    const float sd = (float)sqrt(m2 / 31.0);
    const float thr = sigma * (sd + 1e-8f);
    uint32_t om = 0;
    float am = 0.0f;
    for (int i = 0; i < 32; ++i) {
      const int o = fabsf(x[i] - mu) > thr;
      om |= (uint32_t)o << i;
      if (o) x[i] = mu;
      am = max_nan(am, fabsf(x[i]));
    }
    if (!isnan(am) && am < 1e-8f) am = 1e-8f;
    const float delta = am / half;
    scales[g] = oracle_f32_to_bf16(delta);
    if (omask_out) omask_out[g] = om;
    uint32_t code[32];
    for (int i = 0; i < 32; ++i) {
      const float noise = (dither[g * 32 + i] - 0.5f) * delta;
      const float a = x[i] + noise;
      const float v = a / delta + half;
      float vc = isnan(v) ? 0.0f : v;
      if (vc < 0.0f) vc = 0.0f;
      if (vc > maxc) vc = maxc;
      code[i] = (uint32_t)nearbyintf(vc); /* default rounding mode: half to even */
    }
    if (bits == 4) {
      for (int j = 0; j < 16; ++j) codes[g * 16 + j] = (uint8_t)((code[2 * j] << 4) | code[2 * j + 1]);
    } else if (bits == 2) {
      for (int j = 0; j < 8; ++j)
        codes[g * 8 + j] = (uint8_t)((code[4 * j] << 6) | (code[4 * j + 1] << 4) | (code[4 * j + 2] << 2) |
                                     code[4 * j + 3]);
    } else {
      for (int j = 0; j < 32; ++j) codes[g * 32 + j] = (uint8_t)code[j];
    }
  }
}

/* out = bf16((code - half) * float(bf16 delta)); then out[idx[k]] = val[k]. */
void oracle_nbit_decode(const uint16_t* scales, const uint8_t* codes, int64_t n_groups, int bits,
                        const int32_t* idx, const uint16_t* val, int64_t n_out, uint16_t* dst) {
  const float half = (float)((1 << bits) - 1) / 2.0f;
  for (int64_t g = 0; g < n_groups; ++g) {
    const float delta = bf16_to_f32(scales[g]);
    for (int i = 0; i < 32; ++i) {
      uint32_t c;
      if (bits == 4) {
        uint8_t b = codes[g * 16 + i / 2];
        c = (i & 1) ? (b & 0xFu) : (b >> 4);
      } else if (bits == 2) {
        uint8_t b = codes[g * 8 + i / 4];
        c = (b >> (6 - 2 * (i & 3))) & 3u;
      } else {
        c = codes[g * 32 + i];
      }
      dst[g * 32 + i] = oracle_f32_to_bf16(((float)c - half) * delta);
    }
  }
  const int64_t n_elems = n_groups * 32;
  for (int64_t k = 0; k < n_out; ++k)
    if (idx[k] >= 0 && idx[k] < n_elems) dst[idx[k]] = val[k];
}

/* ------------------------------------------------------------ XXH64 */
static const uint64_t XP1 = 0x9E3779B185EBCA87ull, XP2 = 0xC2B2AE3D27D4EB4Full,
                      XP3 = 0x165667B19E3779F9ull, XP4 = 0x85EBCA77C2B2AE63ull,
                      XP5 = 0x27D4EB2F165667C5ull;
static uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static uint64_t rd64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }
static uint32_t rd32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
static uint64_t xround(uint64_t acc, uint64_t in) { acc += in * XP2; acc = rotl64(acc, 31); return acc * XP1; }
static uint64_t xmerge(uint64_t h, uint64_t v) { h ^= xround(0, v); return h * XP1 + XP4; }

uint64_t oracle_xxh64(const uint8_t* p, int64_t len, uint64_t seed) {
  const uint8_t* end = p + len;
  uint64_t h;
  if (len >= 32) {
    uint64_t v1 = seed + XP1 + XP2, v2 = seed + XP2, v3 = seed, v4 = seed - XP1;
    const uint8_t* limit = end - 32;
    do {
      v1 = xround(v1, rd64(p)); v2 = xround(v2, rd64(p + 8));
      v3 = xround(v3, rd64(p + 16)); v4 = xround(v4, rd64(p + 24));
      p += 32;
    } while (p <= limit);
    h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
    h = xmerge(h, v1); h = xmerge(h, v2); h = xmerge(h, v3); h = xmerge(h, v4);
  } else {
    h = seed + XP5;
  }
  h += (uint64_t)len;
  while (p + 8 <= end) { h ^= xround(0, rd64(p)); h = rotl64(h, 27) * XP1 + XP4; p += 8; }
  if (p + 4 <= end) { h ^= (uint64_t)rd32(p) * XP1; h = rotl64(h, 23) * XP2 + XP3; p += 4; }
  while (p < end) { h ^= (uint64_t)(*p) * XP5; h = rotl64(h, 11) * XP1; ++p; }
  h ^= h >> 33; h *= XP2; h ^= h >> 29; h *= XP3; h ^= h >> 32;
  return h;
}

void oracle_xxh64_items(const uint8_t* data, int64_t n_items, int64_t item_bytes, int64_t stride,
                        uint64_t seed, uint64_t* out) {
  for (int64_t i = 0; i < n_items; ++i) out[i] = oracle_xxh64(data + i * stride, item_bytes, seed);
}

/* ------------------------------------------------------------ Philox */
void oracle_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Uniforms U = (b + 0.5) / 256 that the PHILOX mode of the kernel uses for
 * elements [offset, offset + n), b being byte (e & 15) (little-endian order
 * over the four output words) of Philox4x32-10(counter = e >> 4, key = seed). */
void oracle_philox_dither(int64_t n, uint64_t seed, uint64_t offset, float* out) {
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint64_t cached = ~0ull;
  uint32_t r[4] = {0, 0, 0, 0};
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t e = offset + (uint64_t)i;
    const uint64_t c = e >> 4;
    if (c != cached) {
      const uint32_t ctr[4] = {(uint32_t)c, (uint32_t)(c >> 32), 0u, 0u};
      oracle_philox4x32_10(ctr, key, r);
      cached = c;
    }
    const int f = (int)(e & 15u);
    const uint32_t b = (r[f >> 2] >> (8 * (f & 3))) & 0xFFu;
    out[i] = ((float)b + 0.5f) * (1.0f / 256.0f);
  }
}

/* ------------------------------------------------------------ FP8 (E4M3FN) codec */
/* bf16 -> float8_e4m3fn as torch's cast computes it (ashkv/codecs/fp8.py:51-60
 * calls tensor.to(torch.float8_e4m3fn)): round to nearest even over the
 * E4M3FN grid (bias 7, subnormal step 2^-9, largest finite 448), with NO
 * saturation: a magnitude that rounds past 448 (> 464), an infinity or a NaN
 * becomes the NaN code 0x7F with the input's sign. */
static uint8_t fp8_from_f32(float f) {
  const uint8_t sign = (f32_to_bits(f) >> 24) & 0x80u;
  const float a = fabsf(f);
  if (!(a <= 464.0f)) return (uint8_t)(sign | 0x7Fu);
  if (a < 0x1p-6f) /* subnormal range: multiples of 2^-9 (8 rounds up to the smallest normal) */
    return (uint8_t)(sign | (uint8_t)nearbyintf(a * 512.0f));
  int e;
  frexpf(a, &e);                                  /* a = m * 2^e, m in [0.5, 1) */
  e -= 1;                                         /* a = 1.f * 2^e, e in [-6, 8] */
  const int steps = (int)nearbyintf(ldexpf(a, 3 - e)); /* 8..16 eighths of 2^e */
  return (uint8_t)(sign | (((e + 7) << 3) + steps - 8)); /* 16 carries into the exponent */
}

void oracle_fp8_encode(const uint16_t* src, int64_t n, uint8_t* dst) {
  for (int64_t i = 0; i < n; ++i) dst[i] = fp8_from_f32(bf16_to_f32(src[i]));
}

/* float8_e4m3fn -> bf16 (fp8.py:71-79: view(float8_e4m3fn).to(bfloat16)).
 * Every finite E4M3FN value is exact in bf16; NaN codes (0x7F, 0xFF) become
 * `nan_bits` (0x7FFF from torch's CUDA cast, which the reference uses
 * whenever a GPU is present). */
void oracle_fp8_decode(const uint8_t* src, int64_t n, uint16_t nan_bits, uint16_t* dst) {
  for (int64_t i = 0; i < n; ++i) {
    const uint8_t c = src[i];
    const int e = (c >> 3) & 15, m = c & 7;
    if (e == 15 && m == 7) { dst[i] = nan_bits; continue; }
    const float mag = e == 0 ? ldexpf((float)m, -9) : ldexpf((float)(8 + m), e - 10);
    dst[i] = oracle_f32_to_bf16((c & 0x80) ? -mag : mag);
  }
}

/* ------------------------------------------------------------ INT4 group codec */
/* numpy's float32 -> int8 cast on x86 (the cast ashkv/codecs/int4.py:61
 * applies after np.round): truncate to int32 (NaN, infinities and values
 * outside int32 give INT32_MIN) and keep the low byte. */
static int8_t np_f32_to_i8(float r) {
  int32_t v = INT32_MIN;
  if (r > -2147483648.0f && r < 2147483648.0f) v = (int32_t)r;
  return (int8_t)(uint8_t)(uint32_t)v;
}

/* torch CPU float32 -> bf16 (int4.py:72, :112): round to nearest even, every
 * NaN written as `nan_bits` (0xFFFF from torch's vectorised CPU cast). */
static uint16_t bf16_cpu(float f, uint16_t nan_bits) {
  return isnan(f) ? nan_bits : oracle_f32_to_bf16(f);
}

/* INT4Codec.encode (int4.py:38-75) over n bf16 values zero-padded to
 * n_groups * group_size: am = maximum(max|x|, 1e-8) with NaN propagating
 * (np.max / np.maximum), q = clip(int8(round_half_even(x*7/am)), -8, 7),
 * nibble = q + 8, high nibble = even element; scale = bf16(am).
 * packed holds n_groups*group_size/2 bytes (the caller checks evenness). */
void oracle_int4_encode(const uint16_t* src, int64_t n, int32_t group_size, int64_t n_groups,
                        uint16_t nan_bits, uint16_t* scales, uint8_t* packed) {
  const int64_t total = n_groups * group_size;
  for (int64_t i = 0; i < total / 2; ++i) packed[i] = 0;
  for (int64_t g = 0; g < n_groups; ++g) {
    float am = 0.0f;
    int nan_seen = 0;
    for (int32_t k = 0; k < group_size; ++k) {
      const int64_t i = g * group_size + k;
      const float x = i < n ? bf16_to_f32(src[i]) : 0.0f;
      if (isnan(x)) nan_seen = 1;
      else if (fabsf(x) > am) am = fabsf(x);
    }
    if (nan_seen) am = NAN;
    else if (am < 1e-8f) am = 1e-8f;
    scales[g] = bf16_cpu(am, nan_bits);
    for (int32_t k = 0; k < group_size; ++k) {
      const int64_t i = g * group_size + k;
      const float x = i < n ? bf16_to_f32(src[i]) : 0.0f;
      const float prod = x * 7.0f;
      const float v = prod / am;
      int q = np_f32_to_i8(nearbyintf(v));
      if (q < -8) q = -8;
      if (q > 7) q = 7;
      const uint8_t nib = (uint8_t)(q + 8) & 15u;
      if ((i & 1) == 0) packed[i >> 1] |= (uint8_t)(nib << 4);
      else packed[i >> 1] |= nib;
    }
  }
}

/* INT4Codec.decode (int4.py:77-112): out = bf16(float(nibble - 8) * float(scale) / 7). */
void oracle_int4_decode(const uint16_t* scales, const uint8_t* packed, int64_t n_groups, int32_t group_size,
                        uint16_t nan_bits, uint16_t* dst) {
  const int64_t total = n_groups * group_size;
  for (int64_t i = 0; i < total; ++i) {
    const uint8_t b = packed[i >> 1];
    const int q = ((i & 1) == 0 ? (b >> 4) : (b & 15)) - 8;
    const float p = (float)q * bf16_to_f32(scales[i / group_size]);
    dst[i] = bf16_cpu(p / 7.0f, nan_bits);
  }
}
