// Mixed-tier page migration: one launch moves every page of a transition list
// from its current tier's representation to its target tier's (sm_100a).
//
// Replaces the per-page migrate() ladder (ashkv/runtime/migrate.py:35-191)
// for the transitions the controller plans (ashkv/runtime/controller.py:88-104:
// one step hotter on promotion, one step colder on demotion), with the codec
// of each tier edge as the resolver assigns it
// (ashkv/compiler/codec_resolver.py:56-95): BF16 <-> FP8 slot (INT8 or FP8
// codec), FP8 slot <-> INT4 (INT4Codec or the dithered 4-bit codec), INT4 <->
// ARCHIVE (the dithered INT2 codec).  The reference's migrate applies the
// edge's codec to the page's stored bytes; here a page is decoded from its
// current format to bf16 and encoded into the target format, so every tier
// holds a compressed image of the page's bf16 values.
//
// A page is 2*T token rows of row_len bf16 (its K rows, then its V rows) of one
// layer: E = 2 * T * row_len elements.  Per list entry one CTA
//   1. checks the entry the way migrate() does (pinned -> skipped, already at
//      target -> skipped, a tier without a codec -> skipped) and takes a slot
//      of the target tier's store (free stack, popped with an atomic);
//   2. decodes the page (into a bf16 staging tile in shared memory for the
//      staged edges: 64-byte rows of 32 elements, 16-byte chunks XOR-swizzled
//      so thread-per-group and thread-per-chunk access are both free of bank
//      conflicts);
//   3. encodes it into the target slot (or the page's KV-pool rows);
//   4. commits tier and slot in the device page table and records the slot it
//      gave up.  ashkv_release_slots pushes recorded slots back afterwards, so
//      stacks are only popped in this kernel and only pushed in that one.
// Entries are resolved 32 at a time by one warp (list -> page -> table
// columns -> slot) so that chain of dependent loads is paid once per batch.
// Two launches share a list.  The direct pass moves the edges that need no
// staging tile (BF16 -> INT8 row by row, BF16 -> FP8 chunk by chunk, and every
// decode into BF16, which first copies the compressed slot into shared memory
// with cp.async) and reports the entries that do not move.  With two or more
// compressed tiers it also moves compressed -> INT8 / FP8 / INT4 pages: the
// raw slot copy is decoded chunk by chunk straight into the target's encoder
// (dithered sources overlay their outliers from a per-group index of the
// sorted outlier list), so that compute-heavy work runs beside the
// memory-bound BF16 edges of the same list.  The staged pass (the bf16 tile,
// and the dithered encoder's per-page outlier ranking) takes the edges into
// the dithered formats and BF16 -> INT4.
#include <algorithm>

#include "common.cuh"
#include "fp8_conv.cuh"
#include "int4_group.cuh"
#include "nbit_group.cuh"

namespace ashkv {
namespace {

constexpr int kThreads = 256;  // largest CTA; smaller pages take smaller CTAs (block_threads)
constexpr int kWarps = kThreads / 32;
// Threads / warps of the running CTA: one page per CTA, and the CTA is sized to
// the page (a 128-wide row's page gets one warp) so that no warp idles.
#define kNT int(blockDim.x)
#define kNW int(blockDim.x >> 5)
__host__ __device__ constexpr int block_threads(int row) { return row >= 1024 ? 256 : row / 4; }
constexpr int kTiers = 6;
constexpr int kBatch = 32;
constexpr int kMaxElems = 65536;  // 128 KiB of staging; outlier indices fit in 16 bits
constexpr int kDirectBlocks = 3;  // CTAs per SM of the direct pass (registers <= 85)
constexpr int kStagedBlocks = 3;  // CTAs per SM of the staged pass (registers <= 85, 3 x 68 KiB)

struct Store {
  uint8_t* data;
  int64_t slot_bytes;
  int32_t n_slots;
  int32_t format;
  int32_t* free_stack;
  int32_t* free_top;
};

struct MigParams {
  int8_t* tier;
  const int32_t* pin;
  const int32_t* layer_id;
  const int32_t* token_start;
  int32_t* page_slot;
  int64_t n_pages;
  const int8_t* target;
  const int32_t* list;
  const int32_t* count;
  int32_t max_entries;
  const uint64_t* layer_k;
  const uint64_t* layer_v;
  int32_t n_layers;
  int32_t T;
  int32_t row_len;
  int64_t row_stride;
  Store store[kTiers];
  float sigma;
  int32_t outlier_cap;
  uint32_t round_keys[20];
  int32_t* entry_status;
  int32_t* released;
  int32_t first_offset;  // direct pass: byte offset of the outlier index after the raw slot copy
};

struct Entry {
  uint64_t kbase, vbase;  // K / V row of the page's first token in the pool
  int32_t page, cur, tgt, layer, ts, old_slot, new_slot, status;
};

__host__ __device__ __forceinline__ int64_t int8_codes_offset(int T) { return (4 * int64_t(T) + 15) / 16 * 16; }

// Slot layouts (E elements, offsets in bytes):
//   INT8   [2T fp16 scales | pad to 16 | E int8 codes]           (the hooks' per-token layout)
//   FP8    [E e4m3fn bytes]
//   INT4   [E/64 bf16 scales | E/2 nibble bytes]                 (INT4Codec, group 64)
//   NBIT*  [u32 n_out, 3 x u32 0 | E/32 bf16 delta | E*bits/8 codes | cap x u32 outliers]
//          outlier entry = (element index in the page << 16) | bf16 bits, ascending
__host__ __device__ __forceinline__ int64_t nbit_delta_off() { return 16; }
__host__ __device__ __forceinline__ int64_t nbit_codes_off(int64_t E) { return 16 + E / 16; }
__host__ __device__ __forceinline__ int64_t nbit_entries_off(int64_t E, int bits) {
  return nbit_codes_off(E) + E * bits / 8;
}

int64_t slot_bytes_for(int32_t format, int64_t E, int32_t cap) {
  int64_t b = -1;
  switch (format) {
    case ASHKV_PAGE_INT8: b = -1; break;  // needs T; computed by the caller
    case ASHKV_PAGE_FP8: b = E; break;
    case ASHKV_PAGE_INT4: b = E / 32 + E / 2; break;
    case ASHKV_PAGE_NBIT4: b = nbit_entries_off(E, 4) + 4 * int64_t(cap); break;
    case ASHKV_PAGE_NBIT2: b = nbit_entries_off(E, 2) + 4 * int64_t(cap); break;
    default: break;
  }
  return b;
}

// Bytes of a slot that hold data (rounded up to 16; slots are rounded to 256).
__host__ __device__ __forceinline__ int64_t used_bytes(int32_t format, int64_t E, int T, int32_t cap) {
  int64_t b = 0;
  switch (format) {
    case ASHKV_PAGE_INT8: b = int8_codes_offset(T) + E; break;
    case ASHKV_PAGE_FP8: b = E; break;
    case ASHKV_PAGE_INT4: b = E / 32 + E / 2; break;
    case ASHKV_PAGE_NBIT4: b = nbit_entries_off(E, 4) + 4 * int64_t(cap); break;
    case ASHKV_PAGE_NBIT2: b = nbit_entries_off(E, 2) + 4 * int64_t(cap); break;
    default: break;
  }
  return (b + 15) / 16 * 16;
}

// Byte offset of element e in the staging tile: group g = e / 32 is a 64-byte
// row; 16-byte chunk k of it sits at position k ^ ((g >> 1) & 3).
__device__ __forceinline__ uint32_t stage_off(uint32_t e) {
  const uint32_t g = e >> 5;
  return (g << 6) + ((((e >> 3) & 3u) ^ ((g >> 1) & 3u)) << 4) + ((e & 7u) << 1);
}
__device__ __forceinline__ uint4 lds_chunk(const uint8_t* stage, uint32_t e) {
  return *reinterpret_cast<const uint4*>(stage + stage_off(e));
}
__device__ __forceinline__ void sts_chunk(uint8_t* stage, uint32_t e, uint4 v) {
  *reinterpret_cast<uint4*>(stage + stage_off(e)) = v;
}

__device__ __forceinline__ uint16_t* pool_row(const MigParams& p, const Entry& en, int r) {
  const int T = p.T;
  return reinterpret_cast<uint16_t*>(r < T ? en.kbase : en.vbase) + int64_t(r < T ? r : r - T) * p.row_stride;
}
// Chunk k (8 elements) of the page -> its address in the pool.
template <int ROW>
__device__ __forceinline__ uint16_t* pool_chunk(const MigParams& p, const Entry& en, int k) {
  constexpr int CPR = ROW / 8;
  return pool_row(p, en, k / CPR) + (k % CPR) * 8;
}

// 16-byte asynchronous global -> shared copy: no register staging, so every
// chunk of a page can be in flight at once; cp.async.wait_all completes them.
__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_addr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ uint2 ld_nc_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

// ---------------------------------------------------------------- 8-element decoders
// Eight INT8 codes with scale s -> eight bf16 (the reference decode).
__device__ __forceinline__ uint4 int8_dec8(uint2 cw, float s) {
  const Recip y = make_recip(127.0f);
  const f2 YHI = pk2(y.hi, y.hi), YLO = pk2(y.lo, y.lo), S = pk2(s, s);
  const bool fast = int8_dec_fast(s);
  const uint32_t ww[2] = {cw.x, cw.y};
  uint32_t o[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    f2 F0, F1;
    int8x4_to_f2(ww[h], F0, F1);
    if (fast) {
      o[2 * h] = f32x2_to_bf16x2_pk(div2_short(mul2(F0, S), YHI, YLO));
      o[2 * h + 1] = f32x2_to_bf16x2_pk(div2_short(mul2(F1, S), YHI, YLO));
    } else {
      float a, b;
      upk2(F0, a, b);
      o[2 * h] = f32x2_to_bf16x2(__fdiv_rn(__fmul_rn(a, s), 127.0f), __fdiv_rn(__fmul_rn(b, s), 127.0f));
      upk2(F1, a, b);
      o[2 * h + 1] = f32x2_to_bf16x2(__fdiv_rn(__fmul_rn(a, s), 127.0f), __fdiv_rn(__fmul_rn(b, s), 127.0f));
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
__device__ __forceinline__ uint4 fp8_dec8(uint2 c) {
  return make_uint4(bf16x2_from_fp8x2(c.x & 0xFFFFu), bf16x2_from_fp8x2(c.x >> 16),
                    bf16x2_from_fp8x2(c.y & 0xFFFFu), bf16x2_from_fp8x2(c.y >> 16));
}
__device__ __forceinline__ uint4 int4_dec8(uint32_t c, uint16_t scale) {
  uint32_t o[4];
  unpack_nibbles8(c, bf16_to_f32(scale), o);
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------- decoders (slot -> staging)
template <int ROW>
__device__ void stage_from_pool(const MigParams& p, const Entry& en, uint8_t* stage, int n8) {
  const uint32_t base = smem_u32(stage);
  for (int k = threadIdx.x; k < n8; k += kNT) cp_async16(base + stage_off(uint32_t(k) * 8u), pool_chunk<ROW>(p, en, k));
  cp_async_wait_all();
}

template <int ROW>
__device__ void stage_from_int8(const uint8_t* slot, int T, uint8_t* stage, int n8) {
  constexpr int CPR = ROW / 8;
  const uint8_t* codes = slot + int8_codes_offset(T);
  const Recip y = make_recip(127.0f);
  const f2 YHI = pk2(y.hi, y.hi), YLO = pk2(y.lo, y.lo);
  constexpr int U = 4;
  (void)YHI; (void)YLO;
  for (int k0 = threadIdx.x; k0 < n8; k0 += U * kNT) {
    uint2 cw[U];
    uint16_t sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + u * kNT;
      if (k < n8) {
        cw[u] = ld_nc_v2(codes + int64_t(k) * 8);
        sc[u] = reinterpret_cast<const uint16_t*>(slot)[k / CPR];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + u * kNT;
      if (k < n8) sts_chunk(stage, uint32_t(k) * 8u, int8_dec8(cw[u], f16_to_f32(sc[u])));
    }
  }
}

__device__ void stage_from_fp8(const uint8_t* slot, uint8_t* stage, int n8) {
  constexpr int U = 4;
  for (int k0 = threadIdx.x; k0 < n8; k0 += U * kNT) {
    uint2 c[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k0 + u * kNT < n8) c[u] = ld_nc_v2(slot + int64_t(k0 + u * kNT) * 8);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k0 + u * kNT < n8) sts_chunk(stage, uint32_t(k0 + u * kNT) * 8u, fp8_dec8(c[u]));
  }
}

__device__ void stage_from_int4(const uint8_t* slot, int64_t E, uint8_t* stage, int n8) {
  const uint16_t* scales = reinterpret_cast<const uint16_t*>(slot);
  const uint32_t* nib = reinterpret_cast<const uint32_t*>(slot + E / 32);
  constexpr int U = 4;
  for (int k0 = threadIdx.x; k0 < n8; k0 += U * kNT) {
    uint32_t c[U];
    uint16_t sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + u * kNT;
      if (k < n8) { c[u] = nib[k]; sc[u] = scales[k >> 3]; }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k0 + u * kNT < n8) sts_chunk(stage, uint32_t(k0 + u * kNT) * 8u, int4_dec8(c[u], sc[u]));
  }
}

template <int BITS>
__device__ void stage_from_nbit(const uint8_t* slot, int64_t E, int32_t cap, uint8_t* stage) {
  const uint16_t* delta = reinterpret_cast<const uint16_t*>(slot + nbit_delta_off());
  const uint8_t* codes = slot + nbit_codes_off(E);
  const int n_groups = int(E / 32);
  constexpr float half = float((1 << BITS) - 1) * 0.5f;
  for (int g = threadIdx.x; g < n_groups; g += kNT) {
    GroupCodes<BITS> gc;
    load_group<BITS>(delta, codes, g, gc);
    uint32_t o[16];
    group_bf16<BITS>(gc, half, o);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      sts_chunk(stage, uint32_t(g) * 32u + 8u * c, make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]));
  }
  __syncthreads();  // dense values first, then the outliers overwrite theirs
  const uint32_t n_out = min(*reinterpret_cast<const uint32_t*>(slot), uint32_t(cap));
  const uint32_t* ent = reinterpret_cast<const uint32_t*>(slot + nbit_entries_off(E, BITS));
  for (uint32_t j = threadIdx.x; j < n_out; j += kNT) {
    const uint32_t e = ent[j];
    const uint32_t idx = e >> 16;
    if (idx < uint32_t(E)) *reinterpret_cast<uint16_t*>(stage + stage_off(idx)) = uint16_t(e & 0xFFFFu);
  }
}

// ---------------------------------------------------------------- encoders (staging -> slot)
template <int ROW>
__device__ void pool_from_stage(const MigParams& p, const Entry& en, const uint8_t* stage, int n8) {
  constexpr int CPR = ROW / 8;
  for (int k = threadIdx.x; k < n8; k += kNT)
    *reinterpret_cast<uint4*>(pool_row(p, en, k / CPR) + (k % CPR) * 8) = lds_chunk(stage, uint32_t(k) * 8u);
}

// TEAM lanes per row, NCH chunks of 8 per lane (the row kernels' mapping).
template <int ROW>
__device__ void int8_from_stage(const uint8_t* stage, int T, uint8_t* slot) {
  constexpr int TEAM = ROW >= 1024 ? 32 : ROW / 32;
  constexpr int NCH = ROW / (8 * TEAM);
  constexpr int RPW = 32 / TEAM;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TEAM, lin = lane % TEAM;
  uint8_t* codes = slot + int8_codes_offset(T);
  for (int r0 = warp * RPW; r0 < 2 * T; r0 += kNW * RPW) {  // warp-uniform loop
    const int r = r0 + sub;
    const bool on = r < 2 * T;
    uint32_t w[4 * NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint4 v = on ? lds_chunk(stage, uint32_t(r) * ROW + uint32_t(c * TEAM + lin) * 8u) : make_uint4(0, 0, 0, 0);
      w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
    }
    const float am = fmaxf(team_absmax_bf16<TEAM>(w), 1e-8f);
    if (!on) continue;
    if (lin == 0) reinterpret_cast<uint16_t*>(slot)[r] = f32_to_f16(am);
    const Int8Div d = int8_div(am);
#pragma unroll
    for (int c = 0; c < NCH; ++c)
      *reinterpret_cast<uint2*>(codes + int64_t(r) * ROW + (c * TEAM + lin) * 8) =
          make_uint2(int8_codes4_bf16(w[4 * c], w[4 * c + 1], d), int8_codes4_bf16(w[4 * c + 2], w[4 * c + 3], d));
  }
}

__device__ void fp8_from_stage(const uint8_t* stage, uint8_t* slot, int n8) {
  for (int k = threadIdx.x; k < n8; k += kNT) {
    const uint4 v = lds_chunk(stage, uint32_t(k) * 8u);
    *reinterpret_cast<uint2*>(slot + int64_t(k) * 8) =
        make_uint2(fp8x2_from_bf16x2(v.x) | (fp8x2_from_bf16x2(v.y) << 16),
                   fp8x2_from_bf16x2(v.z) | (fp8x2_from_bf16x2(v.w) << 16));
  }
}

// INT4Codec, group 64: two lanes per group, each with one 32-element staging row.
__device__ void int4_from_stage(const uint8_t* stage, int64_t E, uint8_t* slot) {
  uint16_t* scales = reinterpret_cast<uint16_t*>(slot);
  uint8_t* nib = slot + E / 32;
  const int n_rows = int(E / 32), lane = threadIdx.x & 31;
  for (int base = threadIdx.x & ~31; base < n_rows; base += kNT) {  // warp-uniform
    const int g = base + lane;
    const bool on = g < n_rows;
    float x[4][8];
    float m = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      unpack_chunk(on ? lds_chunk(stage, uint32_t(g) * 32u + 8u * c) : make_uint4(0, 0, 0, 0), x[c]);
      m = chunk_max(m, x[c]);
    }
    m = max_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    if (!on) continue;
    const float am = group_max_finish(m);
    if ((g & 1) == 0) scales[g >> 1] = static_cast<uint16_t>(bf16_cpu(am));
    const GroupDiv d = group_div(am);
    uint32_t o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) o[c] = pack_chunk(x[c], d);
    *reinterpret_cast<uint4*>(nib + int64_t(g) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------- direct paths (no staging tile)
// BF16 -> INT8 walks the page row by row, BF16 -> FP8 chunk by chunk, and a
// decode into BF16 needs no tile either: warps stream the page with several
// rows in flight.  A compressed source is first copied whole into shared
// memory with cp.async (all of its bytes in flight), then decoded from there
// into the pool rows.

// BF16 pool rows -> INT8 slot: TEAM lanes per row, NCH chunks per lane, U row
// groups loaded before any is encoded.
template <int ROW>
__device__ void int8_from_pool(const MigParams& p, const Entry& en, uint8_t* slot) {
  constexpr int TEAM = ROW >= 1024 ? 32 : ROW / 32;
  constexpr int NCH = ROW / (8 * TEAM);
  constexpr int RPW = 32 / TEAM;
  constexpr int U = NCH <= 4 ? 2 : 1;
  const int T = p.T;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TEAM, lin = lane % TEAM;
  uint8_t* codes = slot + int8_codes_offset(T);
  for (int r0 = warp * RPW * U; r0 < 2 * T; r0 += kNW * RPW * U) {  // warp-uniform
    uint32_t w[U][4 * NCH];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r = r0 + u * RPW + sub;
      const uint16_t* row = r < 2 * T ? pool_row(p, en, r) : nullptr;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const uint4 v = row ? ld_nc_v4(row + (c * TEAM + lin) * 8) : make_uint4(0, 0, 0, 0);
        w[u][4 * c] = v.x; w[u][4 * c + 1] = v.y; w[u][4 * c + 2] = v.z; w[u][4 * c + 3] = v.w;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r = r0 + u * RPW + sub;
      const float am = fmaxf(team_absmax_bf16<TEAM>(w[u]), 1e-8f);
      if (r >= 2 * T) continue;
      if (lin == 0) reinterpret_cast<uint16_t*>(slot)[r] = f32_to_f16(am);
      const Int8Div d = int8_div(am);
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        *reinterpret_cast<uint2*>(codes + int64_t(r) * ROW + (c * TEAM + lin) * 8) = make_uint2(
            int8_codes4_bf16(w[u][4 * c], w[u][4 * c + 1], d), int8_codes4_bf16(w[u][4 * c + 2], w[u][4 * c + 3], d));
    }
  }
}

// BF16 pool rows -> FP8 slot, U chunks in flight per thread.
template <int ROW>
__device__ void fp8_from_pool(const MigParams& p, const Entry& en, uint8_t* slot, int n8) {
  constexpr int U = 4;
  for (int k0 = threadIdx.x; k0 < n8; k0 += U * kNT) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k0 + u * kNT < n8) v[u] = ld_nc_v4(pool_chunk<ROW>(p, en, k0 + u * kNT));
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + u * kNT;
      if (k >= n8) continue;
      *reinterpret_cast<uint2*>(slot + int64_t(k) * 8) =
          make_uint2(fp8x2_from_bf16x2(v[u].x) | (fp8x2_from_bf16x2(v[u].y) << 16),
                     fp8x2_from_bf16x2(v[u].z) | (fp8x2_from_bf16x2(v[u].w) << 16));
    }
  }
}

// Copy `bytes` (a multiple of 16) of a slot into shared memory.
__device__ __forceinline__ void raw_copy(const uint8_t* slot, int64_t bytes, uint8_t* raw) {
  const uint32_t base = smem_u32(raw);
  for (int64_t o = int64_t(threadIdx.x) * 16; o < bytes; o += kNT * 16) cp_async16(base + uint32_t(o), slot + o);
  cp_async_wait_all();
  __syncthreads();
}

// INT8 / FP8 / INT4 bytes in shared memory -> BF16 pool rows.
template <int ROW, int FMT>
__device__ void pool_from_raw(const MigParams& p, const Entry& en, const uint8_t* raw, int64_t E, int n8) {
  constexpr int CPR = ROW / 8;
  for (int k = threadIdx.x; k < n8; k += kNT) {
    uint4 o;
    if constexpr (FMT == ASHKV_PAGE_INT8) {
      const uint2 cw = *reinterpret_cast<const uint2*>(raw + int8_codes_offset(p.T) + int64_t(k) * 8);
      o = int8_dec8(cw, f16_to_f32(reinterpret_cast<const uint16_t*>(raw)[k / CPR]));
    } else if constexpr (FMT == ASHKV_PAGE_FP8) {
      o = fp8_dec8(*reinterpret_cast<const uint2*>(raw + int64_t(k) * 8));
    } else {
      o = int4_dec8(reinterpret_cast<const uint32_t*>(raw + E / 32)[k], reinterpret_cast<const uint16_t*>(raw)[k >> 3]);
    }
    *reinterpret_cast<uint4*>(pool_chunk<ROW>(p, en, k)) = o;
  }
}

// Dithered N-bit bytes in shared memory -> BF16 pool rows; a group never crosses a row.
template <int ROW, int BITS>
__device__ void pool_from_nbit(const MigParams& p, const Entry& en, const uint8_t* raw, int64_t E) {
  const uint16_t* delta = reinterpret_cast<const uint16_t*>(raw + nbit_delta_off());
  const uint8_t* codes = raw + nbit_codes_off(E);
  const int n_groups = int(E / 32);
  constexpr float half = float((1 << BITS) - 1) * 0.5f;
  for (int g = threadIdx.x; g < n_groups; g += kNT) {
    GroupCodes<BITS> gc;
    load_group<BITS>(delta, codes, g, gc);
    uint32_t o[16];
    group_bf16<BITS>(gc, half, o);
    uint16_t* dst = pool_chunk<ROW>(p, en, 4 * g);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
  }
  __syncthreads();  // dense values first, then the outliers overwrite theirs
  const uint32_t n_out = min(*reinterpret_cast<const uint32_t*>(raw), uint32_t(p.outlier_cap));
  const uint32_t* ent = reinterpret_cast<const uint32_t*>(raw + nbit_entries_off(E, BITS));
  for (uint32_t j = threadIdx.x; j < n_out; j += kNT) {
    const uint32_t e = ent[j];
    const uint32_t idx = e >> 16;
    if (idx < uint32_t(E)) pool_row(p, en, int(idx / ROW))[idx % ROW] = uint16_t(e & 0xFFFFu);
  }
}

// ---------------------------------------------------------------- compressed -> compressed, direct
// A compressed source slot, copied whole into shared memory (`raw`), read chunk
// by chunk (8 elements) as the bf16 values its decoder gives, so that an edge
// between two compressed tiers needs no bf16 staging tile: the target encoder
// pulls its chunks straight from the raw bytes.  Dithered sources keep their
// outliers in a sorted list; `first[g]` is the first list entry of group g or
// later (built once per page), so a chunk finds its outliers in a few steps.

// Eight codes of a dithered group (chunk c of group g) -> eight bf16, as group_bf16 decodes them.
template <int BITS>
__device__ __forceinline__ uint4 nbit_chunk(const uint8_t* raw, int64_t E, int k) {
  constexpr float half = float((1 << BITS) - 1) * 0.5f;
  const int g = k >> 2, c = k & 3;
  const float delta = bf16_to_f32(reinterpret_cast<const uint16_t*>(raw + nbit_delta_off())[g]);
  const f2 DEL = pk2(delta, delta), NH = pk2(-half, -half), N23 = pk2(-8388608.0f, -8388608.0f);
  auto pair = [&](float a, float b) { return f32x2_to_bf16x2_pk(mul2(add2(add2(pk2(a, b), N23), NH), DEL)); };
  const uint8_t* codes = raw + nbit_codes_off(E) + int64_t(g) * (4 * BITS);
  uint32_t o[4];
  if constexpr (BITS == 4) {  // word c: elements 8c .. 8c+7, byte j = (elem 2j) << 4 | elem 2j+1
    const uint32_t w = reinterpret_cast<const uint32_t*>(codes)[c];
    const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu, lo = w & 0x0F0F0F0Fu;
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pair(code_plus_2p23(hi, j), code_plus_2p23(lo, j));
  } else {  // bytes 2c, 2c+1 of the group: four codes each, the first in the top bits
    const uint32_t w = reinterpret_cast<const uint16_t*>(codes)[c];
    const uint32_t c0 = (w >> 6) & 0x0303u, c1 = (w >> 4) & 0x0303u, c2 = (w >> 2) & 0x0303u, c3 = w & 0x0303u;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      o[2 * j] = pair(code_plus_2p23(c0, j), code_plus_2p23(c1, j));
      o[2 * j + 1] = pair(code_plus_2p23(c2, j), code_plus_2p23(c3, j));
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// first[g] = index of the first outlier entry whose element lies in group g or
// later, for every group of the page (n_out where none does).  Entries are
// ascending by element index, as the encoder writes them.
template <int BITS>
__device__ void build_outlier_index(const uint8_t* raw, int64_t E, int32_t cap, uint16_t* first) {
  const uint32_t n_out = min(*reinterpret_cast<const uint32_t*>(raw), uint32_t(cap));
  const uint32_t* ent = reinterpret_cast<const uint32_t*>(raw + nbit_entries_off(E, BITS));
  const int n_groups = int(E / 32);
  for (uint32_t j = threadIdx.x; j < n_out; j += kNT) {
    const int gj = min(int(ent[j] >> 21), n_groups - 1);  // element index >> 5
    const int gp = j == 0 ? -1 : min(int(ent[j - 1] >> 21), n_groups - 1);
    for (int g = gp + 1; g <= gj; ++g) first[g] = uint16_t(j);
  }
  const int g_last = n_out == 0 ? -1 : min(int(ent[n_out - 1] >> 21), n_groups - 1);
  for (int g = g_last + 1 + int(threadIdx.x); g < n_groups; g += kNT) first[g] = uint16_t(n_out);
}

// Overwrite chunk k's outliers (elements 8k .. 8k+7) in v.
template <int BITS>
__device__ __forceinline__ uint4 overlay_outliers(uint4 v, const uint8_t* raw, int64_t E, int32_t cap,
                                                  const uint16_t* first, int k) {
  const uint32_t n_out = min(*reinterpret_cast<const uint32_t*>(raw), uint32_t(cap));
  const uint32_t* ent = reinterpret_cast<const uint32_t*>(raw + nbit_entries_off(E, BITS));
  const uint32_t lo = uint32_t(k) * 8u, hi = lo + 8u;
  for (uint32_t j = first[k >> 2]; j < n_out; ++j) {
    const uint32_t e = ent[j], idx = e >> 16;
    if (idx >= hi) break;
    if (idx < lo) continue;
    const uint32_t i = idx - lo, bits = e & 0xFFFFu;
    const uint32_t keep = (i & 1u) ? 0x0000FFFFu : 0xFFFF0000u, put = (i & 1u) ? (bits << 16) : bits;
    switch (i >> 1) {
      case 0: v.x = (v.x & keep) | put; break;
      case 1: v.y = (v.y & keep) | put; break;
      case 2: v.z = (v.z & keep) | put; break;
      default: v.w = (v.w & keep) | put; break;
    }
  }
  return v;
}

// Chunk k of a compressed page in shared memory, decoded to bf16.
template <int ROW, int FS>
__device__ __forceinline__ uint4 raw_chunk(const uint8_t* raw, int T, int64_t E, int32_t cap, const uint16_t* first,
                                           int k) {
  if constexpr (FS == ASHKV_PAGE_INT8) {
    const uint2 cw = *reinterpret_cast<const uint2*>(raw + int8_codes_offset(T) + int64_t(k) * 8);
    return int8_dec8(cw, f16_to_f32(reinterpret_cast<const uint16_t*>(raw)[k / (ROW / 8)]));
  } else if constexpr (FS == ASHKV_PAGE_FP8) {
    return fp8_dec8(*reinterpret_cast<const uint2*>(raw + int64_t(k) * 8));
  } else if constexpr (FS == ASHKV_PAGE_INT4) {
    return int4_dec8(reinterpret_cast<const uint32_t*>(raw + E / 32)[k], reinterpret_cast<const uint16_t*>(raw)[k >> 3]);
  } else {
    constexpr int BITS = FS == ASHKV_PAGE_NBIT4 ? 4 : 2;
    return overlay_outliers<BITS>(nbit_chunk<BITS>(raw, E, k), raw, E, cap, first, k);
  }
}

// -> INT8 slot: TEAM lanes per row, NCH chunks per lane (int8_from_stage's mapping).
template <int ROW, int FS>
__device__ void int8_from_raw(const uint8_t* raw, int T, int64_t E, int32_t cap, const uint16_t* first,
                              uint8_t* slot) {
  constexpr int TEAM = ROW >= 1024 ? 32 : ROW / 32;
  constexpr int NCH = ROW / (8 * TEAM);
  constexpr int RPW = 32 / TEAM;
  constexpr int CPR = ROW / 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TEAM, lin = lane % TEAM;
  uint8_t* codes = slot + int8_codes_offset(T);
  for (int r0 = warp * RPW; r0 < 2 * T; r0 += kNW * RPW) {  // warp-uniform
    const int r = r0 + sub;
    const bool on = r < 2 * T;
    uint32_t w[4 * NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint4 v = on ? raw_chunk<ROW, FS>(raw, T, E, cap, first, r * CPR + c * TEAM + lin) : make_uint4(0, 0, 0, 0);
      w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
    }
    const float am = fmaxf(team_absmax_bf16<TEAM>(w), 1e-8f);
    if (!on) continue;
    if (lin == 0) reinterpret_cast<uint16_t*>(slot)[r] = f32_to_f16(am);
    const Int8Div d = int8_div(am);
#pragma unroll
    for (int c = 0; c < NCH; ++c)
      *reinterpret_cast<uint2*>(codes + int64_t(r) * ROW + (c * TEAM + lin) * 8) =
          make_uint2(int8_codes4_bf16(w[4 * c], w[4 * c + 1], d), int8_codes4_bf16(w[4 * c + 2], w[4 * c + 3], d));
  }
}

// -> FP8 slot, chunk by chunk.
template <int ROW, int FS>
__device__ void fp8_from_raw(const uint8_t* raw, int T, int64_t E, int32_t cap, const uint16_t* first, uint8_t* slot,
                             int n8) {
  for (int k = threadIdx.x; k < n8; k += kNT) {
    const uint4 v = raw_chunk<ROW, FS>(raw, T, E, cap, first, k);
    *reinterpret_cast<uint2*>(slot + int64_t(k) * 8) =
        make_uint2(fp8x2_from_bf16x2(v.x) | (fp8x2_from_bf16x2(v.y) << 16),
                   fp8x2_from_bf16x2(v.z) | (fp8x2_from_bf16x2(v.w) << 16));
  }
}

// -> INT4 slot (group 64): two lanes per group, four chunks (32 elements) per lane.
template <int ROW, int FS>
__device__ void int4_from_raw(const uint8_t* raw, int T, int64_t E, int32_t cap, const uint16_t* first,
                              uint8_t* slot) {
  uint16_t* scales = reinterpret_cast<uint16_t*>(slot);
  uint8_t* nib = slot + E / 32;
  const int n_rows = int(E / 32), lane = threadIdx.x & 31;
  for (int base = threadIdx.x & ~31; base < n_rows; base += kNT) {  // warp-uniform
    const int g = base + lane;
    const bool on = g < n_rows;
    float x[4][8];
    float m = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      unpack_chunk(on ? raw_chunk<ROW, FS>(raw, T, E, cap, first, 4 * g + c) : make_uint4(0, 0, 0, 0), x[c]);
      m = chunk_max(m, x[c]);
    }
    m = max_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
    if (!on) continue;
    const float am = group_max_finish(m);
    if ((g & 1) == 0) scales[g >> 1] = static_cast<uint16_t>(bf16_cpu(am));
    const GroupDiv d = group_div(am);
    uint32_t o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) o[c] = pack_chunk(x[c], d);
    *reinterpret_cast<uint4*>(nib + int64_t(g) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// One compressed -> compressed edge from the raw source bytes (FT: INT8, FP8 or INT4).
template <int ROW, int FS>
__device__ void xcode_from_raw(const MigParams& p, int ft, const uint8_t* raw, const uint16_t* first, int64_t E,
                               uint8_t* dst) {
  const int T = p.T;
  if (ft == ASHKV_PAGE_INT8) int8_from_raw<ROW, FS>(raw, T, E, p.outlier_cap, first, dst);
  else if (ft == ASHKV_PAGE_FP8) fp8_from_raw<ROW, FS>(raw, T, E, p.outlier_cap, first, dst, int(E / 8));
  else int4_from_raw<ROW, FS>(raw, T, E, p.outlier_cap, first, dst);
}

// A compressed -> INT8 / FP8 / INT4 page: the source slot copied whole into
// shared memory, then transcoded chunk by chunk (a dithered source first
// indexes its outliers).  Called by every thread of the CTA.
template <int ROW>
__device__ __forceinline__ void xcode_page(const MigParams& p, int fs, int ft, const uint8_t* src, uint8_t* raw,
                                           uint8_t* smem, int64_t E, uint8_t* dst) {
  raw_copy(src, used_bytes(fs, E, p.T, p.outlier_cap), raw);
  uint16_t* first = reinterpret_cast<uint16_t*>(smem + p.first_offset);
  switch (fs) {
    case ASHKV_PAGE_INT8: xcode_from_raw<ROW, ASHKV_PAGE_INT8>(p, ft, raw, first, E, dst); break;
    case ASHKV_PAGE_FP8: xcode_from_raw<ROW, ASHKV_PAGE_FP8>(p, ft, raw, first, E, dst); break;
    case ASHKV_PAGE_INT4: xcode_from_raw<ROW, ASHKV_PAGE_INT4>(p, ft, raw, first, E, dst); break;
    case ASHKV_PAGE_NBIT4:
      build_outlier_index<4>(raw, E, p.outlier_cap, first);
      __syncthreads();
      xcode_from_raw<ROW, ASHKV_PAGE_NBIT4>(p, ft, raw, first, E, dst);
      break;
    default:
      build_outlier_index<2>(raw, E, p.outlier_cap, first);
      __syncthreads();
      xcode_from_raw<ROW, ASHKV_PAGE_NBIT2>(p, ft, raw, first, E, dst);
      break;
  }
  __syncthreads();  // the raw copy and the outlier index are free again
}

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, off);
    if (lane >= off) inc += t;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  uint32_t before = 0;
  total = 0;
#pragma unroll
  for (int w = 0; w < kNW; ++w) {
    const uint32_t t = s_warp[w];
    before += w < warp ? t : 0u;
    total += t;
  }
  return before + inc - v;
}

// Dithered N-bit: one thread per 32-element group (encode_group), then the
// page's outliers ranked by a block scan.  Returns false on outlier overflow.
template <int BITS>
__device__ bool nbit_from_stage(const MigParams& p, const Entry& en, const uint8_t* stage, int64_t E, uint8_t* slot,
                                uint32_t* s_omask, uint32_t* s_warp) {
  NbitEncParams np{};
  np.sigma = p.sigma;
  np.half_states = float((1 << BITS) - 1) * 0.5f;
#pragma unroll
  for (int k = 0; k < 20; ++k) np.round_keys[k] = p.round_keys[k];
  np.dither_offset = uint64_t(en.page) * uint64_t(E);
  np.scales = reinterpret_cast<uint16_t*>(slot + nbit_delta_off());
  np.codes = slot + nbit_codes_off(E);
  const int n_groups = int(E / 32), lane = threadIdx.x & 31;
  const uint32_t stage_base = smem_u32(stage);
  for (int base = threadIdx.x & ~31; base < n_groups; base += kNT) {  // warp-uniform
    const int g = base + lane;
    const bool on = g < n_groups;
    const uint32_t tile = stage_base + uint32_t(base) * 64u;
    const SmemGroup src{tile, tile + uint32_t(lane) * 64u, uint32_t(lane >> 1) & 3u};
    const uint32_t om = encode_group<BITS, ASHKV_DITHER_PHILOX>(src, np, g, on);
    if (on) s_omask[g] = om;
  }
  __syncthreads();
  // groups [g0, g0 + per) of this thread, in order
  const int per = (n_groups + kNT - 1) / kNT;
  const int g0 = threadIdx.x * per;
  uint32_t cnt = 0;
  for (int j = 0; j < per; ++j)
    if (g0 + j < n_groups) cnt += uint32_t(__popc(s_omask[g0 + j]));
  uint32_t total;
  uint32_t pos = block_exclusive_scan(cnt, s_warp, total);
  const uint32_t cap = uint32_t(p.outlier_cap);
  uint32_t* ent = reinterpret_cast<uint32_t*>(slot + nbit_entries_off(E, BITS));
  if (total <= cap) {
    for (int j = 0; j < per; ++j) {
      const int g = g0 + j;
      if (g >= n_groups) break;
      uint32_t m = s_omask[g];
      while (m) {
        const uint32_t b = uint32_t(__ffs(m) - 1);
        m &= m - 1;
        const uint32_t idx = uint32_t(g) * 32u + b;
        ent[pos++] = (idx << 16) | *reinterpret_cast<const uint16_t*>(stage + stage_off(idx));
      }
    }
  }
  if (threadIdx.x == 0) {
    uint4 hdr = make_uint4(total <= cap ? total : 0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(slot) = hdr;
  }
  return total <= cap;
}

__device__ __forceinline__ int fmt_of(const MigParams& p, int t) {
  return (t >= 0 && t < kTiers) ? p.store[t].format : ASHKV_PAGE_NONE;
}

// Entries are processed by two launches over the same list.  The direct pass
// moves the pages whose edge needs no staging tile (BF16 -> INT8 / FP8, and
// every edge into BF16) and reports every entry that does not move; it marks
// the other moving entries kDeferred without taking a slot, and the staged
// pass (staging tile, the dithered encoder) moves only those.
// kDirectX is the direct pass of a tier set with two or more compressed tiers: it
// also moves compressed -> INT8 / FP8 / INT4 pages (from the raw source copy), so
// that work overlaps the memory-bound BF16 edges of the same list; a tier set
// with one compressed tier launches the plain kDirect code.
constexpr int kDirect = 0, kStaged = 1, kDirectX = 2;
constexpr int32_t kDeferred = 100;
constexpr int32_t kNotMine = 101;

template <int MODE>
__device__ __forceinline__ bool direct_edge(int fs, int ft) {
  if (ft == ASHKV_PAGE_BF16) return true;
  if (fs == ASHKV_PAGE_BF16) return ft == ASHKV_PAGE_INT8 || ft == ASHKV_PAGE_FP8;
  return MODE == kDirectX && (ft == ASHKV_PAGE_INT8 || ft == ASHKV_PAGE_FP8 || ft == ASHKV_PAGE_INT4);
}

// Resolve entry i: the migrate() ladder's checks, then the slot.  Called by all
// 32 lanes of a warp (lanes with !valid take part in the collectives only); the
// slots are popped with one atomic per target tier and warp, lanes ranked by
// their position in the ballot.
template <int MODE>
__device__ Entry resolve(const MigParams& p, int64_t i, bool valid) {
  const int lane = threadIdx.x & 31;
  Entry e{};
  e.status = ASHKV_MIGRATE_BAD_PAGE;
  e.old_slot = e.new_slot = -1;
  e.tgt = -1;
  bool pop = false;
  do {
    if (!valid || (MODE == kStaged && p.entry_status[i] != kDeferred)) {
      e.status = kNotMine;
      break;
    }
    const int32_t page = p.list[i];
    e.page = page;
    if (page < 0 || page >= p.n_pages) break;
    e.cur = p.tier[page];
    e.tgt = p.target[page];
    e.layer = p.layer_id[page];
    e.ts = p.token_start[page];
    e.old_slot = p.page_slot[page];
    const int32_t pin = p.pin ? p.pin[page] : 0;
    if (pin > 0) { e.status = ASHKV_MIGRATE_PINNED; break; }
    if (e.cur == e.tgt) { e.status = ASHKV_MIGRATE_SAME_TIER; break; }
    const int fs = fmt_of(p, e.cur), ft = fmt_of(p, e.tgt);
    if (fs == ASHKV_PAGE_NONE || ft == ASHKV_PAGE_NONE) { e.status = ASHKV_MIGRATE_NO_CODEC; break; }
    if (e.layer < 0 || e.layer >= p.n_layers || e.ts < 0) break;
    if (fs != ASHKV_PAGE_BF16 && (e.old_slot < 0 || e.old_slot >= p.store[e.cur].n_slots)) break;
    e.kbase = p.layer_k[e.layer] + uint64_t(e.ts) * uint64_t(p.row_stride) * 2u;
    e.vbase = p.layer_v[e.layer] + uint64_t(e.ts) * uint64_t(p.row_stride) * 2u;
    if (MODE != kStaged && !direct_edge<MODE>(fs, ft)) { e.status = kDeferred; break; }
    e.status = ASHKV_MIGRATE_OK;
    pop = ft != ASHKV_PAGE_BF16;
  } while (false);
#pragma unroll 1
  for (int t = 1; t < kTiers; ++t) {
    const bool mine = pop && e.tgt == t;
    const unsigned m = __ballot_sync(0xFFFFFFFFu, mine);
    if (!m) continue;
    const int leader = __ffs(m) - 1, want = __popc(m);
    int32_t old = 0;
    if (lane == leader) old = atomicSub(p.store[t].free_top, want);
    old = __shfl_sync(0xFFFFFFFFu, old, leader);
    const int taken = old <= 0 ? 0 : (old < want ? old : want);
    if (lane == leader && taken < want) atomicAdd(p.store[t].free_top, want - taken);
    if (mine) {
      const int rank = __popc(m & ((1u << lane) - 1u));
      const int32_t pos = old - 1 - rank;
      if (rank >= taken) {
        e.status = ASHKV_MIGRATE_NO_SLOT;
      } else if (pos >= p.store[t].n_slots || (e.new_slot = p.store[t].free_stack[pos]) < 0 ||
                 e.new_slot >= p.store[t].n_slots) {  // corrupt stack: leave it popped, report it
        e.status = ASHKV_MIGRATE_BAD_PAGE;
        e.new_slot = -1;
      }
    }
  }
  return e;
}

template <int ROW, int MODE>
__global__ void __launch_bounds__(kThreads, MODE == kStaged ? kStagedBlocks : kDirectBlocks)
    migrate_pages_kernel(const MigParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ Entry s_ent[kBatch];
  __shared__ uint32_t s_warp[kWarps];
  __shared__ int32_t s_ok;
  const int T = p.T;
  const int64_t E = 2 * int64_t(T) * ROW;
  const int n8 = int(E / 8);
  uint8_t* stage = smem;  // direct pass: the raw copy of a compressed source; staged pass: the bf16 tile
  uint32_t* s_omask = reinterpret_cast<uint32_t*>(smem + E * 2);
  const int32_t count = min(*p.count, p.max_entries);
  for (int64_t b0 = blockIdx.x; b0 < count; b0 += int64_t(kBatch) * gridDim.x) {
    const int64_t left = (count - b0 + gridDim.x - 1) / gridDim.x;
    const int nb = left < kBatch ? int(left) : kBatch;
    if (threadIdx.x < 32) {
      const Entry e = resolve<MODE>(p, b0 + int64_t(threadIdx.x) * gridDim.x, int(threadIdx.x) < nb);
      if (int(threadIdx.x) < nb) s_ent[threadIdx.x] = e;
    }
    __syncthreads();
    for (int k = 0; k < nb; ++k) {
      const Entry en = s_ent[k];
      const int64_t i = b0 + int64_t(k) * gridDim.x;
      if (en.status == kNotMine) continue;
      bool ok = en.status == ASHKV_MIGRATE_OK;
      if (ok) {
        const int fs = p.store[en.cur].format, ft = p.store[en.tgt].format;
        const uint8_t* src = fs == ASHKV_PAGE_BF16 ? nullptr
                                                   : p.store[en.cur].data + int64_t(en.old_slot) * p.store[en.cur].slot_bytes;
        uint8_t* dst = ft == ASHKV_PAGE_BF16 ? nullptr
                                             : p.store[en.tgt].data + int64_t(en.new_slot) * p.store[en.tgt].slot_bytes;
        if constexpr (MODE != kStaged) {
          if (fs == ASHKV_PAGE_BF16 && ft == ASHKV_PAGE_INT8) {
            int8_from_pool<ROW>(p, en, dst);
          } else if (fs == ASHKV_PAGE_BF16) {
            fp8_from_pool<ROW>(p, en, dst, n8);
          } else if (MODE == kDirect || ft == ASHKV_PAGE_BF16) {  // into BF16
            raw_copy(src, used_bytes(fs, E, T, p.outlier_cap), stage);
            switch (fs) {
              case ASHKV_PAGE_INT8: pool_from_raw<ROW, ASHKV_PAGE_INT8>(p, en, stage, E, n8); break;
              case ASHKV_PAGE_FP8: pool_from_raw<ROW, ASHKV_PAGE_FP8>(p, en, stage, E, n8); break;
              case ASHKV_PAGE_INT4: pool_from_raw<ROW, ASHKV_PAGE_INT4>(p, en, stage, E, n8); break;
              case ASHKV_PAGE_NBIT4: pool_from_nbit<ROW, 4>(p, en, stage, E); break;
              default: pool_from_nbit<ROW, 2>(p, en, stage, E); break;
            }
            __syncthreads();  // the raw copy is free again
          } else {
            xcode_page<ROW>(p, fs, ft, src, stage, smem, E, dst);
          }
        } else {
          switch (fs) {
            case ASHKV_PAGE_BF16: stage_from_pool<ROW>(p, en, stage, n8); break;
            case ASHKV_PAGE_INT8: stage_from_int8<ROW>(src, T, stage, n8); break;
            case ASHKV_PAGE_FP8: stage_from_fp8(src, stage, n8); break;
            case ASHKV_PAGE_INT4: stage_from_int4(src, E, stage, n8); break;
            case ASHKV_PAGE_NBIT4: stage_from_nbit<4>(src, E, p.outlier_cap, stage); break;
            default: stage_from_nbit<2>(src, E, p.outlier_cap, stage); break;
          }
          __syncthreads();
          switch (ft) {
            case ASHKV_PAGE_BF16: pool_from_stage<ROW>(p, en, stage, n8); break;
            case ASHKV_PAGE_INT8: int8_from_stage<ROW>(stage, T, dst); break;
            case ASHKV_PAGE_FP8: fp8_from_stage(stage, dst, n8); break;
            case ASHKV_PAGE_INT4: int4_from_stage(stage, E, dst); break;
            case ASHKV_PAGE_NBIT4: ok = nbit_from_stage<4>(p, en, stage, E, dst, s_omask, s_warp); break;
            default: ok = nbit_from_stage<2>(p, en, stage, E, dst, s_omask, s_warp); break;
          }
          if (threadIdx.x == 0) s_ok = ok;
          __syncthreads();  // staging, s_omask and s_warp are free again; s_ok visible
          ok = s_ok != 0;
        }
      }
      if (threadIdx.x == 0) {
        int32_t status = en.status, rel = -1;
        if (en.status == kDeferred) {
          // moved by the staged pass
        } else if (en.status == ASHKV_MIGRATE_OK && ok) {
          p.tier[en.page] = int8_t(en.tgt);
          p.page_slot[en.page] = en.new_slot;  // -1 when the page returns to its BF16 rows
          if (en.old_slot >= 0 && p.store[en.cur].format != ASHKV_PAGE_BF16) rel = (en.cur << 24) | en.old_slot;
        } else if (en.status == ASHKV_MIGRATE_OK) {
          status = ASHKV_MIGRATE_OVERFLOW;
          rel = (en.tgt << 24) | en.new_slot;
        }
        p.entry_status[i] = status;
        p.released[i] = rel;
      }
    }
    __syncthreads();  // s_ent is rewritten by the next batch
  }
}

struct ReleaseParams {
  const int32_t* released;
  const int32_t* count;
  int32_t max_entries;
  Store store[kTiers];
  uint32_t* status;
};

// Pushes with one atomic per tier and warp (lanes ranked in the ballot).
__global__ void __launch_bounds__(256) release_slots_kernel(const ReleaseParams p) {
  const int32_t count = min(*p.count, p.max_entries);
  const int lane = threadIdx.x & 31;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i0 = int64_t(blockIdx.x) * blockDim.x + (threadIdx.x & ~31); i0 < count; i0 += stride) {
    const int64_t i = i0 + lane;
    const int32_t v = i < count ? p.released[i] : -1;
    int t = v < 0 ? 0 : (v >> 24);
    const int32_t slot = v & 0xFFFFFF;
    if (v >= 0 && (t <= 0 || t >= kTiers || !p.store[t].free_stack || slot >= p.store[t].n_slots)) {
      if (p.status) atomicOr(p.status, ASHKV_FLAG_INDEX_RANGE);
      t = 0;
    }
#pragma unroll 1
    for (int tt = 1; tt < kTiers; ++tt) {
      const unsigned m = __ballot_sync(0xFFFFFFFFu, t == tt);
      if (!m) continue;
      const int leader = __ffs(m) - 1;
      int32_t base = 0;
      if (lane == leader) base = atomicAdd(p.store[tt].free_top, __popc(m));
      base = __shfl_sync(0xFFFFFFFFu, base, leader);
      if (t == tt) {
        const int32_t pos = base + __popc(m & ((1u << lane) - 1u));
        if (pos >= 0 && pos < p.store[tt].n_slots) p.store[tt].free_stack[pos] = slot;
        else if (p.status) atomicOr(p.status, ASHKV_FLAG_INDEX_RANGE);
      }
    }
  }
}

bool row_ok(int32_t row) { return row == 128 || row == 256 || row == 512 || row == 1024 || row == 2048; }

template <int ROW>
ashkv_status_t launch_migrate(const MigParams& p, bool xcode_direct, size_t raw_smem, size_t stage_smem,
                              cudaStream_t st) {
  const int sms = sm_count() > 0 ? sm_count() : 148;
  constexpr int NT = block_threads(ROW);
  constexpr int CTA_SCALE = kThreads / NT;  // CTAs per SM grow as CTAs shrink
  auto direct = xcode_direct ? migrate_pages_kernel<ROW, kDirectX> : migrate_pages_kernel<ROW, kDirect>;
  cudaError_t e = cudaFuncSetAttribute(direct, cudaFuncAttributeMaxDynamicSharedMemorySize, int(raw_smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(migrate_pages_kernel<ROW, kStaged>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(stage_smem));
  if (e != cudaSuccess) {
    set_error("migrate_pages (shared memory attribute)", e);
    return ASHKV_LAUNCH_ERROR;
  }
  const int64_t gd = std::min<int64_t>(p.max_entries, int64_t(sms) * kDirectBlocks * CTA_SCALE);
  direct<<<unsigned(gd > 0 ? gd : 1), NT, raw_smem, st>>>(p);
  const ashkv_status_t rc = check_launch("migrate_pages (direct pass)");
  if (rc != ASHKV_OK) return rc;
  const int64_t gs = std::min<int64_t>(p.max_entries, int64_t(sms) * kStagedBlocks * CTA_SCALE);
  migrate_pages_kernel<ROW, kStaged><<<unsigned(gs > 0 ? gs : 1), NT, stage_smem, st>>>(p);
  return check_launch("migrate_pages (staged pass)");
}

bool copy_stores(const ashkv_tier_store_t* stores, Store (&out)[kTiers], bool need_data) {
  if (!stores) return false;
  for (int t = 0; t < kTiers; ++t) {
    const ashkv_tier_store_t& s = stores[t];
    out[t] = Store{static_cast<uint8_t*>(s.d_data), s.slot_bytes, s.n_slots, s.format, s.d_free_stack, s.d_free_top};
    if (t == 0) {
      if (s.format != ASHKV_PAGE_BF16) return false;
      continue;
    }
    if (s.format == ASHKV_PAGE_NONE) continue;
    if (s.format < ASHKV_PAGE_INT8 || s.format > ASHKV_PAGE_NBIT2) return false;
    if (s.n_slots < 0 || s.n_slots > 0xFFFFFF || !s.d_free_stack || !s.d_free_top) return false;
    if (need_data && (!s.d_data || !aligned(s.d_data, 16) || s.slot_bytes % 16)) return false;
  }
  return true;
}

}  // namespace
}  // namespace ashkv

using namespace ashkv;

extern "C" int64_t ashkv_page_slot_bytes(int32_t format, int32_t tokens_per_page, int32_t row_len,
                                         int32_t outlier_cap) {
  if (tokens_per_page <= 0 || row_len <= 0 || outlier_cap < 0) return -1;
  const int64_t E = 2 * int64_t(tokens_per_page) * row_len;
  int64_t b = format == ASHKV_PAGE_INT8 ? int8_codes_offset(tokens_per_page) + E : slot_bytes_for(format, E, outlier_cap);
  if (b < 0) return -1;
  return (b + 255) / 256 * 256;
}

extern "C" ashkv_status_t ashkv_migrate_pages(
    int8_t* d_tier, const int32_t* d_pin, const int32_t* d_layer_id, const int32_t* d_token_start,
    int32_t* d_page_slot, int64_t n_pages, const int8_t* d_target, const int32_t* d_list, const int32_t* d_count,
    int32_t max_entries, const uint64_t* d_layer_k, const uint64_t* d_layer_v, int32_t n_layers,
    int32_t tokens_per_page, int32_t row_len, int64_t row_stride, const ashkv_tier_store_t* stores, float sigma,
    uint64_t seed, int32_t outlier_cap, int32_t* d_entry_status, int32_t* d_released, void* stream) {
  MigParams p{};
  p.tier = d_tier; p.pin = d_pin; p.layer_id = d_layer_id; p.token_start = d_token_start; p.page_slot = d_page_slot;
  p.n_pages = n_pages; p.target = d_target; p.list = d_list; p.count = d_count; p.max_entries = max_entries;
  p.layer_k = d_layer_k; p.layer_v = d_layer_v; p.n_layers = n_layers; p.T = tokens_per_page; p.row_len = row_len;
  p.row_stride = row_stride; p.sigma = sigma; p.outlier_cap = outlier_cap;
  p.entry_status = d_entry_status; p.released = d_released;
  if (max_entries < 0 || n_pages < 0 || n_layers <= 0 || tokens_per_page <= 0 || outlier_cap < 0) {
    set_message("ashkv_migrate_pages: negative size or no layers");
    return ASHKV_BAD_ARGUMENT;
  }
  if (max_entries == 0) return ASHKV_OK;
  if (!d_tier || !d_layer_id || !d_token_start || !d_page_slot || !d_target || !d_list || !d_count || !d_layer_k ||
      !d_layer_v || !d_entry_status || !d_released) {
    set_message("ashkv_migrate_pages: null device pointer");
    return ASHKV_BAD_ARGUMENT;
  }
  if (!row_ok(row_len) || (row_stride * 2) % 16 || row_stride < row_len) {
    set_message("ashkv_migrate_pages: row_len must be 128, 256, 512, 1024 or 2048 with a 16-byte row stride");
    return ASHKV_BAD_ARGUMENT;
  }
  const int64_t E = 2 * int64_t(tokens_per_page) * row_len;
  if (E > kMaxElems || E % 1024) {
    set_message("ashkv_migrate_pages: a page (2 * tokens_per_page * row_len) must be a multiple of 1024 and at most "
                "65536 elements");
    return ASHKV_BAD_ARGUMENT;
  }
  if (!copy_stores(stores, p.store, true)) {
    set_message("ashkv_migrate_pages: bad tier store table (store 0 must be the BF16 pool)");
    return ASHKV_BAD_ARGUMENT;
  }
  for (int t = 1; t < kTiers; ++t) {
    const Store& s = p.store[t];
    if (s.format == ASHKV_PAGE_NONE) continue;
    const int64_t need = ashkv_page_slot_bytes(s.format, tokens_per_page, row_len, outlier_cap);
    if (s.slot_bytes < need) {
      set_message("ashkv_migrate_pages: a tier store's slots are smaller than its format needs");
      return ASHKV_BAD_ARGUMENT;
    }
  }
  if ((p.store[1].format == ASHKV_PAGE_NBIT4 || p.store[2].format == ASHKV_PAGE_NBIT4 ||
       p.store[3].format == ASHKV_PAGE_NBIT4 || p.store[1].format == ASHKV_PAGE_NBIT2 ||
       p.store[2].format == ASHKV_PAGE_NBIT2 || p.store[3].format == ASHKV_PAGE_NBIT2) && !(sigma > 0.0f)) {
    set_message("ashkv_migrate_pages: sigma must be positive for the dithered formats");
    return ASHKV_BAD_ARGUMENT;
  }
  philox_round_keys(seed, p.round_keys);
  const size_t smem = size_t(E) * 2 + size_t(E / 32) * 4;
  size_t raw = 16;
  for (int t = 1; t < kTiers; ++t)
    if (p.store[t].format != ASHKV_PAGE_NONE)
      raw = std::max<size_t>(raw, size_t(used_bytes(p.store[t].format, E, tokens_per_page, outlier_cap)));
  // Two or more compressed tiers: compressed -> INT8 / FP8 / INT4 edges can occur,
  // and the direct pass takes them (the raw source copy, then the per-group
  // outlier index of a dithered source).  With one, every edge has a BF16 end.
  int compressed_tiers = 0;
  for (int t = 1; t < kTiers; ++t) compressed_tiers += p.store[t].format != ASHKV_PAGE_NONE;
  const bool xcode_direct = compressed_tiers >= 2;
  p.first_offset = int32_t(raw);  // used_bytes is a multiple of 16
  const size_t raw_smem = xcode_direct ? raw + size_t(E / 32) * 2 : raw;
  const size_t stage_smem = smem;
  if (raw_smem > size_t(200) * 1024) {
    set_message("ashkv_migrate_pages: outlier_cap too large for one page in shared memory");
    return ASHKV_BAD_ARGUMENT;
  }
  cudaStream_t st = as_stream(stream);
  switch (row_len) {
    case 128: return launch_migrate<128>(p, xcode_direct, raw_smem, stage_smem, st);
    case 256: return launch_migrate<256>(p, xcode_direct, raw_smem, stage_smem, st);
    case 512: return launch_migrate<512>(p, xcode_direct, raw_smem, stage_smem, st);
    case 1024: return launch_migrate<1024>(p, xcode_direct, raw_smem, stage_smem, st);
    default: return launch_migrate<2048>(p, xcode_direct, raw_smem, stage_smem, st);
  }
}

extern "C" ashkv_status_t ashkv_release_slots(const int32_t* d_released, const int32_t* d_count, int32_t max_entries,
                                              const ashkv_tier_store_t* stores, uint32_t* d_status, void* stream) {
  ReleaseParams p{};
  p.released = d_released; p.count = d_count; p.max_entries = max_entries; p.status = d_status;
  if (max_entries < 0) return ASHKV_BAD_ARGUMENT;
  if (max_entries == 0) return ASHKV_OK;
  if (!d_released || !d_count || !copy_stores(stores, p.store, false)) {
    set_message("ashkv_release_slots: null pointer or bad tier store table");
    return ASHKV_BAD_ARGUMENT;
  }
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t g = std::min<int64_t>((int64_t(max_entries) + 255) / 256, int64_t(sms) * 4);
  release_slots_kernel<<<unsigned(g > 0 ? g : 1), 256, 0, as_stream(stream)>>>(p);
  return check_launch("release_slots");
}
