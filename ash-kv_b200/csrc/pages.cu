// Batched page migration kernels: gather + INT8 encode into shadow-arena
// slots (demotion) and INT8 decode + scatter back into the KV pool
// (promotion), driven by device-resident transition lists.
//
// Replaces the per-page loop around migrate() (ashkv/runtime/migrate.py:35-191)
// for the BF16 <-> INT8 transition with the hooks' INT8 layout
// (ashkv/adapters/sglang/hooks.py:83-137): one fp16 absmax scale per token over
// all local heads.  A page is `tokens_per_page` consecutive token rows of one
// layer; page-table row p names it by (layer_id[p], token_start[p]).  The K
// and V rows of a page are found at layer_k[l] + (token_start + j) * row_stride
// (and layer_v likewise).
//
// Slot layout in the arena (slot_bytes per slot, 16-byte aligned):
//   [0, 2T)                  fp16 scales of the K rows
//   [2T, 4T)                 fp16 scales of the V rows
//   [S0, S0 + T*row)         int8 K codes,  S0 = round_up(4T, 16)
//   [S0 + T*row, S0 + 2T*row) int8 V codes
//
// Slots come from a device free stack (free_stack[0 .. *free_top)).  List
// entry i takes free_stack[*free_top - 1 - i], so assignment is deterministic
// and needs no atomics; ashkv_slots_commit then lowers *free_top.  The list
// length is read on the device (d_count), so no host synchronisation sits
// between the policy kernel and these kernels.
#include <algorithm>

#include "common.cuh"

namespace ashkv {
namespace {

constexpr int kThreads = 256;
// decode: row groups whose codes a warp loads before converting any (4 for
// full-warp rows; 2 when a warp holds several rows, which is already 2 x RPW rows)
template <int TEAM>
constexpr int rows_in_flight() { return TEAM == 32 ? 4 : 2; }


struct PagesParams {
  const uint64_t* layer_k;
  const uint64_t* layer_v;
  int32_t n_layers;
  const int32_t* layer_id;
  const int32_t* token_start;
  const int32_t* list;
  const int32_t* count;
  int32_t max_entries;
  int32_t tokens_per_page;
  int32_t row_len;
  int64_t row_stride;
  uint8_t* arena;
  int64_t slot_bytes;
  int64_t n_slots;
  int32_t* free_stack;
  const int32_t* free_top;
  int32_t* page_slot;
  int32_t* entry_status;  // per list entry: 0 ok, 1 no slot, 2 bad page / slot
  int32_t free_slots;     // decode: push the slot back onto the free stack
  int32_t* free_top_rw;
};

__host__ __device__ __forceinline__ int64_t codes_offset(int T) { return (4 * int64_t(T) + 15) / 16 * 16; }

// Row mapping: TEAM consecutive lanes hold one row, NCH chunks of 8 elements per
// lane (row_len = TEAM * NCH * 8), so a warp covers RPW = 32 / TEAM rows at a time.
// Every supported row width uses NCH = 4 (8 for 2048), which keeps the per-lane
// work per row -- the row maximum's shuffles, the divisor, the scale -- spread
// over 32 elements whatever the number of local heads.  `lin` is the lane's index
// within its team, `on` whether its row exists.

// One lane's share of a row (NCH chunks of 8 bf16).
template <int NCH>
struct RowIn {
  uint4 ch[NCH];
};

template <int TEAM, int NCH>
__device__ __forceinline__ void load_row_in(const uint16_t* src, int lin, bool on, RowIn<NCH>& ri) {
#pragma unroll
  for (int c = 0; c < NCH; ++c) ri.ch[c] = on ? ld_nc_v4(src + (c * TEAM + lin) * 8) : make_uint4(0, 0, 0, 0);
}

// Encode one loaded row into int8 codes + fp16 scale.  Called by every lane of the
// warp (the row maximum is a shuffle reduction within the team).
template <int TEAM, int NCH>
__device__ __forceinline__ void encode_row(const RowIn<NCH>& ri, int8_t* codes, uint16_t* scale, int lin, bool on) {
  uint32_t words[4 * NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    words[4 * c] = ri.ch[c].x; words[4 * c + 1] = ri.ch[c].y;
    words[4 * c + 2] = ri.ch[c].z; words[4 * c + 3] = ri.ch[c].w;
  }
  const float am = fmaxf(team_absmax_bf16<TEAM>(words), 1e-8f);
  if (!on) return;
  if (lin == 0) *scale = f32_to_f16(am);
  const Int8Div d = int8_div(am);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const uint32_t w[4] = {ri.ch[c].x, ri.ch[c].y, ri.ch[c].z, ri.ch[c].w};
    *reinterpret_cast<uint2*>(codes + (c * TEAM + lin) * 8) =
        make_uint2(int8_codes4_bf16(w[0], w[1], d), int8_codes4_bf16(w[2], w[3], d));
  }
}

// A row's codes as held by one lane (NCH chunks of 8 bytes) and its scale.
template <int NCH>
struct RowCodes {
  uint2 w[NCH];
  float scale;
};
template <int TEAM, int NCH>
__device__ __forceinline__ void load_row_codes(const int8_t* codes, const uint16_t* scale, int lin, bool on,
                                               RowCodes<NCH>& rc) {
  if (!on) return;
  rc.scale = f16_to_f32(*scale);
#pragma unroll
  for (int c = 0; c < NCH; ++c) rc.w[c] = *reinterpret_cast<const uint2*>(codes + (c * TEAM + lin) * 8);
}

template <int TEAM, int NCH>
__device__ __forceinline__ void decode_row(const RowCodes<NCH>& rc, uint16_t* dst, int lin, bool on) {
  if (!on) return;
  const float scale = rc.scale;
  const bool fast = int8_dec_fast(scale);
  const Recip y = make_recip(127.0f);
  const f2 S = pk2(scale, scale), YHI = pk2(y.hi, y.hi), YLO = pk2(y.lo, y.lo);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int e0 = (c * TEAM + lin) * 8;
    const uint32_t ww[2] = {rc.w[c].x, rc.w[c].y};
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      f2 F0, F1;  // float(code) of bytes 0,1 and 2,3 of ww[h]
      int8x4_to_f2(ww[h], F0, F1);
      if (fast) {
        o[2 * h] = f32x2_to_bf16x2_pk(div2_short(mul2(F0, S), YHI, YLO));
        o[2 * h + 1] = f32x2_to_bf16x2_pk(div2_short(mul2(F1, S), YHI, YLO));
      } else {
        float a, b;
        upk2(F0, a, b);
        o[2 * h] = f32x2_to_bf16x2(__fdiv_rn(__fmul_rn(a, scale), 127.0f), __fdiv_rn(__fmul_rn(b, scale), 127.0f));
        upk2(F1, a, b);
        o[2 * h + 1] = f32x2_to_bf16x2(__fdiv_rn(__fmul_rn(a, scale), 127.0f), __fdiv_rn(__fmul_rn(b, scale), 127.0f));
      }
    }
    *reinterpret_cast<uint4*>(dst + e0) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// A CTA walks its list entries (blockIdx.x, + gridDim.x, ...) in batches of kBatch:
// the first kBatch threads resolve one entry each (list -> page -> layer, slot ->
// row pointers) into shared memory, so that the chain of dependent index loads is
// paid once per batch instead of once per page, then all warps stream the rows.
constexpr int kBatch = 32;
constexpr int kWarps = kThreads / 32;

struct PageRef {
  const uint16_t* k;  // K row of the page's first token
  const uint16_t* v;
  uint8_t* base;      // arena slot
  int32_t page;
  int32_t slot;       // -1: entry skipped (status already written)
};

__device__ __forceinline__ int batch_len(int64_t b0, int32_t count) {
  const int64_t left = (count - b0 + gridDim.x - 1) / gridDim.x;
  return left < kBatch ? int(left) : kBatch;
}

__device__ __forceinline__ PageRef page_ref(const PagesParams& p, int32_t page, int32_t l, int32_t slot) {
  const int64_t off = int64_t(p.token_start[page]) * p.row_stride;
  return PageRef{reinterpret_cast<const uint16_t*>(p.layer_k[l]) + off,
                 reinterpret_cast<const uint16_t*>(p.layer_v[l]) + off,
                 p.arena + int64_t(slot) * p.slot_bytes, page, slot};
}

// Warps of a CTA in groups of `wpp` per page: a pass of one warp covers SPAN =
// U * RPW consecutive rows of its page, so a page of 2T rows takes
// ceil(2T / SPAN) warps (at most kWarps) and the CTA streams kWarps / wpp pages
// of its batch at once.
struct WarpPlan {
  int wpp, ppp, slot, wi;  // warps per page, pages per pass, this warp's page slot and index in its group
};
template <int SPAN>
__device__ __forceinline__ WarpPlan warp_plan(int T, int warp) {
  WarpPlan w;
  w.wpp = min((2 * T + SPAN - 1) / SPAN, kWarps);
  w.ppp = kWarps / w.wpp;
  w.slot = warp / w.wpp;
  w.wi = warp - w.slot * w.wpp;
  return w;
}

template <int TEAM, int NCH>
__global__ void __launch_bounds__(kThreads, NCH <= 4 ? 3 : 1) encode_pages_kernel(const PagesParams p) {
  __shared__ PageRef s_ref[kBatch];
  constexpr int RPW = 32 / TEAM;                     // rows per warp-wide load
  constexpr int U = NCH <= 2 ? 2 : 1;                // row groups whose loads are in flight together
  constexpr int SPAN = U * RPW;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TEAM, lin = lane % TEAM;
  const int32_t count = min(*p.count, p.max_entries);
  const int32_t top = *p.free_top;
  const int T = p.tokens_per_page;
  const int64_t c0 = codes_offset(T);
  const WarpPlan wp = warp_plan<SPAN>(T, warp);
  for (int64_t b0 = blockIdx.x; b0 < count; b0 += int64_t(kBatch) * gridDim.x) {
    const int nb = batch_len(b0, count);
    if (threadIdx.x < nb) {
      const int64_t i = b0 + int64_t(threadIdx.x) * gridDim.x;
      const int32_t page = p.list[i];
      PageRef ref{nullptr, nullptr, nullptr, page, -1};
      int32_t status = 1;  // no free slot
      if (i < top) {
        const int32_t l = p.layer_id[page];
        const int32_t slot = p.free_stack[top - 1 - i];
        status = 2;
        if (l >= 0 && l < p.n_layers && slot >= 0 && slot < p.n_slots) {
          ref = page_ref(p, page, l, slot);
          p.page_slot[page] = slot;
          status = 0;
        }
      }
      p.entry_status[i] = status;
      s_ref[threadIdx.x] = ref;
    }
    __syncthreads();
    if (wp.slot < wp.ppp) {
      for (int e = wp.slot; e < nb; e += wp.ppp) {
        const PageRef ref = s_ref[e];
        if (ref.slot < 0) continue;
        for (int r0 = wp.wi * SPAN; r0 < 2 * T; r0 += wp.wpp * SPAN) {
          RowIn<NCH> ri[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int r = r0 + u * RPW + sub;
            const int j = r >= T ? r - T : r;
            load_row_in<TEAM, NCH>((r >= T ? ref.v : ref.k) + j * p.row_stride, lin, r < 2 * T, ri[u]);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int r = r0 + u * RPW + sub;
            encode_row<TEAM, NCH>(ri[u], reinterpret_cast<int8_t*>(ref.base + c0 + int64_t(r) * p.row_len),
                                  reinterpret_cast<uint16_t*>(ref.base) + r, lin, r < 2 * T);
          }
        }
      }
    }
    __syncthreads();  // s_ref is rewritten by the next batch
  }
}

template <int TEAM, int NCH>
__global__ void __launch_bounds__(kThreads, TEAM < 32 ? 3 : 1) decode_pages_kernel(const PagesParams p) {
  __shared__ PageRef s_ref[kBatch];
  constexpr int RPW = 32 / TEAM;
  constexpr int U = rows_in_flight<TEAM>();
  constexpr int SPAN = U * RPW;  // all codes of a pass are loaded before any is converted
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TEAM, lin = lane % TEAM;
  const int32_t count = min(*p.count, p.max_entries);
  const int T = p.tokens_per_page;
  const int64_t c0 = codes_offset(T);
  const WarpPlan wp = warp_plan<SPAN>(T, warp);
  for (int64_t b0 = blockIdx.x; b0 < count; b0 += int64_t(kBatch) * gridDim.x) {
    const int nb = batch_len(b0, count);
    if (threadIdx.x < nb) {
      const int64_t i = b0 + int64_t(threadIdx.x) * gridDim.x;
      const int32_t page = p.list[i];
      const int32_t l = p.layer_id[page];
      const int32_t slot = p.page_slot[page];
      PageRef ref{nullptr, nullptr, nullptr, page, -1};
      int32_t status = 2;
      if (l >= 0 && l < p.n_layers && slot >= 0 && slot < p.n_slots) {
        ref = page_ref(p, page, l, slot);
        status = 0;
      }
      p.entry_status[i] = status;
      s_ref[threadIdx.x] = ref;
    }
    __syncthreads();
    if (wp.slot < wp.ppp) {
      for (int e = wp.slot; e < nb; e += wp.ppp) {
        const PageRef ref = s_ref[e];
        if (ref.slot < 0) continue;
        for (int r0 = wp.wi * SPAN; r0 < 2 * T; r0 += wp.wpp * SPAN) {
          RowCodes<NCH> rc[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int r = r0 + u * RPW + sub;
            load_row_codes<TEAM, NCH>(reinterpret_cast<const int8_t*>(ref.base + c0 + int64_t(r) * p.row_len),
                                      reinterpret_cast<const uint16_t*>(ref.base) + r, lin, r < 2 * T, rc[u]);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int r = r0 + u * RPW + sub;
            const int j = r >= T ? r - T : r;
            decode_row<TEAM, NCH>(rc[u], const_cast<uint16_t*>(r >= T ? ref.v : ref.k) + j * p.row_stride, lin,
                                  r < 2 * T);
          }
        }
      }
    }
    __syncthreads();  // every warp is done reading the batch's slots before they are released
    if (threadIdx.x < nb && p.free_slots) {
      const PageRef ref = s_ref[threadIdx.x];
      if (ref.slot >= 0) {
        p.page_slot[ref.page] = -1;
        const int32_t pos = atomicAdd(p.free_top_rw, 1);
        if (pos < p.n_slots) p.free_stack[pos] = ref.slot;
      }
    }
    __syncthreads();  // s_ref is rewritten by the next batch
  }
}

__global__ void slots_commit_kernel(const int32_t* count, int32_t max_entries, int32_t* free_top) {
  const int32_t c = min(*count, max_entries);
  const int32_t t = *free_top;
  *free_top = t - min(c, t);
}

// Row lengths head_num_local * 128 for 1..16 local heads (powers of two).
bool pick_nch(int32_t row_len, int& nch) {
  nch = row_len;
  return row_len == 128 || row_len == 256 || row_len == 512 || row_len == 1024 || row_len == 2048;
}

ashkv_status_t validate(const PagesParams& p) {
  if (p.n_layers <= 0 || p.tokens_per_page <= 0 || p.max_entries < 0 || p.n_slots < 0) return ASHKV_BAD_ARGUMENT;
  if (!p.layer_k || !p.layer_v || !p.layer_id || !p.token_start || !p.list || !p.count || !p.arena ||
      !p.page_slot || !p.entry_status)
    return ASHKV_BAD_ARGUMENT;
  const int64_t need = codes_offset(p.tokens_per_page) + 2 * int64_t(p.tokens_per_page) * p.row_len;
  if (p.slot_bytes < need || (p.slot_bytes % 16) || !aligned(p.arena, 16)) return ASHKV_BAD_ARGUMENT;
  if ((p.row_stride * 2) % 16) return ASHKV_BAD_ARGUMENT;
  return ASHKV_OK;
}

unsigned grid_for(int32_t max_entries) {
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t g = std::min<int64_t>(max_entries, int64_t(sms) * 8);
  return unsigned(g > 0 ? g : 1);
}

}  // namespace
}  // namespace ashkv

using namespace ashkv;

#define ASHKV_PAGES_DISPATCH(KERNEL, NAME)                                                  \
  switch (nch) {                                                                           \
    case 128: KERNEL<4, 4><<<grid_for(p.max_entries), kThreads, 0, st>>>(p); break;        \
    case 256: KERNEL<8, 4><<<grid_for(p.max_entries), kThreads, 0, st>>>(p); break;        \
    case 512: KERNEL<16, 4><<<grid_for(p.max_entries), kThreads, 0, st>>>(p); break;       \
    case 1024: KERNEL<32, 4><<<grid_for(p.max_entries), kThreads, 0, st>>>(p); break;      \
    default: KERNEL<32, 8><<<grid_for(p.max_entries), kThreads, 0, st>>>(p); break;        \
  }                                                                                        \
  return check_launch(NAME);

extern "C" int64_t ashkv_int8_page_slot_bytes(int32_t tokens_per_page, int32_t row_len) {
  const int64_t need = codes_offset(tokens_per_page) + 2 * int64_t(tokens_per_page) * row_len;
  return (need + 255) / 256 * 256;
}

extern "C" ashkv_status_t ashkv_int8_encode_pages(
    const uint64_t* d_layer_k, const uint64_t* d_layer_v, int32_t n_layers, const int32_t* d_layer_id,
    const int32_t* d_token_start, const int32_t* d_list, const int32_t* d_count, int32_t max_entries,
    int32_t tokens_per_page, int32_t row_len, int64_t row_stride, void* d_arena, int64_t slot_bytes,
    int64_t n_slots, int32_t* d_free_stack, int32_t* d_free_top, int32_t* d_page_slot, int32_t* d_entry_status,
    void* stream) {
  PagesParams p{};
  p.layer_k = d_layer_k; p.layer_v = d_layer_v; p.n_layers = n_layers; p.layer_id = d_layer_id;
  p.token_start = d_token_start; p.list = d_list; p.count = d_count; p.max_entries = max_entries;
  p.tokens_per_page = tokens_per_page; p.row_len = row_len; p.row_stride = row_stride;
  p.arena = static_cast<uint8_t*>(d_arena); p.slot_bytes = slot_bytes; p.n_slots = n_slots;
  p.free_stack = d_free_stack; p.free_top = d_free_top; p.page_slot = d_page_slot; p.entry_status = d_entry_status;
  if (max_entries == 0) return ASHKV_OK;
  int nch = 0;
  if (!pick_nch(row_len, nch) || !d_free_stack || !d_free_top) return ASHKV_BAD_ARGUMENT;
  const ashkv_status_t v = validate(p);
  if (v != ASHKV_OK) return v;
  cudaStream_t st = as_stream(stream);
  ASHKV_PAGES_DISPATCH(encode_pages_kernel, "int8_encode_pages")
}

extern "C" ashkv_status_t ashkv_slots_commit(const int32_t* d_count, int32_t max_entries, int32_t* d_free_top,
                                             void* stream) {
  if (!d_count || !d_free_top || max_entries < 0) return ASHKV_BAD_ARGUMENT;
  slots_commit_kernel<<<1, 1, 0, as_stream(stream)>>>(d_count, max_entries, d_free_top);
  return check_launch("slots_commit");
}

extern "C" ashkv_status_t ashkv_int8_decode_pages(
    const uint64_t* d_layer_k, const uint64_t* d_layer_v, int32_t n_layers, const int32_t* d_layer_id,
    const int32_t* d_token_start, const int32_t* d_list, const int32_t* d_count, int32_t max_entries,
    int32_t tokens_per_page, int32_t row_len, int64_t row_stride, const void* d_arena, int64_t slot_bytes,
    int64_t n_slots, int32_t* d_page_slot, int32_t free_slots, int32_t* d_free_stack, int32_t* d_free_top,
    int32_t* d_entry_status, void* stream) {
  PagesParams p{};
  p.layer_k = d_layer_k; p.layer_v = d_layer_v; p.n_layers = n_layers; p.layer_id = d_layer_id;
  p.token_start = d_token_start; p.list = d_list; p.count = d_count; p.max_entries = max_entries;
  p.tokens_per_page = tokens_per_page; p.row_len = row_len; p.row_stride = row_stride;
  p.arena = static_cast<uint8_t*>(const_cast<void*>(d_arena)); p.slot_bytes = slot_bytes; p.n_slots = n_slots;
  p.page_slot = d_page_slot; p.entry_status = d_entry_status; p.free_slots = free_slots;
  p.free_stack = d_free_stack; p.free_top_rw = d_free_top;
  if (max_entries == 0) return ASHKV_OK;
  int nch = 0;
  if (!pick_nch(row_len, nch)) return ASHKV_BAD_ARGUMENT;
  if (free_slots && (!d_free_stack || !d_free_top)) return ASHKV_BAD_ARGUMENT;
  const ashkv_status_t v = validate(p);
  if (v != ASHKV_OK) return v;
  cudaStream_t st = as_stream(stream);
  ASHKV_PAGES_DISPATCH(decode_pages_kernel, "int8_decode_pages")
}
