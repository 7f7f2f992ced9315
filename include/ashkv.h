/*
 * ashkv.h — C ABI of libashkv_cuda.so, the sm_100a kernels behind ASH-KV's
 * KV-page codec and demote/promote hot path.
 *
 * Conventions shared by every entry point:
 *   - Plain pointers and sizes only.  Pointers named d_* are device pointers;
 *     `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every call is asynchronous on `stream`, performs no host synchronisation
 *     and allocates nothing; all buffers are owned by the caller.
 *   - The return value is an ashkv_status_t.  Conditions that only the device
 *     can see (outlier-list overflow, out-of-range indices) are OR-ed as
 *     ASHKV_FLAG_* bits into the caller's device status word `d_status`, which
 *     the caller reads back whenever it chooses.
 *   - No C++ exception crosses this boundary.
 *
 * Each declaration cites the reference interface it replaces (paths are
 * relative to the ASH-KV source tree).
 */
#ifndef ASHKV_H_
#define ASHKV_H_

#include <stdint.h>

#if defined(__GNUC__)
#define ASHKV_API __attribute__((visibility("default")))
#else
#define ASHKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host return values) --------------------------------- */
typedef int32_t ashkv_status_t;
#define ASHKV_OK               0
#define ASHKV_BAD_ARGUMENT     1
#define ASHKV_OUTLIER_OVERFLOW 2
#define ASHKV_LAUNCH_ERROR     3
#define ASHKV_TIMEOUT          4

/* ---- device status-word flags (OR-ed into *d_status) ------------------- */
#define ASHKV_FLAG_OUTLIER_OVERFLOW 0x1u  /* a bucket had more outliers than its capacity */
#define ASHKV_FLAG_INDEX_RANGE      0x2u  /* an index pointed outside its buffer; that element was skipped */
#define ASHKV_FLAG_TIMEOUT          0x4u  /* a bounded wait inside a kernel gave up; its outputs are incomplete */

/* ---- element-type tags -------------------------------------------------- */
#define ASHKV_DTYPE_BF16 0
#define ASHKV_DTYPE_FP16 1

/* ---- N-bit codec constants ---------------------------------------------- */
#define ASHKV_NBIT_GROUP          32    /* elements per quantisation group */
#define ASHKV_NBIT_BUCKET_GROUPS  32    /* groups per outlier bucket (one warp's groups) */
#define ASHKV_NBIT_BUCKET_ELEMS   1024  /* elements per outlier bucket */
#define ASHKV_DITHER_TENSOR 0           /* uniform U in [0,1) read from a caller fp32 tensor */
#define ASHKV_DITHER_PHILOX 1           /* dither generated in-kernel: Philox4x32-10(seed) */

/* ---- flags for the INT8 codec ------------------------------------------- */
#define ASHKV_INT8_FP32_PRODUCT 0x1u  /* v*127 in fp32 (Triton 2.x typing) instead of the input dtype */

/* Library version (major*10000 + minor*100 + patch). */
ASHKV_API int32_t ashkv_version(void);

/* Human-readable text for a status code; static storage, never NULL. */
ASHKV_API const char* ashkv_status_string(ashkv_status_t status);

/* Text of the last CUDA error seen by this thread inside the library. */
ASHKV_API const char* ashkv_last_error(void);

/* Number of streaming multiprocessors of the current device (0 on error). */
ASHKV_API int32_t ashkv_device_sm_count(void);

/* ========================================================================
 * INT8 per-row absmax codec.
 * Replaces the Triton `_int8_encode_kernel` / `_int8_decode_kernel`
 * (ashkv/codecs/int8.py:50-81 and :98-116) as used by INT8Codec
 * (ashkv/codecs/int8.py:149-221) and the SGLang hooks
 * (ashkv/adapters/sglang/hooks.py:104-128, :220-236).
 *
 * encode, per row r of `row_len` elements:
 *   am      = max(max_i |x_i|, 1e-8)              (fp32, NaN ignored)
 *   s_i     = round_to_input_dtype(x_i * 127)      (fp32 product if ASHKV_INT8_FP32_PRODUCT)
 *   q       = s_i / am                              (PTX div.full.f32, as the Triton
 *                                                    kernel divides on the GPU)
 *   code_i  = low byte of int32(trunc(q + (q > 0 ? 0.5 : -0.5)))  (saturating, NaN -> 0;
 *                                                    Triton's fp32 -> int8 cast)
 *   scale_r = am rounded to scale_dtype
 * Row r is read from d_src + (d_row_index ? d_row_index[r] : r) * src_row_stride
 * (elements), written to d_codes + r * codes_row_stride (bytes).  Its scale
 * goes to byte offset (r / scales_per_slot) * scale_slot_stride
 * + (r % scales_per_slot) * 2 of d_scales; scales_per_slot == 1 with
 * scale_slot_stride == 2 is a plain contiguous scale array.
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_int8_encode_rows(
    const void* d_src, int32_t src_dtype, int64_t n_rows, int32_t row_len,
    int64_t src_row_stride, const int64_t* d_row_index,
    void* d_codes, int64_t codes_row_stride,
    void* d_scales, int32_t scale_dtype, int32_t scales_per_slot, int64_t scale_slot_stride,
    uint32_t flags, void* stream);

/* The same encode over n_layers layers in one launch, for the SGLang demote
 * hook, which encodes the same token rows of every layer
 * (ashkv/adapters/sglang/hooks.py:93-137 loops over layers with one Triton
 * launch each): layer l reads its rows from d_layer_src[l] (16-byte aligned),
 * writes codes at d_codes + l * layer_codes_offset and scales at d_scales +
 * l * layer_scales_offset (bytes), with the per-layer addressing above.
 * n_layers is at most 65535. */
ASHKV_API ashkv_status_t ashkv_int8_encode_rows_layers(
    const uint64_t* d_layer_src, int32_t n_layers, int32_t src_dtype, int64_t n_rows, int32_t row_len,
    int64_t src_row_stride, const int64_t* d_row_index,
    void* d_codes, int64_t codes_row_stride, int64_t layer_codes_offset,
    void* d_scales, int32_t scale_dtype, int32_t scales_per_slot, int64_t scale_slot_stride,
    int64_t layer_scales_offset, uint32_t flags, void* stream);

/* decode, per element: out = round_to_out_dtype(bf16((float)code * (float)scale / 127)).
 * Row r is written to d_dst + (d_row_index ? d_row_index[r] : r) * dst_row_stride.
 * Scale addressing mirrors ashkv_int8_encode_rows. */
ASHKV_API ashkv_status_t ashkv_int8_decode_rows(
    const void* d_codes, int64_t codes_row_stride,
    const void* d_scales, int32_t scale_dtype, int32_t scales_per_slot, int64_t scale_slot_stride,
    int64_t n_rows, int32_t row_len,
    void* d_dst, int32_t dst_dtype, int64_t dst_row_stride, const int64_t* d_row_index,
    void* stream);

/* ========================================================================
 * Dithered N-bit codec with 3-sigma outlier isolation (bits = 2, 4 or 8).
 * Replaces DitheredNBitCodec.encode/decode (ashkv/codecs/nbit_dithered.py:43-167)
 * and DitheredINT2Codec.encode/decode (ashkv/codecs/int2_dithered.py:36-147).
 *
 * Input: n_groups groups of 32 bf16 elements, contiguous.  Per group:
 *   mu      = fp32 mean (8 strided fp32 partial sums, then summed in order)
 *   sd      = fp32(sqrt(M2 / 31)), M2 accumulated in fp64
 *   outlier = |x - mu| > sigma * (sd + 1e-8)
 *   x'      = outlier ? mu : x
 *   delta   = max(max|x'|, 1e-8) / ((2^bits - 1) / 2)
 *   code    = clamp(rint((x' + (U - 0.5) * delta) / delta + half), 0, 2^bits - 1)
 * Outputs: d_scales (bf16 delta per group), d_codes (MSB-first packing,
 * 32*bits/8 bytes per group), and the outlier list in buckets of 32 groups:
 * d_bucket_counts[b] is the number of outliers of bucket b (even when it
 * exceeds bucket_cap), d_bucket_entries[b*bucket_cap + j] =
 * (element index within the bucket << 16) | bf16 bits, ascending.
 * dither_mode ASHKV_DITHER_TENSOR reads U = d_dither[e] (fp32 in [0, 1), one
 * per element, what torch.rand returns in the reference); ASHKV_DITHER_PHILOX
 * derives U = (b + 0.5) / 256 from byte b = (e & 15) of the four output words
 * (little-endian) of Philox4x32-10(key = seed, counter = (dither_elem_offset
 * + e) / 16); dither_elem_offset must be a multiple of 16.
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_nbit_encode(
    const void* d_src, int64_t n_groups, int32_t bits, float sigma,
    int32_t dither_mode, const float* d_dither, uint64_t seed, uint64_t dither_elem_offset,
    void* d_scales, void* d_codes,
    uint32_t* d_bucket_counts, uint32_t* d_bucket_entries, int32_t bucket_cap,
    uint32_t* d_status, void* stream);

/* Decode groups, then overwrite the bucketed outliers:
 *   out = bf16(((float)code - half) * (float)bf16_delta); out[idx] = val. */
ASHKV_API ashkv_status_t ashkv_nbit_decode(
    const void* d_scales, const void* d_codes, int64_t n_groups, int32_t bits,
    const uint32_t* d_bucket_counts, const uint32_t* d_bucket_entries, int32_t bucket_cap,
    void* d_dst, uint32_t* d_status, void* stream);

/* Exclusive scan of min(count, cap) over the buckets, then gather the bucketed
 * outliers into the reference blob's flat form: d_out_index[k] (int32 element
 * index within the call, ascending) and d_out_value[k] (bf16 bits).
 * d_total receives the number of outliers written.  d_offsets holds
 * ashkv_nbit_flatten_scratch_ints(n_buckets) uint32 of caller scratch; on
 * return d_offsets[b] is bucket b's first position in the flat list and
 * d_offsets[n_buckets] the total. */
ASHKV_API int64_t ashkv_nbit_flatten_scratch_ints(int64_t n_buckets);
ASHKV_API ashkv_status_t ashkv_nbit_outliers_flatten(
    const uint32_t* d_bucket_counts, const uint32_t* d_bucket_entries, int32_t bucket_cap,
    int64_t n_buckets, uint32_t* d_offsets,
    int32_t* d_out_index, uint16_t* d_out_value, uint32_t* d_total, void* stream);

/* Decode from the blob form: dense dequantisation followed by a scatter of a
 * flat outlier list (any order; indices outside [0, n_groups*32) are skipped
 * and flagged with ASHKV_FLAG_INDEX_RANGE). */
ASHKV_API ashkv_status_t ashkv_nbit_decode_flat(
    const void* d_scales, const void* d_codes, int64_t n_groups, int32_t bits,
    const int32_t* d_out_index, const uint16_t* d_out_value, int64_t n_outliers,
    void* d_dst, uint32_t* d_status, void* stream);

/* ========================================================================
 * XXH64 of many equal-sized items (pages), one 64-bit digest per item.
 * Replaces checksum() (ashkv/codecs/checksum.py:26-37, xxhash.xxh64(...).intdigest())
 * as applied per page by migrate's verify step (ashkv/runtime/migrate.py:151-176)
 * and PageTable's bf16/current checksums (ashkv/contracts/page.py:43-44).
 * Item i occupies item_bytes bytes at d_data + i * item_stride.
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_xxh64_items(
    const void* d_data, int64_t n_items, int64_t item_bytes, int64_t item_stride,
    uint64_t seed, uint64_t* d_out, void* stream);

/* ========================================================================
 * Page-table policy.
 * ashkv_score replaces score_vectorized (ashkv/runtime/score.py:15-52):
 *   R = clip(((w_T*T + w_S*S) + w_N*N) + w_P*P, 0, 1), one fp32 rounding per
 *   operation, NaN kept.
 * ashkv_desired_tiers replaces desired_tiers (ashkv/runtime/controller.py:32-106):
 *   boost = min((pressure - p_emergency) * 2, 0.15) if pressure >= p_emergency else 0
 *   up = theta_high + delta; down = theta_low + boost - delta   (double, then fp32)
 *   target = cur; if R >= up and cur > BF16: target = next_hotter[cur];
 *   if R <= down and cur < INT4: target = next_colder[cur]   (demotion wins).
 *   next_colder / next_hotter are HOST arrays of 6 int8 (one per Tier), as
 *   compiled by compile_controller (ashkv/compiler/runtime_builder.py:80-122).
 *   Tiers outside [0, 6) are left unchanged.
 * ashkv_policy_step fuses both and emits the ascending page-row lists of
 * demotions (target > cur) and promotions (target < cur); d_counts[0..1] get
 * their lengths.  d_scratch holds ashkv_policy_scratch_ints(n) int32.
 * d_R may be NULL in ashkv_policy_step.
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_score(const float* d_T, const float* d_S, const float* d_N, const float* d_P,
                                     int64_t n, float w_T, float w_S, float w_N, float w_P, float* d_R,
                                     void* stream);

ASHKV_API ashkv_status_t ashkv_desired_tiers(const float* d_R, const int8_t* d_cur, int64_t n, double pressure,
                                             double theta_high, double theta_low, double delta,
                                             double p_emergency, const int8_t* next_colder,
                                             const int8_t* next_hotter, int8_t* d_target, void* stream);

ASHKV_API int64_t ashkv_policy_scratch_ints(int64_t n);

ASHKV_API ashkv_status_t ashkv_policy_step(
    const float* d_T, const float* d_S, const float* d_N, const float* d_P, const int8_t* d_cur, int64_t n,
    float w_T, float w_S, float w_N, float w_P, double pressure, double theta_high, double theta_low,
    double delta, double p_emergency, const int8_t* next_colder, const int8_t* next_hotter,
    float* d_R, int8_t* d_target, int32_t* d_demote_list, int32_t* d_promote_list, int32_t* d_counts,
    int32_t* d_scratch, void* stream);

/* ========================================================================
 * Pitched copy (cudaMemcpy2DAsync, direction inferred from the pointers):
 * `height` rows of `width` bytes from src (row pitch src_pitch) to dst (row
 * pitch dst_pitch).  Used by the SGLang promote path to move only the used
 * bytes of each compressed host slot (ashkv/adapters/sglang/hooks.py:198-216
 * moves whole slots through a host-side gather instead).
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_memcpy2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                                        int64_t width, int64_t height, void* stream);

/* ========================================================================
 * Fill: the 32-bit pattern `value` repeated over `bytes` bytes of device
 * memory at d_dst (4-byte aligned, bytes a multiple of 4), with 32-byte
 * streaming stores.  Clears staging buffers and host-slot tails, and is the
 * plain write stream the write-dominated decoders are measured against.
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_fill32(void* d_dst, int64_t bytes, uint32_t value, void* stream);

/* ========================================================================
 * Indexed row copies: for r < n_rows and s < n_sub, `width` bytes from
 *   src + (d_src_index ? d_src_index[r] : r) * src_row_stride + s * src_sub_stride
 * to
 *   dst + (d_dst_index ? d_dst_index[r] : r) * dst_row_stride + s * dst_sub_stride,
 * in one kernel.  Used by the SGLang hooks for host pool rows that are not one
 * contiguous run (ashkv/adapters/sglang/hooks.py:118-137 scatters them with a
 * host-side index assignment per layer, :198-216 gathers them likewise).
 * dst and src are device memory or page-locked host memory mapped for the
 * current device (read and written through that mapping); anything else is
 * refused with ASHKV_BAD_ARGUMENT before any launch.  Index lists are device
 * memory; an index outside [0, dst_rows) / [0, src_rows) skips that row and
 * sets ASHKV_FLAG_INDEX_RANGE in *d_status (if given).  Addresses, strides
 * and width are multiples of 16 bytes.
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_copy_rows_indexed(
    void* dst, int64_t dst_row_stride, int64_t dst_sub_stride, const int64_t* d_dst_index, int64_t dst_rows,
    const void* src, int64_t src_row_stride, int64_t src_sub_stride, const int64_t* d_src_index, int64_t src_rows,
    int64_t width, int64_t n_sub, int64_t n_rows, uint32_t* d_status, void* stream);

/* ========================================================================
 * Batched BF16 <-> INT8 page migration over device-resident lists.
 * Replaces the per-page migrate() loop (ashkv/runtime/migrate.py:35-191) for
 * the BF16 -> FP8/INT8-slot transition and its promotion, with the SGLang
 * hooks' INT8 layout (one fp16 scale per token over the local heads,
 * ashkv/adapters/sglang/hooks.py:83-137).
 *   page p = tokens_per_page rows of row_len bf16 starting at token
 *   d_token_start[p] of layer d_layer_id[p]; K rows at d_layer_k[l] +
 *   token * row_stride (elements), V rows likewise.  row_len must be 128 or a
 *   power-of-two multiple of 256 up to 2048.
 *   Entry i < min(*d_count, max_entries) of d_list is encoded into arena slot
 *   d_free_stack[*d_free_top - 1 - i] (slot_bytes each, see
 *   ashkv_int8_page_slot_bytes); d_page_slot[p] records it; d_entry_status[i]
 *   = 0 ok, 1 no free slot, 2 bad page/slot.  ashkv_slots_commit then pops
 *   the used slots off the stack.
 * ashkv_int8_decode_pages decodes the slot of each listed page back into the
 * K/V rows; with free_slots != 0 it pushes the slot back on the stack and
 * sets d_page_slot[p] = -1.
 * ======================================================================== */
ASHKV_API int64_t ashkv_int8_page_slot_bytes(int32_t tokens_per_page, int32_t row_len);

ASHKV_API ashkv_status_t ashkv_int8_encode_pages(
    const uint64_t* d_layer_k, const uint64_t* d_layer_v, int32_t n_layers, const int32_t* d_layer_id,
    const int32_t* d_token_start, const int32_t* d_list, const int32_t* d_count, int32_t max_entries,
    int32_t tokens_per_page, int32_t row_len, int64_t row_stride, void* d_arena, int64_t slot_bytes,
    int64_t n_slots, int32_t* d_free_stack, int32_t* d_free_top, int32_t* d_page_slot, int32_t* d_entry_status,
    void* stream);

ASHKV_API ashkv_status_t ashkv_slots_commit(const int32_t* d_count, int32_t max_entries, int32_t* d_free_top,
                                            void* stream);

ASHKV_API ashkv_status_t ashkv_int8_decode_pages(
    const uint64_t* d_layer_k, const uint64_t* d_layer_v, int32_t n_layers, const int32_t* d_layer_id,
    const int32_t* d_token_start, const int32_t* d_list, const int32_t* d_count, int32_t max_entries,
    int32_t tokens_per_page, int32_t row_len, int64_t row_stride, const void* d_arena, int64_t slot_bytes,
    int64_t n_slots, int32_t* d_page_slot, int32_t free_slots, int32_t* d_free_stack, int32_t* d_free_top,
    int32_t* d_entry_status, void* stream);

/* ========================================================================
 * Mixed-tier page migration over device-resident transition lists.
 * Replaces the per-page migrate() ladder (ashkv/runtime/migrate.py:35-191)
 * for every (current, target) tier edge the controller plans
 * (ashkv/runtime/controller.py:88-104), each running the codec the resolver
 * puts on that tier (ashkv/compiler/codec_resolver.py:56-95).
 *
 * A page p is 2 * tokens_per_page rows of row_len bf16: its K rows, then its
 * V rows, at token d_token_start[p] of layer d_layer_id[p] of the KV pool
 * (K rows at d_layer_k[l] + token * row_stride elements, V likewise).  Each
 * tier t holds its pages in stores[t] (a host array of six entries indexed by
 * tier: BF16, FP8, INT4, ARCHIVE, CPU, DISK): store 0 must have format
 * ASHKV_PAGE_BF16 (the pool rows themselves); a tier whose format is
 * ASHKV_PAGE_NONE has no codec.  Other stores are arrays of n_slots slots of
 * slot_bytes (>= ashkv_page_slot_bytes) with a device free stack
 * (d_free_stack[0 .. *d_free_top)).
 *
 * ashkv_migrate_pages, for each entry i < min(*d_count, max_entries) of
 * d_list (page p, current tier d_tier[p], target d_target[p]):
 *   pinned (d_pin[p] > 0) -> ASHKV_MIGRATE_PINNED, already at target ->
 *   ASHKV_MIGRATE_SAME_TIER, a tier without a codec -> ASHKV_MIGRATE_NO_CODEC,
 *   bad layer / slot -> ASHKV_MIGRATE_BAD_PAGE, empty target stack ->
 *   ASHKV_MIGRATE_NO_SLOT; otherwise the page is decoded from its current
 *   slot (or pool rows) and encoded into a slot popped from the target store
 *   (or its pool rows), and d_tier[p], d_page_slot[p] are updated (-1 for
 *   BF16).  A dithered page with more outliers than outlier_cap is not moved
 *   (ASHKV_MIGRATE_OVERFLOW).  d_entry_status[i] gets the status and
 *   d_released[i] the slot given up, as (tier << 24) | slot, or -1.
 *   Dithered formats draw Philox4x32-10(seed) at counter (p * E + e) / 8 for
 *   element e of page p (E = 2 * tokens_per_page * row_len), sigma as in
 *   DitheredNBitCodec.  row_len is 128, 256, 512, 1024 or 2048; E is a
 *   multiple of 1024 and at most 65536.  A page must appear at most once per
 *   call.
 * ashkv_release_slots then pushes every recorded slot back on its store's
 * free stack.  Run it after ashkv_migrate_pages and before the next one
 * (pops and pushes never share a launch).
 * ======================================================================== */
#define ASHKV_PAGE_NONE  (-1)  /* the tier has no codec */
#define ASHKV_PAGE_BF16  0     /* the page's rows in the KV pool */
#define ASHKV_PAGE_INT8  1     /* [2T fp16 row scales | pad to 16 | int8 codes] (the hooks' layout) */
#define ASHKV_PAGE_FP8   2     /* FP8Codec: e4m3fn bytes */
#define ASHKV_PAGE_INT4  3     /* INT4Codec, group 64: [E/64 bf16 scales | E/2 nibble bytes] */
#define ASHKV_PAGE_NBIT4 4     /* DitheredNBitCodec(bits=4): [u32 n_out, 12 B | E/32 bf16 delta | codes | outliers] */
#define ASHKV_PAGE_NBIT2 5     /* DitheredINT2Codec: the same layout with 2-bit codes */

#define ASHKV_MIGRATE_OK        0
#define ASHKV_MIGRATE_NO_SLOT   1
#define ASHKV_MIGRATE_BAD_PAGE  2
#define ASHKV_MIGRATE_PINNED    3
#define ASHKV_MIGRATE_SAME_TIER 4
#define ASHKV_MIGRATE_NO_CODEC  5
#define ASHKV_MIGRATE_OVERFLOW  6

typedef struct {
  void* d_data;          /* n_slots * slot_bytes bytes, 16-byte aligned */
  int64_t slot_bytes;    /* multiple of 16 */
  int32_t n_slots;       /* at most 2^24 - 1 */
  int32_t format;        /* ASHKV_PAGE_* */
  int32_t* d_free_stack; /* [n_slots] */
  int32_t* d_free_top;   /* [1] */
} ashkv_tier_store_t;

/* Bytes of one slot of `format` (rounded up to 256); -1 for a bad argument. */
ASHKV_API int64_t ashkv_page_slot_bytes(int32_t format, int32_t tokens_per_page, int32_t row_len,
                                        int32_t outlier_cap);

ASHKV_API ashkv_status_t ashkv_migrate_pages(
    int8_t* d_tier, const int32_t* d_pin, const int32_t* d_layer_id, const int32_t* d_token_start,
    int32_t* d_page_slot, int64_t n_pages, const int8_t* d_target, const int32_t* d_list, const int32_t* d_count,
    int32_t max_entries, const uint64_t* d_layer_k, const uint64_t* d_layer_v, int32_t n_layers,
    int32_t tokens_per_page, int32_t row_len, int64_t row_stride, const ashkv_tier_store_t* stores, float sigma,
    uint64_t seed, int32_t outlier_cap, int32_t* d_entry_status, int32_t* d_released, void* stream);

ASHKV_API ashkv_status_t ashkv_release_slots(const int32_t* d_released, const int32_t* d_count, int32_t max_entries,
                                             const ashkv_tier_store_t* stores, uint32_t* d_status, void* stream);

/* ========================================================================
 * ashkv_policy_step without a scratch argument.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory while
 * they plan a step (an engine that has reserved nearly all HBM for its KV
 * pool, or a plain C/FFI caller without a caching allocator).  The per-block
 * counts live in a static 32 KiB device array inside the library, held by
 * every GPU that loads it until the process exits, which limits the page
 * table to ASHKV_POLICY_NOALLOC_MAX_PAGES entries (larger n returns
 * ASHKV_BAD_ARGUMENT with a message in ashkv_last_error()).  The first call
 * on each device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * All calls share the array: calls whose kernels overlap on the GPU race.
 * The function allocates nothing.
 * ======================================================================== */
#define ASHKV_POLICY_NOALLOC_MAX_PAGES 4194304
ASHKV_API ashkv_status_t ashkv_policy_step_noalloc(
    const float* d_T, const float* d_S, const float* d_N, const float* d_P, const int8_t* d_cur, int64_t n,
    float w_T, float w_S, float w_N, float w_P, double pressure, double theta_high, double theta_low,
    double delta, double p_emergency, const int8_t* next_colder, const int8_t* next_hotter,
    float* d_R, int8_t* d_target, int32_t* d_demote_list, int32_t* d_promote_list, int32_t* d_counts,
    void* stream);

/* ========================================================================
 * ashkv_policy_step with the allocator pressure read from device memory
 * (one fp32 value, e.g. the result of the ranks' MAX all-reduce), so a
 * step needs no host read-back between the pressure exchange and the
 * plan.  The thresholds are computed in the kernel with the same double
 * operations as ashkv_policy_step applies to (double)*d_pressure, so both
 * give identical lists.  d_scratch may be NULL: the static scratch of
 * ashkv_policy_step_noalloc is used then (same limits and sharing rule).
 * No counterpart in the reference, whose pressure is a host float
 * (ashkv/runtime/controller.py:32-106).
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_policy_step_device_pressure(
    const float* d_T, const float* d_S, const float* d_N, const float* d_P, const int8_t* d_cur, int64_t n,
    float w_T, float w_S, float w_N, float w_P, const float* d_pressure, double theta_high, double theta_low,
    double delta, double p_emergency, const int8_t* next_colder, const int8_t* next_hotter,
    float* d_R, int8_t* d_target, int32_t* d_demote_list, int32_t* d_promote_list, int32_t* d_counts,
    int32_t* d_scratch, void* stream);

/* ========================================================================
 * FP8 codec: bf16 <-> float8_e4m3fn, one byte per element.
 * Replaces FP8Codec (ashkv/codecs/fp8.py:32-79), i.e. torch's casts
 * tensor.to(torch.float8_e4m3fn) and view(float8_e4m3fn).to(bfloat16):
 *   encode: round to nearest even, no saturation -- |x| > 464, inf and NaN
 *           give 0x7F | sign (E4M3FN's NaN);
 *   decode: exact; NaN codes give bf16 0x7FFF (torch's CUDA cast).
 * n elements; any alignment (16/32-byte aligned buffers take the vector path).
 * ======================================================================== */
ASHKV_API ashkv_status_t ashkv_fp8_encode(const void* d_src_bf16, int64_t n, void* d_dst_fp8, void* stream);
ASHKV_API ashkv_status_t ashkv_fp8_decode(const void* d_src_fp8, int64_t n, void* d_dst_bf16, void* stream);

/* ========================================================================
 * INT4 group codec.  Replaces INT4Codec (ashkv/codecs/int4.py:38-112),
 * which the reference runs in numpy on the host.  The n bf16 inputs are
 * zero-padded to n_groups = ceil(n / group_size) groups; per group
 *   am = maximum(max|x|, 1e-8) (NaN propagates), scale = bf16(am),
 *   q  = clip(int8(round_half_even(x*7/am)), -8, 7)  (numpy's x86 int8 cast:
 *        NaN / inf give 0), stored as q + 8, even element in the high nibble;
 * decode: bf16(float(q) * float(scale) / 7).  Every NaN written as bf16 is
 * 0xFFFF (torch's CPU cast, where the reference computes).
 * d_scales: n_groups bf16; d_packed: n_groups * group_size / 2 bytes (the
 * padded count must be even, else ASHKV_BAD_ARGUMENT); d_dst: n_groups *
 * group_size bf16.  ashkv_int4_group_count(n, group_size) = n_groups.
 * ======================================================================== */
ASHKV_API int64_t ashkv_int4_group_count(int64_t n, int32_t group_size);
ASHKV_API ashkv_status_t ashkv_int4_encode(const void* d_src_bf16, int64_t n, int32_t group_size,
                                           void* d_scales_bf16, void* d_packed, void* stream);
ASHKV_API ashkv_status_t ashkv_int4_decode(const void* d_scales_bf16, const void* d_packed, int64_t n_groups,
                                           int32_t group_size, void* d_dst_bf16, void* stream);

/* ========================================================================
 * Attention-derived page features (the S and N inputs of ashkv_score).
 * Saliency restates the attention mass per key of the reference simulator
 * (ashkv/tests/simulator.py:66-80): for query rows q [n_q, heads_q, head_dim]
 * and key rows k [n_k, heads_kv, head_dim] (bf16, contiguous, 16-byte
 * aligned; query head h reads key head h / (heads_q / heads_kv)),
 *   P[h,i,:] = softmax_j(scale * q_i . k_j), keys j <= q_pos0 + i only,
 *   d_token_saliency[j] = sum over h and i of P[h,i,j]          (fp32).
 * Scores run on the tensor cores (tcgen05, fp32 accumulation in TMEM),
 * so results match an fp32 evaluation to fp32 accumulation-order accuracy.
 * head_dim must be 64 or 128; d_scratch holds
 * ashkv_saliency_scratch_floats(heads_q, n_q, n_k) floats.
 * ashkv_page_features: per page of tokens_per_page consecutive keys,
 *   d_S[p] = (sum of the page's token saliency) / (largest page sum),
 *   d_N[p] = mean over the page's tokens t of
 *            ||k_t - k_{t-1}||^2 / (||k_t||^2 + ||k_{t-1}||^2) / 2  (0 for t = 0),
 * k rows of row_len = heads_kv * head_dim bf16; d_s_raw: n_pages floats of
 * scratch.  With d_token_saliency NULL only d_N is written.  The reference
 * defines no page-level saliency and no novelty producer; these are this
 * library's definitions, both in [0, 1].
 * ======================================================================== */
ASHKV_API int64_t ashkv_saliency_scratch_floats(int32_t heads_q, int64_t n_q, int64_t n_k);
ASHKV_API ashkv_status_t ashkv_attention_saliency(const void* d_q, const void* d_k, int32_t heads_q, int32_t heads_kv,
                                                  int32_t head_dim, int64_t n_q, int64_t n_k, int64_t q_pos0,
                                                  float scale, float* d_scratch, float* d_token_saliency,
                                                  uint32_t* d_status, void* stream);
ASHKV_API ashkv_status_t ashkv_page_features(const float* d_token_saliency, const void* d_k, int32_t row_len,
                                             int64_t n_k, int32_t tokens_per_page, float* d_s_raw, float* d_S,
                                             float* d_N, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ASHKV_H_ */
