// Page-table policy kernels: score, desired tier, transition lists (sm_100a).
//
// Restates score_vectorized (ashkv/runtime/score.py:15-52) and desired_tiers
// (ashkv/runtime/controller.py:32-106) of the reference.  The reference runs
// five-plus numpy passes over a snapshot copy of the page table on the host;
// here one kernel reads the four feature columns and the tier column once and
// writes R and the target tier, and a second kernel turns the per-block
// transition counts into two stable (ascending page-row) lists: pages to
// demote (target colder than current) and pages to promote.
//
// Numerics: each product and sum is a separate fp32 IEEE operation in the
// reference's left-to-right order ((wT*T + wS*S) + wN*N) + wP*P; clip keeps
// NaN; the thresholds are computed on the host in double exactly as the
// reference's Python floats and rounded once to fp32, as numpy does when it
// compares a float32 array with a Python float.
#include "common.cuh"

namespace ashkv {
namespace {

constexpr int kThreads = 256;
constexpr int kItems = 4;
constexpr int kPagesPerBlock = kThreads * kItems;
constexpr int kTiers = 6;

struct PolicyParams {
  const float* T; const float* S; const float* N; const float* P;
  const int8_t* cur;
  int64_t n;
  float wT, wS, wN, wP;
  float up, down;             // promote / demote thresholds (fp32)
  const float* pressure_dev;  // when set, up/down come from this device value and th_*
  double th_high, th_low, th_delta, th_emergency;
  int8_t next_colder[kTiers];
  int8_t next_hotter[kTiers];
  int do_score, do_tiers;
  const float* R_in;          // when !do_score
  float* R_out;               // nullable
  int8_t* target_out;         // nullable
  int32_t* block_counts;      // [2 * n_blocks] (demote, promote), nullable
};

__device__ __forceinline__ float score1(const PolicyParams& p, int64_t i) {
  float r = __fmul_rn(p.wT, p.T[i]);
  r = __fadd_rn(r, __fmul_rn(p.wS, p.S[i]));
  r = __fadd_rn(r, __fmul_rn(p.wN, p.N[i]));
  r = __fadd_rn(r, __fmul_rn(p.wP, p.P[i]));
  r = r < 0.0f ? 0.0f : r;  // comparisons are false for NaN: NaN stays NaN
  r = r > 1.0f ? 1.0f : r;
  return r;
}

__device__ __forceinline__ int8_t tier1(const PolicyParams& p, float up, float down, float r, int8_t c) {
  int8_t t = c;
  if (c < 0 || c >= kTiers) return t;  // out-of-table tiers never move
  if (r >= up && c > 0) t = p.next_hotter[c];
  if (r <= down && c < 2) t = p.next_colder[c];  // demotion applied second: it wins
  return t;
}

// The thresholds from a pressure held in device memory: the host's double
// arithmetic (fill_params) with every operation rounded on its own.
__device__ __forceinline__ void device_thresholds(const PolicyParams& p, float& up, float& down) {
  const double pr = double(*p.pressure_dev);
  double boost = 0.0;
  if (pr >= p.th_emergency) {
    boost = __dmul_rn(__dadd_rn(pr, -p.th_emergency), 2.0);
    boost = boost < 0.15 ? boost : 0.15;
  }
  up = __double2float_rn(__dadd_rn(p.th_high, p.th_delta));
  down = __double2float_rn(__dadd_rn(__dadd_rn(p.th_low, boost), -p.th_delta));
}

__global__ void __launch_bounds__(kThreads) policy_kernel(const PolicyParams p) {
  __shared__ int32_t s_cnt[2];
  if (threadIdx.x < 2) s_cnt[threadIdx.x] = 0;
  __syncthreads();
  int32_t nd = 0, np = 0;
  float up = p.up, down = p.down;
  if (p.do_tiers && p.pressure_dev) device_thresholds(p, up, down);
  const int64_t base = int64_t(blockIdx.x) * kPagesPerBlock + threadIdx.x;
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int64_t i = base + int64_t(k) * kThreads;
    if (i >= p.n) break;
    const float r = p.do_score ? score1(p, i) : p.R_in[i];
    if (p.R_out) p.R_out[i] = r;
    if (p.do_tiers) {
      const int8_t c = p.cur[i];
      const int8_t t = tier1(p, up, down, r, c);
      if (p.target_out) p.target_out[i] = t;
      nd += t > c;
      np += t < c;
    }
  }
  if (!p.block_counts) return;
  // warp reduce then one atomic per warp into shared
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    nd += __shfl_xor_sync(0xFFFFFFFFu, nd, off);
    np += __shfl_xor_sync(0xFFFFFFFFu, np, off);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&s_cnt[0], nd);
    atomicAdd(&s_cnt[1], np);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    p.block_counts[2 * blockIdx.x] = s_cnt[0];
    p.block_counts[2 * blockIdx.x + 1] = s_cnt[1];
  }
}

// Writes the transition lists.  Block b covers the same pages as block b of
// policy_kernel; its list offsets are the sums of the earlier blocks' counts.
__global__ void __launch_bounds__(kThreads) compact_kernel(const int8_t* cur, const int8_t* target, int64_t n,
                                                           const int32_t* block_counts, int32_t* demote_list,
                                                           int32_t* promote_list, int32_t* totals) {
  __shared__ int32_t s_warp[2][kThreads / 32];
  __shared__ int32_t s_base[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // 1. offsets of this block: reduce counts of blocks [0, blockIdx.x)
  int32_t bd = 0, bp = 0;
  for (int64_t b = threadIdx.x; b < blockIdx.x; b += kThreads) {
    bd += block_counts[2 * b];
    bp += block_counts[2 * b + 1];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    bd += __shfl_xor_sync(0xFFFFFFFFu, bd, off);
    bp += __shfl_xor_sync(0xFFFFFFFFu, bp, off);
  }
  if (lane == 0) { s_warp[0][warp] = bd; s_warp[1][warp] = bp; }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t a = 0, c = 0;
    for (int w = 0; w < kThreads / 32; ++w) { a += s_warp[0][w]; c += s_warp[1][w]; }
    s_base[0] = a; s_base[1] = c;
    if (blockIdx.x == gridDim.x - 1) {
      totals[0] = a + block_counts[2 * blockIdx.x];
      totals[1] = c + block_counts[2 * blockIdx.x + 1];
    }
  }
  __syncthreads();
  // 2. stable in-block ranks, in page order (k-major over the strided layout)
  int32_t run_d = s_base[0], run_p = s_base[1];
  const int64_t base = int64_t(blockIdx.x) * kPagesPerBlock;
  for (int k = 0; k < kItems; ++k) {
    const int64_t i = base + int64_t(k) * kThreads + threadIdx.x;
    int32_t fd = 0, fp = 0;
    if (i < n) {
      const int8_t c = cur[i], t = target[i];
      fd = t > c; fp = t < c;
    }
    const unsigned md = __ballot_sync(0xFFFFFFFFu, fd), mp = __ballot_sync(0xFFFFFFFFu, fp);
    const unsigned lt = (1u << lane) - 1u;
    __syncthreads();  // s_warp reuse
    if (lane == 0) { s_warp[0][warp] = __popc(md); s_warp[1][warp] = __popc(mp); }
    __syncthreads();
    int32_t wd = 0, wp = 0, td = 0, tp = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      if (w < warp) { wd += s_warp[0][w]; wp += s_warp[1][w]; }
      td += s_warp[0][w]; tp += s_warp[1][w];
    }
    if (fd) demote_list[run_d + wd + __popc(md & lt)] = int32_t(i);
    if (fp) promote_list[run_p + wp + __popc(mp & lt)] = int32_t(i);
    run_d += td; run_p += tp;
  }
}

void fill_params(PolicyParams& p, double pressure, double theta_high, double theta_low, double delta,
                 double p_emergency, const int8_t* next_colder, const int8_t* next_hotter) {
  // Same double-precision arithmetic as the reference's Python floats.
  double boost = 0.0;
  if (pressure >= p_emergency) {
    boost = (pressure - p_emergency) * 2.0;
    boost = boost < 0.15 ? boost : 0.15;
  }
  const double up = theta_high + delta;
  const double down = (theta_low + boost) - delta;
  p.up = float(up);
  p.down = float(down);
  for (int i = 0; i < kTiers; ++i) {
    p.next_colder[i] = next_colder[i];
    p.next_hotter[i] = next_hotter[i];
  }
}

}  // namespace
}  // namespace ashkv

using namespace ashkv;

extern "C" ashkv_status_t ashkv_score(const float* d_T, const float* d_S, const float* d_N, const float* d_P,
                                      int64_t n, float w_T, float w_S, float w_N, float w_P, float* d_R,
                                      void* stream) {
  if (n < 0) return ASHKV_BAD_ARGUMENT;
  if (n == 0) return ASHKV_OK;
  if (!d_T || !d_S || !d_N || !d_P || !d_R) return ASHKV_BAD_ARGUMENT;
  const int64_t blocks = (n + kPagesPerBlock - 1) / kPagesPerBlock;
  if (blocks > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;
  PolicyParams p{};
  p.T = d_T; p.S = d_S; p.N = d_N; p.P = d_P; p.n = n;
  p.wT = w_T; p.wS = w_S; p.wN = w_N; p.wP = w_P;
  p.do_score = 1; p.do_tiers = 0; p.R_out = d_R;
  policy_kernel<<<unsigned(blocks), kThreads, 0, as_stream(stream)>>>(p);
  return check_launch("score");
}

extern "C" ashkv_status_t ashkv_desired_tiers(const float* d_R, const int8_t* d_cur, int64_t n, double pressure,
                                              double theta_high, double theta_low, double delta,
                                              double p_emergency, const int8_t* next_colder,
                                              const int8_t* next_hotter, int8_t* d_target, void* stream) {
  if (n < 0 || !next_colder || !next_hotter) return ASHKV_BAD_ARGUMENT;
  if (n == 0) return ASHKV_OK;
  if (!d_R || !d_cur || !d_target) return ASHKV_BAD_ARGUMENT;
  const int64_t blocks = (n + kPagesPerBlock - 1) / kPagesPerBlock;
  if (blocks > 0x7FFFFFFF) return ASHKV_BAD_ARGUMENT;
  PolicyParams p{};
  p.n = n; p.cur = d_cur; p.R_in = d_R; p.do_score = 0; p.do_tiers = 1; p.target_out = d_target;
  fill_params(p, pressure, theta_high, theta_low, delta, p_emergency, next_colder, next_hotter);
  policy_kernel<<<unsigned(blocks), kThreads, 0, as_stream(stream)>>>(p);
  return check_launch("desired_tiers");
}

extern "C" int64_t ashkv_policy_scratch_ints(int64_t n) {
  return 2 * ((n + kPagesPerBlock - 1) / kPagesPerBlock) + 2;
}

namespace ashkv {
namespace {

// Shared by the host-pressure and device-pressure entry points.
ashkv_status_t policy_step_impl(
    const float* d_T, const float* d_S, const float* d_N, const float* d_P, const int8_t* d_cur, int64_t n,
    float w_T, float w_S, float w_N, float w_P, double pressure, const float* d_pressure, double theta_high,
    double theta_low, double delta, double p_emergency, const int8_t* next_colder, const int8_t* next_hotter,
    float* d_R, int8_t* d_target, int32_t* d_demote_list, int32_t* d_promote_list, int32_t* d_counts,
    int32_t* d_scratch, void* stream) {
  if (n < 0 || !next_colder || !next_hotter) return ASHKV_BAD_ARGUMENT;
  if (n > 0x7FFFFFFFLL) return ASHKV_BAD_ARGUMENT;  // list entries are int32 page rows
  cudaStream_t st = as_stream(stream);
  if (n == 0) {
    if (d_counts && cudaMemsetAsync(d_counts, 0, 2 * sizeof(int32_t), st) != cudaSuccess)
      return check_launch("policy_step_memset");
    return ASHKV_OK;
  }
  if (!d_T || !d_S || !d_N || !d_P || !d_cur || !d_target || !d_demote_list || !d_promote_list || !d_counts ||
      !d_scratch)
    return ASHKV_BAD_ARGUMENT;
  const int64_t blocks = (n + kPagesPerBlock - 1) / kPagesPerBlock;
  PolicyParams p{};
  p.T = d_T; p.S = d_S; p.N = d_N; p.P = d_P; p.cur = d_cur; p.n = n;
  p.wT = w_T; p.wS = w_S; p.wN = w_N; p.wP = w_P;
  p.do_score = 1; p.do_tiers = 1; p.R_out = d_R; p.target_out = d_target; p.block_counts = d_scratch;
  fill_params(p, pressure, theta_high, theta_low, delta, p_emergency, next_colder, next_hotter);
  p.pressure_dev = d_pressure;
  p.th_high = theta_high; p.th_low = theta_low; p.th_delta = delta; p.th_emergency = p_emergency;
  policy_kernel<<<unsigned(blocks), kThreads, 0, st>>>(p);
  ashkv_status_t s = check_launch("policy_step");
  if (s != ASHKV_OK) return s;
  compact_kernel<<<unsigned(blocks), kThreads, 0, st>>>(d_cur, d_target, n, d_scratch, d_demote_list,
                                                        d_promote_list, d_counts);
  return check_launch("policy_compact");
}

}  // namespace
}  // namespace ashkv

extern "C" ashkv_status_t ashkv_policy_step(
    const float* d_T, const float* d_S, const float* d_N, const float* d_P, const int8_t* d_cur, int64_t n,
    float w_T, float w_S, float w_N, float w_P, double pressure, double theta_high, double theta_low,
    double delta, double p_emergency, const int8_t* next_colder, const int8_t* next_hotter,
    float* d_R, int8_t* d_target, int32_t* d_demote_list, int32_t* d_promote_list, int32_t* d_counts,
    int32_t* d_scratch, void* stream) {
  return policy_step_impl(d_T, d_S, d_N, d_P, d_cur, n, w_T, w_S, w_N, w_P, pressure, nullptr, theta_high,
                          theta_low, delta, p_emergency, next_colder, next_hotter, d_R, d_target, d_demote_list,
                          d_promote_list, d_counts, d_scratch, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free policy step.
//
// Some callers cannot allocate device memory when they plan a step: a serving
// engine that reserves almost all of HBM for its KV pool at start-up leaves
// nothing for a per-step cudaMalloc (it can fail, or fragment the pool), and
// plain C/FFI callers have no caching allocator to borrow a scratch buffer
// from.  ashkv_policy_step_noalloc needs no scratch argument: the per-block
// transition counts live in the static device array below, so the caller
// passes only inputs and outputs.
//
// The array is a file-scope __device__ object: every GPU that loads the
// library holds it (32 KiB) until the process exits.  It bounds the page
// table at ASHKV_POLICY_NOALLOC_MAX_PAGES entries.  All calls share it, so
// two calls whose kernels overlap on the GPU (e.g. on different streams)
// race; calls on one stream are ordered and safe.  Nothing in it needs to
// start at zero: the first kernel writes every count the second one reads.
// ---------------------------------------------------------------------------
#include <mutex>

namespace ashkv {
namespace {

constexpr int64_t kNoallocMaxBlocks = (ASHKV_POLICY_NOALLOC_MAX_PAGES + kPagesPerBlock - 1) / kPagesPerBlock;
static __device__ __align__(256) int32_t g_policy_scratch[2 * kNoallocMaxBlocks + 2];

constexpr int kMaxDevices = 64;
int32_t* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_policy_scratch on the current device (looked up once per
// device: in host code the symbol name is only a host-side stand-in).
ashkv_status_t scratch_for_current_device(int32_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("policy_step_noalloc: cudaGetDevice", e);
    return ASHKV_LAUNCH_ERROR;
  }
  if (dev < 0 || dev >= kMaxDevices) return ASHKV_BAD_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_policy_scratch);
    if (e != cudaSuccess || !p) {
      set_error("policy_step_noalloc: cudaGetSymbolAddress", e);
      cudaGetLastError();
      return ASHKV_LAUNCH_ERROR;
    }
    g_scratch_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return ASHKV_OK;
}

}  // namespace
}  // namespace ashkv

extern "C" ashkv_status_t ashkv_policy_step_noalloc(
    const float* d_T, const float* d_S, const float* d_N, const float* d_P, const int8_t* d_cur, int64_t n,
    float w_T, float w_S, float w_N, float w_P, double pressure, double theta_high, double theta_low,
    double delta, double p_emergency, const int8_t* next_colder, const int8_t* next_hotter,
    float* d_R, int8_t* d_target, int32_t* d_demote_list, int32_t* d_promote_list, int32_t* d_counts,
    void* stream) {
  if (n > ASHKV_POLICY_NOALLOC_MAX_PAGES) {
    set_message("policy_step_noalloc: the page table has more entries than the static scratch holds "
                "(ASHKV_POLICY_NOALLOC_MAX_PAGES = 4194304); use ashkv_policy_step with caller scratch");
    return ASHKV_BAD_ARGUMENT;
  }
  int32_t* scratch = nullptr;
  const ashkv_status_t s = scratch_for_current_device(&scratch);
  if (s != ASHKV_OK) return s;
  return ashkv_policy_step(d_T, d_S, d_N, d_P, d_cur, n, w_T, w_S, w_N, w_P, pressure, theta_high, theta_low,
                           delta, p_emergency, next_colder, next_hotter, d_R, d_target, d_demote_list,
                           d_promote_list, d_counts, scratch, stream);
}

extern "C" ashkv_status_t ashkv_policy_step_device_pressure(
    const float* d_T, const float* d_S, const float* d_N, const float* d_P, const int8_t* d_cur, int64_t n,
    float w_T, float w_S, float w_N, float w_P, const float* d_pressure, double theta_high, double theta_low,
    double delta, double p_emergency, const int8_t* next_colder, const int8_t* next_hotter,
    float* d_R, int8_t* d_target, int32_t* d_demote_list, int32_t* d_promote_list, int32_t* d_counts,
    int32_t* d_scratch, void* stream) {
  if (!d_pressure) return ASHKV_BAD_ARGUMENT;
  int32_t* scratch = d_scratch;
  if (!scratch) {
    if (n > ASHKV_POLICY_NOALLOC_MAX_PAGES) {
      set_message("policy_step_device_pressure: without caller scratch the page table is limited to "
                  "ASHKV_POLICY_NOALLOC_MAX_PAGES = 4194304 entries");
      return ASHKV_BAD_ARGUMENT;
    }
    const ashkv_status_t s = scratch_for_current_device(&scratch);
    if (s != ASHKV_OK) return s;
  }
  return policy_step_impl(d_T, d_S, d_N, d_P, d_cur, n, w_T, w_S, w_N, w_P, 0.0, d_pressure, theta_high,
                          theta_low, delta, p_emergency, next_colder, next_hotter, d_R, d_target, d_demote_list,
                          d_promote_list, d_counts, scratch, stream);
}
