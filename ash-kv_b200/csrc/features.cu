// Attention-derived page features on sm_100a: saliency (tcgen05 tensor cores,
// TMEM accumulators, TMA-fed shared memory) and key novelty.
//
// Saliency restates the reference simulator's attention mass per key
// (ashkv/tests/simulator.py:66-80):
//   s[h,i,j]  = (q_i . k_j) * scale,  masked to -inf unless key position j <= query position
//   P[h,i,:]  = softmax_j(s[h,i,:])
//   sal[j]    = sum over heads h and queries i of P[h,i,j]
// in two tensor-core passes over the score tiles (the softmax normaliser of
// every query row first, then each key row's column mass), with fp32
// accumulation in TMEM.  The reference keeps only this per-token quantity;
// per page it is summed over the page's tokens and divided by the largest
// page's mass (S in [0, 1]), and the novelty input is the mean over the page
// of ||k_t - k_{t-1}||^2 / (||k_t||^2 + ||k_{t-1}||^2) / 2 (in [0, 1]).
//
// Tiles: 128 queries x 128 keys per MMA group (M = N = 128, K = head_dim in
// steps of 16), bf16 operands in 128-byte-swizzled K-major shared memory
// (one 16 KiB chunk per 64 elements of head_dim), one fp32 accumulator of 128
// TMEM columns per tile.  One CTA per SM: a producer warp issues the TMA loads
// (4 B-tile stages, 160 KiB with the A tile) and the MMAs into 4 accumulators
// (all 512 TMEM columns), so up to three tiles' MMAs run ahead of the
// epilogue and the loads run further ahead still; no epilogue thread issues
// anything.  Sixteen warps share a tile's epilogue: warp w reads TMEM
// lanes 32 (w % 4) .. + 31 (accumulator rows) and columns 32 (w / 4) .. + 31,
// so each thread handles 32 values per tile; pass 1 keeps an online max/sum
// per (row, column group), pass 2 (keys x queries) a sum per (key row, column
// group), merged through shared memory at the end.  The causal mask is
// evaluated only for column groups that cross the diagonal.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace ashkv {
namespace {

constexpr int kTile = 128;                   // rows of a query or key tile
constexpr int kChunkBytes = kTile * 128;     // 128 rows x 64 bf16 (one swizzle atom column) = 16 KiB
constexpr int kEpiWarps = 16;                // TMEM lane quadrant (warp % 4) x 32-column group (warp / 4)
constexpr int kThreadsF = (kEpiWarps + 1) * 32;  // + one producer warp (TMA loads and MMA issue)
constexpr int kColGroups = 4;
constexpr uint32_t kPolls = 1u << 24;        // bounded mbarrier waits
constexpr int kSB = 4;                       // B tile stages
constexpr int kAcc = 4;                      // 128-column fp32 accumulators
constexpr uint32_t kAccCols = 128 * kAcc;    // the whole TMEM of the SM: one CTA per SM

// ---------------------------------------------------------------- tcgen05 / TMA wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(smem_dst)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A * B^T, A: M x K and B: N x K, both K-major bf16 in shared memory.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
               :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate),
                  "r"(0u), "r"(0u), "r"(0u), "r"(0u) : "memory");
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 128 bytes stacked every 1024 bytes (stride byte offset), sm_100 version 1.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = uint64_t((smem_addr >> 4) & 0x3FFFu);  // start address (16-byte units)
  d |= uint64_t(1) << 16;                              // leading byte offset: unused for swizzled K-major
  d |= uint64_t(1024 >> 4) << 32;                      // stride byte offset
  d |= uint64_t(1) << 46;                              // descriptor version
  d |= uint64_t(2) << 61;                              // SWIZZLE_128B
  return d;
}
// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major, M = N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t(kTile) >> 3) << 17) |
                            ((uint32_t(kTile) >> 4) << 24);

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y,
                                            int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      :: "r"(smem_u32(smem_dst)), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// Two 2^x on an fp32 pair.
__device__ __forceinline__ f2 ex2_2(f2 x) {
  float a, b;
  upk2(x, a, b);
  return pk2(ex2(a), ex2(b));
}

struct SalParams {
  int32_t heads_q, group, nch;  // group = heads_q / heads_kv; nch = head_dim / 64
  int64_t n_q, n_k, q_pos0;
  float c;                      // scale * log2(e)
  float* lse2;                  // [heads_q, n_q]: log2 of sum_j 2^(s_ij * c)
  float* colsum;                // [heads_q, n_k]
  uint32_t* status;
};

// Loads `rows` tile t (all head_dim chunks) of head `head` into dst, arriving on bar.
__device__ __forceinline__ void load_tile(const CUtensorMap* map, uint8_t* dst, uint64_t* bar, int nch, int head,
                                          int64_t t) {
  mbar_arrive_expect_tx(bar, uint32_t(nch * kChunkBytes));
  for (int c = 0; c < nch; ++c) tma_load_3d(dst + c * kChunkBytes, map, bar, c * 64, head, int32_t(t * kTile));
}

// One tile's MMA group: acc (+)= A_tile * B_tile^T over head_dim.
__device__ __forceinline__ void mma_tile(uint32_t acc, const uint8_t* a, const uint8_t* b, int nch) {
  const uint32_t sa = smem_u32(a), sb = smem_u32(b);
  for (int c = 0; c < nch; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j)  // K = 16 per MMA: 32 bytes further along the swizzled row
      umma_bf16(acc, sw128_kmajor_desc(sa + c * kChunkBytes + j * 32), sw128_kmajor_desc(sb + c * kChunkBytes + j * 32),
                kIdesc, (c | j) != 0);
}

// Shared layout of both passes: [A tile][B stage 0] .. [B stage kSB-1], 1024-byte aligned.
struct PassSmem {
  uint8_t* a;
  uint32_t stage_bytes;  // one tile: nch chunks
  __device__ __forceinline__ uint8_t* b(int i) const { return a + uint32_t(i + 1) * stage_bytes; }
};
__device__ __forceinline__ PassSmem carve(uint8_t* raw, int nch) {
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  PassSmem s;
  s.a = base;
  s.stage_bytes = uint32_t(nch) * kChunkBytes;
  return s;
}
struct PassBars {
  uint64_t a, b[kSB], bfree[kSB], full[kAcc], empty[kAcc];
};
__device__ __forceinline__ void init_bars(PassBars& br) {
  mbar_init(&br.a, 1);
#pragma unroll
  for (int i = 0; i < kSB; ++i) { mbar_init(&br.b[i], 1); mbar_init(&br.bfree[i], 1); }
#pragma unroll
  for (int i = 0; i < kAcc; ++i) { mbar_init(&br.full[i], 1); mbar_init(&br.empty[i], kEpiWarps); }
  mbar_init_fence();
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// The pipelined loop shared by both passes.  A (the CTA's fixed tile) is
// loaded once; B tiles t = t0 .. t0 + nt - 1 stream through kSB shared-memory
// stages into kAcc TMEM accumulators.  One producer warp (its lane 0) issues
// the TMA loads and the MMAs: tile i's MMA once its B stage has landed and the
// epilogue warps have drained accumulator i % kAcc, and the refill of tile
// i - 1's stage once that MMA has completed.  The epilogue warps copy their 32
// values of tile i out of TMEM, release the accumulator and run epi(i, v).
// Returns false (and sets ASHKV_FLAG_TIMEOUT) if a bounded wait gave up; all
// issued MMAs and TMA loads have completed when it returns.
template <class Epi>
__device__ bool run_tiles(const CUtensorMap* amap, int a_head, int64_t a_tile, const CUtensorMap* bmap, int b_head,
                          int64_t t0, int nt, int nch, const PassSmem& sm, PassBars& br, uint32_t tmem,
                          uint32_t* status, Epi epi) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  volatile __shared__ int s_fail;
  if (tid == 0) s_fail = 0;
  __syncthreads();
  // producer's record, for the clean-up: B loads issued up to `loaded` and awaited up
  // to `waited`, MMAs issued up to `issued` and seen complete up to `done`
  int loaded = -1, waited = -1, issued = -1, done = -1;
  bool a_ok = true;
  if (warp == kEpiWarps) {
    if (lane == 0) {
      load_tile(amap, sm.a, &br.a, nch, a_head, a_tile);
      for (int t = 0; t < kSB && t < nt; ++t) {
        load_tile(bmap, sm.b(t), &br.b[t], nch, b_head, t0 + t);
        loaded = t;
      }
      a_ok = mbar_wait_bounded(&br.a, 0, kPolls);
      bool ok = a_ok;
      for (int i = 0; ok && i < nt; ++i) {
        const int st = i % kSB, ac = i % kAcc;
        ok = mbar_wait_bounded(&br.b[st], (i / kSB) & 1, kPolls);
        if (!ok) break;
        waited = i;
        if (i >= kAcc && !(ok = mbar_wait_bounded(&br.empty[ac], ((i / kAcc) - 1) & 1, kPolls))) break;
        tc_fence_after();
        mma_tile(tmem + uint32_t(ac) * 128u, sm.a, sm.b(st), nch);
        umma_commit(&br.full[ac]);
        umma_commit(&br.bfree[st]);
        issued = i;
        const int j = i - 1;  // tile j's MMA is the one before: refill its stage once it has completed
        if (j >= 0 && j + kSB < nt) {
          if (!(ok = mbar_wait_bounded(&br.bfree[j % kSB], (j / kSB) & 1, kPolls))) break;
          done = j;
          load_tile(bmap, sm.b(j % kSB), &br.b[j % kSB], nch, b_head, t0 + j + kSB);
          loaded = j + kSB;
        }
      }
      if (!ok) s_fail = 1;
    }
    __syncwarp();
  } else {
    const uint32_t my_lanes = (uint32_t((warp & 3) * 32) << 16) + uint32_t(warp >> 2) * 32u;
    for (int i = 0; i < nt; ++i) {
      const int ac = i % kAcc;
      if (!mbar_wait_bounded(&br.full[ac], (i / kAcc) & 1, kPolls)) {
        s_fail = 1;
        break;
      }
      tc_fence_after();
      float v[32];
      tmem_ld32(tmem + my_lanes + uint32_t(ac) * 128u, v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&br.empty[ac]);  // this warp is done with the accumulator
      epi(i, v);
    }
  }
  __syncthreads();
  const bool ok = !s_fail;
  if (warp == kEpiWarps && lane == 0) {
    if (!ok) atomicOr(status, ASHKV_FLAG_TIMEOUT);
    // every issued MMA and TMA load completes before TMEM and shared memory are released
    for (int t = done + 1; t <= issued; ++t) mbar_wait_bounded(&br.bfree[t % kSB], (t / kSB) & 1, kPolls);
    if (!a_ok) mbar_wait_bounded(&br.a, 0, kPolls);
    for (int t = waited + 1; t <= loaded; ++t) mbar_wait_bounded(&br.b[t % kSB], (t / kSB) & 1, kPolls);
  }
  tc_fence_before();
  __syncthreads();
  return ok;
}

// Pass 1: CTA (query tile qt, query head h): log2-sum-exp2 of every query row.
// Query tiles run in reverse order so the longest (most key tiles) start first.
__global__ void __launch_bounds__(kThreadsF, 1) saliency_rows_kernel(const __grid_constant__ CUtensorMap tq,
                                                                     const __grid_constant__ CUtensorMap tk,
                                                                     const SalParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ PassBars br;
  __shared__ uint32_t s_tmem;
  __shared__ float s_m[kColGroups][kTile], s_l[kColGroups][kTile];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = (warp & 3) * 32 + (tid & 31), cg = warp >> 2;
  const int qt = int(gridDim.x) - 1 - int(blockIdx.x), h = blockIdx.y, hk = h / p.group;
  const int64_t qrow = int64_t(qt) * kTile + row, qpos = p.q_pos0 + qrow;
  const int64_t q_hi = min(int64_t(qt + 1) * kTile, p.n_q) - 1;
  const int64_t k_hi = min(p.q_pos0 + q_hi, p.n_k - 1);  // the last key any row of the tile attends
  const int nt = k_hi < 0 ? 0 : int(k_hi / kTile) + 1;
  const PassSmem sm = carve(smem_raw, p.nch);
  if (warp == 0) tmem_alloc(&s_tmem, kAccCols);
  if (tid == 0) init_bars(br);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  float m = -INFINITY, l = 0.0f;
  const float c = p.c;
  if (nt > 0) {
    run_tiles(&tq, h, qt, &tk, hk, 0, nt, p.nch, sm, br, tmem, p.status,
              [&](int i, float (&v)[32]) {
                const int64_t k0 = int64_t(i) * kTile + cg * 32;
                float mx = -INFINITY;
                if (k0 + 31 <= qpos && k0 + 31 < p.n_k) {  // the whole column group is visible: fp32 pairs
                  const f2 C2 = pk2(c, c);
                  f2 V[16];
#pragma unroll
                  for (int j = 0; j < 16; ++j) {
                    V[j] = mul2(pk2(v[2 * j], v[2 * j + 1]), C2);
                    float a, b;
                    upk2(V[j], a, b);
                    mx = max3f(mx, a, b);
                  }
                  const float mn = fmaxf(m, mx);
                  const f2 NMN = pk2(-mn, -mn);
                  f2 S = pk2(0.0f, 0.0f);
#pragma unroll
                  for (int j = 0; j < 16; ++j) S = add2(S, ex2_2(add2(V[j], NMN)));
                  float s0, s1;
                  upk2(S, s0, s1);
                  l = (m == -INFINITY ? 0.0f : l * ex2(m - mn)) + (s0 + s1);
                  m = mn;
                  return;
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j) {
                    v[j] = (k0 + j <= qpos && k0 + j < p.n_k) ? v[j] * c : -INFINITY;
                    mx = fmaxf(mx, v[j]);
                  }
                }
                if (mx == -INFINITY) return;
                const float mn = fmaxf(m, mx);
                float sum = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) sum += ex2(v[j] - mn);
                l = (m == -INFINITY ? 0.0f : l * ex2(m - mn)) + sum;
                m = mn;
              });
  }
  // merge the four column groups of each row
  if (warp < kEpiWarps) {
    s_m[cg][row] = m;
    s_l[cg][row] = l;
  }
  __syncthreads();
  if (cg == 0 && qrow < p.n_q) {
    float M = -INFINITY;
#pragma unroll
    for (int g = 0; g < kColGroups; ++g) M = fmaxf(M, s_m[g][row]);
    float L = 0.0f;
    if (M != -INFINITY)
#pragma unroll
      for (int g = 0; g < kColGroups; ++g)
        if (s_l[g][row] > 0.0f) L += s_l[g][row] * ex2(s_m[g][row] - M);
    p.lse2[int64_t(h) * p.n_q + qrow] = L > 0.0f ? M + __log2f(L) : INFINITY;
  }
  if (warp == 0) {
    tmem_dealloc(tmem, kAccCols);
    tmem_relinquish();
  }
}

// Pass 2: CTA (key tile kt, query head h): sum over the query rows of
// 2^(s * c - lse2[q]) for every key row of the tile (scores computed as K Q^T).
__global__ void __launch_bounds__(kThreadsF, 1) saliency_cols_kernel(const __grid_constant__ CUtensorMap tq,
                                                                     const __grid_constant__ CUtensorMap tk,
                                                                     const SalParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ PassBars br;
  __shared__ uint32_t s_tmem;
  __shared__ float s_sum[kColGroups][kTile];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = (warp & 3) * 32 + (tid & 31), cg = warp >> 2;
  const int kt = blockIdx.x, h = blockIdx.y, hk = h / p.group;
  const int64_t kpos = int64_t(kt) * kTile + row;
  // queries that can attend a key of this tile: query position >= kt * 128
  int64_t q_lo = int64_t(kt) * kTile - p.q_pos0;
  if (q_lo < 0) q_lo = 0;
  const int64_t n_qt = (p.n_q + kTile - 1) / kTile;
  const int64_t t0 = q_lo / kTile;
  const int nt = t0 < n_qt ? int(n_qt - t0) : 0;
  const PassSmem sm = carve(smem_raw, p.nch);
  if (warp == 0) tmem_alloc(&s_tmem, kAccCols);
  if (tid == 0) init_bars(br);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const float c = p.c;
  const float* lse = p.lse2 + int64_t(h) * p.n_q;
  float acc_sum = 0.0f;
  if (nt > 0) {
    run_tiles(&tk, hk, kt, &tq, h, t0, nt, p.nch, sm, br, tmem, p.status,
              [&](int i, float (&v)[32]) {
                const int64_t qc = (t0 + i) * kTile + cg * 32;
                const bool full = p.q_pos0 + qc >= kpos && qc + 31 < p.n_q;  // every query of the group sees this key
                if (full && (reinterpret_cast<uintptr_t>(lse + qc) & 15u) == 0) {
                  const float4* l4 = reinterpret_cast<const float4*>(lse + qc);  // the group's row normalisers
                  const f2 C2 = pk2(c, c);
                  f2 S = pk2(0.0f, 0.0f);
#pragma unroll
                  for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 n4 = __ldg(l4 + j4);
                    S = add2(S, ex2_2(fma2(pk2(v[4 * j4], v[4 * j4 + 1]), C2, pk2(-n4.x, -n4.y))));
                    S = add2(S, ex2_2(fma2(pk2(v[4 * j4 + 2], v[4 * j4 + 3]), C2, pk2(-n4.z, -n4.w))));
                  }
                  float s0, s1;
                  upk2(S, s0, s1);
                  acc_sum += s0 + s1;
                } else if (full) {
#pragma unroll
                  for (int j = 0; j < 32; ++j) acc_sum += ex2(fmaf(v[j], c, -__ldg(lse + qc + j)));
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j) {
                    const bool valid = p.q_pos0 + qc + j >= kpos && qc + j < p.n_q;
                    acc_sum += valid ? ex2(fmaf(v[j], c, -lse[qc + j])) : 0.0f;
                  }
                }
              });
  }
  if (warp < kEpiWarps) s_sum[cg][row] = acc_sum;
  __syncthreads();
  if (cg == 0 && kpos < p.n_k)
    p.colsum[int64_t(h) * p.n_k + kpos] = (s_sum[0][row] + s_sum[1][row]) + (s_sum[2][row] + s_sum[3][row]);
  if (warp == 0) {
    tmem_dealloc(tmem, kAccCols);
    tmem_relinquish();
  }
}

// sal[k] = sum over query heads of colsum[h, k].
__global__ void head_sum_kernel(const float* __restrict__ colsum, int32_t heads, int64_t n_k, float* __restrict__ sal) {
  for (int64_t k = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; k < n_k; k += int64_t(gridDim.x) * blockDim.x) {
    float s = 0.0f;
    for (int h = 0; h < heads; ++h) s += colsum[int64_t(h) * n_k + k];
    sal[k] = s;
  }
}

// One CTA per page: raw saliency mass (sum of the page's token saliency) and
// novelty (mean over its tokens of ||k_t - k_{t-1}||^2 / (||k_t||^2 + ||k_{t-1}||^2) / 2).
// Warp w takes tokens t0 + w, t0 + w + 8, ...; the warps' partial sums are added
// in warp order, so the result is the same on every run.  Rows are read as
// 16-byte chunks when row_len is a multiple of 8 and k is 16-byte aligned (VEC),
// else element by element.
template <bool VEC>
__device__ __forceinline__ void token_sums(const uint16_t* a, const uint16_t* b, int32_t row_len, int lane, float& dd,
                                           float& nn) {
  dd = 0.0f;
  nn = 0.0f;
  if constexpr (VEC) {
#pragma unroll 4
    for (int e = lane * 8; e < row_len; e += 256) {
      const uint4 va = ld_nc_v4(a + e), vb = ld_nc_v4(b + e);
      const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x0 = bf16lo(wa[j]), x1 = bf16hi(wa[j]), y0 = bf16lo(wb[j]), y1 = bf16hi(wb[j]);
        dd = fmaf(x0 - y0, x0 - y0, fmaf(x1 - y1, x1 - y1, dd));
        nn = fmaf(x0, x0, fmaf(y0, y0, fmaf(x1, x1, fmaf(y1, y1, nn))));
      }
    }
  } else {
    for (int e = lane; e < row_len; e += 32) {
      const float x = bf16_to_f32(a[e]), y = bf16_to_f32(b[e]);
      dd = fmaf(x - y, x - y, dd);
      nn = fmaf(x, x, fmaf(y, y, nn));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    dd += __shfl_xor_sync(0xFFFFFFFFu, dd, off);
    nn += __shfl_xor_sync(0xFFFFFFFFu, nn, off);
  }
}

constexpr int kRawWarps = 8;

template <bool VEC>
__global__ void __launch_bounds__(kRawWarps * 32) page_raw_kernel(const float* __restrict__ sal,
                                                                  const uint16_t* __restrict__ k, int32_t row_len,
                                                                  int64_t n_k, int32_t tokens_per_page,
                                                                  int64_t n_pages, float* __restrict__ s_raw,
                                                                  float* __restrict__ novelty) {
  __shared__ float s_nov[kRawWarps], s_mass[kRawWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t pg = blockIdx.x; pg < n_pages; pg += gridDim.x) {
    const int64_t t0 = pg * tokens_per_page;
    const int64_t t1 = min(t0 + tokens_per_page, n_k);
    float nov = 0.0f, mass = 0.0f;
    for (int64_t t = t0 + warp; t < t1; t += kRawWarps) {
      if (sal) mass += sal[t];
      if (t == 0) continue;
      float dd, nn;
      token_sums<VEC>(k + t * row_len, k + (t - 1) * row_len, row_len, lane, dd, nn);
      nov += nn > 0.0f ? 0.5f * dd / nn : 0.0f;
    }
    if (lane == 0) {
      s_nov[warp] = nov;
      s_mass[warp] = mass;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float n_sum = 0.0f, m_sum = 0.0f;
      for (int w = 0; w < kRawWarps; ++w) {
        n_sum += s_nov[w];
        m_sum += s_mass[w];
      }
      if (s_raw) s_raw[pg] = m_sum;
      novelty[pg] = n_sum / float(t1 - t0);
    }
    __syncthreads();  // s_nov / s_mass are rewritten for the next page
  }
}

// One CTA: S[p] = s_raw[p] / max_p s_raw[p] (0 when every page has zero mass).
__global__ void __launch_bounds__(1024) page_normalise_kernel(const float* __restrict__ s_raw, int64_t n_pages,
                                                              float* __restrict__ s_out) {
  __shared__ float s_max[32];
  float m = 0.0f;
  for (int64_t i = threadIdx.x; i < n_pages; i += blockDim.x) m = fmaxf(m, s_raw[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = m;
  __syncthreads();
  m = 0.0f;
  for (int w = 0; w < int(blockDim.x / 32); ++w) m = fmaxf(m, s_max[w]);
  const float inv = m > 0.0f ? 1.0f / m : 0.0f;
  for (int64_t i = threadIdx.x; i < n_pages; i += blockDim.x) s_out[i] = s_raw[i] * inv;
}

// [n, heads, head_dim] bf16 as a 3-D tensor map; box = 64 elements x 1 head x 128 tokens, 128-byte swizzle.
bool make_qk_tmap(CUtensorMap* map, const void* ptr, int64_t n, int32_t heads, int32_t head_dim) {
  auto fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
  if (!fn || !aligned(ptr, 16) || n <= 0 || n > 0x7FFFFFFFLL) return false;
  cuuint64_t dims[3] = {cuuint64_t(head_dim), cuuint64_t(heads), cuuint64_t(n)};
  cuuint64_t strides[2] = {cuuint64_t(head_dim) * 2, cuuint64_t(heads) * head_dim * 2};
  cuuint32_t box[3] = {64, 1, uint32_t(kTile)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

unsigned grid_for(int64_t items, int threads) {
  const int64_t need = (items + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count() > 0 ? sm_count() : 148) * 8;
  return unsigned(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace
}  // namespace ashkv

using namespace ashkv;

extern "C" int64_t ashkv_saliency_scratch_floats(int32_t heads_q, int64_t n_q, int64_t n_k) {
  if (heads_q <= 0 || n_q < 0 || n_k < 0) return -1;
  return int64_t(heads_q) * (n_q + n_k);
}

extern "C" ashkv_status_t ashkv_attention_saliency(const void* d_q, const void* d_k, int32_t heads_q, int32_t heads_kv,
                                                   int32_t head_dim, int64_t n_q, int64_t n_k, int64_t q_pos0,
                                                   float scale, float* d_scratch, float* d_token_saliency,
                                                   uint32_t* d_status, void* stream) {
  if (heads_q <= 0 || heads_kv <= 0 || heads_q % heads_kv || (head_dim != 64 && head_dim != 128)) {
    set_message("ashkv_attention_saliency: heads_q must be a multiple of heads_kv and head_dim 64 or 128");
    return ASHKV_BAD_ARGUMENT;
  }
  if (n_q < 0 || n_k < 0 || n_q > (int64_t(1) << 30) || n_k > (int64_t(1) << 30)) return ASHKV_BAD_ARGUMENT;
  if (n_k == 0) return ASHKV_OK;
  if (!d_q || !d_k || !d_scratch || !d_token_saliency || !d_status) return ASHKV_BAD_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  SalParams p;
  p.heads_q = heads_q; p.group = heads_q / heads_kv; p.nch = head_dim / 64;
  p.n_q = n_q; p.n_k = n_k; p.q_pos0 = q_pos0;
  p.c = scale * 1.4426950408889634f;
  p.lse2 = d_scratch;
  p.colsum = d_scratch + int64_t(heads_q) * n_q;
  p.status = d_status;
  if (n_q == 0) {
    if (cudaMemsetAsync(d_token_saliency, 0, size_t(n_k) * sizeof(float), st) != cudaSuccess)
      return check_launch("ashkv_attention_saliency");
    return ASHKV_OK;
  }
  CUtensorMap tq, tk;
  if (!make_qk_tmap(&tq, d_q, n_q, heads_q, head_dim) || !make_qk_tmap(&tk, d_k, n_k, heads_kv, head_dim)) {
    set_message("ashkv_attention_saliency: cannot build the tensor maps (16-byte aligned buffers needed)");
    return ASHKV_BAD_ARGUMENT;
  }
  // Always the head_dim 128 size: one CTA per SM, which holds all 512 TMEM columns.
  const int smem = (1 + kSB) * 2 * kChunkBytes + 1024;
  if (cudaFuncSetAttribute(saliency_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(saliency_cols_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return check_launch("ashkv_attention_saliency smem attribute");
  const dim3 grid_rows{unsigned((n_q + kTile - 1) / kTile), unsigned(heads_q)};
  saliency_rows_kernel<<<grid_rows, kThreadsF, smem, st>>>(tq, tk, p);
  const dim3 grid_cols{unsigned((n_k + kTile - 1) / kTile), unsigned(heads_q)};
  saliency_cols_kernel<<<grid_cols, kThreadsF, smem, st>>>(tq, tk, p);
  head_sum_kernel<<<grid_for(n_k, 256), 256, 0, st>>>(p.colsum, heads_q, n_k, d_token_saliency);
  return check_launch("ashkv_attention_saliency");
}

extern "C" ashkv_status_t ashkv_page_features(const float* d_token_saliency, const void* d_k, int32_t row_len,
                                              int64_t n_k, int32_t tokens_per_page, float* d_s_raw, float* d_S,
                                              float* d_N, void* stream) {
  if (n_k < 0 || row_len <= 0 || tokens_per_page <= 0) return ASHKV_BAD_ARGUMENT;
  if (n_k == 0) return ASHKV_OK;
  if (!d_k || !d_N || (d_token_saliency && (!d_s_raw || !d_S))) return ASHKV_BAD_ARGUMENT;
  cudaStream_t st = as_stream(stream);
  const int64_t n_pages = (n_k + tokens_per_page - 1) / tokens_per_page;
  const auto* kb = static_cast<const uint16_t*>(d_k);
  float* s_raw = d_token_saliency ? d_s_raw : nullptr;
  const unsigned grid = grid_for(n_pages * 256, 256);  // one CTA per page, at most 8 per SM
  if (row_len % 8 == 0 && aligned(d_k, 16))
    page_raw_kernel<true><<<grid, kRawWarps * 32, 0, st>>>(d_token_saliency, kb, row_len, n_k, tokens_per_page,
                                                           n_pages, s_raw, d_N);
  else
    page_raw_kernel<false><<<grid, kRawWarps * 32, 0, st>>>(d_token_saliency, kb, row_len, n_k, tokens_per_page,
                                                            n_pages, s_raw, d_N);
  if (d_token_saliency) page_normalise_kernel<<<1, 1024, 0, st>>>(d_s_raw, n_pages, d_S);
  return check_launch("ashkv_page_features");
}
