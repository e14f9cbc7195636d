// QKV projection GEMM on the 5th-generation tensor cores (tcgen05).
//
// out[M, N] = A[M, K] . W[N, K]^T (+ bias), bf16 operands, fp32 accumulation
// in TMEM, bf16 output.  Replaces the three cuBLAS `F.linear` calls of the
// reference prologue (sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:287-289)
// with one GEMM over the concatenated [3*dim, dim] weight.
//
// FP8 variant (kFp8): e4m3 operands with one fp32 scale per row of A (token)
// and per row of W (output channel), the reference's row-wise FP8 prologue
// (`torch._scaled_mm(x_fp8, w_fp8.t(), scale_a, scale_b, bias, out_dtype=bf16)`,
// fused_qkv_rope.py:270-285 with the recipe of ops/quantization/fp8_linear.py:45-61):
// the accumulator times scale_a[m] times scale_b[n], plus the bias, rounded to
// bf16.  The shared-memory tiles, the TMA boxes and the descriptors are the
// same bytes as in bf16 (128-byte rows: 128 e4m3 or 64 bf16 values; every MMA
// consumes 32 bytes of each row: K = 32 e4m3 or 16 bf16).
//
// Persistent kernel: one CTA per SM walks the 128 x 256 output tiles
// (tile = blockIdx.x + i * gridDim.x, rasterised in groups of 16 M-tiles so
// the tiles in flight at one time share A and W through L2).  K step 64 (one
// 128-byte swizzle atom), 4-stage TMA ring that runs across tile boundaries.
// Warp roles: warp 0 issues TMA loads, warp 1 owns TMEM and issues the MMAs
// from one elected thread (tcgen05.mma M=128 N=256 K=16) into one of two
// 256-column accumulators, warps 2..5 drain the other accumulator (each warp
// reads the 32 TMEM lanes its warp id allows) and write bf16 rows, optionally
// with each row's sum of squares of its bf16 outputs per 256-column tile (the
// qk-RMSNorm statistics).  The epilogue of tile i thus overlaps the MMAs of
// tile i+1.
//
// Optional side job (warps 6..9): work items of the streaming norm pass of an
// EARLIER chunk of rows (norm_block), e.g. the Ulysses scatter of chunk c-1
// while the tensor cores project chunk c; the side job shares nothing with the
// GEMM but the SM.
#include "common.cuh"
#include "kernels.h"

namespace rola {

namespace gemm {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int OFF_BAR = STAGES * STAGE_BYTES;
constexpr int OFF_NORM = OFF_BAR + 1024;  // side-job shared memory
constexpr int SMEM_BYTES = OFF_NORM + 1024 /*alignment*/;
constexpr int THREADS = 192;
constexpr int THREADS_SIDE = THREADS + kNormThreads;
constexpr int GROUP_M = 16;
constexpr int ACC_COLS = 2 * BN;  // two accumulators
}  // namespace gemm

template <bool kFp8>
__global__ void __launch_bounds__(gemm::THREADS_SIDE, 1)
    gemm_tcgen05(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                 const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out, int64_t ldo,
                 float* __restrict__ ssq, int M, int N, int K, const __grid_constant__ NormRopeParams side,
                 int side_items, const float* __restrict__ scale_a, const float* __restrict__ scale_b) {
  using namespace gemm;
  constexpr int BKE = kFp8 ? 2 * BK : BK;  // K elements per 128-byte stage row
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + OFF_BAR;
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2], drain
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto acc_full = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto acc_empty = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain = bar0 + 8u * (2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 256);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 264);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int nk = K / BKE;
  // my tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_tiles = blockIdx.x < num_tiles ? (num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  auto tile_coords = [&](int lt, int& m0, int& n_tile) {
    const int tile = blockIdx.x + lt * gridDim.x;
    const int per_group = GROUP_M * num_n;
    const int g = tile / per_group, r = tile % per_group;
    const int gm = min(GROUP_M, num_m - g * GROUP_M);
    m0 = (g * GROUP_M + r % gm) * BM;
    n_tile = r / gm;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(acc_full(a), 1);
      mbar_init(acc_empty(a), 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), ACC_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        int m0, n_tile;
        tile_coords(lt, m0, n_tile);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(empty(s), ((it / STAGES) & 1) ^ 1, abort_flag, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + s * STAGE_BYTES;
          mbar_expect_tx(full(s), STAGE_BYTES);
          tma_load_2d(sa, &ta, full(s), kb * BKE, m0);
          tma_load_2d(sa + A_BYTES, &tb, full(s), kb * BKE, n_tile * BN);
        }
      }
      // make sure no load is still writing shared memory when the CTA exits
      for (int k = max(0, it - STAGES); k < it; ++k)
        mbar_wait(full(k % STAGES), (k / STAGES) & 1, abort_flag, kDevTimeoutLoad);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = kFp8 ? idesc_e4m3_f32(BM, BN) : idesc_bf16_f32(BM, BN, false, false);
      bool ok = true;
      int it = 0;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int a = lt & 1;
        // the epilogue has drained this accumulator (tile lt - 2)
        if (!mbar_wait(acc_empty(a), ((lt >> 1) & 1) ^ 1, abort_flag, kDevTimeoutSoftmax)) break;
        tc_fence_after();
        const uint32_t acc = tmem + a * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(full(s), (it / STAGES) & 1, abort_flag, kDevTimeoutLoad)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + s * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = sdesc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t db = sdesc_sw128(sb + kk * 32, 16, 1024);
            if constexpr (kFp8) {
              mma_f8_ss(acc, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            } else {
              mma_bf16_ss(acc, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(empty(s));
        }
        if (ok) mma_commit(acc_full(a));
      }
      // every MMA issued has completed before TMEM is freed, also on the abort
      // path (where mbar_wait would return at once): bounded, ignores the flag
      mma_commit(drain);
      mbar_wait_until(drain, 0, globaltimer_ns() + kWaitLimitNs);
    }
  } else if (warp < 6) {
    // epilogue warps 2..5: TMEM lane quadrant = warp % 4
    const int q = warp & 3;
    const int row = q * 32 + lane;
    for (int lt = 0; lt < my_tiles; ++lt) {
      const int a = lt & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full(a), (lt >> 1) & 1, abort_flag, kDevTimeoutMma));
      if (!ok) break;
      tc_fence_after();
      int m0, n_tile;
      tile_coords(lt, m0, n_tile);
      const int gm_row = m0 + row;
      const uint32_t acc = tmem + a * BN + ((uint32_t)(q * 32) << 16);
      float ss = 0.f;  // sum of squares of this row's bf16 outputs in this tile
      float row_scale = 1.f;
      if (kFp8 && gm_row < M) row_scale = scale_a[gm_row];
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(acc + c * 32, v);
        tmem_ld_wait();
        if (gm_row < M) {
          const int col = n_tile * BN + c * 32;
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
          if (kFp8) {
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] = (f[i] * row_scale) * __ldg(scale_b + col + i);
          }
          if (bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] += bf2f(bias[col + i]);
          }
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)gm_row * ldo + col);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 u;
            u.x = pack_bf2(f[8 * i + 0], f[8 * i + 1]);
            u.y = pack_bf2(f[8 * i + 2], f[8 * i + 3]);
            u.z = pack_bf2(f[8 * i + 4], f[8 * i + 5]);
            u.w = pack_bf2(f[8 * i + 6], f[8 * i + 7]);
            dst[i] = u;
          }
          if (ssq) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float r = rbf(f[i]);
              ss = fmaf(r, r, ss);
            }
          }
        }
      }
      // the accumulator may be overwritten once every warp's loads completed
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(a));
      if (ssq && gm_row < M) ssq[(int64_t)gm_row * (N / BN) + n_tile] = ss;
    }
  } else {
    // side job, warps 6..9 (only launched with side_items > 0)
    uint8_t* nsm = gbase + OFF_NORM;
    const int ngrp = (side.H + kNormHeads - 1) / kNormHeads;
    for (int item = blockIdx.x; item < side_items; item += gridDim.x)
      norm_block<true, false, false, kNormRingCompact>(side, item / ngrp, item % ngrp, 0, nsm,
                                                        threadIdx.x - THREADS, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, ACC_COLS);
  }
}

static int g_num_sms = 0;

int launch_gemm_bf16(const CUtensorMap& ta, const CUtensorMap& tb, const __nv_bfloat16* bias, __nv_bfloat16* out,
                     int64_t ldo, float* ssq, int M, int N, int K, const NormRopeParams* side, cudaStream_t s,
                     const float* scale_a, const float* scale_b) {
  using namespace gemm;
  const bool fp8 = scale_a != nullptr;
  if (N % BN != 0 || K % (fp8 ? 2 * BK : BK) != 0 || M <= 0 || fp8 != (scale_b != nullptr)) return -1;
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) return (int)cudaGetLastError();
  }
  int side_items = 0, smem = SMEM_BYTES;
  NormRopeParams sp{};
  if (side) {
    // norm-only pass of B = 1 rows with the compact ring, items = blocks x head groups
    if (side->B != 1 || side->ssq == nullptr || !side->compact) return -1;
    sp = *side;
    side_items = sp.NB * ((sp.H + kNormHeads - 1) / kNormHeads);
    const int nslots = 2 + (sp.v_dst[0] != nullptr) + (sp.x != nullptr && sp.g_dst[0] != nullptr);
    smem += norm_smem_bytes(kNormRingCompact, nslots, sp.blk, true);
    if (smem > 227 * 1024) return -1;
  }
  const int num_tiles = ((M + BM - 1) / BM) * (N / BN);
  const int grid = num_tiles < g_num_sms ? num_tiles : g_num_sms;
  const int threads = side_items ? THREADS_SIDE : THREADS;
  if (fp8) {
    cudaFuncSetAttribute(gemm_tcgen05<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    gemm_tcgen05<true><<<grid, threads, smem, s>>>(ta, tb, bias, out, ldo, ssq, M, N, K, sp, side_items, scale_a,
                                                   scale_b);
  } else {
    cudaFuncSetAttribute(gemm_tcgen05<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    gemm_tcgen05<false><<<grid, threads, smem, s>>>(ta, tb, bias, out, ldo, ssq, M, N, K, sp, side_items, nullptr,
                                                    nullptr);
  }
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Two-SM variant (bf16, no side job): a cluster of two CTAs computes a 256 x 256
// output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16).  Each
// CTA stages its own 128 rows of A and its half (128 rows) of the W tile, so
// every SM pulls 32 KB instead of 48 KB from L2 per K step of 64; the freed
// shared memory holds a 6-stage ring.  The even CTA of the pair (the leader)
// issues the MMAs, which read both CTAs' shared memory and write each CTA's
// 128 accumulator rows into its own tensor memory; both CTAs' loads complete
// on the leader's stage barriers (the leader arms them for both), the MMA
// completions are signalled to both CTAs' barriers, and both CTAs' epilogue
// warps release an accumulator on the leader's barrier.  Loads carry no
// multicast.  Same per-element arithmetic as the single-SM kernel: the K steps
// accumulate in the same order into fp32.
// ---------------------------------------------------------------------------
namespace gemm2 {
constexpr int BM = 128;                      // rows of A per CTA (256 per pair)
constexpr int BN = 256;                      // output columns per pair
constexpr int BK = 64, STAGES = 6;
constexpr int A_BYTES = BM * BK * 2;         // 16 KB
constexpr int B_BYTES = (BN / 2) * BK * 2;   // 16 KB: this CTA's half of the W tile
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int OFF_BAR = STAGES * STAGE_BYTES;  // 192 KB
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024 /*alignment*/;
constexpr int THREADS = 192;
constexpr int GROUP_M = 8;                   // 256-row M tiles per raster group
constexpr int ACC_COLS = 2 * BN;             // two accumulators
}  // namespace gemm2

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the shared::cluster address of the variable at shared::cta address `a` in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory, completing on an mbarrier of either CTA of the pair
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.cta_group::2 [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at shared::cta offset `bar` in both CTAs of the pair once
// every tcgen05 op issued so far by this thread completes
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
// arrive on the issuing CTA's own barrier
__device__ __forceinline__ void mma_commit_pair_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm2::THREADS, 1)
    gemm2sm_tcgen05(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                    const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out, int64_t ldo,
                    float* __restrict__ ssq, int M, int N, int K) {
  using namespace gemm2;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + OFF_BAR;
  // barriers: full[S] (leader), empty[S], acc_full[2], acc_empty[2] (leader), drain (leader)
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto acc_full = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto acc_empty = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain = bar0 + 8u * (2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * (2 * STAGES + 5));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 8 * (2 * STAGES + 5) + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int num_m = (M + 2 * BM - 1) / (2 * BM), num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int nk = K / BK;
  const int my_tiles = cluster < num_tiles ? (num_tiles - 1 - cluster) / nclusters + 1 : 0;
  auto tile_coords = [&](int lt, int& m0, int& n_tile) {  // m0: first of the pair's 256 rows
    const int tile = cluster + lt * nclusters;
    const int per_group = GROUP_M * num_n;
    const int g = tile / per_group, r = tile % per_group;
    const int gm = min(GROUP_M, num_m - g * GROUP_M);
    m0 = (g * GROUP_M + r % gm) * 2 * BM;
    n_tile = r / gm;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(acc_full(a), 1);
      mbar_init(acc_empty(a), 8);  // the epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
  }
  if (warp == 1) {  // one warp of each CTA allocates the pair's tensor memory
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)ACC_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      // ----------------------------------------------------------------- TMA
      int it = 0;
      bool ok = true;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        int m0, n_tile;
        tile_coords(lt, m0, n_tile);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(empty(s), ((it / STAGES) & 1) ^ 1, abort_flag, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + s * STAGE_BYTES;
          const uint32_t fb = mapa_shared(full(s), 0);
          if (rank == 0) mbar_expect_tx(full(s), 2 * STAGE_BYTES);  // both CTAs' bytes
          tma_load_2d_pair(sa, &ta, fb, kb * BK, m0 + (int)rank * BM);
          tma_load_2d_pair(sa + A_BYTES, &tb, fb, kb * BK, n_tile * BN + (int)rank * (BN / 2));
        }
      }
      // the leader sees every load of both CTAs complete on its barriers: no
      // copy is still writing shared memory when the pair passes the final
      // cluster barrier (the waits ignore the abort flag and share one limit)
      if (rank == 0) {
        const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
        bool drained = true;
        for (int k = max(0, it - STAGES); k < it && drained; ++k)
          drained = mbar_wait_until(full(k % STAGES), (k / STAGES) & 1, deadline);
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && elect_one()) {
      // ----------------------------------------------------------------- MMA
      const uint32_t idesc = idesc_bf16_f32(2 * BM, BN, false, false);
      bool ok = true;
      int it = 0;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int a = lt & 1;
        // both CTAs' epilogues have drained this accumulator (tile lt - 2)
        if (!mbar_wait(acc_empty(a), ((lt >> 1) & 1) ^ 1, abort_flag, kDevTimeoutSoftmax)) break;
        tc_fence_after();
        const uint32_t acc = tmem + a * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(full(s), (it / STAGES) & 1, abort_flag, kDevTimeoutLoad)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + s * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_bf16_ss_pair(acc, sdesc_sw128(sa + kk * 32, 16, 1024), sdesc_sw128(sb + kk * 32, 16, 1024), idesc,
                             (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit_pair(empty(s));
        }
        if (ok) mma_commit_pair(acc_full(a));
      }
      // every MMA of the pair has completed before either CTA frees its TMEM
      // (the cluster barrier below), also on the abort path
      mma_commit_pair_local(drain);
      mbar_wait_until(drain, 0, globaltimer_ns() + kWaitLimitNs);
    }
  } else {
    // ------------------------------------------------- epilogue warps 2..5
    const int q = warp & 3;
    const int row = q * 32 + lane;
    for (int lt = 0; lt < my_tiles; ++lt) {
      const int a = lt & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full(a), (lt >> 1) & 1, abort_flag, kDevTimeoutMma));
      if (!ok) break;
      tc_fence_after();
      int m0, n_tile;
      tile_coords(lt, m0, n_tile);
      const int gm_row = m0 + (int)rank * BM + row;
      const uint32_t acc = tmem + a * BN + ((uint32_t)(q * 32) << 16);
      float ss = 0.f;  // sum of squares of this row's bf16 outputs in this tile
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(acc + c * 32, v);
        tmem_ld_wait();
        if (gm_row < M) {
          const int col = n_tile * BN + c * 32;
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
          if (bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] += bf2f(bias[col + i]);
          }
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)gm_row * ldo + col);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 u;
            u.x = pack_bf2(f[8 * i + 0], f[8 * i + 1]);
            u.y = pack_bf2(f[8 * i + 2], f[8 * i + 3]);
            u.z = pack_bf2(f[8 * i + 4], f[8 * i + 5]);
            u.w = pack_bf2(f[8 * i + 6], f[8 * i + 7]);
            dst[i] = u;
          }
          if (ssq) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float r = rbf(f[i]);
              ss = fmaf(r, r, ss);
            }
          }
        }
      }
      // the accumulator may be overwritten once every warp of both CTAs read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) {
          mbar_arrive(acc_empty(a));
        } else {
          mbar_arrive_remote(mapa_shared(acc_empty(a), 0));
        }
      }
      if (ssq && gm_row < M) ssq[(int64_t)gm_row * (N / BN) + n_tile] = ss;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its pair may still use its memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)ACC_COLS)
                 : "memory");
  }
}

int launch_gemm_bf16_2sm(const CUtensorMap& ta, const CUtensorMap& tb_half, const __nv_bfloat16* bias,
                         __nv_bfloat16* out, int64_t ldo, float* ssq, int M, int N, int K, cudaStream_t s) {
  using namespace gemm2;
  if (N % BN != 0 || K % BK != 0 || M <= 0) return -1;
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) return (int)cudaGetLastError();
  }
  const int num_tiles = ((M + 2 * BM - 1) / (2 * BM)) * (N / BN);
  const int clusters = num_tiles < g_num_sms / 2 ? num_tiles : g_num_sms / 2;
  cudaFuncSetAttribute(gemm2sm_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  gemm2sm_tcgen05<<<2 * clusters, THREADS, SMEM_BYTES, s>>>(ta, tb_half, bias, out, ldo, ssq, M, N, K);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Row-wise e4m3 quantization (the FP8 GEMM's operands), restating
// quantize_activation_rowwise / quantize_weight_rowwise
// (sparkdiffusion/ops/quantization/fp8_linear.py:45-61): scale = amax|row| / 448
// + 1e-12 in fp32; q = e4m3(bf16(x / bf16(scale))), the bf16 quotient rounded
// to nearest even as torch divides bf16 tensors, then rounded to nearest even
// e4m3 (|q| <= 448 (1 + 2^-8) here, inside e4m3's range).  One CTA per row.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));  // hi -> upper byte
  return r;
}

__global__ void __launch_bounds__(128) quantize_rows_e4m3_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld,
                                                                 int K, uint8_t* __restrict__ xq,
                                                                 float* __restrict__ scale) {
  __shared__ float s_red[4];
  const int64_t m = blockIdx.x;
  const __nv_bfloat16* row = x + m * ld;
  float amax = 0.f;
  for (int c = threadIdx.x * 8; c < K; c += 128 * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float a, b;
      unpack_bf2(w[e], a, b);
      amax = fmaxf(amax, fmaxf(fabsf(a), fabsf(b)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
  const float sc = __fadd_rn(__fdiv_rn(amax, 448.0f), 1e-12f);
  const float sc_bf = rbf(sc);
  if (threadIdx.x == 0) scale[m] = sc;
  uint8_t* qrow = xq + m * (int64_t)K;
  for (int c = threadIdx.x * 8; c < K; c += 128 * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint16_t q[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float a, b;
      unpack_bf2(w[e], a, b);
      q[e] = cvt_e4m3x2(rbf(__fdiv_rn(a, sc_bf)), rbf(__fdiv_rn(b, sc_bf)));
    }
    *reinterpret_cast<uint2*>(qrow + c) =
        make_uint2((uint32_t)q[0] | ((uint32_t)q[1] << 16), (uint32_t)q[2] | ((uint32_t)q[3] << 16));
  }
}

int launch_quantize_rows_e4m3(const __nv_bfloat16* x, int64_t ld, int M, int K, uint8_t* xq, float* scale,
                              cudaStream_t s) {
  quantize_rows_e4m3_kernel<<<M, 128, 0, s>>>(x, ld, K, xq, scale);
  return (int)cudaGetLastError();
}

}  // namespace rola
