// QKV projection GEMM on the 5th-generation tensor cores (tcgen05).
//
// out[M, N] = A[M, K] . W[N, K]^T (+ bias), bf16 operands, fp32 accumulation
// in TMEM, bf16 output.  Replaces the three cuBLAS `F.linear` calls of the
// reference prologue (sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:287-289)
// with one GEMM over the concatenated [3*dim, dim] weight.
//
// CTA tile 128 x 256, K step 64 (one 128-byte swizzle atom), 4-stage TMA ring.
// Warp roles: warp 0 issues TMA loads, warp 1 owns TMEM and issues the MMAs
// from one elected thread (tcgen05.mma M=128 N=256 K=16), warps 2..5 drain the
// accumulator from TMEM (each warp reads the 32 TMEM lanes its warp id allows)
// and write bf16 rows (optionally also each row's sum of squares of its bf16
// outputs per 256-column tile, which the qk-RMSNorm pass consumes).  Tiles are rasterised in groups of 16 M-tiles so the
// CTAs resident at one time share A and W tiles through L2.
#include "common.cuh"
#include "kernels.h"

namespace rola {

namespace gemm {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*barriers*/ + 1024 /*alignment*/;
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;
}  // namespace gemm

__global__ void __launch_bounds__(gemm::THREADS, 1)
    gemm_bf16_tcgen05(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                      const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out, int64_t ldo,
                      float* __restrict__ ssq, int M, int N, int K) {
  using namespace gemm;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + STAGES * STAGE_BYTES;
  // barriers: full[S], empty[S], acc_full, drain
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t acc_full = bar0 + 8u * (2 * STAGES);
  const uint32_t drain = acc_full + 8u;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + STAGES * STAGE_BYTES + 256);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + STAGES * STAGE_BYTES + 264);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = N / BN;
  // grouped rasterisation
  const int bid = blockIdx.x;
  const int per_group = GROUP_M * num_n;
  const int g = bid / per_group, r = bid % per_group;
  const int gm = min(GROUP_M, num_m - g * GROUP_M);
  const int m_tile = g * GROUP_M + r % gm, n_tile = r / gm;
  const int m0 = m_tile * BM, n0 = n_tile * BN;
  const int nk = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait(empty(s), ((kb / STAGES) & 1) ^ 1, abort_flag, kDevTimeoutMma)) break;
        const uint32_t sa = base + s * STAGE_BYTES;
        mbar_expect_tx(full(s), STAGE_BYTES);
        tma_load_2d(sa, &ta, full(s), kb * BK, m0);
        tma_load_2d(sa + A_BYTES, &tb, full(s), kb * BK, n0);
        ++issued;
      }
      // make sure no load is still writing shared memory when the CTA exits
      for (int kb = max(0, issued - STAGES); kb < issued; ++kb)
        mbar_wait(full(kb % STAGES), (kb / STAGES) & 1, abort_flag, kDevTimeoutLoad);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN, false, false);
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait(full(s), (kb / STAGES) & 1, abort_flag, kDevTimeoutLoad)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = base + s * STAGE_BYTES;
        const uint32_t sb = sa + A_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t da = sdesc_sw128(sa + kk * 32, 16, 1024);
          const uint64_t db = sdesc_sw128(sb + kk * 32, 16, 1024);
          mma_bf16_ss(tmem, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(empty(s));
      }
      if (ok) mma_commit(acc_full);
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, kDevTimeoutMma);
    }
  } else {
    // epilogue warps 2..5: TMEM lane quadrant = warp % 4
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag, kDevTimeoutMma));
    tc_fence_after();
    if (ok) {
      const int gm_row = m0 + row;
      float ss = 0.f;  // sum of squares of this row's bf16 outputs in this tile
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
        tmem_ld_wait();
        if (gm_row < M) {
          const int col = n0 + c * 32;
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
      if (ssq && gm_row < M) ssq[(int64_t)gm_row * (N / BN) + n_tile] = ss;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

int launch_gemm_bf16(const CUtensorMap& ta, const CUtensorMap& tb, const __nv_bfloat16* bias, __nv_bfloat16* out,
                     int64_t ldo, float* ssq, int M, int N, int K, cudaStream_t s) {
  using namespace gemm;
  if (N % BN != 0 || K % BK != 0 || M <= 0) return -1;
  cudaFuncSetAttribute(gemm_bf16_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  const int num_m = (M + BM - 1) / BM, num_n = N / BN;
  gemm_bf16_tcgen05<<<num_m * num_n, THREADS, SMEM_BYTES, s>>>(ta, tb, bias, out, ldo, ssq, M, N, K);
  return (int)cudaGetLastError();
}

}  // namespace rola
