// Block-sparse online-softmax attention on tcgen05, fused with the low-rank
// correction and the gate (one epilogue).
//
// Restates `_rola_fwd_kernel` (sparkdiffusion/ops/fused_kernel/
// fused_sparse_attn.py:55-144): for query block m of head (b, h) iterate the
// selected key blocks j of the LUT, s = (q.k) * D^-1/2 * log2(e) in fp32,
// columns past L masked to -inf for a partial block, base-2 online softmax,
// P rounded to bf16 before P.V, o = acc / l.  The epilogue then restates
// o_lr = q_lr . C (fused_lowrank.py:360-362) and `_gate_fusion_kernel`
// (fused_gate.py:67-127), storing the gated output [B, L, H*D] directly.
//
// One CTA per (query block, batch*head), 6 warps:
//   warp 0      TMA producer: Q once, then K_j and V_j (two 64-column boxes
//               each) into a 2-stage ring, gathered by LUT block index; the
//               low-rank operands q_lr and C^T for the epilogue.
//   warp 1      TMEM owner and MMA issuer (one elected thread):
//               S_i = Q K_i^T into one of two TMEM S buffers, O += P_i V_i.
//   warps 2..5  softmax: thread = query row = TMEM lane; reads S from TMEM,
//               keeps the running max/sum, writes P (bf16, 128B-swizzled) to
//               shared memory, rescales O in TMEM when the running max grows
//               by more than `rescale_threshold` (log2 units; 0 = every growth,
//               exactly the reference's recurrence; larger values keep a stale
//               max, which leaves acc / l unchanged but moves the bf16
//               rounding of P), and finally runs the epilogue.
// TMEM columns: S0 [0,128), S1 [128,256), O [256,384); o_lr reuses S0.
#include "common.cuh"
#include "kernels.h"

namespace rola {

namespace attn {
constexpr int THREADS = 192;
constexpr int TILE = 16384;  // one [128 rows x 64 bf16] box, 128B swizzle
constexpr int OFF_Q = 0;
constexpr int OFF_K = 2 * TILE;        // 2 stages x 2 boxes
constexpr int OFF_V = OFF_K + 4 * TILE;
constexpr int OFF_P = OFF_V + 4 * TILE;
constexpr int OFF_E = OFF_P + 2 * TILE;  // q_lr box, C^T box
constexpr int OFF_BAR = OFF_E + 2 * TILE;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
}  // namespace attn

// barrier slots
enum : int {
  B_Q = 0, B_KF0, B_KF1, B_VF0, B_VF1, B_KVE0, B_KVE1, B_SF0, B_SF1, B_SFREE0, B_SFREE1,
  B_PF, B_OF, B_EPI, B_LR, B_DRAIN, B_COUNT
};

__device__ __forceinline__ int lut_block(const AttnParams& p, const int32_t* lut_row, int i) {
  int j = lut_row[i];
  if (j < 0 || j >= p.NBk) {
    set_device_error(kDevBadIndex);
    j = j < 0 ? 0 : p.NBk - 1;
  }
  return j;
}

__global__ void __launch_bounds__(attn::THREADS, 1)
    sparse_attn_tcgen05(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tqlr,
                        const __grid_constant__ CUtensorMap tct, const AttnParams p) {
  using namespace attn;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + OFF_BAR;
  auto bar = [&](int i) { return bars + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * B_COUNT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int topk = p.topk;
  const int32_t* lut_row = p.lut + ((int64_t)bh * p.NBq + m) * topk;

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    mbar_init(bar(B_KF0), 1);
    mbar_init(bar(B_KF1), 1);
    mbar_init(bar(B_VF0), 1);
    mbar_init(bar(B_VF1), 1);
    mbar_init(bar(B_KVE0), 1);
    mbar_init(bar(B_KVE1), 1);
    mbar_init(bar(B_SF0), 1);
    mbar_init(bar(B_SF1), 1);
    mbar_init(bar(B_SFREE0), 4);
    mbar_init(bar(B_SFREE1), 4);
    mbar_init(bar(B_PF), 4);
    mbar_init(bar(B_OF), 1);
    mbar_init(bar(B_EPI), 1);
    mbar_init(bar(B_LR), 1);
    mbar_init(bar(B_DRAIN), 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    if (p.has_lowrank) {
      prefetch_tmap(&tqlr);
      prefetch_tmap(&tct);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA
    if (elect_one()) {
      mbar_expect_tx(bar(B_Q), 2 * TILE);
      tma_load_4d(base + OFF_Q, &tq, bar(B_Q), 0, m * 128, h, b);
      tma_load_4d(base + OFF_Q + TILE, &tq, bar(B_Q), 64, m * 128, h, b);
      if (p.has_lowrank) {
        mbar_expect_tx(bar(B_EPI), 2 * TILE);
        tma_load_4d(base + OFF_E, &tqlr, bar(B_EPI), 0, m * 128, h, b);
        tma_load_3d(base + OFF_E + TILE, &tct, bar(B_EPI), 0, 0, bh);
      }
      int issued = 0;
      for (int i = 0; i < topk; ++i) {
        const int s = i & 1;
        if (!mbar_wait(bar(B_KVE0 + s), ((i >> 1) & 1) ^ 1, abort_flag, kDevTimeoutMma)) break;
        const int j = lut_block(p, lut_row, i);
        const uint32_t sk = base + OFF_K + s * 2 * TILE;
        const uint32_t sv = base + OFF_V + s * 2 * TILE;
        mbar_expect_tx(bar(B_KF0 + s), 2 * TILE);
        tma_load_4d(sk, &tk, bar(B_KF0 + s), 0, j * 128, h, b);
        tma_load_4d(sk + TILE, &tk, bar(B_KF0 + s), 64, j * 128, h, b);
        mbar_expect_tx(bar(B_VF0 + s), 2 * TILE);
        tma_load_4d(sv, &tv, bar(B_VF0 + s), 0, j * 128, h, b);
        tma_load_4d(sv + TILE, &tv, bar(B_VF0 + s), 64, j * 128, h, b);
        ++issued;
      }
      // drain: no TMA may still target shared memory when the CTA exits
      mbar_wait(bar(B_Q), 0, abort_flag, kDevTimeoutLoad);
      if (p.has_lowrank) mbar_wait(bar(B_EPI), 0, abort_flag, kDevTimeoutLoad);
      for (int i = max(0, issued - 2); i < issued; ++i) {
        mbar_wait(bar(B_KF0 + (i & 1)), (i >> 1) & 1, abort_flag, kDevTimeoutLoad);
        mbar_wait(bar(B_VF0 + (i & 1)), (i >> 1) & 1, abort_flag, kDevTimeoutLoad);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16_f32(128, 128, false, false);
      const uint32_t id_pv = idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_wait(bar(B_Q), 0, abort_flag, kDevTimeoutLoad);
      auto issue_pv = [&](int i) -> bool {
        const int s = i & 1;
        if (!mbar_wait(bar(B_PF), i & 1, abort_flag, kDevTimeoutSoftmax)) return false;
        if (!mbar_wait(bar(B_VF0 + s), (i >> 1) & 1, abort_flag, kDevTimeoutLoad)) return false;
        tc_fence_after();
        const uint32_t sv = base + OFF_V + s * 2 * TILE;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t da = sdesc_sw128(base + OFF_P + (kk >> 2) * TILE + (kk & 3) * 32, 16, 1024);
          const uint64_t db = sdesc_sw128(sv + kk * 2048, TILE, 1024);
          mma_bf16_ss(tO, da, db, id_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar(B_KVE0 + s));
        mma_commit(bar(B_OF));
        return true;
      };
      for (int i = 0; i < topk && ok; ++i) {
        const int s = i & 1;
        ok = mbar_wait(bar(B_KF0 + s), (i >> 1) & 1, abort_flag, kDevTimeoutLoad) &&
             mbar_wait(bar(B_SFREE0 + s), ((i >> 1) & 1) ^ 1, abort_flag, kDevTimeoutSoftmax);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sk = base + OFF_K + s * 2 * TILE;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * TILE + (kk & 3) * 32;
          mma_bf16_ss(tS[s], sdesc_sw128(base + OFF_Q + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), id_qk,
                      kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(B_SF0 + s));
        if (i >= 1) ok = issue_pv(i - 1);
      }
      if (ok) ok = issue_pv(topk - 1);
      if (ok && p.has_lowrank) {
        // o_lr = q_lr . C into S0 once the softmax released the last S0 use
        const int last0 = ((topk - 1) & 1) == 0 ? topk - 1 : topk - 2;
        ok = mbar_wait(bar(B_EPI), 0, abort_flag, kDevTimeoutLoad) &&
             mbar_wait(bar(B_SFREE0), (last0 >> 1) & 1, abort_flag, kDevTimeoutSoftmax);
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_bf16_ss(tS[0], sdesc_sw128(base + OFF_E + kk * 32, 16, 1024),
                        sdesc_sw128(base + OFF_E + TILE + kk * 32, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(B_LR));
        }
      }
      mma_commit(bar(B_DRAIN));
      mbar_wait(bar(B_DRAIN), 0, abort_flag, kDevTimeoutMma);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float scale = p.qk_scale;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint8_t* sP = gbase + OFF_P;
    for (int i = 0; i < topk; ++i) {
      const int s = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_SF0 + s), (i >> 1) & 1, abort_flag, kDevTimeoutMma))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS[s] + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_SFREE0 + s));

      const int j = lut_block(p, lut_row, i);
      const int valid = p.L - j * 128;
      float mx = -INFINITY;
      if (valid < 128) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          if (c >= valid) sv[c] = __float_as_uint(-INFINITY);
        }
      }
#pragma unroll
      for (int c = 0; c < 128; ++c) mx = fmaxf(mx, __uint_as_float(sv[c]));
      const float m_new = fmaxf(m_run, mx * scale);
      float m_use = m_run, alpha = 1.f;
      bool rescale = false;
      if (i == 0) {
        m_use = m_new;
      } else if (m_new - m_run > p.rescale_threshold) {
        m_use = m_new;
        alpha = ex2_approx(m_run - m_new);
        rescale = true;
      }
      float rs = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(sv[2 * c]), scale, -m_use));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sv[2 * c + 1]), scale, -m_use));
        rs += p0 + p1;
        pk[c] = pack_bf2(p0, p1);
      }
      l_run = l_run * alpha + rs;
      m_run = m_use;

      if (i >= 1) {
        // P buffer and O are in use by P_{i-1} V_{i-1} until it completes
        if (!__all_sync(0xffffffffu, mbar_wait(bar(B_OF), (i - 1) & 1, abort_flag, kDevTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t ov[32];
            tmem_ld32(tO + lane_off + c * 32, ov);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st32(tO + lane_off + c * 32, ov);
          }
          tmem_st_wait();
        }
      }
      // P row -> shared memory, 128B-swizzled K-major layout (two 64-column boxes)
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {
        const int box = c16 >> 3, chunk = c16 & 7;
        uint4 u = make_uint4(pk[4 * c16], pk[4 * c16 + 1], pk[4 * c16 + 2], pk[4 * c16 + 3]);
        *reinterpret_cast<uint4*>(sP + box * TILE + row * 128 + ((chunk ^ (row & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PF));
    }

    // ------------------------------------------------------------ epilogue
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_OF), (topk - 1) & 1, abort_flag, kDevTimeoutMma));
    tc_fence_after();
    bool lowrank = false;
    if (ok && p.has_lowrank)
      lowrank = __all_sync(0xffffffffu, mbar_wait(bar(B_LR), 0, abort_flag, kDevTimeoutMma));
    ok = ok && (lowrank || !p.has_lowrank);
    if (ok) {
      tc_fence_after();
      const int t = m * 128 + row;
      const float inv_l = 1.0f / l_run;
      // pass 1: row statistics of o_sparse (bf16 chain) and of o_lr
      float ss_os = 0.f, ss_lr = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
        tmem_ld32(tO + lane_off + c * 32, ov);
        uint32_t lv[32];
        if (lowrank) tmem_ld32(tS[0] + lane_off + c * 32, lv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float os = rbf(__uint_as_float(ov[e]) * inv_l);
          ss_os += rbf(os * os);
          if (lowrank) {
            const float lr = rbf(__uint_as_float(lv[e]));
            ss_lr = fmaf(lr, lr, ss_lr);
          }
        }
      }
      float os_rms = 1.f, lr_scale = 0.f, gate = 0.f;
      if (lowrank) {
        const float os_mean = rbf(ss_os * (1.0f / 128.0f));
        const float os_mean_eps = rbf(os_mean + 1e-5f);
        os_rms = rbf(sqrtf(os_mean_eps));
        lr_scale = rsqrtf(ss_lr * (1.0f / 128.0f) + p.eps_lr);
        gate = (p.gate != nullptr && t < p.L) ? bf2f(p.gate[((int64_t)b * p.L + t) * p.H + h]) : 0.f;
      }
      // pass 2: fuse and store (TMEM loads by the whole warp, stores only for rows < L)
      const bool store = t < p.L;
      {
        const int64_t orow = (int64_t)b * p.o_sB + (int64_t)h * p.o_sH + (int64_t)t * p.o_sT;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(tO + lane_off + c * 32, ov);
          uint32_t lv[32];
          if (lowrank) tmem_ld32(tS[0] + lane_off + c * 32, lv);
          tmem_ld_wait();
          float os[32], fo[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            os[e] = rbf(__uint_as_float(ov[e]) * inv_l);
            if (lowrank) {
              const float lrn = rbf(rbf(__uint_as_float(lv[e])) * lr_scale);
              fo[e] = (os[e] / os_rms + gate * lrn) * os_rms;
            } else {
              fo[e] = os[e];
            }
          }
          if (p.out && store) {
            uint4* dst = reinterpret_cast<uint4*>(p.out + orow + c * 32);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              dst[v4] = make_uint4(pack_bf2(fo[8 * v4], fo[8 * v4 + 1]), pack_bf2(fo[8 * v4 + 2], fo[8 * v4 + 3]),
                                   pack_bf2(fo[8 * v4 + 4], fo[8 * v4 + 5]), pack_bf2(fo[8 * v4 + 6], fo[8 * v4 + 7]));
          }
          if (p.o_sparse && store) {
            uint4* dst = reinterpret_cast<uint4*>(p.o_sparse + orow + c * 32);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              dst[v4] = make_uint4(pack_bf2(os[8 * v4], os[8 * v4 + 1]), pack_bf2(os[8 * v4 + 2], os[8 * v4 + 3]),
                                   pack_bf2(os[8 * v4 + 4], os[8 * v4 + 5]), pack_bf2(os[8 * v4 + 6], os[8 * v4 + 7]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch_sparse_attn(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tqlr,
                       const CUtensorMap& tct, const AttnParams& p, cudaStream_t s) {
  using namespace attn;
  cudaFuncSetAttribute(sparse_attn_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  dim3 grid(p.NBq, p.B * p.H);
  sparse_attn_tcgen05<<<grid, THREADS, SMEM_BYTES, s>>>(tq, tk, tv, tqlr, tct, p);
  return (int)cudaGetLastError();
}

}  // namespace rola
