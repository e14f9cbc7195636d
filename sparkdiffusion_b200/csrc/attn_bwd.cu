// Backward of the block-sparse attention on tcgen05 (the training path).
//
// The reference's training forward (sparkdiffusion/networks/wan_rola_attention.py:
// 293-327) runs the block-sparse softmax attention through the external SLA
// package (`_attention.apply(q, k, v, sparse_map, lut, real_topk, BLKQ, BLKK)`,
// :320-321), whose backward gives dq, dk, dv of
//     o_i = sum_{j in sel(i)} softmax_j(q_i . k_j / sqrt(D)) v_j
// where sel(i) are the key blocks the query block of row i selected.  This
// file computes exactly that gradient from the forward's per-row log-sum-exp
// (written by sparse_attn_tcgen05), without atomics:
//
//   delta[r]  = sum_d dO[r, d] O[r, d]                            (delta kernel)
//   P         = exp2(q.k * D^-1/2 log2(e) - lse2[r])   (recomputed, fp32)
//   dP        = dO V^T,  dS = P (dP - delta[r])
//   dQ        = D^-1/2 dS K        query-stationary over the LUT  (dq kernel)
//   dV = P^T dO,  dK = D^-1/2 dS^T Q   key-stationary over the inverse LUT
//                                                                  (dkdv kernel)
// P and dS are rounded to bf16 where they feed an MMA (as the forward rounds
// P before P.V); every accumulation is fp32 in tensor memory.
//
// Both kernels keep a 128-row tile stationary (Q and dO of a query tile, or K
// and V of a key tile) and walk the other side in steps of 64 rows: a
// 128-row block is two steps, a 64-row block (block size 64) one step whose
// selection bits say which 64-row half of the stationary tile selected it.  The S / dP
// accumulators of a step are multi-buffered in tensor memory, and the
// softmax warpgroups take the steps in turn, so the MMA warp computes the
// next steps' S and dP while step i's P and dS are computed, and several
// steps' exp2 work runs at once.
//
// Warp 0 lane 0: TMA producer (no multicast).  Warp 1: tensor memory owner
// and MMA issuer (one elected thread).  The softmax warpgroups (thread = TMEM
// lane = stationary-tile row) take the steps in turn: the dq kernel has three
// (512 threads, three S / dP buffers, so the MMA warp runs two steps ahead),
// the dkdv kernel two buffers (its two 128-column accumulators fill the rest
// of the tensor memory) with both of its warpgroups on every step, 32
// columns each.  The CTA's warpgroups 1 and 2 (the first two softmax
// warpgroups; warps 0-3 are the producer, the MMA issuer and two idle warps)
// then store one 64-column half of the accumulators each.  Every mbarrier wait
// is bounded (error flag + abort, as in the forward); on the abort path the
// producer still drains its loads and the MMA issuer its MMAs (bounded waits
// that ignore the abort flag) before the tensor memory is freed.
#include "common.cuh"
#include "kernels.h"

namespace rola {

namespace bwd {
constexpr int DQ_THREADS = 512;      // dq kernel: three softmax warpgroups
constexpr int DQ_NBUF = 3;           // dq kernel: S / dP buffers in tensor memory (steps in flight)
constexpr int DQ_ACC = 128 * DQ_NBUF;  // dq kernel: TMEM column of the dQ accumulator
constexpr int BOX = 8192;          // [64 rows x 64 bf16] box, 128-byte swizzle
constexpr int HALF = 2 * BOX;      // 64 rows x 128 d: one step's operand
constexpr int TILE = 2 * HALF;     // 128 rows x 128 d: the stationary operands
constexpr int BOX128 = 2 * BOX;    // [128 rows x 64 bf16] (two 64-row boxes stacked)
constexpr int THREADS = 384;      // dkdv kernel: two softmax warpgroups, both on every step
constexpr int KV_STAGES = 4;  // dkdv ring
constexpr int DQ_STAGES = 5;  // dq ring
constexpr int MAX_STAGES = 5;
// dq kernel: Q and dO of the query tile, then the ring of (K, V) 64-row steps
constexpr int DQ_OFF_Q = 0, DQ_OFF_DO = TILE, DQ_OFF_RING = 2 * TILE;
constexpr int DQ_ENTRY = 2 * HALF;
constexpr int DQ_OFF_BAR = DQ_OFF_RING + DQ_STAGES * DQ_ENTRY;  // 224 KB
// dkdv kernel: K and V of the key tile, then the ring of (Q, dO, lse2, delta) 64-row steps
constexpr int KV_OFF_K = 0, KV_OFF_V = TILE, KV_OFF_RING = 2 * TILE;
constexpr int KV_ENTRY = 2 * HALF + 1024;  // + 64 lse2 + 64 delta (fp32), padded to keep 1024-byte alignment
constexpr int KV_OFF_BAR = KV_OFF_RING + KV_STAGES * KV_ENTRY;  // 196 KB
constexpr int BAR_BYTES = 256;
constexpr int DQ_SMEM = DQ_OFF_BAR + BAR_BYTES + 1024;
constexpr int KV_SMEM = KV_OFF_BAR + BAR_BYTES + 1024;
static_assert(KV_ENTRY % 1024 == 0, "ring entries keep the 1024-byte swizzle alignment");
static_assert(KV_SMEM <= 227 * 1024 && DQ_SMEM <= 227 * 1024, "shared memory per CTA");
constexpr float kSmScale = 0.08838834764831845f;  // 128^-1/2
}  // namespace bwd

enum : int {
  G_TILE = 0,                        // stationary tiles loaded
  G_FULL0,                           // ring entry s loaded: G_FULL0 + s
  G_EMPTY0 = G_FULL0 + bwd::MAX_STAGES,  // ring entry s consumed (MMA commit)
  G_SF0 = G_EMPTY0 + bwd::MAX_STAGES,    // S and dP of a step in TMEM buffer b: G_SF0 + b
  G_DS0 = G_SF0 + 3,                     // dS (and P) of a step in TMEM buffer b, 4 warp arrivals: G_DS0 + b
  G_ACC = G_DS0 + 3,                     // accumulators final
  G_COUNT
};
static_assert(8 * G_COUNT + 16 <= bwd::BAR_BYTES, "barrier region too small");
static_assert(bwd::DQ_NBUF <= 3, "barrier slots for three buffers");

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// block index of a LUT / inverse-table entry (selection bits and the -1
// padding of a paired table stripped; error flag on an index outside [0, nb))
__device__ __forceinline__ int entry_block(int32_t e, int nb) {
  if (e < 0) return 0;
  int j = e & 0x0fffffff;
  if (j >= nb) {
    set_device_error(kDevBadIndex);
    j = nb - 1;
  }
  return j;
}

// the 64 rows starting at row r0 of map m (64-row boxes), both column halves
__device__ __forceinline__ void load_half(uint32_t dst, const CUtensorMap* m, uint32_t bar, int r0, int h, int b) {
  tma_load_4d(dst, m, bar, 0, r0, h, b);
  tma_load_4d(dst + bwd::BOX, m, bar, 64, r0, h, b);
}
// the 128 rows starting at row r0 as two stacked 64-row boxes per column half
__device__ __forceinline__ void load_tile(uint32_t dst, const CUtensorMap* m, uint32_t bar, int r0, int h, int b) {
  tma_load_4d(dst, m, bar, 0, r0, h, b);
  tma_load_4d(dst + bwd::BOX, m, bar, 0, r0 + 64, h, b);
  tma_load_4d(dst + bwd::BOX128, m, bar, 64, r0, h, b);
  tma_load_4d(dst + bwd::BOX128 + bwd::BOX, m, bar, 64, r0 + 64, h, b);
}

// X[128 x 64] = A[128 x 128] B[64 x 128]^T over D: A a stationary 128-row
// tile, B one step's 64-row operand, both K-major
__device__ __forceinline__ void mma_step_ss(uint32_t d_tmem, uint32_t sa, uint32_t sb, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t ka = (kk >> 2) * bwd::BOX128 + (kk & 3) * 32;
    const uint32_t kb = (kk >> 2) * bwd::BOX + (kk & 3) * 32;
    mma_bf16_ss(d_tmem, sdesc_sw128(sa + ka, 16, 1024), sdesc_sw128(sb + kb, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}
// X[128 x 128] (+)= A[128 x 64] B[64 x 128]: A packed bf16 in TMEM (32
// columns), B one step's 64-row operand read MN-major
__device__ __forceinline__ void mma_step_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t sb, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_bf16_ts(d_tmem, a_tmem + 8 * kk, sdesc_sw128(sb + kk * 2048, bwd::BOX, 1024), idesc,
                (acc || kk > 0) ? 1u : 0u);
}

// ---------------------------------------------------------------------------
// delta[bh, t] = sum_d dO . O (fp32, fixed order), 0 on the padding rows [L, Lpad)
// ---------------------------------------------------------------------------
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, int64_t o_sB, int64_t o_sH, int64_t o_sT,
                                      const __nv_bfloat16* __restrict__ dout, int64_t d_sB, int64_t d_sH,
                                      int64_t d_sT, int B, int H, int L, int Lpad, float* __restrict__ delta) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = g >> 4;  // 16 lanes per (b, h, t) row
  const int sub = threadIdx.x & 15;
  const bool live = row < (int64_t)B * H * Lpad;
  const int64_t bh = live ? row / Lpad : 0;
  const int t = live ? (int)(row % Lpad) : 0;
  float acc = 0.f;
  if (live && t < L) {
    const int b = (int)(bh / H), h = (int)(bh % H);
    const uint4 ov = *reinterpret_cast<const uint4*>(o + b * o_sB + h * o_sH + t * o_sT + sub * 8);
    const uint4 dv = *reinterpret_cast<const uint4*>(dout + b * d_sB + h * d_sH + t * d_sT + sub * 8);
    const uint32_t oa[4] = {ov.x, ov.y, ov.z, ov.w}, da[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float o0, o1, d0, d1;
      unpack_bf2(oa[e], o0, o1);
      unpack_bf2(da[e], d0, d1);
      acc = fmaf(o0, d0, acc);
      acc = fmaf(o1, d1, acc);
    }
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (live && sub == 0) delta[row] = acc;
}

// ---------------------------------------------------------------------------
// inverse LUT: map[bh][j][i] = 1 when query block i selected key block j, then
// per key tile the ascending list of the query blocks that selected it
// ---------------------------------------------------------------------------
__global__ void lut_scatter_kernel(const int32_t* __restrict__ lut, int BH, int NBq, int NBk, int topk,
                                   uint8_t* __restrict__ map) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)BH * NBq * topk) return;
  const int64_t bh = g / ((int64_t)NBq * topk);
  const int i = (int)((g / topk) % NBq);
  const int j = lut[g];
  if (j < 0 || j >= NBk) {
    set_device_error(kDevBadIndex);
    return;
  }
  map[(bh * NBk + j) * NBq + i] = 1;
}

// one warp per (bh, 128-row key tile J).  Row layout (width NBq + 2 int32):
// [count, entries...].  Block 128: entries are the query blocks that selected
// key block J.  Block 64: entries are the 64-row query blocks i that selected
// key block 2J or 2J+1, as i | bit 28 (selected 2J) | bit 29 (selected 2J+1).
__global__ void lut_invert_kernel(const uint8_t* __restrict__ map, int BH, int NBq, int NBk, int blk64, int width,
                                  int32_t* __restrict__ inv) {
  const int NKT = blk64 ? (NBk + 1) / 2 : NBk;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)BH * NKT) return;
  const int64_t bh = w / NKT;
  const int J = (int)(w % NKT);
  const int j0 = blk64 ? 2 * J : J;
  const uint8_t* m0 = map + (bh * NBk + j0) * NBq;
  const uint8_t* m1 = (blk64 && j0 + 1 < NBk) ? m0 + NBq : nullptr;
  int32_t* out = inv + w * width;
  int n = 0;
  for (int base = 0; base < NBq; base += 32) {
    const int i = base + lane;
    int bits = 0;
    if (i < NBq) {
      bits = m0[i];
      if (m1) bits |= m1[i] << 1;
    }
    const uint32_t ball = __ballot_sync(0xffffffffu, bits != 0);
    if (bits) out[1 + n + __popc(ball & ((1u << lane) - 1u))] = blk64 ? (i | (bits << 28)) : i;
    n += __popc(ball);
  }
  if (lane == 0) out[0] = n;
}

// Tensor memory (512 columns): S (or S^T) of buffer b at [128 b, 128 b + 64),
// dP (or dP^T) at [128 b + 64, 128 b + 128); P^T and dS (dS^T) packed bf16
// over the first 32 columns of those.  dq kernel: three buffers, dQ at
// [384, 512).  dkdv kernel: two buffers (each warpgroup packs its 32 columns'
// P^T / dS^T over the first 16 of them), dV at [256, 384), dK at [384, 512).

// ---------------------------------------------------------------------------
// dq kernel: one CTA per (128-row query tile, b*h)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(bwd::DQ_THREADS, 1)
    attn_bwd_dq_tcgen05(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                        const AttnBwdParams p) {
  using namespace bwd;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + DQ_OFF_BAR;
  auto bar = [&](int i) { return bars + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + DQ_OFF_BAR + 8 * G_COUNT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + DQ_OFF_BAR + 8 * G_COUNT + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int m = blockIdx.x;  // 128-row query tile
  const bool two = p.blk64 != 0;
  // LUT row of this tile.  Block 128: topk key blocks, two 64-key steps each.
  // Block 64: the paired table's union (count of pairs first), one step per entry.
  const int ent = two ? 2 * p.topk + 1 : p.topk;
  const int32_t* row = p.lut + ((int64_t)bh * p.NQT + m) * ent + (two ? 1 : 0);
  const int n = two ? 2 * max(1, min(row[-1], p.topk)) : 2 * p.topk;  // steps
  // key rows of step i
  auto step_key = [&](int i) {
    return two ? 64 * entry_block(row[i], p.NBk) : 128 * entry_block(row[i >> 1], p.NBk) + 64 * (i & 1);
  };

  if (threadIdx.x == 0) {
    mbar_init(bar(G_TILE), 1);
    for (int s = 0; s < DQ_STAGES; ++s) {
      mbar_init(bar(G_FULL0 + s), 1);
      mbar_init(bar(G_EMPTY0 + s), 1);
    }
    for (int t = 0; t < DQ_NBUF; ++t) {
      mbar_init(bar(G_SF0 + t), 1);
      mbar_init(bar(G_DS0 + t), 4);
    }
    mbar_init(bar(G_ACC), 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    prefetch_tmap(&tdo);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      mbar_expect_tx(bar(G_TILE), 2 * TILE);
      load_tile(base + DQ_OFF_Q, &tq, bar(G_TILE), 128 * m, h, b);
      load_tile(base + DQ_OFF_DO, &tdo, bar(G_TILE), 128 * m, h, b);
      for (int i = 0; i < n; ++i) {
        const int s = i % DQ_STAGES;
        if (!mbar_wait(bar(G_EMPTY0 + s), ((i / DQ_STAGES) & 1) ^ 1, abort_flag, kDevTimeoutMma)) break;
        const uint32_t dst = base + DQ_OFF_RING + s * DQ_ENTRY;
        mbar_expect_tx(bar(G_FULL0 + s), 2 * HALF);
        const int r0 = step_key(i);
        load_half(dst, &tk, bar(G_FULL0 + s), r0, h, b);
        load_half(dst + HALF, &tv, bar(G_FULL0 + s), r0, h, b);
      }
      // drain: no TMA may still target shared memory when the CTA exits
      const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
      bool drained = mbar_wait_until(bar(G_TILE), 0, deadline);
      for (int i = max(0, n - DQ_STAGES); i < n && drained; ++i)
        drained = mbar_wait_until(bar(G_FULL0 + i % DQ_STAGES), (i / DQ_STAGES) & 1, deadline);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    // order: S_i, dP_i, then dQ += dS_{i-2} K_{i-2} once step i-2's dS is in
    // TMEM, so the tensor core computes S_i / dP_i while steps i-2 and i-1
    // are in the softmax (three buffers, three softmax warpgroups)
    if (elect_one()) {
      const uint32_t id_s = idesc_bf16_f32(128, 64, false, false);
      const uint32_t id_q = idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_wait(bar(G_TILE), 0, abort_flag, kDevTimeoutLoad);
      auto issue_dq = [&](int i) {
        if (!mbar_wait(bar(G_DS0 + i % DQ_NBUF), (i / DQ_NBUF) & 1, abort_flag, kDevTimeoutSoftmax)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t sk = base + DQ_OFF_RING + (i % DQ_STAGES) * DQ_ENTRY;
        mma_step_ts(tmem + DQ_ACC, tmem + 128 * (i % DQ_NBUF), sk, id_q, i > 0);  // dQ += dS K
        mma_commit(bar(G_EMPTY0 + i % DQ_STAGES));
      };
      for (int i = 0; i < n && ok; ++i) {
        const int s = i % DQ_STAGES;
        if (!mbar_wait(bar(G_FULL0 + s), (i / DQ_STAGES) & 1, abort_flag, kDevTimeoutLoad)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sk = base + DQ_OFF_RING + s * DQ_ENTRY, sv = sk + HALF;
        const uint32_t tb = tmem + 128 * (i % DQ_NBUF);
        mma_step_ss(tb, base + DQ_OFF_Q, sk, id_s);        // S  = Q K^T
        mma_step_ss(tb + 64, base + DQ_OFF_DO, sv, id_s);  // dP = dO V^T
        mma_commit(bar(G_SF0 + i % DQ_NBUF));
        if (i >= DQ_NBUF - 1) issue_dq(i - (DQ_NBUF - 1));
      }
      for (int i = max(0, n - (DQ_NBUF - 1)); i < n && ok; ++i) issue_dq(i);
      mma_commit(bar(G_ACC));
      // every MMA issued has completed before TMEM is freed, also on the abort path
      mbar_wait_until(bar(G_ACC), 0, globaltimer_ns() + kWaitLimitNs);
    }
  } else if (warp >= 4) {
    // -------------------------------------- dS of alternate steps, then the dQ epilogue
    const int wg = (warp - 4) >> 2;  // steps i with i % 3 == wg; warpgroups 0 and 1: epilogue columns [64 wg, 64 wg + 64)
    const int q = warp & 3;
    const int r = q * 32 + lane;  // query row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t tS = tmem + lane_off + 128 * wg, tdP = tS + 64;
    const int tok = 128 * m + r;
    const float lse = p.lse[(int64_t)bh * p.Lpad + tok];
    const float dlt = p.delta[(int64_t)bh * p.Lpad + tok];
    const uint64_t sc2 = f2_pack(p.qk_scale, p.qk_scale), nl2 = f2_pack(-lse, -lse);
    bool ok = true;
    for (int i = wg; i < n; i += DQ_NBUF) {
      if (!__all_sync(0xffffffffu, mbar_wait(bar(G_SF0 + wg), (i / DQ_NBUF) & 1, abort_flag, kDevTimeoutMma))) {
        ok = false;
        break;
      }
      tc_fence_after();
      int valid;  // valid key columns of this step for this row
      if (!two) {
        valid = min(64, max(0, p.L - step_key(i)));
      } else {
        const int32_t e = row[i];
        valid = (e < 0 || !((e >> (28 + (r >> 6))) & 1)) ? 0 : min(64, p.L - 64 * (e & 0x0fffffff));
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + 32 * c, sv);
        tmem_ld32(tdP + 32 * c, dv);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int col = 32 * c + 2 * e;
          float x0, x1;
          f2_unpack(fma_f32x2(f2_pack(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2, nl2), x0, x1);
          const float p0 = col < valid ? ex2_approx(x0) : 0.f;
          const float p1 = col + 1 < valid ? ex2_approx(x1) : 0.f;
          w[e] = pack_bf2(p0 * (__uint_as_float(dv[2 * e]) - dlt), p1 * (__uint_as_float(dv[2 * e + 1]) - dlt));
        }
        tmem_st16(tS + 16 * c, w);  // packed dS over the first 32 S columns of the buffer
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(G_DS0 + wg));
    }
    if (wg == 2) ok = false;  // the third warpgroup has no epilogue columns
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(G_ACC), 0, abort_flag, kDevTimeoutMma));
    tc_fence_after();
    if (ok) {
      const uint32_t tQ = tmem + DQ_ACC + lane_off + 64 * wg;
      uint32_t v[64];
      tmem_ld32(tQ, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tQ + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld_wait();
      if (tok < p.L) {
        uint4* dst = reinterpret_cast<uint4*>(p.dq + (int64_t)b * p.g_sB + (int64_t)h * p.g_sH + (int64_t)tok * p.g_sT +
                                              64 * wg);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w4[e] = pack_bf2(__uint_as_float(v[8 * c + 2 * e]) * kSmScale, __uint_as_float(v[8 * c + 2 * e + 1]) * kSmScale);
          dst[c] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
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

// ---------------------------------------------------------------------------
// dk/dv kernel: one CTA per (128-row key tile, b*h).  Both softmax
// warpgroups work on every step, 32 query columns each, so a step's P^T /
// dS^T take half the time on the chain (S^T, dP^T) -> softmax -> (dV, dK);
// the two S^T / dP^T buffers let the next step's S^T and dP^T run meanwhile.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(bwd::THREADS, 1)
    attn_bwd_dkdv_tcgen05(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                          const AttnBwdParams p) {
  using namespace bwd;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + KV_OFF_BAR;
  auto bar = [&](int i) { return bars + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + KV_OFF_BAR + 8 * G_COUNT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + KV_OFF_BAR + 8 * G_COUNT + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int J = blockIdx.x;  // 128-row key tile
  const bool two = p.blk64 != 0;
  const int32_t* row = p.inv + ((int64_t)bh * p.NKT + J) * p.inv_width;
  const int cnt = max(0, min(row[0], p.inv_width - 1));
  const int32_t* ents = row + 1;
  // steps: block 128, two 64-row halves of each query block; block 64, one per entry
  const int n = two ? cnt : 2 * cnt;
  auto step_query = [&](int i) {
    return two ? 64 * entry_block(ents[i], p.NBq) : 128 * entry_block(ents[i >> 1], p.NBq) + 64 * (i & 1);
  };

  if (threadIdx.x == 0) {
    mbar_init(bar(G_TILE), 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(bar(G_FULL0 + s), 1);
      mbar_init(bar(G_EMPTY0 + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(G_SF0 + t), 1);
      mbar_init(bar(G_DS0 + t), 8);
    }
    mbar_init(bar(G_ACC), 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    prefetch_tmap(&tdo);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      mbar_expect_tx(bar(G_TILE), 2 * TILE);
      load_tile(base + KV_OFF_K, &tk, bar(G_TILE), 128 * J, h, b);
      load_tile(base + KV_OFF_V, &tv, bar(G_TILE), 128 * J, h, b);
      const float* lse_row = p.lse + (int64_t)bh * p.Lpad;
      const float* dlt_row = p.delta + (int64_t)bh * p.Lpad;
      for (int i = 0; i < n; ++i) {
        const int s = i % KV_STAGES;
        if (!mbar_wait(bar(G_EMPTY0 + s), ((i / KV_STAGES) & 1) ^ 1, abort_flag, kDevTimeoutMma)) break;
        const uint32_t dst = base + KV_OFF_RING + s * KV_ENTRY;
        mbar_expect_tx(bar(G_FULL0 + s), 2 * HALF + 512);
        const int r0 = step_query(i);
        load_half(dst, &tq, bar(G_FULL0 + s), r0, h, b);
        load_half(dst + HALF, &tdo, bar(G_FULL0 + s), r0, h, b);
        bulk_load(dst + 2 * HALF, lse_row + r0, 256, bar(G_FULL0 + s));
        bulk_load(dst + 2 * HALF + 256, dlt_row + r0, 256, bar(G_FULL0 + s));
      }
      const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
      bool drained = mbar_wait_until(bar(G_TILE), 0, deadline);
      for (int i = max(0, n - KV_STAGES); i < n && drained; ++i)
        drained = mbar_wait_until(bar(G_FULL0 + i % KV_STAGES), (i / KV_STAGES) & 1, deadline);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (elect_one()) {
      const uint32_t id_s = idesc_bf16_f32(128, 64, false, false);
      const uint32_t id_a = idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_wait(bar(G_TILE), 0, abort_flag, kDevTimeoutLoad);
      auto issue_acc = [&](int i) {
        if (!mbar_wait(bar(G_DS0 + (i & 1)), (i >> 1) & 1, abort_flag, kDevTimeoutSoftmax)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t sq = base + KV_OFF_RING + (i % KV_STAGES) * KV_ENTRY, sdo = sq + HALF;
        const uint32_t tb = tmem + 128 * (i & 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // dV += P^T dO, dK += dS^T Q; queries 16 kk.. of warpgroup kk / 2
          const uint32_t a = 32 * (kk >> 1) + 8 * (kk & 1);
          mma_bf16_ts(tmem + 256, tb + a, sdesc_sw128(sdo + kk * 2048, BOX, 1024), id_a, (i > 0 || kk > 0) ? 1u : 0u);
          mma_bf16_ts(tmem + 384, tb + 64 + a, sdesc_sw128(sq + kk * 2048, BOX, 1024), id_a,
                      (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar(G_EMPTY0 + i % KV_STAGES));
      };
      for (int i = 0; i < n && ok; ++i) {
        const int s = i % KV_STAGES;
        if (!mbar_wait(bar(G_FULL0 + s), (i / KV_STAGES) & 1, abort_flag, kDevTimeoutLoad)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sq = base + KV_OFF_RING + s * KV_ENTRY, sdo = sq + HALF;
        const uint32_t tb = tmem + 128 * (i & 1);
        mma_step_ss(tb, base + KV_OFF_K, sq, id_s);        // S^T  = K Q^T
        mma_step_ss(tb + 64, base + KV_OFF_V, sdo, id_s);  // dP^T = V dO^T
        mma_commit(bar(G_SF0 + (i & 1)));
        if (i > 0) issue_acc(i - 1);
      }
      if (ok && n > 0) issue_acc(n - 1);
      mma_commit(bar(G_ACC));
      // every MMA issued has completed before TMEM is freed, also on the abort path
      mbar_wait_until(bar(G_ACC), 0, globaltimer_ns() + kWaitLimitNs);
    }
  } else if (warp >= 4) {
    // ---------- P^T, dS^T of query columns [32 wg, 32 wg + 32) of every step, then the dK/dV epilogue
    const int wg = (warp - 4) >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;  // key row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint64_t sc2 = f2_pack(p.qk_scale, p.qk_scale);
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int s = i % KV_STAGES;
      const uint32_t tS = tmem + lane_off + 128 * (i & 1) + 32 * wg, tdP = tS + 64;
      bool got = mbar_wait(bar(G_SF0 + (i & 1)), (i >> 1) & 1, abort_flag, kDevTimeoutMma);
      // the step's lse2 / delta (bulk copies) are visible once its load barrier completed
      got = got && mbar_wait(bar(G_FULL0 + s), (i / KV_STAGES) & 1, abort_flag, kDevTimeoutLoad);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      bool sel = true;  // block 64: did this step's query block select this key row's block?
      if (two) {
        const int32_t e = ents[i];
        sel = e >= 0 && ((e >> (28 + (r >> 6))) & 1);
      }
      const float* lse_s = reinterpret_cast<const float*>(gbase + KV_OFF_RING + s * KV_ENTRY + 2 * HALF) + 32 * wg;
      const float* dlt_s = lse_s + 64;
      {
        uint32_t sv[32], dv[32];
        tmem_ld32(tS, sv);
        tmem_ld32(tdP, dv);
        tmem_ld_wait();
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 l2 = *reinterpret_cast<const float2*>(lse_s + 2 * e);
          const float2 d2 = *reinterpret_cast<const float2*>(dlt_s + 2 * e);
          float x0, x1;
          f2_unpack(fma_f32x2(f2_pack(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2,
                              f2_pack(-l2.x, -l2.y)),
                    x0, x1);
          const float p0 = sel ? ex2_approx(x0) : 0.f;
          const float p1 = sel ? ex2_approx(x1) : 0.f;
          wp[e] = pack_bf2(p0, p1);
          wd[e] = pack_bf2(p0 * (__uint_as_float(dv[2 * e]) - d2.x), p1 * (__uint_as_float(dv[2 * e + 1]) - d2.y));
        }
        tmem_st16(tS, wp);   // packed P^T over the first 16 of this warpgroup's S^T columns
        tmem_st16(tdP, wd);  // packed dS^T over the first 16 of its dP^T columns
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(G_DS0 + (i & 1)));
    }
    if (ok && n > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(G_ACC), 0, abort_flag, kDevTimeoutMma));
    tc_fence_after();
    const int tok = 128 * J + r;
    if (ok) {
      // both accumulators are read (warp-collective TMEM loads, every lane)
      // and packed before the per-row store condition diverges the warp
      uint32_t pk[2][32];
#pragma unroll
      for (int which = 0; which < 2; ++which) {  // dV, then dK (scaled by D^-1/2)
        uint32_t v[64];
        if (n > 0) {
          const uint32_t tA = tmem + 256 + 128 * which + lane_off + 64 * wg;
          tmem_ld32(tA, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          tmem_ld32(tA + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e) v[e] = 0u;  // no query block selected this key tile
        }
        const float sc = which ? kSmScale : 1.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e)
          pk[which][e] = pack_bf2(__uint_as_float(v[2 * e]) * sc, __uint_as_float(v[2 * e + 1]) * sc);
      }
      if (tok < p.L) {
        const int64_t goff = (int64_t)b * p.g_sB + (int64_t)h * p.g_sH + (int64_t)tok * p.g_sT + 64 * wg;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          uint4* dst = reinterpret_cast<uint4*>((which ? p.dk : p.dv) + goff);
#pragma unroll
          for (int c = 0; c < 8; ++c)
            dst[c] = make_uint4(pk[which][4 * c], pk[which][4 * c + 1], pk[which][4 * c + 2], pk[which][4 * c + 3]);
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

int launch_attn_bwd_delta(const __nv_bfloat16* o, int64_t o_sB, int64_t o_sH, int64_t o_sT, const __nv_bfloat16* dout,
                          int64_t d_sB, int64_t d_sH, int64_t d_sT, int B, int H, int L, int Lpad, float* delta,
                          cudaStream_t s) {
  const int64_t threads = (int64_t)B * H * Lpad * 16;
  attn_bwd_delta_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(o, o_sB, o_sH, o_sT, dout, d_sB, d_sH, d_sT,
                                                                        B, H, L, Lpad, delta);
  return (int)cudaGetLastError();
}

int launch_lut_invert(const int32_t* lut, int BH, int NBq, int NBk, int topk, int blk64, uint8_t* map, int32_t* inv,
                      int width, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(map, 0, (size_t)BH * NBq * NBk, s);
  if (e != cudaSuccess) return (int)e;
  const int64_t n = (int64_t)BH * NBq * topk;
  lut_scatter_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(lut, BH, NBq, NBk, topk, map);
  const int64_t warps = (int64_t)BH * (blk64 ? (NBk + 1) / 2 : NBk);
  lut_invert_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(map, BH, NBq, NBk, blk64, width, inv);
  return (int)cudaGetLastError();
}

int launch_attn_bwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                    const AttnBwdParams& p, cudaStream_t s) {
  using namespace bwd;
  cudaFuncSetAttribute(attn_bwd_dq_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM);
  cudaFuncSetAttribute(attn_bwd_dkdv_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, KV_SMEM);
  attn_bwd_dq_tcgen05<<<dim3(p.NQT, p.B * p.H), DQ_THREADS, DQ_SMEM, s>>>(tq, tk, tv, tdo, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  attn_bwd_dkdv_tcgen05<<<dim3(p.NKT, p.B * p.H), THREADS, KV_SMEM, s>>>(tq, tk, tv, tdo, p);
  return (int)cudaGetLastError();
}

}  // namespace rola
