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
// Block size 64 runs on 128-row tiles as in the forward: the dq kernel takes
// the paired LUT of launch_pair_blocks (two 64-row key blocks stacked per key
// tile, selection bits per query half); the dkdv kernel takes an inverse
// table whose entries are 64-row query blocks with two selection bits (key
// block 2J, key block 2J+1 of key tile J), stacked two per query tile.
//
// Both kernels: 384 threads.  Warp 0 lane 0 is the TMA producer (no
// multicast), warp 1 owns tensor memory and issues the MMAs (one elected
// thread), warpgroups 1 and 2 each take one 64-column half of the S / dP tile
// for all 128 rows (thread = TMEM lane = tile row) and then the epilogue of
// that half.  Every mbarrier wait is bounded (error flag + abort, as in the
// forward).
#include "common.cuh"
#include "kernels.h"

namespace rola {

namespace bwd {
constexpr int THREADS = 384;
constexpr int TILE = 16384;  // [128 rows x 64 bf16] box, 128-byte swizzle
constexpr int SLOT = 2 * TILE;  // one 128 x 128 bf16 tile
constexpr int STAGES = 2;
// dq kernel: Q and dO of the query tile, then the ring of (K, V) key tiles
constexpr int DQ_OFF_Q = 0, DQ_OFF_DO = SLOT, DQ_OFF_RING = 2 * SLOT;
constexpr int DQ_ENTRY = 2 * SLOT;
constexpr int DQ_OFF_BAR = DQ_OFF_RING + STAGES * DQ_ENTRY;  // 192 KB
// dkdv kernel: K and V of the key tile, then the ring of (Q, dO, lse2, delta) query tiles
constexpr int KV_OFF_K = 0, KV_OFF_V = SLOT, KV_OFF_RING = 2 * SLOT;
constexpr int KV_ENTRY = 2 * SLOT + 1024;  // + 128 lse2 + 128 delta (fp32)
constexpr int KV_OFF_BAR = KV_OFF_RING + STAGES * KV_ENTRY;  // 194 KB
constexpr int BAR_BYTES = 256;
constexpr int DQ_SMEM = DQ_OFF_BAR + BAR_BYTES + 1024;
constexpr int KV_SMEM = KV_OFF_BAR + BAR_BYTES + 1024;
static_assert(KV_ENTRY % 1024 == 0, "ring entries keep the 1024-byte swizzle alignment");
constexpr float kSmScale = 0.08838834764831845f;  // 128^-1/2
}  // namespace bwd

enum : int {
  G_TILE = 0,          // stationary tiles loaded (Q, dO / K, V)
  G_FULL0,             // ring entry s loaded: G_FULL0 + s
  G_EMPTY0 = G_FULL0 + bwd::STAGES,  // ring entry s consumed (MMA commit)
  G_SF = G_EMPTY0 + bwd::STAGES,     // S and dP of the current block in TMEM
  G_DS,                // dS (dq) / P^T and dS^T (dkdv) in TMEM, 8 warp arrivals
  G_ACC,               // accumulators final
  G_COUNT
};
static_assert(8 * G_COUNT + 16 <= bwd::BAR_BYTES, "barrier region too small");

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// key block of entry i of a 128-block LUT row (clamped, error flag on a bad index)
__device__ __forceinline__ int bwd_block(const int32_t* row, int i, int nb) {
  int j = row[i];
  if (j < 0 || j >= nb) {
    set_device_error(kDevBadIndex);
    j = j < 0 ? 0 : nb - 1;
  }
  return j;
}
// 64-row block of a paired / inverse entry (padding -1 -> block 0, masked by the caller)
__device__ __forceinline__ int bwd_block64(int32_t e, int nb) {
  if (e < 0) return 0;
  int j = e & 0x0fffffff;
  if (j >= nb) {
    set_device_error(kDevBadIndex);
    j = nb - 1;
  }
  return j;
}

// load a 128-row tile (two 64-column boxes) of map m at rows r0 (and, block 64,
// the lower 64 rows from r1)
__device__ __forceinline__ void load_tile(uint32_t dst, const CUtensorMap* m, uint32_t bar, int r0, int r1, bool two,
                                          int h, int b) {
  if (!two) {
    tma_load_4d(dst, m, bar, 0, r0, h, b);
    tma_load_4d(dst + bwd::TILE, m, bar, 64, r0, h, b);
  } else {
    tma_load_4d(dst, m, bar, 0, r0, h, b);
    tma_load_4d(dst + bwd::TILE / 2, m, bar, 0, r1, h, b);
    tma_load_4d(dst + bwd::TILE, m, bar, 64, r0, h, b);
    tma_load_4d(dst + bwd::TILE + bwd::TILE / 2, m, bar, 64, r1, h, b);
  }
}

// issue X (+)= A B^T over D = 128 with both operands K-major 128 x 128 tiles
__device__ __forceinline__ void mma_tile_ss(uint32_t d_tmem, uint32_t sa, uint32_t sb, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t off = (kk >> 2) * bwd::TILE + (kk & 3) * 32;
    mma_bf16_ss(d_tmem, sdesc_sw128(sa + off, 16, 1024), sdesc_sw128(sb + off, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}
// issue X (+)= A B with A packed bf16 in TMEM (each warpgroup's 64 K-columns
// packed into the first 32 TMEM columns of its half) and B an MN-major tile
__device__ __forceinline__ void mma_tile_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t sb, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    mma_bf16_ts(d_tmem, a_tmem + 64 * (kk >> 2) + 8 * (kk & 3), sdesc_sw128(sb + kk * 2048, bwd::TILE, 1024), idesc,
                (acc || kk > 0) ? 1u : 0u);
  }
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

// one warp per (bh, key tile J).  Row layout (width NBq + 2 int32): [count,
// entries...].  Block 128: entries are query blocks, count = their number.
// Block 64: entries are 64-row query blocks i | bit 28 (selected key block 2J)
// | bit 29 (selected key block 2J+1), padded with -1 to an even number; count
// = number of stacked pairs.
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
  if (lane == 0) {
    if (blk64 && (n & 1)) out[1 + n] = -1;
    out[0] = blk64 ? (n + 1) / 2 : n;
  }
}

// ---------------------------------------------------------------------------
// dq kernel: one CTA per (128-row query tile, b*h)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(bwd::THREADS, 1)
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
  // LUT row of this tile: block 128 the plain row, block 64 the paired row (count first)
  const int ent = two ? 2 * p.topk + 1 : p.topk;
  const int32_t* row = p.lut + ((int64_t)bh * p.NQT + m) * ent + (two ? 1 : 0);
  const int n = two ? max(1, min(row[-1], p.topk)) : p.topk;

  if (threadIdx.x == 0) {
    mbar_init(bar(G_TILE), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(G_FULL0 + s), 1);
      mbar_init(bar(G_EMPTY0 + s), 1);
    }
    mbar_init(bar(G_SF), 1);
    mbar_init(bar(G_DS), 8);
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
  const uint32_t tmem = *tmem_slot;  // S/dS [0,128), dP [128,256), dQ [256,384)

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      mbar_expect_tx(bar(G_TILE), 2 * SLOT);
      load_tile(base + DQ_OFF_Q, &tq, bar(G_TILE), 128 * m, 128 * m + 64, two, h, b);
      load_tile(base + DQ_OFF_DO, &tdo, bar(G_TILE), 128 * m, 128 * m + 64, two, h, b);
      bool ok = true;
      for (int i = 0; i < n && ok; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(bar(G_EMPTY0 + s), ((i / STAGES) & 1) ^ 1, abort_flag, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        const uint32_t dst = base + DQ_OFF_RING + s * DQ_ENTRY;
        mbar_expect_tx(bar(G_FULL0 + s), 2 * SLOT);
        int r0, r1 = 0;
        if (!two) {
          r0 = 128 * bwd_block(row, i, p.NBk);
        } else {
          r0 = 64 * bwd_block64(row[2 * i], p.NBk);
          r1 = 64 * bwd_block64(row[2 * i + 1], p.NBk);
        }
        load_tile(dst, &tk, bar(G_FULL0 + s), r0, r1, two, h, b);
        load_tile(dst + SLOT, &tv, bar(G_FULL0 + s), r0, r1, two, h, b);
      }
      // drain: no TMA may still target shared memory when the CTA exits
      const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
      bool drained = mbar_wait_until(bar(G_TILE), 0, deadline);
      for (int i = max(0, n - STAGES); i < n && drained; ++i)
        drained = mbar_wait_until(bar(G_FULL0 + i % STAGES), (i / STAGES) & 1, deadline);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (elect_one()) {
      const uint32_t id_ss = idesc_bf16_f32(128, 128, false, false);
      const uint32_t id_ts = idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_wait(bar(G_TILE), 0, abort_flag, kDevTimeoutLoad);
      for (int i = 0; i < n && ok; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(bar(G_FULL0 + s), (i / STAGES) & 1, abort_flag, kDevTimeoutLoad)) break;
        tc_fence_after();
        const uint32_t sk = base + DQ_OFF_RING + s * DQ_ENTRY, sv = sk + SLOT;
        mma_tile_ss(tmem, base + DQ_OFF_Q, sk, id_ss);          // S  = Q K^T
        mma_tile_ss(tmem + 128, base + DQ_OFF_DO, sv, id_ss);   // dP = dO V^T
        mma_commit(bar(G_SF));
        if (!mbar_wait(bar(G_DS), i & 1, abort_flag, kDevTimeoutSoftmax)) break;
        tc_fence_after();
        mma_tile_ts(tmem + 256, tmem, sk, id_ts, i > 0);        // dQ += dS K
        mma_commit(bar(G_EMPTY0 + s));
      }
      mma_commit(bar(G_ACC));
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------- dS, then the dQ epilogue
    const int hc = (warp - 4) >> 2;  // key half (columns) of this warpgroup
    const int q = warp & 3;
    const int r = q * 32 + lane;      // tile row = TMEM lane
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t tS = tmem + lane_off + 64 * hc, tdP = tmem + 128 + lane_off + 64 * hc;
    const int tok = 128 * m + r;
    const float lse = p.lse[(int64_t)bh * p.Lpad + tok];
    const float dlt = p.delta[(int64_t)bh * p.Lpad + tok];
    const uint64_t sc2 = f2_pack(p.qk_scale, p.qk_scale), nl2 = f2_pack(-lse, -lse);
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      if (!__all_sync(0xffffffffu, mbar_wait(bar(G_SF), i & 1, abort_flag, kDevTimeoutMma))) {
        ok = false;
        break;
      }
      tc_fence_after();
      int valid;  // valid key columns of this half for this row
      if (!two) {
        valid = min(64, max(0, p.L - 128 * bwd_block(row, i, p.NBk) - 64 * hc));
      } else {
        const int32_t e = row[2 * i + hc];
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
          const float d0 = p0 * (__uint_as_float(dv[2 * e]) - dlt);
          const float d1 = p1 * (__uint_as_float(dv[2 * e + 1]) - dlt);
          w[e] = pack_bf2(d0, d1);
        }
        tmem_st16(tS + 16 * c, w);  // packed dS over the S columns of this half
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(G_DS));
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(G_ACC), 0, abort_flag, kDevTimeoutMma));
    tc_fence_after();
    if (ok) {
      const uint32_t tQ = tmem + 256 + lane_off + 64 * hc;
      uint32_t v[64];
      tmem_ld32(tQ, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tQ + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld_wait();
      if (tok < p.L) {
        uint4* dst = reinterpret_cast<uint4*>(p.dq + (int64_t)b * p.g_sB + (int64_t)h * p.g_sH + (int64_t)tok * p.g_sT +
                                              64 * hc);
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
// dk/dv kernel: one CTA per (128-row key tile, b*h)
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
  // query tiles to visit (block 64: stacked pairs of entries)
  const int n = max(0, min(row[0], two ? (p.inv_width - 1) / 2 : p.inv_width - 1));
  const int32_t* ents = row + 1;

  if (threadIdx.x == 0) {
    mbar_init(bar(G_TILE), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(G_FULL0 + s), 1);
      mbar_init(bar(G_EMPTY0 + s), 1);
    }
    mbar_init(bar(G_SF), 1);
    mbar_init(bar(G_DS), 8);
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
  const uint32_t tmem = *tmem_slot;  // S^T/P^T [0,128), dP^T/dS^T [128,256), dV [256,384), dK [384,512)

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      mbar_expect_tx(bar(G_TILE), 2 * SLOT);
      load_tile(base + KV_OFF_K, &tk, bar(G_TILE), 128 * J, 128 * J + 64, two, h, b);
      load_tile(base + KV_OFF_V, &tv, bar(G_TILE), 128 * J, 128 * J + 64, two, h, b);
      bool ok = true;
      for (int i = 0; i < n && ok; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(bar(G_EMPTY0 + s), ((i / STAGES) & 1) ^ 1, abort_flag, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        const uint32_t dst = base + KV_OFF_RING + s * KV_ENTRY;
        mbar_expect_tx(bar(G_FULL0 + s), 2 * SLOT + 1024);
        const int64_t srow = (int64_t)bh * p.Lpad;
        if (!two) {
          const int qi = bwd_block(ents, i, p.NBq);
          load_tile(dst, &tq, bar(G_FULL0 + s), 128 * qi, 0, false, h, b);
          load_tile(dst + SLOT, &tdo, bar(G_FULL0 + s), 128 * qi, 0, false, h, b);
          bulk_load(dst + 2 * SLOT, p.lse + srow + 128 * qi, 512, bar(G_FULL0 + s));
          bulk_load(dst + 2 * SLOT + 512, p.delta + srow + 128 * qi, 512, bar(G_FULL0 + s));
        } else {
          const int i0 = bwd_block64(ents[2 * i], p.NBq), i1 = bwd_block64(ents[2 * i + 1], p.NBq);
          load_tile(dst, &tq, bar(G_FULL0 + s), 64 * i0, 64 * i1, true, h, b);
          load_tile(dst + SLOT, &tdo, bar(G_FULL0 + s), 64 * i0, 64 * i1, true, h, b);
          bulk_load(dst + 2 * SLOT, p.lse + srow + 64 * i0, 256, bar(G_FULL0 + s));
          bulk_load(dst + 2 * SLOT + 256, p.lse + srow + 64 * i1, 256, bar(G_FULL0 + s));
          bulk_load(dst + 2 * SLOT + 512, p.delta + srow + 64 * i0, 256, bar(G_FULL0 + s));
          bulk_load(dst + 2 * SLOT + 768, p.delta + srow + 64 * i1, 256, bar(G_FULL0 + s));
        }
      }
      const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
      bool drained = mbar_wait_until(bar(G_TILE), 0, deadline);
      for (int i = max(0, n - STAGES); i < n && drained; ++i)
        drained = mbar_wait_until(bar(G_FULL0 + i % STAGES), (i / STAGES) & 1, deadline);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (elect_one()) {
      const uint32_t id_ss = idesc_bf16_f32(128, 128, false, false);
      const uint32_t id_ts = idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_wait(bar(G_TILE), 0, abort_flag, kDevTimeoutLoad);
      for (int i = 0; i < n && ok; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(bar(G_FULL0 + s), (i / STAGES) & 1, abort_flag, kDevTimeoutLoad)) break;
        tc_fence_after();
        const uint32_t sq = base + KV_OFF_RING + s * KV_ENTRY, sdo = sq + SLOT;
        mma_tile_ss(tmem, base + KV_OFF_K, sq, id_ss);          // S^T  = K Q^T
        mma_tile_ss(tmem + 128, base + KV_OFF_V, sdo, id_ss);   // dP^T = V dO^T
        mma_commit(bar(G_SF));
        if (!mbar_wait(bar(G_DS), i & 1, abort_flag, kDevTimeoutSoftmax)) break;
        tc_fence_after();
        mma_tile_ts(tmem + 256, tmem, sdo, id_ts, i > 0);       // dV += P^T dO
        mma_tile_ts(tmem + 384, tmem + 128, sq, id_ts, i > 0);  // dK += dS^T Q
        mma_commit(bar(G_EMPTY0 + s));
      }
      mma_commit(bar(G_ACC));
    }
  } else if (warp >= 4) {
    // ---------------------------------------------- P^T, dS^T, then the dK/dV epilogue
    const int hc = (warp - 4) >> 2;  // query half (columns) of this warpgroup
    const int q = warp & 3;
    const int r = q * 32 + lane;      // key row = TMEM lane
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t tS = tmem + lane_off + 64 * hc, tdP = tmem + 128 + lane_off + 64 * hc;
    const uint64_t sc2 = f2_pack(p.qk_scale, p.qk_scale);
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int s = i % STAGES;
      bool got = mbar_wait(bar(G_SF), i & 1, abort_flag, kDevTimeoutMma);
      // the entry's lse2 / delta (bulk copies) are visible once its load barrier completed
      got = got && mbar_wait(bar(G_FULL0 + s), (i / STAGES) & 1, abort_flag, kDevTimeoutLoad);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      bool sel = true;  // this key row's block was selected by this half's query block
      if (two) {
        const int32_t e = ents[2 * i + hc];
        sel = e >= 0 && ((e >> (28 + (r >> 6))) & 1);
      }
      const float* lse_s = reinterpret_cast<const float*>(gbase + KV_OFF_RING + s * KV_ENTRY + 2 * SLOT) + 64 * hc;
      const float* dlt_s = lse_s + 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + 32 * c, sv);
        tmem_ld32(tdP + 32 * c, dv);
        tmem_ld_wait();
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 l2 = *reinterpret_cast<const float2*>(lse_s + 32 * c + 2 * e);
          const float2 d2 = *reinterpret_cast<const float2*>(dlt_s + 32 * c + 2 * e);
          float x0, x1;
          f2_unpack(fma_f32x2(f2_pack(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2,
                              f2_pack(-l2.x, -l2.y)),
                    x0, x1);
          const float p0 = sel ? ex2_approx(x0) : 0.f;
          const float p1 = sel ? ex2_approx(x1) : 0.f;
          wp[e] = pack_bf2(p0, p1);
          wd[e] = pack_bf2(p0 * (__uint_as_float(dv[2 * e]) - d2.x), p1 * (__uint_as_float(dv[2 * e + 1]) - d2.y));
        }
        tmem_st16(tS + 16 * c, wp);   // packed P^T over the S^T columns of this half
        tmem_st16(tdP + 16 * c, wd);  // packed dS^T over the dP^T columns of this half
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(G_DS));
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
          const uint32_t tA = tmem + 256 + 128 * which + lane_off + 64 * hc;
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
        const int64_t goff = (int64_t)b * p.g_sB + (int64_t)h * p.g_sH + (int64_t)tok * p.g_sT + 64 * hc;
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
  attn_bwd_dq_tcgen05<<<dim3(p.NQT, p.B * p.H), THREADS, DQ_SMEM, s>>>(tq, tk, tv, tdo, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  attn_bwd_dkdv_tcgen05<<<dim3(p.NKT, p.B * p.H), THREADS, KV_SMEM, s>>>(tq, tk, tv, tdo, p);
  return (int)cudaGetLastError();
}

}  // namespace rola
