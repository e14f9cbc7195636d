// Block-sparse online-softmax attention on tcgen05, fused with the low-rank
// correction and the gate (one epilogue).
//
// Restates `_rola_fwd_kernel` (sparkdiffusion/ops/fused_kernel/
// fused_sparse_attn.py:55-144): for query block m of head (b, h) iterate the
// selected key blocks j of the LUT, s = (q.k) * D^-1/2 * log2(e) in fp32,
// columns past L masked to -inf for a partial block, base-2 online softmax,
// P rounded to bf16 before P.V, o = acc / l.  The epilogue then restates
// o_lr = q_lr . C (fused_lowrank.py:360-362) and `_gate_fusion_kernel`
// (fused_gate.py:67-127), storing the gated output directly.
//
// One CTA per (pair of query blocks, batch*head): the two 128-row tiles A and
// B have their own LUT rows and run ping-pong, so the tensor core executes one
// tile's MMAs while the other tile's softmax runs.  Four warpgroups with
// registers rebalanced by setmaxnreg (launch: 512 threads x 128):
//   WG0 (56 regs)   warp 0 lane 0: TMA producer.  Q of both tiles once, then
//                   the K and V blocks of both LUTs through one 5-slot ring in
//                   exactly the order the MMAs consume them (K_A0 K_B0 | V_A0
//                   K_A1 V_B0 K_B1 | ...), then the epilogue operands (q_lr
//                   tiles and C^T, and the hidden-state tiles when the gate is
//                   computed from x).  No multicast.
//                   warp 1: TMEM owner and MMA issuer (one elected thread):
//                   S = Q K^T (smem x smem) and O += P V with P read from TMEM
//                   (tcgen05.mma with the A operand in tensor memory).
//   WG1, WG2 (176)  softmax of tile A / tile B: thread = query row = TMEM lane.
//                   Per KV block the whole S row is loaded at once, the row max
//                   taken, the row's O rescale factor published, and
//                   P = exp2(s*scale - m) written back over the S columns as
//                   packed bf16, handed to the MMA in chunks of 32 keys so that
//                   P V starts while the rest of P is computed; then the fused
//                   epilogue.
//   WG3 (96)        correction: rescales O in TMEM by the published factors
//                   while the softmax computes P (every growth of the running
//                   max when `rescale_threshold` is 0: the reference's
//                   recurrence exactly); the MMA issuer waits for the
//                   corrected O, then for each P chunk before its K steps.
// TMEM columns: S/P of tile t at [128 t, 128 t + 128), O of tile t at
// [256 + 128 t, ...); the epilogue's o_lr reuses the S columns.
#include "common.cuh"
#include "kernels.h"

namespace rola {

namespace attn {
constexpr int THREADS = 512;
constexpr int LAUNCH_REGS = 128;            // 65536 / 512
constexpr int REGS_LOAD = 56, REGS_CORR = 96, REGS_SOFTMAX = 176;
static_assert(128 * REGS_LOAD + 128 * REGS_CORR + 2 * 128 * REGS_SOFTMAX <= THREADS * LAUNCH_REGS,
              "register split exceeds the pool");
constexpr int TILE = 16384;                 // one [128 rows x 64 bf16] box, 128B swizzle
constexpr int SLOT = 2 * TILE;              // one 128x128 K or V block
constexpr int NSLOTS = 5;
constexpr int OFF_Q = 0;                    // 2 tiles x 2 boxes
constexpr int OFF_RING = 4 * TILE;          // 5 slots
constexpr int OFF_BAR = OFF_RING + NSLOTS * SLOT;  // 224 KB
constexpr int OFF_ALPHA = OFF_BAR + 512;    // per-row O rescale factors of both tiles [2][128] fp32
constexpr int SMEM_BYTES = OFF_ALPHA + 1024 + 1024;
constexpr int PCHUNKS = 4;                  // P handed to the MMA in 4 chunks of 32 keys
}  // namespace attn

// barrier slots
enum : int {
  B_Q = 0,
  B_FULL0,                       // ring slot s full (TMA): B_FULL0 + s
  B_EMPTY0 = B_FULL0 + 5,        // ring slot s consumed (MMA commit): B_EMPTY0 + s
  B_SF0 = B_EMPTY0 + 5, B_SF1,   // S of tile t ready (MMA -> softmax)
  B_PF0,                         // P chunk c of tile t in TMEM (softmax -> MMA): B_PF0 + 4 t + c, 4 arrivals
  B_OF0 = B_PF0 + 8, B_OF1,      // last P V of tile t complete
  B_LR0, B_LR1,                  // o_lr of tile t in TMEM
  B_AR0, B_AR1,                  // rescale factors of tile t published (softmax -> correction), 4 arrivals
  B_OC0, B_OC1,                  // O of tile t rescaled (correction -> MMA), 4 arrivals
  B_DRAIN,
  B_COUNT
};
// barriers, then the abort flag, the TMEM address and the epilogue's per-warp flags
static_assert(8 * B_COUNT + 16 + 32 <= attn::OFF_ALPHA - attn::OFF_BAR, "barrier region too small");

// block size 64: one entry of a tile's paired union (launch_pair_blocks) -> the
// key block (padding -1 -> block 0, which the softmax masks out entirely)
__device__ __forceinline__ int pair_block(const AttnParams& p, int32_t e) {
  if (e < 0) return 0;
  int j = e & 0x0fffffff;
  if (j >= p.NBk) {
    set_device_error(kDevBadIndex);
    j = p.NBk - 1;
  }
  return j;
}
// valid columns (0..64) of the 64-column half holding entry e, for a row of
// query block `half` (0 or 1) of the tile: none unless that block selected it
__device__ __forceinline__ int pair_valid(const AttnParams& p, int32_t e, int half) {
  if (e < 0 || !((e >> (28 + half)) & 1)) return 0;
  return min(64, p.L - (e & 0x0fffffff) * 64);
}

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
                        const __grid_constant__ CUtensorMap tct, const __grid_constant__ CUtensorMap tx,
                        const AttnParams p) {
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
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int m0 = 2 * blockIdx.x;                              // first 128-row query tile
  const int NQT = p.blk64 ? (p.NBq + 1) / 2 : p.NBq;           // 128-row query tiles
  const int nt = (m0 + 1 < NQT) ? 2 : 1;  // active tiles
  // Row of tile t in p.lut: the LUT row (block 128) or the tile's paired union
  // (block 64: the count, then 2k entries).  Main-loop iterations: the LUT
  // length, or for block 64 the larger key-tile count of the two tiles (the
  // other tile's extra key tiles are padding and fully masked).
  const int ent = p.blk64 ? 2 * p.topk + 1 : p.topk;
  auto tile_row = [&](int t) { return p.lut + ((int64_t)bh * NQT + m0 + t) * ent + (p.blk64 ? 1 : 0); };
  int topk = p.topk;
  if (p.blk64) {
    topk = tile_row(0)[-1];
    if (nt == 2) topk = max(topk, tile_row(1)[-1]);
    topk = max(1, min(topk, p.topk));
  }

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    for (int s = 0; s < NSLOTS; ++s) {
      mbar_init(bar(B_FULL0 + s), 1);
      mbar_init(bar(B_EMPTY0 + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(B_SF0 + t), 1);
      for (int c = 0; c < PCHUNKS; ++c) mbar_init(bar(B_PF0 + PCHUNKS * t + c), 4);
      mbar_init(bar(B_OF0 + t), 1);
      mbar_init(bar(B_LR0 + t), 1);
      mbar_init(bar(B_AR0 + t), 4);
      mbar_init(bar(B_OC0 + t), 4);
    }
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
    if (p.has_x) prefetch_tmap(&tx);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto slot_addr = [&](int r) { return base + OFF_RING + (r % NSLOTS) * SLOT; };

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_LOAD));
  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA
      mbar_expect_tx(bar(B_Q), nt * 2 * TILE);
      for (int t = 0; t < nt; ++t) {
        tma_load_4d(base + OFF_Q + t * 2 * TILE, &tq, bar(B_Q), 0, (m0 + t) * 128, h, b);
        tma_load_4d(base + OFF_Q + t * 2 * TILE + TILE, &tq, bar(B_Q), 64, (m0 + t) * 128, h, b);
      }
      int r = 0;
      bool ok = true;
      // one ring entry: wait until its slot is free, then issue its loads
      auto acquire = [&](int bytes) -> uint32_t {
        const int s = r % NSLOTS;
        if (!mbar_wait(bar(B_EMPTY0 + s), ((r / NSLOTS) & 1) ^ 1, abort_flag, kDevTimeoutMma)) {
          ok = false;
          return 0;
        }
        mbar_expect_tx(bar(B_FULL0 + s), bytes);
        return slot_addr(r);
      };
      auto load_block = [&](const CUtensorMap* m, int t, int i) {
        const uint32_t dst = acquire(SLOT);
        if (!ok) return;
        const int s = r % NSLOTS;
        if (!p.blk64) {
          const int j = lut_block(p, tile_row(t), i);
          tma_load_4d(dst, m, bar(B_FULL0 + s), 0, j * 128, h, b);
          tma_load_4d(dst + TILE, m, bar(B_FULL0 + s), 64, j * 128, h, b);
        } else {
          // two 64-row key blocks stacked into one 128-row block (64-row boxes;
          // the 128-byte swizzle follows the address, so the halves line up)
          const int32_t* row = tile_row(t);
          const int j0 = pair_block(p, row[2 * i]), j1 = pair_block(p, row[2 * i + 1]);
          tma_load_4d(dst, m, bar(B_FULL0 + s), 0, j0 * 64, h, b);
          tma_load_4d(dst + TILE / 2, m, bar(B_FULL0 + s), 0, j1 * 64, h, b);
          tma_load_4d(dst + TILE, m, bar(B_FULL0 + s), 64, j0 * 64, h, b);
          tma_load_4d(dst + TILE + TILE / 2, m, bar(B_FULL0 + s), 64, j1 * 64, h, b);
        }
        ++r;
      };
      for (int t = 0; t < nt && ok; ++t) load_block(&tk, t, 0);
      for (int i = 0; i < topk && ok; ++i) {
        for (int t = 0; t < nt && ok; ++t) {
          load_block(&tv, t, i);
          if (ok && i + 1 < topk) load_block(&tk, t, i + 1);
        }
      }
      if (ok && p.has_lowrank) {
        // epilogue operands: q_lr of each tile in one slot, C^T in the next
        uint32_t dst = acquire(nt * TILE);
        if (ok) {
          const int s = r % NSLOTS;
          for (int t = 0; t < nt; ++t) tma_load_4d(dst + t * TILE, &tqlr, bar(B_FULL0 + s), 0, (m0 + t) * 128, h, b);
          ++r;
        }
        if (ok) dst = acquire(TILE);
        if (ok) {
          tma_load_3d(dst, &tct, bar(B_FULL0 + r % NSLOTS), 0, 0, bh);
          ++r;
        }
      }
      if (p.has_x) {
        // x tile of each query block (this head's 128 columns) for the gate
        for (int t = 0; t < nt && ok; ++t) {
          const uint32_t dst = acquire(SLOT);
          if (!ok) break;
          const int s = r % NSLOTS;
          tma_load_4d(dst, &tx, bar(B_FULL0 + s), 0, (m0 + t) * 128, h, b);
          tma_load_4d(dst + TILE, &tx, bar(B_FULL0 + s), 64, (m0 + t) * 128, h, b);
          ++r;
        }
      }
      // drain: no TMA may still target shared memory when the CTA exits.  The
      // waits ignore the abort flag (on the abort path the copies already
      // issued must still land) and share one wall-time limit.
      const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
      bool drained = mbar_wait_until(bar(B_Q), 0, deadline);
      for (int n = max(0, r - NSLOTS); n < r && drained; ++n)
        drained = mbar_wait_until(bar(B_FULL0 + n % NSLOTS), (n / NSLOTS) & 1, deadline);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16_f32(128, 128, false, false);
      const uint32_t id_pv = idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_wait(bar(B_Q), 0, abort_flag, kDevTimeoutLoad);
      int r = 0;
      // next ring entry (consumption order = load order)
      auto pop = [&]() -> int {
        const int s = r % NSLOTS;
        if (!mbar_wait(bar(B_FULL0 + s), (r / NSLOTS) & 1, abort_flag, kDevTimeoutLoad)) {
          ok = false;
          return -1;
        }
        tc_fence_after();
        return r++;
      };
      auto issue_s = [&](int t) {
        const int e = pop();
        if (e < 0) return;
        const uint32_t sq = base + OFF_Q + t * 2 * TILE;
        const uint32_t sk = slot_addr(e);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * TILE + (kk & 3) * 32;
          mma_bf16_ss(tmem + 128 * t, sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), id_qk,
                      kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(B_EMPTY0 + e % NSLOTS));
        mma_commit(bar(B_SF0 + t));
      };
      for (int t = 0; t < nt && ok; ++t) issue_s(t);
      for (int i = 0; i < topk && ok; ++i) {
        for (int t = 0; t < nt && ok; ++t) {
          if (!mbar_wait(bar(B_OC0 + t), i & 1, abort_flag, kDevTimeoutSoftmax)) {
            ok = false;
            break;
          }
          const int e = pop();
          if (e < 0) break;
          const uint32_t sv = slot_addr(e);
          // P V in the order the softmax hands P over: the K steps of chunk c
          // (32 keys) start as soon as that chunk is in TMEM, so most of P V
          // runs under the softmax's exp2 work instead of after it
          for (int c = 0; c < PCHUNKS && ok; ++c) {
            if (!mbar_wait(bar(B_PF0 + PCHUNKS * t + c), i & 1, abort_flag, kDevTimeoutSoftmax)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int k2 = 0; k2 < 2; ++k2) {
              // A = P from TMEM (16 bf16 of K = 8 packed columns per step), B = V (MN-major)
              const int kk = 2 * c + k2;
              mma_bf16_ts(tmem + 256 + 128 * t, tmem + 128 * t + kk * 8, sdesc_sw128(sv + kk * 2048, TILE, 1024),
                          id_pv, (i > 0 || kk > 0) ? 1u : 0u);
            }
          }
          if (!ok) break;
          mma_commit(bar(B_EMPTY0 + e % NSLOTS));
          if (i + 1 < topk) {
            issue_s(t);  // overwrites P_t(i) in TMEM after P_t(i) V_t(i) in issue order
          } else {
            mma_commit(bar(B_OF0 + t));
          }
        }
      }
      if (ok && p.has_lowrank) {
        const int e0 = pop();
        const int e1 = ok ? pop() : -1;
        if (ok) {
          for (int t = 0; t < nt; ++t) {
            // o_lr = q_lr . C into the (now free) S columns of tile t
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              mma_bf16_ss(tmem + 128 * t, sdesc_sw128(slot_addr(e0) + t * TILE + kk * 32, 16, 1024),
                          sdesc_sw128(slot_addr(e1) + kk * 32, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
            }
            mma_commit(bar(B_LR0 + t));
          }
        }
      }
      // every MMA issued has completed before TMEM is freed, also on the abort
      // path (where mbar_wait would return at once): bounded, ignores the flag
      mma_commit(bar(B_DRAIN));
      mbar_wait_until(bar(B_DRAIN), 0, globaltimer_ns() + kWaitLimitNs);
    }
  }
  } else if (warp >= 12) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CORR));
    // ------------------------------------------------------------ correction
    // O rescale of both tiles, off the softmax's critical path: once a tile's
    // softmax has published the row factors of block i (right after the row
    // max), scale its O in TMEM while that softmax computes P.  O is stable:
    // the last P V of the tile completed before its S of block i.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const float* s_alpha = reinterpret_cast<const float*>(gbase + OFF_ALPHA);
    bool ok = true;
    for (int i = 0; i < topk && ok; ++i) {
      for (int t = 0; t < nt && ok; ++t) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar(B_AR0 + t), i & 1, abort_flag, kDevTimeoutSoftmax))) {
          ok = false;
          break;
        }
        const float alpha = s_alpha[t * 128 + row];
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
          tc_fence_after();
          const uint32_t tO = tmem + 256 + 128 * t + ((uint32_t)(q * 32) << 16);
          const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t ov[64];
            tmem_ld32(tO + h2 * 64, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
            tmem_ld32(tO + h2 * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              float o0, o1;
              f2_unpack(mul_f32x2(f2_pack(__uint_as_float(ov[2 * e]), __uint_as_float(ov[2 * e + 1])), a2), o0, o1);
              ov[2 * e] = __float_as_uint(o0);
              ov[2 * e + 1] = __float_as_uint(o1);
            }
            tmem_st32(tO + h2 * 64, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
            tmem_st32(tO + h2 * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
          }
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_OC0 + t));
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_SOFTMAX));
    // -------------------------------------------------------------- softmax
    const int t = (warp - 4) >> 2;  // tile of this warpgroup
    const int q = warp & 3;         // TMEM lane quadrant of this warp
    if (t < nt) {
      const int row = q * 32 + lane;
      const uint32_t lane_off = (uint32_t)(q * 32) << 16;
      const uint32_t tS = tmem + 128 * t + lane_off;
      const uint32_t tO = tmem + 256 + 128 * t + lane_off;
      const int32_t* lut_row = tile_row(t);
      const float scale = p.qk_scale;
      // the row's gate value (computed by the norm pass), loaded before the main
      // loop so that its latency is hidden behind it
      const int tok_row = (m0 + t) * 128 + row;
      const float gate_pref = (p.has_lowrank && !p.has_x && p.gate != nullptr && tok_row < p.L)
                                  ? bf2f(p.gate[((int64_t)b * p.L + tok_row) * p.H + h])
                                  : 0.f;
      // block 64: a tile's first key tiles may be entirely masked for this row
      // (blocks only the other query block selected), so the running max starts
      // finite: exp2(-inf - m) is then 0 instead of NaN, and the first real
      // block's rescale factor exp2(-FLT_MAX - m) is 0
      float m_run = p.blk64 ? -FLT_MAX : -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int i = 0; i < topk; ++i) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar(B_SF0 + t), i & 1, abort_flag, kDevTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // valid columns of each 64-column half of the key tile: past L (a partial
        // last block), or, block 64, every column of a key block this row's query
        // block did not select
        int valid_lo, valid_hi;
        if (!p.blk64) {
          const int valid = p.L - lut_block(p, lut_row, i) * 128;
          valid_lo = min(valid, 64);
          valid_hi = min(valid - 64, 64);
        } else {
          valid_lo = pair_valid(p, lut_row[2 * i], row >> 6);
          valid_hi = pair_valid(p, lut_row[2 * i + 1], row >> 6);
        }
        // the whole S row: four 32-column loads, one wait
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
        tmem_ld_wait();
        if (valid_lo < 64 || valid_hi < 64) {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            if (c >= valid_lo) v[c] = __float_as_uint(-INFINITY);
            if (c >= valid_hi) v[64 + c] = __float_as_uint(-INFINITY);
          }
        }
        // row max: 8 independent chains of three-input maxima
        float mx8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          mx8[k] = __uint_as_float(v[k]);
#pragma unroll
          for (int j = 0; j < 7; ++j)
            mx8[k] = max3f(mx8[k], __uint_as_float(v[k + 8 + 16 * j]), __uint_as_float(v[k + 16 + 16 * j]));
          mx8[k] = fmaxf(mx8[k], __uint_as_float(v[k + 120]));
        }
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
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
        // publish this row's O rescale factor to the correction warpgroup
        reinterpret_cast<float*>(gbase + OFF_ALPHA)[t * 128 + row] = rescale ? alpha : 1.0f;
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_AR0 + t));
        // P = exp2(s*scale - m), packed bf16 over the S columns (already in registers).
        // s*scale - m and the row sums run as packed fp32x2 operations (two
        // columns per instruction), the row sum in two independent pairs.
        // P goes to the MMA in chunks of 32 keys: chunk c is published (its
        // stores waited for, then one arrival per warp) once chunk c + 1 is
        // computed, so the wait costs no exp2 time.
        const uint64_t sc2 = f2_pack(scale, scale), nm2 = f2_pack(-m_use, -m_use);
        uint64_t rs2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
        auto publish_p = [&](int c) {
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_PF0 + PCHUNKS * t + c));
        };
        static_assert(PCHUNKS == 4, "P chunks are 32 keys");
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1;
            f2_unpack(fma_f32x2(f2_pack(__uint_as_float(v[32 * c + 2 * e]), __uint_as_float(v[32 * c + 2 * e + 1])),
                                sc2, nm2),
                      x0, x1);
            const float p0 = ex2_approx(x0);
            const float p1 = ex2_approx(x1);
            rs2[e & 1] = add_f32x2(rs2[e & 1], f2_pack(p0, p1));
            w[e] = pack_bf2(p0, p1);
          }
          if (c > 0) publish_p(c - 1);
          tmem_st16(tS + c * 16, w);
        }
        publish_p(3);
        float rsa, rsb, rsc, rsd;
        f2_unpack(rs2[0], rsa, rsb);
        f2_unpack(rs2[1], rsc, rsd);
        const float rs = (rsa + rsc) + (rsb + rsd);
        l_run = l_run * alpha + rs;
        m_run = m_use;
      }

      // ---------------------------------------------------------- epilogue
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_OF0 + t), 0, abort_flag, kDevTimeoutMma));
      bool lowrank = false;
      if (ok && p.has_lowrank)
        lowrank = __all_sync(0xffffffffu, mbar_wait(bar(B_LR0 + t), 0, abort_flag, kDevTimeoutMma));
      ok = ok && (lowrank || !p.has_lowrank);
      tc_fence_after();
      // Staging tile of the output: the Q tile of this tile is free once its
      // last MMAs completed (OF/LR above).  128 rows x 256 B, the 16-byte
      // chunk k of row r at chunk k ^ (r & 7) (conflict-free both ways).
      uint8_t* stage = gbase + OFF_Q + t * 2 * TILE;
      const bool staged = p.out != nullptr || p.peer_n > 0;
      if (ok) {
        const int tok = (m0 + t) * 128 + row;
        if (p.lse) p.lse[(int64_t)bh * p.lse_ld + tok] = tok < p.L ? m_run + log2f(l_run) : INFINITY;
        const float inv_l = 1.0f / l_run;
        const uint64_t il2 = f2_pack(inv_l, inv_l);
        // one pass over TMEM: the row's o_sparse and o_lr values, rounded to
        // bf16 as the reference materialises them, stay in registers as packed
        // pairs (64 + 64) for the statistics and the fused output
        uint32_t osp[64], lrp[64];
        float ss_os = 0.f, ss_lr = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t ov[16];
          tmem_ld16(tO + c * 16, ov);
          uint32_t lv[16];
          if (lowrank) tmem_ld16(tS + c * 16, lv);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            // o = acc / l as one fp32x2 multiply, rounded to bf16 by one packed
            // conversion; the squares rounded to bf16 by one bf16x2 multiply
            // (the product of two bf16 values is exact in fp32, so this is the
            // fp32 square rounded once)
            float a0, a1;
            f2_unpack(mul_f32x2(f2_pack(__uint_as_float(ov[2 * e]), __uint_as_float(ov[2 * e + 1])), il2), a0, a1);
            const uint32_t op = pack_bf2(a0, a1);
            osp[8 * c + e] = op;
            float q0, q1;
            unpack_bf2(mul_bf16x2(op, op), q0, q1);
            ss_os += q0;
            ss_os += q1;
            if (lowrank) {
              const uint32_t lp = pack_bf2(__uint_as_float(lv[2 * e]), __uint_as_float(lv[2 * e + 1]));
              lrp[8 * c + e] = lp;
              float l0, l1;
              unpack_bf2(lp, l0, l1);
              ss_lr = fmaf(l0, l0, ss_lr);
              ss_lr = fmaf(l1, l1, ss_lr);
            }
          }
        }
        float os_rms = 1.f, lr_scale = 0.f, gate = 0.f;
        if (lowrank) {
          const float os_mean = rbf(ss_os * (1.0f / 128.0f));
          const float os_mean_eps = rbf(os_mean + 1e-5f);
          os_rms = rbf(sqrtf(os_mean_eps));
          lr_scale = rsqrtf(ss_lr * (1.0f / 128.0f) + p.eps_lr);
          if (p.has_x) {
            // gate = bf16(sigmoid(bf16(bf16(x_h . w_g) + b_h))) from this row of the x tile
            // (fused_gate.py:97-114); the x tile is the last ring entry of this tile
            const int r_x = nt * 2 * topk + 2 + t;
            if (__all_sync(0xffffffffu, mbar_wait(bar(B_FULL0 + r_x % NSLOTS), (r_x / NSLOTS) & 1, abort_flag,
                                                  kDevTimeoutLoad))) {
              const uint8_t* xs = gbase + OFF_RING + (r_x % NSLOTS) * SLOT;
              const uint4* wg4 = reinterpret_cast<const uint4*>(p.gate_w);
              float acc = 0.f;
#pragma unroll
              for (int c16 = 0; c16 < 16; ++c16) {
                const int box = c16 >> 3, chunk = c16 & 7;
                const uint4 xv = *reinterpret_cast<const uint4*>(xs + box * TILE + row * 128 + ((chunk ^ (row & 7)) << 4));
                const uint4 wv = __ldg(wg4 + c16);
                const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  float x0, x1, w0, w1;
                  unpack_bf2(xa[e], x0, x1);
                  unpack_bf2(wa[e], w0, w1);
                  acc = fmaf(x0, w0, acc);
                  acc = fmaf(x1, w1, acc);
                }
              }
              const float logit = rbf(rbf(acc) + bf2f(p.gate_b[h]));
              gate = rbf(1.0f / (1.0f + expf(-logit)));
            } else {
              ok = false;  // no gate for these rows: store nothing (the error flag is set)
            }
          } else {
            gate = gate_pref;
          }
        }
        // fuse from registers (os / os_rms as a product with the row's
        // reciprocal: one division per row instead of one per element); the
        // fused row goes to the staging tile (stored out coalesced below),
        // o_sparse directly
        const float inv_rms = 1.0f / os_rms;
        const bool store = ok && tok < p.L;
        const int64_t orow = (int64_t)b * p.o_sB + (int64_t)h * p.o_sH + (int64_t)tok * p.o_sT;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t wo[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (lowrank) {
              float os0, os1, l0, l1;
              unpack_bf2(osp[8 * c + e], os0, os1);
              unpack_bf2(lrp[8 * c + e], l0, l1);
              f2_unpack(mul_f32x2(f2_pack(l0, l1), f2_pack(lr_scale, lr_scale)), l0, l1);
              rbf2(l0, l1);
              // (os / os_rms + gate * l) * os_rms with os / os_rms as os * (1 / os_rms)
              const uint64_t u = fma_f32x2(f2_pack(os0, os1), f2_pack(inv_rms, inv_rms),
                                           mul_f32x2(f2_pack(gate, gate), f2_pack(l0, l1)));
              float r0, r1;
              f2_unpack(mul_f32x2(u, f2_pack(os_rms, os_rms)), r0, r1);
              wo[e] = pack_bf2(r0, r1);
            } else {
              wo[e] = osp[8 * c + e];
            }
          }
          if (staged && ok) {
            *reinterpret_cast<uint4*>(stage + row * 256 + (((2 * c) ^ (row & 7)) << 4)) =
                make_uint4(wo[0], wo[1], wo[2], wo[3]);
            *reinterpret_cast<uint4*>(stage + row * 256 + (((2 * c + 1) ^ (row & 7)) << 4)) =
                make_uint4(wo[4], wo[5], wo[6], wo[7]);
          }
          if (p.o_sparse && store) {
            uint4* dst = reinterpret_cast<uint4*>(p.o_sparse + orow + c * 16);
            dst[0] = make_uint4(osp[8 * c + 0], osp[8 * c + 1], osp[8 * c + 2], osp[8 * c + 3]);
            dst[1] = make_uint4(osp[8 * c + 4], osp[8 * c + 5], osp[8 * c + 6], osp[8 * c + 7]);
          }
        }
      }
      if (staged) {
        // coalesced store of the tile: 16 lanes per row, 2 rows per warp
        // instruction; rows of a warp whose epilogue did not run are skipped.
        // Every warp of the warpgroup reaches the named barrier (no early exit).
        int* ok_flags = reinterpret_cast<int*>(gbase + OFF_BAR + 8 * B_COUNT + 16);
        if (lane == 0) ok_flags[t * 4 + q] = ok ? 1 : 0;
        asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");
        const int tid = q * 32 + lane;
        const int chunk = tid & 15;
#pragma unroll 4
        for (int it = 0; it < 16; ++it) {
          const int r = it * 8 + (tid >> 4);
          const int tk = (m0 + t) * 128 + r;
          if (tk >= p.L || ok_flags[t * 4 + (r >> 5)] == 0) continue;
          const uint4 val = *reinterpret_cast<const uint4*>(stage + r * 256 + ((chunk ^ (r & 7)) << 4));
          __nv_bfloat16* dst;
          if (p.peer_n > 0) {
            // head->sequence exchange: the row goes straight to the rank that owns token tk
            const int owner = tk / p.peer_Ls;
            dst = p.out_peer[owner] + (int64_t)b * p.peer_sB + (int64_t)(tk - owner * p.peer_Ls) * p.peer_sT +
                  (int64_t)(p.head_offset + h) * 128;
          } else {
            dst = p.out + (int64_t)b * p.o_sB + (int64_t)h * p.o_sH + (int64_t)tk * p.o_sT;
          }
          *reinterpret_cast<uint4*>(dst + chunk * 8) = val;
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
                       const CUtensorMap& tct, const CUtensorMap& tx, const AttnParams& p, cudaStream_t s) {
  using namespace attn;
  // setmaxnreg redistributes the block's launch registers; refuse to launch if
  // the compiled kernel holds fewer than the split needs (the increase would wait)
  static int launch_regs = -1;
  if (launch_regs < 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, sparse_attn_tcgen05) != cudaSuccess) return (int)cudaGetLastError();
    launch_regs = fa.numRegs;
  }
  if (launch_regs < LAUNCH_REGS) return -1;
  cudaFuncSetAttribute(sparse_attn_tcgen05, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  const int nqt = p.blk64 ? (p.NBq + 1) / 2 : p.NBq;  // 128-row query tiles
  dim3 grid((nqt + 1) / 2, p.B * p.H);
  sparse_attn_tcgen05<<<grid, THREADS, SMEM_BYTES, s>>>(tq, tk, tv, tqlr, tct, tx, p);
  return (int)cudaGetLastError();
}

}  // namespace rola
