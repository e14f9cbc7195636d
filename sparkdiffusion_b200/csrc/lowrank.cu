// Low-rank correction branch: lr = RoPE_rank(bf16(SiLU(bf16(x . P^T)))) for the
// pre-RoPE normed q and k, and C = bf16(k_lr^T . v) per (batch, head).
//
// Restates `_proj_silu_rope_kernel` (sparkdiffusion/ops/fused_kernel/
// fused_lowrank.py:31-152, HAS_NORM=False as called from
// networks/wan_rola_attention.py:432-439) and the cuBLAS `C = k_lr^T v`
// (fused_lowrank.py:355-358).  The product o_lr = q_lr . C is done inside the
// attention epilogue (attn.cu).
//
// These contractions are small (K = 128 or the 128-token block, N = rank), so
// they use warp-level mma.sync m16n8k16 with ldmatrix fragments.  C is summed
// over the sequence in fp32 partials, one per fixed chunk of kKvChunk 64-token
// tiles, that a second kernel adds in chunk order: C is deterministic,
// independent of the launch grid, hence the same for any number of GPUs.
#include "common.cuh"
#include "kernels.h"

namespace rola {

constexpr int kPadX = 128 + 8;  // padded row (elements) of 128-wide tiles
constexpr int kPadR = 64 + 8;   // padded row of the rank tile

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill rows past L
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// cos/sin of one rank pair of token t (identity past rope_dim or past L)
__device__ __forceinline__ float2 rope_cs(const LowrankParams& p, int t, int pair) {
  if (pair >= p.rope_dim || t >= p.L) return make_float2(1.f, 0.f);
  return make_float2(bf2f(p.cos[(int64_t)t * p.rope_dim + pair]), bf2f(p.sin[(int64_t)t * p.rope_dim + pair]));
}

// SiLU + rank-RoPE on one (even, odd) rank pair; returns packed bf16x2
__device__ __forceinline__ uint32_t silu_rope_pair(float l0, float l1, float2 cs, bool rotate) {
  // every bf16 rounding of the pair is one packed conversion (rbf2)
  float e = l0, o = l1;
  rbf2(e, o);                                           // bf16 linear output (fused_lowrank.py:97)
  e = e * __fdividef(1.0f, 1.0f + __expf(-e));          // silu in fp32, then bf16 (:99-102)
  o = o * __fdividef(1.0f, 1.0f + __expf(-o));
  if (rotate) {                                         // rotated pairs (:104-135)
    rbf2(e, o);
    const float c = cs.x, s = cs.y;
    float ec = e * c, os = o * s, es = e * s, oc = o * c;
    rbf2(ec, os);
    rbf2(es, oc);
    return pack_bf2(ec - os, es + oc);
  }
  return pack_bf2(e, o);
}

// q_lr = RoPE_rank(SiLU(q_normed . P^T)) -> [B*L, H, R]
//
// One CTA per (128-token tile, group of kQHeads heads), 8 warps of 16 tokens.
// The projection matrix is staged once per CTA and the tile's RoPE factors
// fetched once into registers; the q tiles of consecutive heads stream through
// a two-stage cp.async ring, so the next head's 32 KB load runs under this
// head's MMAs, SiLU/RoPE and store.  Per element the arithmetic is the same
// mma.sync sequence (k steps in order) and the same rounding points.
constexpr int kLrT = 128;   // tokens per tile
constexpr int kQHeads = 8;  // heads per CTA
constexpr int kQThreads = 256;

__device__ __forceinline__ void q_issue_tile(__nv_bfloat16* dst, const LowrankParams& p, int bh, int t0) {
  const int b = bh / p.H, h = bh % p.H;
  const __nv_bfloat16* base = p.x + (int64_t)b * p.x_sB + (int64_t)h * p.x_sH;
  for (int i = threadIdx.x; i < kLrT * 16; i += kQThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    const bool ok = t0 + r < p.L;
    cp_async16(smem_u32(dst + r * kPadX + c), base + (int64_t)(ok ? t0 + r : 0) * p.x_sT + c, ok);
  }
}

__global__ void __launch_bounds__(kQThreads, 2) lowrank_q_kernel(LowrankParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sX = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [2][128][136]
  __nv_bfloat16* sP = sX + 2 * kLrT * kPadX;                        // [64][136]
  __nv_bfloat16* sO = sP + 64 * kPadX;                              // q_lr of one head [128 t][72]
  const int t0 = blockIdx.x * kLrT;
  const int bh0 = blockIdx.y * kQHeads;
  const int nh = min(kQHeads, p.B * p.H - bh0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tig = lane & 3;
  q_issue_tile(sX, p, bh0, t0);
  for (int i = threadIdx.x; i < 64 * 16; i += kQThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    cp_async16(smem_u32(sP + r * kPadX + c), p.proj + r * 128 + c, true);
  }
  cp_async_commit();
  // this thread's RoPE factors (tokens 16*warp + g and + 8, rank pairs 4*nt + tig)
  float2 cs[2][8];
#pragma unroll
  for (int half = 0; half < 2; ++half)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) cs[half][nt] = rope_cs(p, t0 + warp * 16 + g + half * 8, nt * 4 + tig);
  for (int j = 0; j < nh; ++j) {
    const int bh = bh0 + j, b = bh / p.H, h = bh % p.H;
    if (j + 1 < nh) q_issue_tile(sX + ((j + 1) & 1) * kLrT * kPadX, p, bh + 1, t0);
    cp_async_commit();
    cp_async_wait_1();  // head j (and the projection) landed
    __syncthreads();
    const __nv_bfloat16* cX = sX + (j & 1) * kLrT * kPadX;
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a0, a1, a2, a3;
      {
        const int mi = lane >> 3;
        const int row = warp * 16 + (lane & 7) + (mi & 1) * 8;
        const int col = ks * 16 + (mi >> 1) * 8;
        ldsm_x4(smem_u32(cX + row * kPadX + col), a0, a1, a2, a3);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
        const int mi = lane >> 3;
        const int n = np * 16 + (lane & 7) + (mi >> 1) * 8;
        const int k = ks * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(sP + n * kPadX + k), b0, b1, b2, b3);
        mma16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int tl = warp * 16 + g + half * 8;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int r = nt * 8 + tig * 2;
        *reinterpret_cast<uint32_t*>(sO + tl * kPadR + r) =
            silu_rope_pair(acc[nt][half * 2], acc[nt][half * 2 + 1], cs[half][nt], (r >> 1) < p.rope_dim);
      }
    }
    __syncthreads();  // sO complete; every warp is done reading this q buffer
    // coalesced store: 8 threads per 128-byte token row of this head
    for (int i = threadIdx.x; i < kLrT * 8; i += kQThreads) {
      const int tl = i >> 3, c = (i & 7) * 8;
      const int t = t0 + tl;
      if (t < p.L)
        *reinterpret_cast<uint4*>(p.lr_out + ((int64_t)b * p.L + t) * p.H * 64 + h * 64 + c) =
            *reinterpret_cast<const uint4*>(sO + tl * kPadR + c);
    }
  }
  cp_async_wait_0();
}

// ---------------------------------------------------------------------------
// C partials: for each fixed chunk of kKvChunk 64-token tiles and each (b, h),
// sum over the chunk's tiles of k_lr^T v (fp32), tiles in order.
//
// Persistent: two CTAs of 8 warps per SM walk work items (chunk, b*H + h); the
// k_normed / v tiles of all of a CTA's items, with the tile's rows of the
// low-rank RoPE tables, stream through one double-buffered cp.async ring that
// runs across item boundaries, so no global load sits between a tile's MMAs.
// Per tile:
//   projection  k_lr[64 t][64 r]  : warp w -> tokens 16*(w%4), ranks 32*(w/4)
//   accumulation C[64 r][128 d]   : warp w -> ranks 16*(w%4), dims 64*(w/4)
// The item's sum goes to its chunk's partial; the partials are added in chunk
// order by lowrank_reduce_kernel, so C does not depend on the grid.
// ---------------------------------------------------------------------------
constexpr int kKvT = 64;                       // tokens per tile
constexpr int kKvTile = kKvT * kPadX;          // elements of one padded [64 x 128] tile
constexpr int kKvStages = 2;
constexpr int kKvThreads = 256;
constexpr int kKvRope = kKvT * 32;             // elements of one tile's rows of a RoPE table (rope_dim <= 32)

// one ring stage: k and v tiles of token rows [t0, t0 + 64) of head (b, h), and
// the same rows of the cos / sin tables (flat, rope_dim per row)
__device__ __forceinline__ void kv_issue_tile(__nv_bfloat16* sXb, __nv_bfloat16* sVb, __nv_bfloat16* sCb,
                                              const LowrankParams& p, int b, int h, int t0) {
  const __nv_bfloat16* xb = p.x + (int64_t)b * p.x_sB + (int64_t)h * p.x_sH;
  const __nv_bfloat16* vb = p.v + (int64_t)b * p.v_sB + (int64_t)h * p.v_sH;
  for (int i = threadIdx.x; i < kKvT * 16; i += kKvThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    const bool ok = t0 + r < p.L;
    const int t = ok ? t0 + r : 0;
    cp_async16(smem_u32(sXb + r * kPadX + c), xb + (int64_t)t * p.x_sT + c, ok);
    cp_async16(smem_u32(sVb + r * kPadX + c), vb + (int64_t)t * p.v_sT + c, ok);
  }
  if (p.rope_dim > 0) {
    // rows t0.. of both tables are contiguous: (valid rows) * rope_dim * 2 bytes each,
    // copied in 16-byte pieces, the last one partial (zero filled)
    const int bytes = (min(kKvT, p.L - t0) * p.rope_dim) * 2;
    const int pieces = (bytes + 15) / 16;
    const uint8_t* cb = reinterpret_cast<const uint8_t*>(p.cos + (int64_t)t0 * p.rope_dim);
    const uint8_t* sb = reinterpret_cast<const uint8_t*>(p.sin + (int64_t)t0 * p.rope_dim);
    for (int i = threadIdx.x; i < 2 * pieces; i += kKvThreads) {
      const int k = i < pieces ? i : i - pieces;
      const uint8_t* src = (i < pieces ? cb : sb) + 16 * k;
      const int n = min(16, bytes - 16 * k);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                       smem_u32(sCb + (i < pieces ? 0 : kKvRope) + 8 * k)),
                   "l"(src), "r"(n)
                   : "memory");
    }
  }
}

// position in this CTA's tile sequence: item (chunk * BH + bh) and tile within the chunk
struct KvCursor {
  int item, j;
};

__global__ void __launch_bounds__(kKvThreads, 2) lowrank_kv_kernel(LowrankParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sX = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [kKvStages][64][136]
  __nv_bfloat16* sV = sX + kKvStages * kKvTile;                     // [kKvStages][64][136]
  __nv_bfloat16* sC = sV + kKvStages * kKvTile;                     // [kKvStages][cos, sin][64 * rope_dim]
  __nv_bfloat16* sP = sC + kKvStages * 2 * kKvRope;                 // [64][136]
  __nv_bfloat16* sK = sP + 64 * kPadX;                              // k_lr [64 t][72]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int BH = p.B * p.H;
  const int ntiles = (p.L + kKvT - 1) / kKvT;
  const int nchunks = (ntiles + kKvChunk - 1) / kKvChunk;
  const int items = nchunks * BH;
  auto chunk_tiles = [&](int item) { return min(kKvChunk, ntiles - (item / BH) * kKvChunk); };
  auto advance = [&](KvCursor& c) {
    if (++c.j == chunk_tiles(c.item)) {
      c.j = 0;
      c.item += gridDim.x;
    }
  };
  auto issue = [&](const KvCursor& c, int slot) {
    const int bh = c.item % BH;
    kv_issue_tile(sX + slot * kKvTile, sV + slot * kKvTile, sC + slot * 2 * kKvRope, p, bh / p.H, bh % p.H,
                  ((c.item / BH) * kKvChunk + c.j) * kKvT);
  };
  KvCursor ld{(int)blockIdx.x, 0}, cur{(int)blockIdx.x, 0};
  // the projection matrix, then the first kKvStages - 1 tiles (one group each)
  for (int i = threadIdx.x; i < 64 * 16; i += kKvThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    cp_async16(smem_u32(sP + r * kPadX + c), p.proj + r * 128 + c, true);
  }
  for (int s = 0; s < kKvStages - 1; ++s) {
    if (ld.item < items) {
      issue(ld, s);
      advance(ld);
    }
    cp_async_commit();
  }
  float cacc[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) cacc[nt][e] = 0.f;
  const int pm = warp & 3, pn = warp >> 2;  // projection: m-tile, rank half
  for (int n = 0; cur.item < items; ++n) {
    if (ld.item < items) {
      issue(ld, (n + kKvStages - 1) % kKvStages);
      advance(ld);
    }
    cp_async_commit();
    asm volatile("cp.async.wait_group %0;" ::"n"(kKvStages - 1) : "memory");  // tile n landed
    __syncthreads();
    const int slot = n % kKvStages;
    const __nv_bfloat16* cX = sX + slot * kKvTile;
    const __nv_bfloat16* cV = sV + slot * kKvTile;
    const __nv_bfloat16* cC = sC + slot * 2 * kKvRope;
    const int chunk = cur.item / BH, bh = cur.item % BH;
    const int t0 = (chunk * kKvChunk + cur.j) * kKvT;
    // projection: 16 tokens x 32 ranks per warp, K = 128
    float acc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a0, a1, a2, a3;
      {
        const int mi = lane >> 3;
        const int row = pm * 16 + (lane & 7) + (mi & 1) * 8;
        const int col = ks * 16 + (mi >> 1) * 8;
        ldsm_x4(smem_u32(cX + row * kPadX + col), a0, a1, a2, a3);
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int mi = lane >> 3;
        const int nn = pn * 32 + np * 16 + (lane & 7) + (mi >> 1) * 8;
        const int k = ks * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(sP + nn * kPadX + k), b0, b1, b2, b3);
        mma16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int tl = pm * 16 + g + half * 8;
      const int t = t0 + tl;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int r = pn * 32 + nt * 8 + tig * 2;
        const int pair = r >> 1;
        uint32_t v = 0u;
        if (t < p.L) {
          // the RoPE factors of (t, pair) from the staged rows (identity past rope_dim)
          float2 cs = make_float2(1.f, 0.f);
          if (pair < p.rope_dim)
            cs = make_float2(bf2f(cC[tl * p.rope_dim + pair]), bf2f(cC[kKvRope + tl * p.rope_dim + pair]));
          v = silu_rope_pair(acc[nt][half * 2], acc[nt][half * 2 + 1], cs, pair < p.rope_dim);
        }
        *reinterpret_cast<uint32_t*>(sK + tl * kPadR + r) = v;
      }
    }
    __syncthreads();
    // C[r, d] += sum_t k_lr[t, r] v[t, d]; warp w: r in [16*(w%4), +16), d in [64*(w/4), +64)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a0, a1, a2, a3;
      {
        const int mi = lane >> 3;
        const int t = ks * 16 + (lane & 7) + (mi >> 1) * 8;
        const int r = pm * 16 + (mi & 1) * 8;
        ldsm_x4_t(smem_u32(sK + t * kPadR + r), a0, a1, a2, a3);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int mi = lane >> 3;
        const int t = ks * 16 + (lane & 7) + (mi & 1) * 8;
        const int d = pn * 64 + np * 16 + (mi >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(cV + t * kPadX + d), b0, b1, b2, b3);
        mma16816(cacc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(cacc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    if (cur.j + 1 == chunk_tiles(cur.item)) {
      // last tile of the item: its sum goes to the chunk's partial
      float* dst = p.c_partial + (((int64_t)chunk * BH + bh) * 64) * 128;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int d = pn * 64 + nt * 8 + tig * 2;
        const int r0 = pm * 16 + g;
        *reinterpret_cast<float2*>(dst + r0 * 128 + d) = make_float2(cacc[nt][0], cacc[nt][1]);
        *reinterpret_cast<float2*>(dst + (r0 + 8) * 128 + d) = make_float2(cacc[nt][2], cacc[nt][3]);
#pragma unroll
        for (int e = 0; e < 4; ++e) cacc[nt][e] = 0.f;
      }
    }
    advance(cur);
    __syncthreads();  // every warp is done with this slot (and sK) before they are refilled
  }
  cp_async_wait_0();
}

__global__ void lowrank_reduce_kernel(const float* __restrict__ part, int splits, int BH, int R,
                                      __nv_bfloat16* __restrict__ C, __nv_bfloat16* __restrict__ Ct) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per = (int64_t)R * 128;
  if (i >= (int64_t)BH * per) return;
  const int64_t bh = i / per;
  const int r = (int)((i % per) / 128), d = (int)(i % 128);
  float acc = 0.f;
  for (int s = 0; s < splits; ++s) acc += part[(int64_t)s * BH * per + i];
  const __nv_bfloat16 v = f2bf(acc);
  if (C) C[i] = v;
  if (Ct) Ct[bh * per + (int64_t)d * R + r] = v;
}

int launch_lowrank_q(const LowrankParams& p, cudaStream_t s) {
  const int smem = (2 * kLrT * kPadX + 64 * kPadX + kLrT * kPadR) * 2;
  cudaFuncSetAttribute(lowrank_q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((p.L + kLrT - 1) / kLrT, (p.B * p.H + kQHeads - 1) / kQHeads);
  lowrank_q_kernel<<<grid, kQThreads, smem, s>>>(p);
  return (int)cudaGetLastError();
}

int launch_lowrank_kv(const LowrankParams& p, cudaStream_t s) {
  const int smem = (2 * kKvStages * kKvTile + 2 * kKvStages * kKvRope + 64 * kPadX + kKvT * kPadR) * 2;
  cudaFuncSetAttribute(lowrank_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int items = lowrank_chunks(p.L) * p.B * p.H;
  const int grid = items < 2 * sms ? items : 2 * sms;  // two CTAs per SM
  lowrank_kv_kernel<<<grid, kKvThreads, smem, s>>>(p);
  return (int)cudaGetLastError();
}

int launch_lowrank_reduce(const float* c_partial, int splits, int BH, int R, __nv_bfloat16* C, __nv_bfloat16* Ct,
                          cudaStream_t s) {
  const int64_t total = (int64_t)BH * R * 128;
  lowrank_reduce_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(c_partial, splits, BH, R, C, Ct);
  return (int)cudaGetLastError();
}

}  // namespace rola
