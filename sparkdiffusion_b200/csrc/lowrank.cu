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
// tiles, that a second kernel adds in chunk order: C is deterministic and the
// same for any number of CTA columns, so for any number of GPUs.
#include "common.cuh"
#include "kernels.h"

namespace rola {

constexpr int kLrT = 128;       // tokens per tile
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

// copy a [128 tokens x 128] bf16 tile of head h into padded smem, zeroing rows >= L;
// element (b,h,t,d) of src sits at src + b*sB + h*sH + t*sT + d
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int64_t sB, int64_t sH,
                                          int64_t sT, int b, int t0, int L, int h) {
  const __nv_bfloat16* base = src + (int64_t)b * sB + (int64_t)h * sH;
  for (int i = threadIdx.x; i < kLrT * 16; i += blockDim.x) {
    const int r = i >> 4, c = (i & 15) * 8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (t0 + r < L) u = *reinterpret_cast<const uint4*>(base + (int64_t)(t0 + r) * sT + c);
    *reinterpret_cast<uint4*>(dst + r * kPadX + c) = u;
  }
}

// Projection of 32 tokens (warp w: tokens 32w..32w+31 of the tile) onto rank 64:
// acc[mt][nt][4] in the m16n8 accumulator layout.
__device__ __forceinline__ void project_warp(const __nv_bfloat16* sX, const __nv_bfloat16* sP, float (&acc)[2][8][4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t a[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int mi = lane >> 3;
      const int row = warp * 32 + mt * 16 + (lane & 7) + (mi & 1) * 8;
      const int col = ks * 16 + (mi >> 1) * 8;
      ldsm_x4(smem_u32(sX + row * kPadX + col), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
    }
#pragma unroll
    for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
      const int mi = lane >> 3;
      const int n = np * 16 + (lane & 7) + (mi >> 1) * 8;
      const int k = ks * 16 + (mi & 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(sP + n * kPadX + k), b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        mma16816(acc[mt][2 * np], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b0, b1);
        mma16816(acc[mt][2 * np + 1], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b2, b3);
      }
    }
  }
}

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
__global__ void __launch_bounds__(128) lowrank_q_kernel(LowrankParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sX = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sP = sX + kLrT * kPadX;
  __nv_bfloat16* sO = sX;  // the q tile is dead after the projection: reuse it for q_lr [128 t][72]
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int t0 = blockIdx.x * kLrT;
  for (int i = threadIdx.x; i < 64 * 16; i += blockDim.x) {
    const int r = i >> 4, c = (i & 15) * 8;
    *reinterpret_cast<uint4*>(sP + r * kPadX + c) = *reinterpret_cast<const uint4*>(p.proj + r * 128 + c);
  }
  load_tile(sX, p.x, p.x_sB, p.x_sH, p.x_sT, b, t0, p.L, h);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tig = lane & 3;
  // this thread's RoPE factors, fetched before the MMAs so their latency hides
  float2 cs[2][2][8];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
        cs[mt][half][nt] = rope_cs(p, t0 + warp * 32 + mt * 16 + g + half * 8, nt * 4 + tig);
  __syncthreads();
  float acc[2][8][4];
  project_warp(sX, sP, acc);
  __syncthreads();  // every warp is done reading sX before it is overwritten
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int tl = warp * 32 + mt * 16 + g + half * 8;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int r = nt * 8 + tig * 2;
        *reinterpret_cast<uint32_t*>(sO + tl * kPadR + r) =
            silu_rope_pair(acc[mt][nt][half * 2], acc[mt][nt][half * 2 + 1], cs[mt][half][nt], (r >> 1) < p.rope_dim);
      }
    }
  __syncthreads();
  // coalesced store: 8 threads per 128-byte token row
  for (int i = threadIdx.x; i < kLrT * 8; i += blockDim.x) {
    const int tl = i >> 3, c = (i & 7) * 8;
    const int t = t0 + tl;
    if (t < p.L)
      *reinterpret_cast<uint4*>(p.lr_out + ((int64_t)b * p.L + t) * p.H * 64 + h * 64 + c) =
          *reinterpret_cast<const uint4*>(sO + tl * kPadR + c);
  }
}

// ---------------------------------------------------------------------------
// partial C = sum over this CTA's token tiles of k_lr^T v (fp32)
//
// 64-token tiles, 8 warps, k_normed/v tiles double-buffered with cp.async so
// the HBM stream of the next tile overlaps the two MMA phases of this one:
//   projection  k_lr[64 t][64 r]  : warp w -> tokens 16*(w%4), ranks 32*(w/4)
//   accumulation C[64 r][128 d]   : warp w -> ranks 16*(w%4), dims 64*(w/4)
// ---------------------------------------------------------------------------
constexpr int kKvT = 64;                       // tokens per tile
constexpr int kKvTile = kKvT * kPadX;          // elements of one padded [64 x 128] tile

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill rows past L
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void kv_issue_tile(__nv_bfloat16* sXb, __nv_bfloat16* sVb, const LowrankParams& p, int b,
                                              int h, int t0) {
  const __nv_bfloat16* xb = p.x + (int64_t)b * p.x_sB + (int64_t)h * p.x_sH;
  const __nv_bfloat16* vb = p.v + (int64_t)b * p.v_sB + (int64_t)h * p.v_sH;
  for (int i = threadIdx.x; i < kKvT * 16; i += blockDim.x) {
    const int r = i >> 4, c = (i & 15) * 8;
    const bool ok = t0 + r < p.L;
    const int t = ok ? t0 + r : 0;
    cp_async16(smem_u32(sXb + r * kPadX + c), xb + (int64_t)t * p.x_sT + c, ok);
    cp_async16(smem_u32(sVb + r * kPadX + c), vb + (int64_t)t * p.v_sT + c, ok);
  }
}

__global__ void __launch_bounds__(256, 2) lowrank_kv_kernel(LowrankParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sX = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [2][64][136]
  __nv_bfloat16* sV = sX + 2 * kKvTile;                             // [2][64][136]
  __nv_bfloat16* sP = sV + 2 * kKvTile;                             // [64][136]
  __nv_bfloat16* sK = sP + 64 * kPadX;                              // k_lr [64 t][72]
  const int split = blockIdx.x;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tig = lane & 3;
  for (int i = threadIdx.x; i < 64 * 16; i += blockDim.x) {
    const int r = i >> 4, c = (i & 15) * 8;
    *reinterpret_cast<uint4*>(sP + r * kPadX + c) = *reinterpret_cast<const uint4*>(p.proj + r * 128 + c);
  }
  float cacc[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) cacc[nt][e] = 0.f;

  // This CTA column owns the chunks split, split + splits, ... of kKvChunk
  // consecutive tiles; each chunk's sum goes to its own partial, so C's
  // summation order depends only on L (not on the number of CTA columns, which
  // follows the heads per GPU).
  const int ntiles = (p.L + kKvT - 1) / kKvT;
  const int nchunks = (ntiles + kKvChunk - 1) / kKvChunk;
  auto next_tile = [&](int t) {  // the tile this CTA processes after tile t (ntiles when done)
    if ((t + 1) % kKvChunk != 0 && t + 1 < ntiles) return t + 1;
    const int c = t / kKvChunk + p.splits;
    return c < nchunks ? c * kKvChunk : ntiles;
  };
  int tile = split < nchunks ? split * kKvChunk : ntiles;
  int buf = 0;
  if (tile < ntiles) kv_issue_tile(sX, sV, p, b, h, tile * kKvT);
  cp_async_commit();
  const int pm = warp & 3, pn = warp >> 2;  // projection: m-tile, rank half
  for (; tile < ntiles; tile = next_tile(tile), buf ^= 1) {
    const int next = next_tile(tile);
    if (next < ntiles) kv_issue_tile(sX + (buf ^ 1) * kKvTile, sV + (buf ^ 1) * kKvTile, p, b, h, next * kKvT);
    cp_async_commit();
    cp_async_wait_1();  // this tile has landed (the next may still be in flight)
    __syncthreads();
    const __nv_bfloat16* cX = sX + buf * kKvTile;
    const __nv_bfloat16* cV = sV + buf * kKvTile;
    const int t0 = tile * kKvT;
    float2 cs[2][4];  // this thread's RoPE factors, fetched before the MMAs
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) cs[half][nt] = rope_cs(p, t0 + pm * 16 + g + half * 8, pn * 16 + nt * 4 + tig);
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
        const int n = pn * 32 + np * 16 + (lane & 7) + (mi >> 1) * 8;
        const int k = ks * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(sP + n * kPadX + k), b0, b1, b2, b3);
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
        uint32_t v = 0u;
        if (t < p.L) v = silu_rope_pair(acc[nt][half * 2], acc[nt][half * 2 + 1], cs[half][nt], (r >> 1) < p.rope_dim);
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
    if ((tile + 1) % kKvChunk == 0 || tile + 1 == ntiles) {
      // last tile of a chunk: its sum goes to the chunk's partial
      float* dst = p.c_partial + (((int64_t)(tile / kKvChunk) * p.B * p.H + bh) * 64) * 128;
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
    __syncthreads();  // both tiles of this buffer consumed before it is refilled
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
  const int smem = (kLrT * kPadX + 64 * kPadX) * 2;
  cudaFuncSetAttribute(lowrank_q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((p.L + kLrT - 1) / kLrT, p.B * p.H);
  lowrank_q_kernel<<<grid, 128, smem, s>>>(p);
  return (int)cudaGetLastError();
}

int launch_lowrank_kv(const LowrankParams& p, cudaStream_t s) {
  const int smem = (4 * kKvTile + 64 * kPadX + kKvT * kPadR) * 2;
  cudaFuncSetAttribute(lowrank_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(p.splits, p.B * p.H);
  lowrank_kv_kernel<<<grid, 256, smem, s>>>(p);
  return (int)cudaGetLastError();
}

int launch_lowrank_reduce(const float* c_partial, int splits, int BH, int R, __nv_bfloat16* C, __nv_bfloat16* Ct,
                          cudaStream_t s) {
  const int64_t total = (int64_t)BH * R * 128;
  lowrank_reduce_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(c_partial, splits, BH, R, C, Ct);
  return (int)cudaGetLastError();
}

}  // namespace rola
