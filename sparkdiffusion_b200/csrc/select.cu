// Block-mask selection: block mean pooling, smooth-K centre, pooled scores
// and top-k.
//
// Restates `mean_pool`/`compress_kernel` (sparkdiffusion/ops/fused_kernel/
// utils.py:19-82), the smooth-K centre `k.mean(dim=-2)` and the selection
// `pooled_q @ pooled_k^T` + `torch.topk` (ops/fused_kernel/
// fused_sparse_attn.py:179-198) with build-defined orders so that the LUT is
// bit-exact against the CPU oracle:
//   * block sums add rows sequentially (row 0 first), fp32;
//   * the centre adds block sums sequentially over blocks, then divides by L;
//   * a score is a chain of fp32 FMAs over d = 0..D-1 (bf16 products are exact);
//   * top-k keeps the k largest scores, ties toward the lower block index, and
//     writes the kept indices in ascending order as int32.
// All of these kernels are HBM/L2 bound integer-and-fp32 work on CUDA cores.
#include "common.cuh"
#include "kernels.h"

namespace rola {

// ---------------------------------------------------------------------------
// generic strided block pooling; one thread per (b, m, h, 8-column chunk)
// ---------------------------------------------------------------------------
__global__ void block_pool_kernel(const __nv_bfloat16* __restrict__ x, int64_t sB, int64_t sH, int64_t sT, int B,
                                  int H, int L, int blk, int NB, const __nv_bfloat16* __restrict__ center,
                                  __nv_bfloat16* __restrict__ out_bf16, float* __restrict__ out_f32) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * NB * H * 16;
  if (gid >= total) return;
  const int chunk = (int)(gid & 15);
  int64_t r = gid >> 4;
  const int h = (int)(r % H);
  r /= H;
  const int m = (int)(r % NB);
  const int b = (int)(r / NB);
  const int d0 = chunk * 8;
  const int t0 = m * blk, t1 = min(L, t0 + blk);
  float c[8];
  if (center) {
    const __nv_bfloat16* cp = center + ((int64_t)b * H + h) * 128 + d0;
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = bf2f(cp[i]);
  }
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const __nv_bfloat16* base = x + b * sB + h * sH + d0;
  for (int t = t0; t < t1; ++t) {
    uint4 u = *reinterpret_cast<const uint4*>(base + (int64_t)t * sT);
    float v[8];
    unpack_bf2(u.x, v[0], v[1]);
    unpack_bf2(u.y, v[2], v[3]);
    unpack_bf2(u.z, v[4], v[5]);
    unpack_bf2(u.w, v[6], v[7]);
    if (center) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = rbf(v[i] - c[i]);  // bf16(k - c), utils.py:46-50
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
  if (out_bf16) {
    const float nx = (float)(t1 - t0);
    uint4 u;
    u.x = pack_bf2(__fdiv_rn(acc[0], nx), __fdiv_rn(acc[1], nx));
    u.y = pack_bf2(__fdiv_rn(acc[2], nx), __fdiv_rn(acc[3], nx));
    u.z = pack_bf2(__fdiv_rn(acc[4], nx), __fdiv_rn(acc[5], nx));
    u.w = pack_bf2(__fdiv_rn(acc[6], nx), __fdiv_rn(acc[7], nx));
    *reinterpret_cast<uint4*>(out_bf16 + (((int64_t)b * H + h) * NB + m) * 128 + d0) = u;
  }
  if (out_f32) {
    float4* o = reinterpret_cast<float4*>(out_f32 + ((int64_t)b * NB + m) * H * 128 + h * 128 + d0);
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

int launch_block_pool(const __nv_bfloat16* x, int64_t sB, int64_t sH, int64_t sT, int B, int H, int L, int blk,
                      const __nv_bfloat16* center, __nv_bfloat16* out_bf16, float* out_f32, cudaStream_t s) {
  const int NB = (L + blk - 1) / blk;
  const int64_t total = (int64_t)B * NB * H * 16;
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  block_pool_kernel<<<(unsigned)blocks, threads, 0, s>>>(x, sB, sH, sT, B, H, L, blk, NB, center, out_bf16, out_f32);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// smooth-K centre from block sums
// ---------------------------------------------------------------------------
__global__ void center_kernel(const float* __restrict__ ksum, int B, int NB, int dim, int L,
                              __nv_bfloat16* __restrict__ center) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (c >= dim) return;
  const float* src = ksum + (int64_t)b * NB * dim + c;
  float acc = 0.f;
  for (int m = 0; m < NB; ++m) acc += src[(int64_t)m * dim];
  center[(int64_t)b * dim + c] = f2bf(__fdiv_rn(acc, (float)L));
}

int launch_center(const float* ksum, int B, int NB, int dim, int L, __nv_bfloat16* center, cudaStream_t s) {
  dim3 grid((dim + 255) / 256, B);
  center_kernel<<<grid, 256, 0, s>>>(ksum, B, NB, dim, L, center);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// pooled scores: 64x64 tile per CTA, 4x4 per thread, d-sequential FMA chains
// ---------------------------------------------------------------------------
constexpr int kSt = 64;
__global__ void __launch_bounds__(256) scores_kernel(const __nv_bfloat16* __restrict__ pq,
                                                     const __nv_bfloat16* __restrict__ pk, int NBq, int NBk,
                                                     float* __restrict__ scores) {
  extern __shared__ float scores_smem[];
  float (*sq)[kSt] = reinterpret_cast<float (*)[kSt]>(scores_smem);               // transposed: [d][m]
  float (*sk)[kSt] = reinterpret_cast<float (*)[kSt]>(scores_smem + 128 * kSt);  // [d][j]
  const int bh = blockIdx.z;
  const int m0 = blockIdx.x * kSt, j0 = blockIdx.y * kSt;
  const __nv_bfloat16* qb = pq + (int64_t)bh * NBq * 128;
  const __nv_bfloat16* kb = pk + (int64_t)bh * NBk * 128;
  for (int i = threadIdx.x; i < kSt * 128; i += blockDim.x) {
    const int r = i >> 7, d = i & 127;
    sq[d][r] = (m0 + r < NBq) ? bf2f(qb[(int64_t)(m0 + r) * 128 + d]) : 0.f;
    sk[d][r] = (j0 + r < NBk) ? bf2f(kb[(int64_t)(j0 + r) * 128 + d]) : 0.f;
  }
  __syncthreads();
  const int tm = (threadIdx.x >> 4) * 4;  // 16 x 16 threads, 4 x 4 each
  const int tj = (threadIdx.x & 15) * 4;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;
#pragma unroll 4
  for (int d = 0; d < 128; ++d) {
    const float4 qv = *reinterpret_cast<const float4*>(&sq[d][tm]);
    const float4 kv = *reinterpret_cast<const float4*>(&sk[d][tj]);
    const float qa[4] = {qv.x, qv.y, qv.z, qv.w};
    const float ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][c] = __fmaf_rn(qa[a], ka[c], acc[a][c]);
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int m = m0 + tm + a;
    if (m >= NBq) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int jj = j0 + tj + c;
      if (jj < NBk) scores[((int64_t)bh * NBq + m) * NBk + jj] = acc[a][c];
    }
  }
}

int launch_scores(const __nv_bfloat16* pq, const __nv_bfloat16* pk, int BH, int NBq, int NBk, float* scores,
                  cudaStream_t s) {
  dim3 grid((NBq + kSt - 1) / kSt, (NBk + kSt - 1) / kSt, BH);
  const int smem = 2 * 128 * kSt * (int)sizeof(float);
  cudaFuncSetAttribute(scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  scores_kernel<<<grid, 256, smem, s>>>(pq, pk, NBq, NBk, scores);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// top-k: one warp per row; k rounds of a warp arg-max over 64-bit keys
// (orderable score << 32 | ~index), so ties go to the lower index.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t orderable(float f) {
  if (f == 0.f) f = 0.f;  // -0 and +0 compare equal
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0u;  // NaN ranks last
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kTopkMaxPerLane = 64;  // NBk <= 2048
__global__ void __launch_bounds__(128) topk_kernel(const float* __restrict__ scores, int rows, int NBk, int k,
                                                   int32_t* __restrict__ lut) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* src = scores + (int64_t)warp * NBk;
  const int per = (NBk + 31) / 32;
  uint32_t key[kTopkMaxPerLane];
  uint64_t selected_lo = 0, selected_hi = 0;  // bit i: element lane + 32 i kept
#pragma unroll
  for (int i = 0; i < kTopkMaxPerLane; ++i) {
    const int j = lane + 32 * i;
    key[i] = (i < per && j < NBk) ? orderable(src[j]) : 0u;
  }
  for (int r = 0; r < k; ++r) {
    // local best: highest key, then lowest index (lowest i for this lane)
    uint64_t best = 0;
#pragma unroll
    for (int i = 0; i < kTopkMaxPerLane; ++i) {
      if (i >= per) break;
      const int j = lane + 32 * i;
      const bool taken = (i < 64) ? ((i < 32 ? (selected_lo >> i) : (selected_hi >> (i - 32))) & 1ull) : false;
      if (j < NBk && !taken) {
        const uint64_t cand = ((uint64_t)key[i] << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)j);
        best = cand > best ? cand : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    const uint32_t jbest = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu);
    if ((int)(jbest & 31) == lane) {
      const int i = (int)(jbest >> 5);
      if (i < 32) selected_lo |= 1ull << i;
      else selected_hi |= 1ull << (i - 32);
    }
  }
  // emit kept indices in ascending order
  int32_t* dst = lut + (int64_t)warp * k;
  int written = 0;
  for (int i = 0; i < per; ++i) {
    const bool kept = (i < 32 ? (selected_lo >> i) : (selected_hi >> (i - 32))) & 1ull;
    const uint32_t ballot = __ballot_sync(0xffffffffu, kept);
    if (kept) {
      const int pos = written + __popc(ballot & ((1u << lane) - 1u));
      dst[pos] = lane + 32 * i;
    }
    written += __popc(ballot);
  }
}

int launch_topk(const float* scores, int rows, int NBk, int k, int32_t* lut, cudaStream_t s) {
  if (NBk > 32 * kTopkMaxPerLane || k > NBk || k < 1) return -1;
  const int threads = 128;
  const int64_t blocks = ((int64_t)rows * 32 + threads - 1) / threads;
  topk_kernel<<<(unsigned)blocks, threads, 0, s>>>(scores, rows, NBk, k, lut);
  return (int)cudaGetLastError();
}


// ---------------------------------------------------------------------------
// fused scores + top-k: one CTA per (64 query blocks, batch*head).  The head's
// pooled K is staged in shared memory with a 65-word row stride (lane j reads
// key block j: 32 different rows, 32 different banks); each lane keeps the
// fp32 scores of its key blocks j = lane + 32 i for 4 query rows in registers,
// every score accumulated over d in order (the same FMA chain as
// scores_kernel), then the warp picks each row's top-k exactly as topk_kernel.
// ---------------------------------------------------------------------------
constexpr int kSelWords = 65;         // smem row stride of pooled K, 32-bit words
constexpr int kSelMaxNBk = 768;       // shared-memory bound of the fused kernel

template <int PER>
__device__ __forceinline__ void warp_topk_emit(const float (&acc)[PER], int per, int NBk, int k, int lane,
                                               int32_t* __restrict__ dst) {
  uint32_t key[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int j = lane + 32 * i;
    key[i] = (i < per && j < NBk) ? orderable(acc[i]) : 0u;
  }
  uint64_t taken = 0;  // bit i: element lane + 32 i kept
  for (int r = 0; r < k; ++r) {
    uint64_t best = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int j = lane + 32 * i;
      if (i < per && j < NBk && !((taken >> i) & 1ull)) {
        const uint64_t cand = ((uint64_t)key[i] << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)j);
        best = cand > best ? cand : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    const uint32_t jbest = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu);
    if ((int)(jbest & 31) == lane) taken |= 1ull << (jbest >> 5);
  }
  int written = 0;
  for (int i = 0; i < per; ++i) {
    const bool kept = (taken >> i) & 1ull;
    const uint32_t ballot = __ballot_sync(0xffffffffu, kept);
    if (kept) dst[written + __popc(ballot & ((1u << lane) - 1u))] = lane + 32 * i;
    written += __popc(ballot);
  }
}

// RW query rows per warp, 16 * RW per CTA (fewer when B*H is small, so that
// the grid still covers the SMs)
template <int PER, int RW>
__global__ void __launch_bounds__(512) select_fused_kernel(const __nv_bfloat16* __restrict__ pq,
                                                           const __nv_bfloat16* __restrict__ pk, int NBq, int NBk,
                                                           int k, int32_t* __restrict__ lut) {
  constexpr int ROWS = 16 * RW;
  extern __shared__ uint32_t sel_smem[];
  // pooled K padded with zero rows to 32 * PER rows, so the score loop runs
  // every column group of every lane with no branch in it
  const int per = (NBk + 31) / 32;
  uint32_t* sk = sel_smem;                                       // [32 * PER][65] words (bf16 pairs)
  uint32_t* sq = sel_smem + ((32 * PER * kSelWords + 3) & ~3);   // [ROWS][64] words, 16-byte aligned
  const int bh = blockIdx.y;
  const int m0 = blockIdx.x * ROWS;
  const uint4* kb = reinterpret_cast<const uint4*>(pk + (int64_t)bh * NBk * 128);
  // staging: eight 16-byte loads in flight per thread before their smem stores
  for (int i0 = threadIdx.x; i0 < NBk * 16; i0 += 8 * blockDim.x) {
    uint4 u[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = i0 + e * blockDim.x;
      u[e] = i < NBk * 16 ? kb[i] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = i0 + e * blockDim.x;
      if (i < NBk * 16) {
        uint32_t* d = sk + (i >> 4) * kSelWords + (i & 15) * 4;
        d[0] = u[e].x;
        d[1] = u[e].y;
        d[2] = u[e].z;
        d[3] = u[e].w;
      }
    }
  }
  for (int i = NBk * kSelWords + threadIdx.x; i < 32 * PER * kSelWords; i += blockDim.x) sk[i] = 0u;
  const uint4* qb = reinterpret_cast<const uint4*>(pq + (int64_t)bh * NBq * 128);
  for (int i = threadIdx.x; i < ROWS * 16; i += blockDim.x) {
    const int r = i >> 4;
    const uint4 u = (m0 + r < NBq) ? qb[(int64_t)m0 * 16 + i] : make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(sq)[i] = u;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const int rr0 = warp * RW;  // the RW query rows of this warp
    if (m0 + rr0 >= NBq) return;
    float acc[RW][PER];
#pragma unroll
    for (int a = 0; a < RW; ++a)
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[a][i] = 0.f;
#pragma unroll 2
    for (int w = 0; w < 64; ++w) {
      float q0[RW], q1[RW];
#pragma unroll
      for (int a = 0; a < RW; ++a) unpack_bf2(sq[(rr0 + a) * 64 + w], q0[a], q1[a]);
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int j = lane + 32 * i;  // rows past NBk are zero (their scores are never selected)
        float k0, k1;
        unpack_bf2(sk[j * kSelWords + w], k0, k1);
#pragma unroll
        for (int a = 0; a < RW; ++a) {
          acc[a][i] = __fmaf_rn(q0[a], k0, acc[a][i]);
          acc[a][i] = __fmaf_rn(q1[a], k1, acc[a][i]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < RW; ++a) {
      const int m = m0 + rr0 + a;
      if (m < NBq) warp_topk_emit<PER>(acc[a], per, NBk, k, lane, lut + ((int64_t)bh * NBq + m) * k);
    }
  }
}

int launch_select_fused(const __nv_bfloat16* pq, const __nv_bfloat16* pk, int BH, int NBq, int NBk, int k,
                        int32_t* lut, cudaStream_t s) {
  if (NBk > kSelMaxNBk || k < 1 || k > NBk) return -1;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  // rows per warp: 4 when the grid covers the SMs twice over, else fewer
  int rw = 4;
  while (rw > 1 && (int64_t)BH * ((NBq + 16 * rw - 1) / (16 * rw)) < 2 * sms) rw >>= 1;
  const int per = (NBk + 31) / 32;
  if (per > 20 && rw > 2) rw = 2;  // 4 x 24 accumulators per thread would spill
  dim3 grid((NBq + 16 * rw - 1) / (16 * rw), BH);
#define ROLA_SEL(P, RW)                                                                                   \
  do {                                                                                                    \
    const int smem = (((32 * (P) * kSelWords + 3) & ~3) + 16 * (RW) * 64) * 4;                          \
    cudaFuncSetAttribute(select_fused_kernel<P, RW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);  \
    select_fused_kernel<P, RW><<<grid, 512, smem, s>>>(pq, pk, NBq, NBk, k, lut);                         \
  } while (0)
#define ROLA_SEL_RW(P)            \
  do {                            \
    if (rw == 4) ROLA_SEL(P, 4);  \
    else if (rw == 2) ROLA_SEL(P, 2); \
    else ROLA_SEL(P, 1);          \
  } while (0)
  if (per <= 4) ROLA_SEL_RW(4);
  else if (per <= 8) ROLA_SEL_RW(8);
  else if (per <= 16) ROLA_SEL_RW(16);
  else if (per <= 20) ROLA_SEL_RW(20);
  else if (rw == 2) ROLA_SEL(24, 2);  // rw <= 2 here (no 4 x 24 instantiation)
  else ROLA_SEL(24, 1);
#undef ROLA_SEL_RW
#undef ROLA_SEL
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Block size 64: the attention kernel's 128-row query tiles hold two 64-token
// query blocks (2t, 2t + 1).  For each tile, the union of the two blocks' kept
// key blocks, ascending, padded with -1 to 2k entries, each entry carrying in
// bits 28-29 which of the two query blocks selected it (bit 28: block 2t, bit
// 29: block 2t + 1), preceded by the number of 128-column key tiles (pairs of
// union entries) the tile needs:
//   paired[bh][t] = { count, e_0, ..., e_{2k-1} }
// The LUT rows may be in any order (an injected LUT, e.g. the reference's).
// ---------------------------------------------------------------------------
__global__ void pair_blocks_kernel(const int32_t* __restrict__ lut, int BH, int NBq, int k, int NBk,
                                   int32_t* __restrict__ paired) {
  const int NT = (NBq + 1) / 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)BH * NT) return;
  const int bh = (int)(i / NT), t = (int)(i % NT);
  int32_t* out = paired + i * (2 * k + 1);
  int u = 0;  // union entries written so far (kept ascending by insertion)
  for (int half = 0; half < 2; ++half) {
    const int m = 2 * t + half;
    if (m >= NBq) break;
    const int32_t* row = lut + ((int64_t)bh * NBq + m) * k;
    for (int e = 0; e < k; ++e) {
      int j = row[e];
      if (j < 0 || j >= NBk) {
        set_device_error(kDevBadIndex);
        j = j < 0 ? 0 : NBk - 1;
      }
      const int32_t bit = 1 << (28 + half);
      int pos = 0;
      while (pos < u && (out[1 + pos] & 0x0fffffff) < j) ++pos;
      if (pos < u && (out[1 + pos] & 0x0fffffff) == j) {
        out[1 + pos] |= bit;
        continue;
      }
      for (int q = u; q > pos; --q) out[1 + q] = out[q];
      out[1 + pos] = j | bit;
      ++u;
    }
  }
  for (int q = u; q < 2 * k; ++q) out[1 + q] = -1;
  out[0] = (u + 1) / 2;
}

int launch_pair_blocks(const int32_t* lut, int BH, int NBq, int k, int NBk, int32_t* paired, cudaStream_t s) {
  const int64_t n = (int64_t)BH * ((NBq + 1) / 2);
  pair_blocks_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(lut, BH, NBq, k, NBk, paired);
  return (int)cudaGetLastError();
}

}  // namespace rola
