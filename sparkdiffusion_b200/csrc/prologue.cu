// Prologue epilogue pass: full-width qk-RMSNorm, interleaved RoPE, block
// pooling of the roped q, block sums of the roped k (for the smooth-K centre)
// and the per-(token, head) gate.
//
// Restates the reference's `_epilogue_kernel` (sparkdiffusion/ops/fused_kernel/
// fused_qkv_rope.py:53-225), the q half of `mean_pool` (ops/fused_kernel/
// utils.py:19-82, as called at fused_sparse_attn.py:179) and the gate logits of
// `_gate_fusion_kernel` (ops/fused_kernel/fused_gate.py:97-114), in one pass
// over the projected rows so that q and k are read from HBM once.
//
// Layout: one CTA per (128-token block m, batch b); thread j owns the 8 hidden
// columns [8j, 8j+8) of every token of the block (16 threads per head), so
// every global access is a coalesced 16-byte vector.  Rows are walked in
// order, which fixes the fp32 summation order of the block sums (row 0 first).
#include "common.cuh"
#include "kernels.h"

namespace rola {



// Output offset of (batch b, token t, hidden column c) in the chunked layout
// [B][H / heads_per_chunk][L][heads_per_chunk * D]: one contiguous block per
// destination rank of the sequence->head all-to-all.  With heads_per_chunk == H
// this is the plain token-major [B, L, H*D] layout.
__device__ __forceinline__ int64_t out_offset(const NormRopeParams& p, int b, int t, int col) {
  const int chunk_cols = p.heads_per_chunk * 128;
  const int chunk = col / chunk_cols;
  return (int64_t)b * p.L * (p.H * 128) + (int64_t)chunk * p.L * chunk_cols + (int64_t)t * chunk_cols +
         (col - chunk * chunk_cols);
}
// same layout for the per-(token, head) gate: [B][H / heads_per_chunk][L][heads_per_chunk]
__device__ __forceinline__ int64_t gate_offset(const NormRopeParams& p, int b, int t, int h) {
  const int chunk = h / p.heads_per_chunk;
  return (int64_t)b * p.L * p.H + (int64_t)chunk * p.L * p.heads_per_chunk + (int64_t)t * p.heads_per_chunk +
         (h - chunk * p.heads_per_chunk);
}

__device__ __forceinline__ void load8(const __nv_bfloat16* src, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(src);
  unpack_bf2(u.x, v[0], v[1]);
  unpack_bf2(u.y, v[2], v[3]);
  unpack_bf2(u.z, v[4], v[5]);
  unpack_bf2(u.w, v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* dst, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf2(v[0], v[1]);
  u.y = pack_bf2(v[2], v[3]);
  u.z = pack_bf2(v[4], v[5]);
  u.w = pack_bf2(v[6], v[7]);
  *reinterpret_cast<uint4*>(dst) = u;
}

// block-wide sum of NV values per thread; `red` holds 2 * NV * 32 floats
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float* red, int parity) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
  }
  float* buf = red + parity * NV * 32;
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) buf[i * 32 + warp] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float s = 0.f;
    for (int w = 0; w < nwarps; ++w) s += buf[i * 32 + w];
    v[i] = s;
  }
}

template <bool NORM, bool ROPE, bool POOL>
__global__ void __launch_bounds__(640) norm_rope_pool_kernel(NormRopeParams p) {
  __shared__ float red[2 * 2 * 32];
  __shared__ float s_rstd[2][256];
  const int m = blockIdx.x, b = blockIdx.y;
  const int dim = p.H * 128;
  // the block is rounded up to whole warps; threads past H*16 only join the reductions
  const bool active = threadIdx.x < p.H * 16;
  const int j = active ? threadIdx.x : 0;
  const int col = j * 8;
  const int h = col >> 7, d0 = col & 127;
  const int t0 = m * p.blk;
  const int t1 = min(p.L, t0 + p.blk);
  const float inv_dim = 1.0f / (float)dim;
  // With the GEMM's per-tile sums of squares the norm needs no block reduction:
  // the rstd of every token of the block is computed up front.
  const bool use_ssq = NORM && p.ssq != nullptr;
  if (use_ssq) {
    const int nt = dim / 256, n = t1 - t0;
    for (int i = threadIdx.x; i < 2 * n; i += blockDim.x) {
      const int which = i / n, tl = i - which * n;
      const float* src = p.ssq + ((int64_t)b * p.L + t0 + tl) * p.ssq_ld + which * nt;
      float s = 0.f;
      for (int k = 0; k < nt; ++k) s += src[k];
      s_rstd[which][tl] = rsqrtf(s * inv_dim + p.eps);
    }
    __syncthreads();
  }

  float wq[8], wk[8];
  if (NORM) {
    load8(p.norm_wq + col, wq);
    load8(p.norm_wk + col, wk);
  }
  float gw[8];
  const bool gate = p.x != nullptr && p.gate_out != nullptr;
  if (gate) load8(p.gate_w + d0, gw);
  const float gbias = gate ? bf2f(p.gate_b[h]) : 0.f;

  float qs[8], ks[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) qs[i] = ks[i] = 0.f;

  // one token ahead in registers so its loads overlap this token's work
  float q[8], k[8], xv[8];
  auto load_tok = [&](int t, float (&qq)[8], float (&kk)[8], float (&xx)[8]) {
    const int64_t row = (int64_t)b * p.L + t;
    load8(p.q_in + row * p.ld_in + col, qq);
    load8(p.k_in + row * p.ld_in + col, kk);
    if (gate) load8(p.x + row * p.ld_x + col, xx);
  };
  if (t0 < t1) load_tok(t0, q, k, xv);
  int parity = 0;
#pragma unroll 1
  for (int t = t0; t < t1; ++t, parity ^= 1) {
    const int64_t row = (int64_t)b * p.L + t;
    float qn[8], kn[8], xn[8];
    if (t + 1 < t1) load_tok(t + 1, qn, kn, xn);
    if (!active) {
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = k[i] = 0.f;
    }
    if (p.v_out != nullptr && active) {
      float v[8];
      load8(p.v_in + row * p.ld_in + col, v);
      store8(p.v_out + out_offset(p, b, t, col), v);
    }
    if (NORM) {
      float rq, rk;
      if (use_ssq) {
        rq = s_rstd[0][t - t0];
        rk = s_rstd[1][t - t0];
      } else {
        float ss[2] = {0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ss[0] = fmaf(q[i], q[i], ss[0]);
          ss[1] = fmaf(k[i], k[i], ss[1]);
        }
        block_sum<2>(ss, red, parity);
        rq = rsqrtf(ss[0] * inv_dim + p.eps);
        rk = rsqrtf(ss[1] * inv_dim + p.eps);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        q[i] = rbf(rbf(q[i] * rq) * wq[i]);  // unit in bf16, then x weight in bf16
        k[i] = rbf(rbf(k[i] * rk) * wk[i]);
      }
      if (p.q_normed && active) store8(p.q_normed + out_offset(p, b, t, col), q);
      if (p.k_normed && active) store8(p.k_normed + out_offset(p, b, t, col), k);
    }
    if (ROPE) {
      const float4* cs = reinterpret_cast<const float4*>(p.cos_sin + (int64_t)t * 128 + d0);
      float qr[8], kr[8];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float4 c = cs[i];  // cos_a, sin_a, cos_b, sin_b
        const int e0 = 4 * i, e1 = 4 * i + 2;
        qr[e0] = rbf(q[e0] * c.x - q[e0 + 1] * c.y);
        qr[e0 + 1] = rbf(q[e0] * c.y + q[e0 + 1] * c.x);
        qr[e1] = rbf(q[e1] * c.z - q[e1 + 1] * c.w);
        qr[e1 + 1] = rbf(q[e1] * c.w + q[e1 + 1] * c.z);
        kr[e0] = rbf(k[e0] * c.x - k[e0 + 1] * c.y);
        kr[e0 + 1] = rbf(k[e0] * c.y + k[e0 + 1] * c.x);
        kr[e1] = rbf(k[e1] * c.z - k[e1 + 1] * c.w);
        kr[e1 + 1] = rbf(k[e1] * c.w + k[e1 + 1] * c.z);
      }
      if (p.q_rope && active) store8(p.q_rope + row * dim + col, qr);
      if (p.k_rope && active) store8(p.k_rope + row * dim + col, kr);
      if (POOL) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          qs[i] += qr[i];
          ks[i] += kr[i];
        }
      }
    }
    if (gate) {
      float g = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) g = fmaf(xv[i], gw[i], g);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) g += __shfl_xor_sync(0xffffffffu, g, o);  // 16 lanes of one head
      if ((j & 15) == 0 && active) {
        const float lin = rbf(g);
        const float logit = rbf(lin + gbias);
        p.gate_out[gate_offset(p, b, t, h)] = f2bf(1.0f / (1.0f + expf(-logit)));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      q[i] = qn[i];
      k[i] = kn[i];
      xv[i] = xn[i];
    }
  }
  if (POOL && active) {
    const float nx = (float)(t1 - t0);
    float pq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) pq[i] = __fdiv_rn(qs[i], nx);
    store8(p.pooled_q + (((int64_t)b * p.H + h) * p.NB + m) * 128 + d0, pq);
    float4* ko = reinterpret_cast<float4*>(p.ksum + ((int64_t)b * p.NB + m) * dim + col);
    ko[0] = make_float4(ks[0], ks[1], ks[2], ks[3]);
    ko[1] = make_float4(ks[4], ks[5], ks[6], ks[7]);
  }
}

int launch_norm_rope_pool(const NormRopeParams& p, bool norm, bool rope, bool pool, cudaStream_t s) {
  dim3 grid(p.NB, p.B);
  dim3 block((p.H * 16 + 31) / 32 * 32);
  if (norm && rope && pool) norm_rope_pool_kernel<true, true, true><<<grid, block, 0, s>>>(p);
  else if (norm && rope) norm_rope_pool_kernel<true, true, false><<<grid, block, 0, s>>>(p);
  else if (norm) norm_rope_pool_kernel<true, false, false><<<grid, block, 0, s>>>(p);
  else if (rope && pool) norm_rope_pool_kernel<false, true, true><<<grid, block, 0, s>>>(p);
  else if (rope) norm_rope_pool_kernel<false, true, false><<<grid, block, 0, s>>>(p);
  else return -1;
  return (int)cudaGetLastError();
}

}  // namespace rola
