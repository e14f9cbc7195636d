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
// Layout: one CTA per (token block m, group of 8 heads, batch b); thread j
// owns 8 hidden columns of every token of the block (16 threads per head), so
// every global access is a coalesced 16-byte vector.  Rows are walked in
// order, which fixes the fp32 summation order of the block sums (row 0 first).
#include "common.cuh"
#include "kernels.h"

namespace rola {



// Destination of (batch b, token t, hidden column col) of a chunked output
// (see NormRopeParams): chunk = col / (heads_per_chunk * D).
__device__ __forceinline__ __nv_bfloat16* chunk_dst(__nv_bfloat16* const (&table)[kMaxChunks],
                                                    const NormRopeParams& p, int b, int t, int col) {
  const int chunk_cols = p.heads_per_chunk * 128;
  const int chunk = col / chunk_cols;
  return table[chunk] + (int64_t)b * p.dst_sB + (int64_t)(p.dst_t0 + t) * chunk_cols + (col - chunk * chunk_cols);
}
__device__ __forceinline__ __nv_bfloat16* gate_dst(const NormRopeParams& p, int b, int t, int h) {
  const int chunk = h / p.heads_per_chunk;
  return p.g_dst[chunk] + (int64_t)b * (p.dst_sB / 128) + (int64_t)(p.dst_t0 + t) * p.heads_per_chunk +
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

// ---------------------------------------------------------------------------
// Streaming pass.  One CTA per (token block m, group of 8 heads, batch b):
// thread j owns hidden columns [8 j, 8 j + 8) of the group (16 threads per
// head) for every token of the block.  The token rows of q, k (and v / x when
// needed) are streamed through a 4-token cp.async ring in shared memory;
// each thread reads back exactly the 16-byte chunks it copied, so the loop
// needs no block-wide barrier.  The full-width RMS statistics come from the
// per-tile sums of squares (QKV GEMM epilogue or row_ssq_kernel).
// ---------------------------------------------------------------------------
constexpr int kNormHeads = 8;                   // heads per CTA
constexpr int kNormThreads = kNormHeads * 16;   // 128
constexpr int kNormRing = 4;                    // tokens in flight (more, smaller CTAs beat a deeper ring)
constexpr int kNormRingCompact = 3;             // co-resident variant (fits beside a GEMM CTA)
constexpr int kNormRow = kNormHeads * 128 * 2;  // bytes of one tensor row segment (2 KB)

__device__ __forceinline__ void cp_async16_ca(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_grp() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_grp() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8]) {
  unpack_bf2(u.x, v[0], v[1]);
  unpack_bf2(u.y, v[2], v[3]);
  unpack_bf2(u.z, v[4], v[5]);
  unpack_bf2(u.w, v[6], v[7]);
}

__device__ __forceinline__ void named_bar_sync(int id) {
  asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory");
}

// Shared memory of one norm work item: the token ring plus [2][blk] rstd.
__host__ __device__ constexpr int norm_smem_bytes(int ring, int nslots, int blk, bool norm) {
  return ring * nslots * kNormRow + (norm ? 2 * blk * 4 : 0);
}

// One work item of the streaming pass: token block m, head group grp, batch b,
// run by 128 threads (j = 0..127, whole warps) that synchronise on the named
// barrier bar_id only, so the item can also run on spare warps of another
// kernel (the QKV GEMM).  nsm: norm_smem_bytes(RING, ...) of shared memory.
template <bool NORM, bool ROPE, bool POOL, int RING>
__device__ __forceinline__ void norm_block(const NormRopeParams& p, int m, int grp, int b, uint8_t* nsm, int j,
                                           int bar_id) {
  const int nslots = 2 + (p.v_dst[0] != nullptr) + (p.x != nullptr && p.g_dst[0] != nullptr);
  const int slot_bytes = nslots * kNormRow;
  float* s_rstd = reinterpret_cast<float*>(nsm + RING * slot_bytes);  // [2][blk]
  const int dim = p.H * 128;
  const int h = grp * kNormHeads + (j >> 4);
  const bool active = h < p.H;
  const int col = active ? h * 128 + (j & 15) * 8 : 0;
  const int d0 = (j & 15) * 8;
  const int t0 = m * p.blk;
  const int t1 = min(p.L, t0 + p.blk);
  const int n = t1 - t0;
  const bool has_v = p.v_dst[0] != nullptr;
  const bool gate = p.x != nullptr && p.g_dst[0] != nullptr;
  const uint32_t ring = smem_u32(nsm);
  auto issue = [&](int tl) {
    if (tl < n && active) {
      const int64_t row = (int64_t)b * p.L + t0 + tl;
      const uint32_t slot = ring + (tl % RING) * slot_bytes + j * 16;
      cp_async16_ca(slot, p.q_in + row * p.ld_in + col);
      cp_async16_ca(slot + kNormRow, p.k_in + row * p.ld_in + col);
      if (has_v) cp_async16_ca(slot + 2 * kNormRow, p.v_in + row * p.ld_in + col);
      if (gate) cp_async16_ca(slot + (2 + has_v) * kNormRow, p.x + row * p.ld_x + col);
    }
    cp_async_commit_grp();  // one group per token, empty past the block
  };
#pragma unroll
  for (int i = 0; i < RING; ++i) issue(i);
  if (NORM) {
    // rstd of every token of the block from the per-tile sums of squares
    // (the barrier first: the previous item of this thread group may still read s_rstd)
    named_bar_sync(bar_id);
    const int per = dim / p.ssq_tile;
    for (int i = j; i < 2 * n; i += kNormThreads) {
      const int which = i / n, tl = i - which * n;
      const float* src = p.ssq + ((int64_t)b * p.L + t0 + tl) * p.ssq_ld + which * per;
      float s = 0.f;
      for (int k = 0; k < per; ++k) s += src[k];
      s_rstd[which * p.blk + tl] = rsqrtf(s * (1.0f / (float)dim) + p.eps);
    }
    named_bar_sync(bar_id);
  }
  float wq[8], wk[8];
  if (NORM && active) {
    load8(p.norm_wq + col, wq);
    load8(p.norm_wk + col, wk);
  }
  float gw[8];
  if (gate && active) load8(p.gate_w + d0, gw);
  const float gbias = (gate && active) ? bf2f(p.gate_b[h]) : 0.f;
  float qs[8], ks[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) qs[i] = ks[i] = 0.f;

#pragma unroll 1
  for (int tl = 0; tl < n; ++tl) {
    cp_async_wait_grp<RING - 1>();  // this token's chunks have landed
    const int t = t0 + tl;
    const int64_t row = (int64_t)b * p.L + t;
    const uint8_t* slot = nsm + (tl % RING) * slot_bytes + j * 16;
    float q[8], k[8], xv[8];
    unpack8(*reinterpret_cast<const uint4*>(slot), q);
    unpack8(*reinterpret_cast<const uint4*>(slot + kNormRow), k);
    uint4 vraw = make_uint4(0, 0, 0, 0);
    if (has_v) vraw = *reinterpret_cast<const uint4*>(slot + 2 * kNormRow);
    if (gate) unpack8(*reinterpret_cast<const uint4*>(slot + (2 + has_v) * kNormRow), xv);
    issue(tl + RING);  // refill the slot just read (own chunks only)
    if (!active) continue;
    if (has_v) *reinterpret_cast<uint4*>(chunk_dst(p.v_dst, p, b, t, col)) = vraw;
    if (NORM) {
      const float rq = s_rstd[tl], rk = s_rstd[p.blk + tl];
      // unit in bf16, then x weight in bf16; every bf16 rounding of a column
      // pair is one packed conversion, and the packed words are what is stored
      uint4 qn, kn;
      uint32_t* qw = reinterpret_cast<uint32_t*>(&qn);
      uint32_t* kw = reinterpret_cast<uint32_t*>(&kn);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float a0 = q[2 * i] * rq, a1 = q[2 * i + 1] * rq;
        float b0 = k[2 * i] * rk, b1 = k[2 * i + 1] * rk;
        rbf2(a0, a1);
        rbf2(b0, b1);
        qw[i] = pack_bf2(a0 * wq[2 * i], a1 * wq[2 * i + 1]);
        kw[i] = pack_bf2(b0 * wk[2 * i], b1 * wk[2 * i + 1]);
        unpack_bf2(qw[i], q[2 * i], q[2 * i + 1]);
        unpack_bf2(kw[i], k[2 * i], k[2 * i + 1]);
      }
      if (p.qn_dst[0]) *reinterpret_cast<uint4*>(chunk_dst(p.qn_dst, p, b, t, col)) = qn;
      if (p.kn_dst[0]) *reinterpret_cast<uint4*>(chunk_dst(p.kn_dst, p, b, t, col)) = kn;
    }
    if (ROPE) {
      const float4* cs = reinterpret_cast<const float4*>(p.cos_sin + (int64_t)t * 128 + d0);
      float qr[8], kr[8];
      uint4 qrp, krp;
      uint32_t* qrw = reinterpret_cast<uint32_t*>(&qrp);
      uint32_t* krw = reinterpret_cast<uint32_t*>(&krp);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float4 c = cs[i];  // cos_a, sin_a, cos_b, sin_b
        const int e0 = 4 * i, e1 = 4 * i + 2;
        qrw[2 * i] = pack_bf2(q[e0] * c.x - q[e0 + 1] * c.y, q[e0] * c.y + q[e0 + 1] * c.x);
        qrw[2 * i + 1] = pack_bf2(q[e1] * c.z - q[e1 + 1] * c.w, q[e1] * c.w + q[e1 + 1] * c.z);
        krw[2 * i] = pack_bf2(k[e0] * c.x - k[e0 + 1] * c.y, k[e0] * c.y + k[e0 + 1] * c.x);
        krw[2 * i + 1] = pack_bf2(k[e1] * c.z - k[e1 + 1] * c.w, k[e1] * c.w + k[e1 + 1] * c.z);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        unpack_bf2(qrw[i], qr[2 * i], qr[2 * i + 1]);
        unpack_bf2(krw[i], kr[2 * i], kr[2 * i + 1]);
      }
      if (p.q_rope) *reinterpret_cast<uint4*>(p.q_rope + row * dim + col) = qrp;
      if (p.k_rope) *reinterpret_cast<uint4*>(p.k_rope + row * dim + col) = krp;
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
      // the 16 lanes of one head (the other half-warp may be an absent head)
      const unsigned half = 0xffffu << (j & 16);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) g += __shfl_xor_sync(half, g, o);
      if ((j & 15) == 0) {
        const float lin = rbf(g);
        const float logit = rbf(lin + gbias);
        *gate_dst(p, b, t, h) = f2bf(1.0f / (1.0f + expf(-logit)));
      }
    }
  }
  cp_async_wait_grp<0>();
  if (POOL && active) {
    const float nx = (float)n;
    float pq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) pq[i] = __fdiv_rn(qs[i], nx);
    store8(p.pooled_q + (((int64_t)b * p.H + h) * p.NB + m) * 128 + d0, pq);
    float4* ko = reinterpret_cast<float4*>(p.ksum + ((int64_t)b * p.NB + m) * dim + col);
    ko[0] = make_float4(ks[0], ks[1], ks[2], ks[3]);
    ko[1] = make_float4(ks[4], ks[5], ks[6], ks[7]);
  }
}

template <bool NORM, bool ROPE, bool POOL, int RING>
__global__ void __launch_bounds__(kNormThreads) norm_stream_kernel(NormRopeParams p) {
  extern __shared__ __align__(16) uint8_t nsm[];
  norm_block<NORM, ROPE, POOL, RING>(p, blockIdx.x, blockIdx.y, blockIdx.z, nsm, threadIdx.x, 0);
}

// per-row sums of squares of q and k over tiles of 128 columns (q tiles, then k tiles)
__global__ void row_ssq_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, int64_t ld,
                               int64_t rows, int dim, float* __restrict__ ssq) {
  const int tiles = dim / 128;
  const int64_t gid = (int64_t)blockIdx.x * (blockDim.x / 16) + (threadIdx.x >> 4);  // (row, which, tile)
  const int sub = threadIdx.x & 15;
  if (gid >= rows * 2 * tiles) return;
  const int64_t row = gid / (2 * tiles);
  const int which = (int)((gid / tiles) % 2), tile = (int)(gid % tiles);
  const __nv_bfloat16* src = (which ? k : q) + row * ld + tile * 128 + sub * 8;
  float v[8];
  load8(src, v);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s = fmaf(v[i], v[i], s);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (sub == 0) ssq[row * 2 * tiles + which * tiles + tile] = s;
}

int launch_row_ssq(const __nv_bfloat16* q, const __nv_bfloat16* k, int64_t ld, int64_t rows, int dim, float* ssq,
                   cudaStream_t s) {
  const int64_t items = rows * 2 * (dim / 128);
  const int per_block = 256 / 16;
  row_ssq_kernel<<<(unsigned)((items + per_block - 1) / per_block), 256, 0, s>>>(q, k, ld, rows, dim, ssq);
  return (int)cudaGetLastError();
}

int launch_norm_rope_pool(const NormRopeParams& p, bool norm, bool rope, bool pool, cudaStream_t s) {
  if (norm && (p.ssq == nullptr || p.ssq_tile <= 0 || (p.H * 128) % p.ssq_tile != 0)) return -1;
  const int nslots = 2 + (p.v_dst[0] != nullptr) + (p.x != nullptr && p.g_dst[0] != nullptr);
  const int ring = p.compact ? kNormRingCompact : kNormRing;
  const int smem = norm_smem_bytes(ring, nslots, p.blk, norm);
  if (smem > 227 * 1024) return -1;
  dim3 grid(p.NB, (p.H + kNormHeads - 1) / kNormHeads, p.B);
#define ROLA_NORM(N, R, P, RING)                                                                          \
  do {                                                                                                    \
    cudaFuncSetAttribute(norm_stream_kernel<N, R, P, RING>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
    cudaFuncSetAttribute(norm_stream_kernel<N, R, P, RING>, cudaFuncAttributePreferredSharedMemoryCarveout,   \
                         cudaSharedmemCarveoutMaxShared);                                                 \
    norm_stream_kernel<N, R, P, RING><<<grid, kNormThreads, smem, s>>>(p);                                \
  } while (0)
  if (p.compact) {
    // the norm-only pass that runs beside the QKV GEMM of the next chunk
    if (!norm || rope || pool) return -1;
    ROLA_NORM(true, false, false, kNormRingCompact);
  } else if (norm && rope && pool) ROLA_NORM(true, true, true, kNormRing);
  else if (norm && rope) ROLA_NORM(true, true, false, kNormRing);
  else if (norm) ROLA_NORM(true, false, false, kNormRing);
  else if (rope && pool) ROLA_NORM(false, true, true, kNormRing);
  else if (rope) ROLA_NORM(false, true, false, kNormRing);
  else return -1;
#undef ROLA_NORM
  return (int)cudaGetLastError();
}

}  // namespace rola
