// Internal kernel launchers of the RoLa B200 library (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rola {

// prologue.cu
constexpr int kMaxChunks = 8;  // destinations of the sequence->head exchange (ranks of one node)
struct NormRopeParams {
  const __nv_bfloat16* q_in;
  const __nv_bfloat16* k_in;
  const __nv_bfloat16* v_in;  // only read when v_dst[0] != nullptr
  int64_t ld_in;              // row stride (elements) of q_in/k_in/v_in
  const __nv_bfloat16* x;     // gate input [B*L, dim] (row stride ld_x) or nullptr
  int64_t ld_x;
  const __nv_bfloat16* norm_wq;  // [dim] or nullptr (no norm)
  const __nv_bfloat16* norm_wk;
  const float* cos_sin;          // [L, D] interleaved fp32, row t = token position t
  const __nv_bfloat16* gate_w;   // [D]
  const __nv_bfloat16* gate_b;   // [H] (already in the data dtype)
  // outputs (any may be nullptr)
  __nv_bfloat16* q_rope;  // [B*L, dim]
  __nv_bfloat16* k_rope;
  // q_normed / k_normed / v / gate go out in head chunks of heads_per_chunk heads:
  // chunk c of token t of batch b lands at
  //   qn_dst[c] + b*dst_sB + (dst_t0 + t)*heads_per_chunk*D + column within the chunk
  //   g_dst[c]  + b*(dst_sB/D) + (dst_t0 + t)*heads_per_chunk + head within the chunk
  // (a null entry 0 disables that output).  One chunk of H heads is the plain
  // token-major layout; p chunks into peers' buffers (dst_t0 = rank * L) is the
  // sequence->head exchange itself.
  __nv_bfloat16* qn_dst[kMaxChunks];
  __nv_bfloat16* kn_dst[kMaxChunks];
  __nv_bfloat16* v_dst[kMaxChunks];
  __nv_bfloat16* g_dst[kMaxChunks];
  int64_t dst_sB;
  int dst_t0;
  __nv_bfloat16* pooled_q;  // [B, H, NB, D]
  float* ksum;              // [B, NB, dim]
  const float* ssq;         // [B*L, ssq_ld] per-tile sums of squares (q tiles, then k tiles); needed to normalise
  int ssq_ld;
  int ssq_tile;             // columns per partial sum (256 from the QKV GEMM, 128 from row_ssq)
  int B, L, H, blk, NB;
  int heads_per_chunk;     // chunked output layout for the all-to-all send buffers (H: plain layout)
  int compact;             // small-footprint variant (3-token ring) that fits beside a QKV GEMM CTA
  float eps;
};
int launch_norm_rope_pool(const NormRopeParams& p, bool norm, bool rope, bool pool, cudaStream_t s);
// ssq[row, :] = sums of squares of q[row] and k[row] over 128-column tiles (q tiles, then k tiles)
int launch_row_ssq(const __nv_bfloat16* q, const __nv_bfloat16* k, int64_t ld, int64_t rows, int dim, float* ssq,
                   cudaStream_t s);

// select.cu ---------------------------------------------------------------
// Generic strided block pooling: element (b, h, t, d) of x sits at
// x + b*sB + h*sH + t*sT + d.  mode 0: out_bf16[b,h,m,:] = bf16(sum/nx) (with
// optional centre [B,H,D] subtracted and rounded per row); mode 1:
// out_f32[b,m,h*D+d] = fp32 block sums (no centre).
int launch_block_pool(const __nv_bfloat16* x, int64_t sB, int64_t sH, int64_t sT, int B, int H, int L, int blk,
                      const __nv_bfloat16* center, __nv_bfloat16* out_bf16, float* out_f32, cudaStream_t s);
// centre[b, c] = bf16(sum_m ksum[b, m, c] / L) (sequential over m)
int launch_center(const float* ksum, int B, int NB, int dim, int L, __nv_bfloat16* center, cudaStream_t s);
// scores[bh, m, j] = sum_d pq[bh, m, d] * pk[bh, j, d] (sequential fp32 FMA over d)
int launch_scores(const __nv_bfloat16* pq, const __nv_bfloat16* pk, int BH, int NBq, int NBk, float* scores,
                  cudaStream_t s);
// lut[bh, m, :] = top-k of scores[bh, m, :] (ties -> lower index), ascending int32
int launch_topk(const float* scores, int rows, int NBk, int k, int32_t* lut, cudaStream_t s);
// block size 64: per 128-row query tile, the union of its two query blocks' kept
// key blocks with selection masks: paired [BH, ceil(NBq/2), 2k + 1] int32
int launch_pair_blocks(const int32_t* lut, int BH, int NBq, int k, int NBk, int32_t* paired, cudaStream_t s);
// scores + top-k in one kernel (NBk <= 768; same results as launch_scores + launch_topk)
int launch_select_fused(const __nv_bfloat16* pq, const __nv_bfloat16* pk, int BH, int NBq, int NBk, int k,
                        int32_t* lut, cudaStream_t s);

// lowrank.cu --------------------------------------------------------------
struct LowrankParams {
  const __nv_bfloat16* x;  // q_normed or k_normed: element (b,h,t,d) at x + b*x_sB + h*x_sH + t*x_sT + d
  int64_t x_sB, x_sH, x_sT;
  const __nv_bfloat16* proj;  // [R, D]
  const __nv_bfloat16* cos;   // [L, rope_dim]
  const __nv_bfloat16* sin;
  const __nv_bfloat16* v;     // element (b,h,t,d) at v + b*v_sB + h*v_sH + t*v_sT + d
  int64_t v_sB, v_sH, v_sT;
  __nv_bfloat16* lr_out;      // q_lr: element (b,t,h,r) at lr_out + (b*L+t)*H*R + h*R + r
  float* c_partial;           // [lowrank_chunks(L), B*H, R, D]
  int B, L, H, R, rope_dim, splits;  // splits: unused by the kernels (the C reduction is persistent)
};
// C partials: one per chunk of kKvChunk 64-token tiles, [lowrank_chunks(L), B*H, R, D] fp32
constexpr int kKvChunk = 16;
inline int lowrank_chunks(int L) { return ((L + 63) / 64 + kKvChunk - 1) / kKvChunk; }
int launch_lowrank_q(const LowrankParams& p, cudaStream_t s);
int launch_lowrank_kv(const LowrankParams& p, cudaStream_t s);
// C[bh, r, d] and Ct[bh, d, r] (bf16) from the fp32 partials (sequential over the chunks)
int launch_lowrank_reduce(const float* c_partial, int splits, int BH, int R, __nv_bfloat16* C, __nv_bfloat16* Ct,
                          cudaStream_t s);

// gemm.cu -----------------------------------------------------------------
// out[M, N] (row stride ldo) = A[M, K] * W[N, K]^T (+ bias[N]), bf16 in/out, fp32 accumulate;
// ssq (optional) [M, N/256]: per-row sum of squares of the bf16 outputs of each 256-column tile
// side (optional): a compact norm-only pass (B = 1) that spare warps of the
// persistent GEMM run alongside the tensor-core work
// scale_a [M], scale_b [N] (both or neither): e4m3 operands (ta, tb over uint8), out = acc*scale_a*scale_b + bias
int launch_gemm_bf16(const CUtensorMap& ta, const CUtensorMap& tb, const __nv_bfloat16* bias, __nv_bfloat16* out,
                     int64_t ldo, float* ssq, int M, int N, int K, const NormRopeParams* side, cudaStream_t s,
                     const float* scale_a = nullptr, const float* scale_b = nullptr);
// the same product on pairs of SMs (256 x 256 tiles, tcgen05 cta_group::2); tb_half
// maps W with 128-row boxes (each CTA of a pair stages half of a W tile).  No side job.
int launch_gemm_bf16_2sm(const CUtensorMap& ta, const CUtensorMap& tb_half, const __nv_bfloat16* bias,
                         __nv_bfloat16* out, int64_t ldo, float* ssq, int M, int N, int K, cudaStream_t s);
// row-wise e4m3 quantization of a bf16 [M, K] matrix (row stride ld): scale[m] =
// amax_k|x|/448 + 1e-12 (fp32), xq = e4m3(bf16(x / bf16(scale))) (fp8_linear.py:51-61)
int launch_quantize_rows_e4m3(const __nv_bfloat16* x, int64_t ld, int M, int K, uint8_t* xq, float* scale,
                              cudaStream_t s);

// attn.cu -----------------------------------------------------------------
struct AttnParams {
  const int32_t* lut;  // [B*H, NBq, topk]
  const __nv_bfloat16* gate;  // [B*L, H] precomputed gate values, or nullptr
  const __nv_bfloat16* gate_w;  // [D] with has_x: the gate is computed from x tiles
  const __nv_bfloat16* gate_b;  // [H]
  int has_x;
  __nv_bfloat16* out;         // fused output, element (b,h,t,d) at out + b*o_sB + h*o_sH + t*o_sT + d (nullptr: skip)
  int64_t o_sB, o_sH, o_sT;
  __nv_bfloat16* o_sparse;    // optional, same layout as out
  // head->sequence exchange fused into the store (peer_n > 0, out unused): row t
  // of head h goes to rank owner = t / peer_Ls at
  //   out_peer[owner] + b*peer_sB + (t - owner*peer_Ls)*peer_sT + (head_offset + h)*D + d
  __nv_bfloat16* out_peer[kMaxChunks];
  int peer_n, peer_Ls, head_offset;
  int64_t peer_sB, peer_sT;
  int B, L, H, NBq, NBk, topk, has_lowrank;
  // block size 64 (blk64 = 1): lut is the paired table of launch_pair_blocks
  // (NBq, NBk count 64-token blocks; topk = k of the 64-block selection); the K
  // and V maps have 64-row boxes
  int blk64;
  float qk_scale;  // D^-1/2 * log2(e)
  float eps_lr;    // finfo(dtype).eps
  float rescale_threshold;  // log2 growth of the running max that triggers an O rescale (0 = always)
  // optional (training): base-2 log-sum-exp of each row, lse[bh * lse_ld + t] =
  // m + log2(l) in units of qk_scale, +inf on the padding rows t in [L, lse_ld)
  float* lse;
  int lse_ld;  // 128 * (number of 128-row query tiles)
};
int launch_sparse_attn(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tqlr,
                       const CUtensorMap& tct, const CUtensorMap& tx, const AttnParams& p, cudaStream_t s);

// attn_bwd.cu -------------------------------------------------------------
struct AttnBwdParams {
  const int32_t* lut;  // dq: [B*H, NQT, topk] (block 128) or the paired table [B*H, NQT, 2 topk + 1] (block 64)
  const int32_t* inv;  // dkdv: inverse table [B*H, NKT, inv_width] of launch_lut_invert
  int inv_width;
  const float* lse;    // [B*H, Lpad] base-2 log-sum-exp of the forward (+inf on padding rows)
  const float* delta;  // [B*H, Lpad] rowsum(dO * O)
  __nv_bfloat16* dq;   // gradients: element (b,h,t,d) at base + b*g_sB + h*g_sH + t*g_sT + d
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t g_sB, g_sH, g_sT;
  int B, L, H;
  int NBq, NBk;        // blocks of the selection (64- or 128-token)
  int NQT, NKT, Lpad;  // 128-row query / key tiles, Lpad = 128 * NQT
  int topk, blk64;
  float qk_scale;      // D^-1/2 * log2(e)
};
// delta[bh, t] = sum_d dO * O in fp32 (0 on t in [L, Lpad))
int launch_attn_bwd_delta(const __nv_bfloat16* o, int64_t o_sB, int64_t o_sH, int64_t o_sT, const __nv_bfloat16* dout,
                          int64_t d_sB, int64_t d_sH, int64_t d_sT, int B, int H, int L, int Lpad, float* delta,
                          cudaStream_t s);
// inverse of a selection lut [BH, NBq, topk]: per 128-row key tile the ascending list
// of the query blocks that selected it, count first; block 64 entries carry two
// selection bits (map: BH*NBq*NBk bytes of scratch; width >= NBq + 1)
int launch_lut_invert(const int32_t* lut, int BH, int NBq, int NBk, int topk, int blk64, uint8_t* map, int32_t* inv,
                      int width, cudaStream_t s);
// dq (query-stationary), then dk and dv (key-stationary); maps as the forward's (rows = block size)
int launch_attn_bwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                    const AttnBwdParams& p, cudaStream_t s);

}  // namespace rola
