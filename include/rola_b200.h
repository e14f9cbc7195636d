/*
 * rola_b200.h -- C ABI of the B200 (sm_100a) RoLa attention forward.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to
 * bf16 (`void*`), fp32 (`float*`) or int32 data in the layout stated beside it,
 * every size is an integer, and `stream` is a cudaStream_t passed as void*.
 * Every entry point returns ROLA_OK (0) or an error code; the message of the
 * last error on the calling thread is available from rola_b200_last_error().
 * Nothing is launched when argument validation fails.  There is no CPU
 * fallback: every entry point launches CUDA kernels built for sm_100a.
 *
 * Shapes: B batch, L tokens, H heads, D = 128 head dim, dim = H*D,
 * blk block size, NB = ceil(L/blk), k = kept key blocks, R low-rank rank (64).
 * "token-major" = [B*L rows, row stride ld] with head h in columns
 * [h*D, h*D + D).  The reference's own layouts are noted per entry point.
 *
 * Reference = AlibabaResearch/SparkDiffusion, paths relative to its root.
 */
#ifndef ROLA_B200_H_
#define ROLA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* rola_stream_t;

#define ROLA_B200_ABI_VERSION 2
#define ROLA_PEER_HANDLE_BYTES 64

#define ROLA_OK 0
#define ROLA_ERR_INVALID 1 /* bad shape, size, alignment or null pointer */
#define ROLA_ERR_CUDA 2    /* a CUDA runtime/driver call or a launch failed */
#define ROLA_ERR_DEVICE 3  /* a kernel recorded a device-side error */

/* device-side error codes reported by rola_b200_device_status() */
#define ROLA_DEV_OK 0
#define ROLA_DEV_TIMEOUT_LOAD 1    /* a bounded wait for a TMA load expired */
#define ROLA_DEV_TIMEOUT_MMA 2     /* a bounded wait for an MMA completion expired */
#define ROLA_DEV_TIMEOUT_SOFTMAX 3 /* a bounded wait for the softmax hand-off expired */
#define ROLA_DEV_BAD_INDEX 4       /* a LUT entry outside [0, NB) (clamped) */

int rola_b200_abi_version(void);
const char* rola_b200_last_error(void);

/* Read (and optionally clear) the device-side error flag of the current device.
 * Synchronises the device.  Returns the ROLA_DEV_* code, or -1 on a CUDA error. */
int rola_b200_device_status(int clear);

/* Self-test of the device-side failure detection (no counterpart in the
 * reference).  Launches one thread that waits on an mbarrier nothing completes,
 * with a wall-time limit of limit_us microseconds (1 .. 1e6): the wait gives
 * up, records ROLA_DEV_TIMEOUT_LOAD in the device error flag and the kernel
 * returns.  Synchronises `stream`; returns ROLA_OK when the wait gave up as it
 * must.  Afterwards rola_b200_device_status() reports the code and the
 * context remains usable. */
int rola_b200_check_wait_timeout(unsigned limit_us, rola_stream_t stream);

/* (a4) QKV projection: out[M, N] (row stride N) = x[M, K] . w[N, K]^T + bias[N].
 * bias may be NULL.  N % 256 == 0, K % 64 == 0.  ssq (NULL to skip): fp32
 * [M, N/256], the sum of squares of each row's bf16 outputs per 256-column
 * tile, consumed by the qk-RMSNorm pass.
 * Replaces the three F.linear calls of fused_qkv_gemm_rope
 * (sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:287-289) with one GEMM over
 * the concatenated weight [Wq; Wk; Wv]. */
int rola_b200_qkv_gemm(const void* x, const void* w, const void* bias, void* out, float* ssq, int64_t M, int64_t N,
                       int64_t K, rola_stream_t stream);

/* (f1) Row-wise FP8 (e4m3) quantization of a bf16 [M, K] matrix with row
 * stride ld: scale[m] = max_k |x[m,k]| / 448 + 1e-12 (fp32) and
 * xq[m, k] = e4m3(bf16(x[m,k] / bf16(scale[m]))), xq dense [M, K] bytes.
 * K % 8 == 0.  For the activations per token, and (once) for the QKV weight
 * per output channel.
 * Replaces quantize_activation_rowwise / quantize_weight_rowwise
 * (sparkdiffusion/ops/quantization/fp8_linear.py:45-61). */
int rola_b200_quantize_rows_e4m3(const void* x, int64_t ld, int64_t M, int64_t K, void* xq, float* scale,
                                 rola_stream_t stream);

/* (f1) FP8 QKV projection: out[M, N] (bf16, row stride N) =
 * bf16((xq . wq^T)[m, n] * x_scale[m] * w_scale[n] + bias[n]), e4m3 operands
 * from rola_b200_quantize_rows_e4m3 (xq [M, K], wq [N, K]), fp32 accumulation.
 * bias may be NULL.  N % 256 == 0, K % 128 == 0.  ssq as rola_b200_qkv_gemm.
 * Replaces the three torch._scaled_mm calls of fused_qkv_gemm_rope's FP8 mode
 * (sparkdiffusion/ops/fused_kernel/fused_qkv_rope.py:270-285). */
int rola_b200_qkv_gemm_fp8(const void* xq, const float* x_scale, const void* wq, const float* w_scale,
                           const void* bias, void* out, float* ssq, int64_t M, int64_t N, int64_t K,
                           rola_stream_t stream);

/* (a4 epilogue, a5 q-pool, a6 block sums, a10 gate) in one pass over the rows.
 * q_raw/k_raw: token-major, row stride ld_raw.  ssq (optional): the
 * [B*L, ssq_ld] sums of squares written by rola_b200_qkv_gemm over the q|k|v
 * row (q tiles first, then k; H even); NULL computes the row statistics first in
 * stream-ordered scratch (cudaMallocAsync).  x: token-major [B*L, dim] (gate
 * input; NULL skips the gate).  norm_wq/norm_wk: [dim] (both NULL = no norm).
 * cos_sin: [L, D] fp32 interleaved (cos0, sin0, cos1, ...).  gate_w: [D],
 * gate_b: [H] bf16.  Outputs (any may be NULL): q_rope, k_rope, q_normed,
 * k_normed token-major [B*L, dim]; gate_out [B*L, H]; pooled_q [B, H, NB, D]
 * bf16; ksum [B, NB, dim] fp32 block sums of k_rope.
 * Replaces _epilogue_kernel (fused_qkv_rope.py:53-225, layout [B*H, L, D] there),
 * mean_pool(q) (utils.py:57-82 via fused_sparse_attn.py:179) and the gate
 * logits of _gate_fusion_kernel (fused_gate.py:97-114). */
int rola_b200_qk_norm_rope(const void* q_raw, const void* k_raw, int64_t ld_raw, const float* ssq, int ssq_ld,
                           const void* x, const void* norm_wq, const void* norm_wk, const float* cos_sin,
                           const void* gate_w, const void* gate_b, int B, int L, int H, int blk, float eps,
                           void* q_rope, void* k_rope, void* q_normed, void* k_normed, void* gate_out, void* pooled_q,
                           float* ksum, rola_stream_t stream);

/* Sequence-parallel half of the prologue epilogue (before the Ulysses
 * all-to-all): qk-RMSNorm and gate on a sequence shard of L tokens, writing
 * q_normed, k_normed and v into send buffers laid out
 * [B][H/heads_per_chunk][L][heads_per_chunk*D] and the gate as
 * [B][H/heads_per_chunk][L][heads_per_chunk] (per batch, one contiguous block
 * per destination rank).  Same reference interface as rola_b200_qk_norm_rope. */
int rola_b200_qk_norm_pack(const void* q_raw, const void* k_raw, const void* v_raw, int64_t ld_raw, const float* ssq,
                           int ssq_ld, const void* x, const void* norm_wq, const void* norm_wk, const void* gate_w,
                           const void* gate_b, int B, int L, int H, int heads_per_chunk, float eps, void* q_send,
                           void* k_send, void* v_send, void* gate_out, rola_stream_t stream);

/* One sequence->head scatter: qk_norm_pack with the exchange fused into its
 * stores.  The rows of heads [r*Hl, (r+1)*Hl) (Hl = H / world) of L tokens
 * per batch (B batches, rows token-major with stride ld_raw; ssq the QKV GEMM
 * sums, row stride ssq_ld) go straight into rank r's buffers q_dst[r],
 * k_dst[r], v_dst[r], each [B, dst_rows, Hl*D], at rows [dst_row0,
 * dst_row0 + L), and the gate into g_dst[r] [B, dst_rows, Hl].  A whole
 * sequence shard of rank rk is L = Ls, dst_rows = world*Ls, dst_row0 = rk*Ls;
 * a chunk of it (B = 1) shifts dst_row0.  The destinations are peer mappings
 * (rola_b200_peer_open); the rows are complete when the kernel completes, so a
 * stream-ordered barrier of all ranks after it makes them visible.
 * world <= ROLA_MAX_RANKS.  No counterpart in the reference, whose context
 * parallelism (sparkdiffusion/utils/a2a_cp.py:146-186) exchanges with NCCL
 * all-to-all. */
#define ROLA_MAX_RANKS 8
typedef struct rola_scatter_args {
  const void* q_raw;
  const void* k_raw;
  const void* v_raw;
  int64_t ld_raw;
  const float* ssq;
  int32_t ssq_ld;
  int32_t B;
  int32_t L;
  int32_t H;
  int32_t world;
  float eps;
  int64_t dst_rows;
  int64_t dst_row0;
  const void* x;
  const void* norm_wq;
  const void* norm_wk;
  const void* gate_w;
  const void* gate_b;
  void* q_dst[ROLA_MAX_RANKS];
  void* k_dst[ROLA_MAX_RANKS];
  void* v_dst[ROLA_MAX_RANKS];
  void* g_dst[ROLA_MAX_RANKS];
} rola_scatter_args;

/* The scatter as its own pass.  compact != 0 selects the small-footprint
 * kernel (3-token ring); 0 the 8-token ring. */
int rola_b200_qk_norm_scatter(const rola_scatter_args* args, int compact, rola_stream_t stream);

/* rola_b200_qkv_gemm on rows of this chunk while four spare warps of every
 * GEMM CTA run the scatter `side` of an earlier chunk (B == 1, ssq given):
 * the NVLink traffic of the exchange hides under the tensor-core work of the
 * next projection.  side == NULL: the same single-SM persistent GEMM with no
 * side job (rola_b200_qkv_gemm may pick the SM-pair kernel instead).  No
 * counterpart in the reference. */
int rola_b200_qkv_gemm_scatter(const void* x, const void* w, const void* bias, void* out, float* ssq, int64_t M,
                               int64_t N, int64_t K, const rola_scatter_args* side, rola_stream_t stream);

/* Head-parallel half (after the all-to-all): RoPE, q-pool and k block sums from
 * the normed q/k (token-major, row stride ld).  Same reference interface as
 * rola_b200_qk_norm_rope. */
int rola_b200_rope_pool(const void* q_normed, const void* k_normed, int64_t ld, const float* cos_sin, int B, int L,
                        int H, int blk, void* q_rope, void* k_rope, void* pooled_q, float* ksum,
                        rola_stream_t stream);

/* (a5) block mean pooling, mean_pool (sparkdiffusion/ops/fused_kernel/utils.py:57-82).
 * Element (b, h, t, d) of x sits at x + b*sB + h*sH + t*sT + d (elements).
 * center: [B, H, D] or NULL; out: [B, H, NB, D] bf16.  Rows are summed in order. */
int rola_b200_mean_pool(const void* x, int64_t sB, int64_t sH, int64_t sT, int B, int H, int L, int blk,
                        const void* center, void* out, rola_stream_t stream);

/* (a6) smooth-K centre, k.mean(dim=-2) (fused_sparse_attn.py:180): center [B, H, D] bf16.
 * ksum_ws: fp32 scratch of B*NB*H*D floats (block sums). */
int rola_b200_smooth_k_center(const void* k, int64_t sB, int64_t sH, int64_t sT, int B, int H, int L, int blk,
                              float* ksum_ws, void* center, rola_stream_t stream);

/* (a6) centre from precomputed block sums ksum [B, NB, dim]. */
int rola_b200_center_from_sums(const float* ksum, int B, int NB, int dim, int L, void* center,
                               rola_stream_t stream);

/* (a7) pooled scores (fp32) and top-k selection: pooled_q [BH, NBq, D],
 * pooled_k [BH, NBk, D] bf16 -> lut [BH, NBq, topk] int32 ascending, ties toward
 * the lower block index.  scores_ws: fp32 scratch of BH*NBq*NBk floats, used
 * only when NBk > 768 (below that the scores stay on chip; NULL is allowed).
 * Replaces `pooled_q @ pooled_k^T` + torch.topk (fused_sparse_attn.py:181-198). */
int rola_b200_block_select(const void* pooled_q, const void* pooled_k, int BH, int NBq, int NBk, int topk,
                           float* scores_ws, int32_t* lut, rola_stream_t stream);

/* Block size 64: per 128-row query tile t (query blocks 2t and 2t + 1 of a
 * 64-token selection lut [BH, NB, topk], rows in any order), the ascending
 * union of the two blocks' kept key blocks, padded with -1 to 2*topk entries,
 * bits 28 and 29 of each entry marking which of the two blocks selected it,
 * preceded by the number of 128-column key tiles (entry pairs) it needs:
 * paired [BH, ceil(NB/2), 2*topk + 1] int32, the lut of rola_b200_sparse_attn
 * with blk == 64.  No counterpart in the reference (its Triton kernel takes
 * 64-row query blocks directly, fused_sparse_attn.py:204-213). */
int rola_b200_pair_blocks(const int32_t* lut, int BH, int NB, int topk, int32_t* paired, rola_stream_t stream);

/* (a9) q_lr = RoPE_rank(SiLU(q_normed . proj_q^T)).  Element (b, h, t, d) of
 * q_normed sits at q_normed + sB*b + sH*h + sT*t + d (elements; 16-byte rows).
 * proj_q [R, D], lr_cos/lr_sin [L, rope_dim] bf16 -> q_lr [B*L, H*R] bf16.  R == 64.
 * Replaces _proj_silu_rope_kernel (sparkdiffusion/ops/fused_kernel/fused_lowrank.py:31-152). */
int rola_b200_lowrank_q(const void* q_normed, int64_t sB, int64_t sH, int64_t sT, const void* proj_q,
                        const void* lr_cos, const void* lr_sin, int rope_dim, int B, int L, int H, int R, void* q_lr,
                        rola_stream_t stream);

/* (a9) C = k_lr^T v per (b, h).  k_normed and v are strided views as in
 * rola_b200_lowrank_q (k_s* and v_s* strides) -> C [B*H, R, D] and
 * Ct [B*H, D, R] bf16 (either may be NULL).  c_partial_ws: fp32 scratch of
 * chunks*B*H*R*D floats, chunks = ceil(ceil(L/64)/16): one partial sum per
 * 1024 tokens, added in order, so C does not depend on the launch.  `splits`
 * (> 0) is accepted for ABI compatibility and ignored: the kernel runs
 * persistent CTAs, two per SM.  R == 64; lr_cos / lr_sin 16-byte aligned.
 * Replaces fused_lowrank.py:331-358 (k_lr projection + cuBLAS k_lr^T v). */
int rola_b200_lowrank_kv(const void* k_normed, int64_t k_sB, int64_t k_sH, int64_t k_sT, const void* v, int64_t v_sB,
                         int64_t v_sH, int64_t v_sT, const void* proj_k, const void* lr_cos, const void* lr_sin,
                         int rope_dim, int B, int L, int H, int R, int splits, float* c_partial_ws, void* C, void* Ct,
                         rola_stream_t stream);

/* (a8 + a9 o_lr + a10) block-sparse attention with the fused low-rank + gate
 * epilogue.  q and k share strides (qk_s*), v has its own (v_s*), out and
 * o_sparse share o_s*: element (b, h, t, d) at p + sB*b + sH*h + sT*t + d, all
 * strides multiples of 8 elements.  lut [B*H, NBq, topk] int32; q_lr [B*L, H*R]
 * and Ct [B*H, D, R] (both NULL: no low-rank branch and out = o_sparse).  The
 * gate is either given as values, gate [B*L, H] bf16, or computed in the
 * epilogue from the hidden states x (strided like q, x_s*) with gate_w [D] and
 * gate_b [H] bf16 (give one of gate / x; neither: gate 0).  out / o_sparse may
 * be NULL (not both).
 * blk == 128: lut is the selection [B*H, NB, topk].  blk == 64 (the
 * reference's default rola_blkq = rola_blkk = 64): lut is the paired table of
 * rola_b200_pair_blocks for the 64-token selection [B*H, NB64, topk]; each
 * 128-row query tile then attends to the union of its two blocks' key blocks,
 * every row only to its own block's.  R == 64.
 * Replaces _rola_fwd_kernel (fused_sparse_attn.py:55-144), the o_lr matmul
 * (fused_lowrank.py:360-362) and _gate_fusion_kernel (fused_gate.py:27-127). */
int rola_b200_sparse_attn(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT, const void* v,
                          int64_t v_sB, int64_t v_sH, int64_t v_sT, const int32_t* lut, int B, int L, int H, int blk,
                          int topk, const void* q_lr, const void* Ct, const void* gate, const void* x, int64_t x_sB,
                          int64_t x_sH, int64_t x_sT, const void* gate_w, const void* gate_b, float eps_lr, void* out,
                          void* o_sparse, int64_t o_sB, int64_t o_sH, int64_t o_sT, rola_stream_t stream);

/* rola_b200_sparse_attn with the head->sequence exchange fused into the
 * epilogue store: this rank computed heads [head_offset, head_offset + H) of
 * all L tokens; output row t goes to rank owner = t / (L / world), into
 * out_dst[owner] [B, L / world, H_total*D] at row t - owner*(L / world),
 * columns (head_offset + h)*D.  Gate values (gate [B*L, H]) and the low-rank
 * branch are required.  world <= 8 and divides L.  No counterpart in the
 * reference (see rola_b200_qk_norm_scatter). */
int rola_b200_sparse_attn_scatter(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT,
                                  const void* v, int64_t v_sB, int64_t v_sH, int64_t v_sT, const int32_t* lut, int B,
                                  int L, int H, int blk, int topk, const void* q_lr, const void* Ct, const void* gate,
                                  float eps_lr, void* const* out_dst, int world, int head_offset, int H_total,
                                  rola_stream_t stream);

/* (f4) Training forward of the block-sparse attention: out = the plain
 * attention output (no low-rank branch, no gate), plus lse [B*H, Lpad] fp32
 * (Lpad = 128 * ceil(L / 128)), the base-2 log-sum-exp of each row in units of
 * D^-1/2 log2(e) (+inf on the padding rows), which the backward reads.  Sizes,
 * strides and the lut convention (paired table for blk 64) as
 * rola_b200_sparse_attn.  Replaces the forward of the external SLA kernel the
 * reference trains with (`_attention.apply`, wan_rola_attention.py:320-321). */
int rola_b200_sparse_attn_fwd_lse(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT,
                                  const void* v, int64_t v_sB, int64_t v_sH, int64_t v_sT, const int32_t* lut, int B,
                                  int L, int H, int blk, int topk, void* out, int64_t o_sB, int64_t o_sH, int64_t o_sT,
                                  float* lse, rola_stream_t stream);

/* Bytes of device workspace rola_b200_sparse_attn_bwd needs (0 for bad sizes). */
size_t rola_b200_sparse_attn_bwd_workspace(int B, int L, int H, int blk);

/* (f4) Backward of the block-sparse attention: dq, dk, dv (bf16, element
 * (b, h, t, d) at p + g_sB*b + g_sH*h + g_sT*t + d) from q, k, v, the forward's
 * out and lse, and dout (out and dout share o_s*).  lut is the selection
 * [B*H, NB, topk] (blk 128 or 64); for blk 64, paired is its
 * rola_b200_pair_blocks table (the forward's lut).  Exact gradient of the
 * forward; no atomics (deterministic).  workspace: 16-byte aligned, at least
 * rola_b200_sparse_attn_bwd_workspace bytes.  Replaces the backward of the
 * external SLA kernel (`_attention.apply`, wan_rola_attention.py:320-321). */
int rola_b200_sparse_attn_bwd(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT, const void* v,
                              int64_t v_sB, int64_t v_sH, int64_t v_sT, const void* out, const void* dout, int64_t o_sB,
                              int64_t o_sH, int64_t o_sT, const int32_t* lut, const int32_t* paired, const float* lse,
                              int B, int L, int H, int blk, int topk, void* dq, void* dk, void* dv, int64_t g_sB,
                              int64_t g_sH, int64_t g_sT, void* workspace, size_t workspace_bytes,
                              rola_stream_t stream);

/* Peer memory of the fused exchanges (CUDA IPC; no counterpart in the
 * reference).  peer_alloc: cudaMalloc of bytes on the current device and its
 * ROLA_PEER_HANDLE_BYTES-byte IPC handle; peer_open: map a handle made by
 * another process of the node; peer_close / peer_free undo them. */
int rola_b200_peer_alloc(size_t bytes, void** ptr, unsigned char* handle);
int rola_b200_peer_open(const unsigned char* handle, void** ptr);
int rola_b200_peer_close(void* ptr);
int rola_b200_peer_free(void* ptr);

/* Allocation-free variant of rola_b200_lowrank_kv.  No counterpart in the
 * reference: SparkDiffusion lets PyTorch allocate every temporary.
 * For callers that cannot provide or allocate device memory for the fp32
 * partial sums: a host framework that owns a fixed device-memory pool and
 * forbids allocations outside it, a latency-critical loop where cudaMalloc /
 * cudaFree (which may synchronise the device) is not acceptable, or a binding
 * with no CUDA allocator at hand.  The partials live in a fixed 16 MiB
 * (4 Mi fp32) array compiled into the library, held by every GPU that loads
 * the library until the process exits; chunks*B*H*R*D (chunks as in
 * rola_b200_lowrank_kv) must not exceed 4 Mi, i.e. at most 512 (chunk, batch,
 * head) partials: C4 with 5 heads per GPU fits, all 40 heads do not (larger
 * requests return ROLA_ERR_INVALID before any work).  The
 * first call on a device looks up the array's device address (issue it before
 * any stream capture on that device).  All calls share the array, so calls that
 * overlap on the GPU race; the array needs no clearing (every partial is
 * overwritten before it is read).  Arguments and outputs as rola_b200_lowrank_kv. */
int rola_b200_lowrank_kv_noalloc(const void* k_normed, int64_t k_sB, int64_t k_sH, int64_t k_sT, const void* v,
                                 int64_t v_sB, int64_t v_sH, int64_t v_sT, const void* proj_k, const void* lr_cos,
                                 const void* lr_sin, int rope_dim, int B, int L, int H, int R, int splits, void* C,
                                 void* Ct, rola_stream_t stream);

/* Workspace bytes needed by rola_b200_rola_forward for these sizes. */
size_t rola_b200_forward_workspace_bytes(int B, int L, int H, int blk, int R, int splits);

/* Whole RoLa attention forward up to (excluding) the output projection, from
 * the hidden states: WanSelfAttentionRoLa.fused_forward minus self.o
 * (sparkdiffusion/networks/wan_rola_attention.py:414-446).
 * x [B*L, dim]; w_qkv [3*dim, dim] (= [Wq; Wk; Wv]); b_qkv [3*dim] or NULL;
 * norm_wq/norm_wk [dim]; cos_sin [L, D] fp32; lr_cos/lr_sin [L, rope_dim];
 * proj_q/proj_k [R, D]; gate_w [D]; gate_b [H] bf16; out [B*L, dim] bf16.
 * workspace: device memory of rola_b200_forward_workspace_bytes() bytes
 * (256-byte aligned); lut_out [B*H, NB, topk] int32 may be NULL. */
int rola_b200_rola_forward(const void* x, const void* w_qkv, const void* b_qkv, const void* norm_wq,
                           const void* norm_wk, const float* cos_sin, const void* lr_cos, const void* lr_sin,
                           int rope_dim, const void* proj_q, const void* proj_k, const void* gate_w,
                           const void* gate_b, int B, int L, int H, int blk, int topk, int R, int splits, float eps,
                           void* workspace, size_t workspace_bytes, void* out, int32_t* lut_out,
                           rola_stream_t stream);

/* Host-buffer pipeline (no counterpart in the reference, which takes device
 * tensors): rola_b200_pipeline_forward uploads one step's hidden states from
 * PINNED host memory x_host, runs rola_b200_rola_forward and downloads the
 * result into pinned out_host, all asynchronously on the pipeline's own
 * upload / compute / download streams with double-buffered device copies of
 * x and out, so consecutive calls overlap step s+1's upload and step s-1's
 * download with step s's kernels.  The step starts after the work already on
 * `stream`; rola_b200_pipeline_wait makes `stream` wait for every submitted
 * step (out_host of a step is complete then).  Host buffers must stay valid
 * until that point.  x_bytes / out_bytes: the largest B*L*dim*2 to submit.
 * Other arguments as rola_b200_rola_forward. */
typedef struct rola_pipeline rola_pipeline;
int rola_b200_pipeline_create(size_t x_bytes, size_t out_bytes, rola_pipeline** out);
int rola_b200_pipeline_forward(rola_pipeline* pl, const void* x_host, const void* w_qkv, const void* b_qkv,
                               const void* norm_wq, const void* norm_wk, const float* cos_sin, const void* lr_cos,
                               const void* lr_sin, int rope_dim, const void* proj_q, const void* proj_k,
                               const void* gate_w, const void* gate_b, int B, int L, int H, int blk, int topk, int R,
                               int splits, float eps, void* workspace, size_t workspace_bytes, void* out_host,
                               rola_stream_t stream);
int rola_b200_pipeline_wait(rola_pipeline* pl, rola_stream_t stream);
int rola_b200_pipeline_destroy(rola_pipeline* pl);

#ifdef __cplusplus
}
#endif

#endif /* ROLA_B200_H_ */
