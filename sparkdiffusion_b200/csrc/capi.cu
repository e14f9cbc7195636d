// extern "C" entry points of librola_b200.so (declared in include/rola_b200.h).
//
// Each entry point validates its arguments on the host (returning
// ROLA_ERR_INVALID with a message and launching nothing), builds the TMA
// tensor maps it needs, and launches the kernels on the caller's stream.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/rola_b200.h"
#include "common.cuh"
#include "kernels.h"

// log2 growth of a row's running max that triggers the O rescale in the
// attention kernel; 0 rescales on every growth (the reference's recurrence)
#ifndef ROLA_RESCALE_THRESHOLD
#define ROLA_RESCALE_THRESHOLD 0.0f
#endif

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(int launch_rc, const char* what) {
  if (launch_rc == 0) return ROLA_OK;
  if (launch_rc < 0) return fail(ROLA_ERR_INVALID, "%s: unsupported configuration", what);
  return fail(ROLA_ERR_CUDA, "%s: %s", what, cudaGetErrorString((cudaError_t)launch_rc));
}

#define ROLA_CHECK(cond, ...)                          \
  do {                                                 \
    if (!(cond)) return fail(ROLA_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define ROLA_TRY(expr)            \
  do {                            \
    int _rc = (expr);             \
    if (_rc != ROLA_OK) return _rc; \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline cudaStream_t S(rola_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }
inline const __nv_bfloat16* BF(const void* p) { return reinterpret_cast<const __nv_bfloat16*>(p); }
inline __nv_bfloat16* BFm(void* p) { return reinterpret_cast<__nv_bfloat16*>(p); }

// ---------------------------------------------------------------------------
// TMA descriptors through the driver entry point (no libcuda link dependency)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// bf16 tensor of rank 2 or 3: dims innermost first, strides (bytes) of dims 1.., box innermost first
int make_map(CUtensorMap* m, const void* ptr, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
             const uint32_t* box, const char* what, bool bytes = false) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ROLA_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
  ROLA_CHECK(aligned16(ptr), "%s: base address must be 16-byte aligned", what);
  for (int i = 0; i < rank - 1; ++i)
    ROLA_CHECK(strides_bytes[i] % 16 == 0, "%s: row strides must be multiples of 16 bytes", what);
  cuuint64_t gd[5], gs[4];
  cuuint32_t bd[5], es[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bd[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = fn(m, bytes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank,
                  const_cast<void*>(ptr), gd, gs, bd, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ROLA_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return ROLA_OK;
}

// token-major [B, L, cols] view (row stride ld elements) with [64 x 128 x 1] boxes
int make_token_map(CUtensorMap* m, const void* ptr, int64_t cols, int64_t ld, int L, int B, const char* what) {
  const uint64_t dims[3] = {(uint64_t)cols, (uint64_t)L, (uint64_t)B};
  const uint64_t strides[2] = {(uint64_t)ld * 2, (uint64_t)ld * 2 * (uint64_t)L};
  const uint32_t box[3] = {64, 128, 1};
  return make_map(m, ptr, 3, dims, strides, box, what);
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Side streams per device for the forward's three independent branches, with
// fork/join events: the selection chain (centre, pooled k, scores + top-k) on a
// stream of the device's greatest priority, so that the hardware dispatches its
// few, latency-bound CTAs ahead of the many queued CTAs of the low-rank C^T and
// q_lr kernels, which run on the other two.
struct ForkJoin {
  cudaStream_t side[3] = {nullptr, nullptr, nullptr};  // low-rank kv, low-rank q, selection
  cudaEvent_t fork = nullptr, join[3] = {nullptr, nullptr, nullptr};
  std::mutex mu;
};
ForkJoin g_forkjoin[64];

int forkjoin_get(ForkJoin** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return fail(ROLA_ERR_CUDA, "rola_forward: no current device");
  ForkJoin& f = g_forkjoin[dev];
  std::lock_guard<std::mutex> lock(f.mu);
  if (f.fork == nullptr) {
    int least = 0, greatest = 0;
    e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
    for (int i = 0; i < 3 && e == cudaSuccess; ++i) {
      e = cudaStreamCreateWithPriority(&f.side[i], cudaStreamNonBlocking, i == 2 ? greatest : least);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&f.join[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&f.fork, cudaEventDisableTiming);
    if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "rola_forward: %s", cudaGetErrorString(e));
  }
  *out = &f;
  return ROLA_OK;
}

}  // namespace

using namespace rola;

extern "C" {

int rola_b200_abi_version(void) { return ROLA_B200_ABI_VERSION; }

const char* rola_b200_last_error(void) { return g_last_error.c_str(); }

int rola_b200_device_status(int clear) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    int z = 0;
    if (cudaMemcpyToSymbol(g_device_error, &z, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

static int qkv_gemm_impl(const void* x, const void* w, const void* bias, void* out, float* ssq, int64_t M, int64_t N,
                         int64_t K, const NormRopeParams* side, rola_stream_t stream, bool allow_pairs = true) {
  ROLA_CHECK(x && w && out, "qkv_gemm: null pointer");
  ROLA_CHECK(M > 0 && M < (1ll << 31), "qkv_gemm: M out of range");
  ROLA_CHECK(N > 0 && N % 256 == 0 && N <= 65536, "qkv_gemm: N must be a positive multiple of 256");
  ROLA_CHECK(K > 0 && K % 64 == 0 && K <= 65536, "qkv_gemm: K must be a positive multiple of 64");
  ROLA_CHECK(aligned16(out), "qkv_gemm: out must be 16-byte aligned");
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, 128};
    ROLA_TRY(make_map(&ta, x, 2, dims, strides, box, "qkv_gemm: x"));
  }
  const bool pairs = allow_pairs && side == nullptr && M >= 256;  // the two-SM kernel (no side job)
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, pairs ? 128u : 256u};
    ROLA_TRY(make_map(&tb, w, 2, dims, strides, box, "qkv_gemm: w"));
  }
  if (pairs)
    return cuda_status(launch_gemm_bf16_2sm(ta, tb, BF(bias), BFm(out), N, ssq, (int)M, (int)N, (int)K, S(stream)),
                       "qkv_gemm");
  return cuda_status(launch_gemm_bf16(ta, tb, BF(bias), BFm(out), N, ssq, (int)M, (int)N, (int)K, side, S(stream)),
                     "qkv_gemm");
}

int rola_b200_qkv_gemm(const void* x, const void* w, const void* bias, void* out, float* ssq, int64_t M, int64_t N,
                       int64_t K, rola_stream_t stream) {
  return qkv_gemm_impl(x, w, bias, out, ssq, M, N, K, nullptr, stream);
}

int rola_b200_quantize_rows_e4m3(const void* x, int64_t ld, int64_t M, int64_t K, void* xq, float* scale,
                                 rola_stream_t stream) {
  ROLA_CHECK(x && xq && scale, "quantize_rows_e4m3: null pointer");
  ROLA_CHECK(M > 0 && M < (1ll << 31) && K > 0 && K % 8 == 0 && K <= 65536 && ld >= K && ld % 8 == 0,
             "quantize_rows_e4m3: bad sizes (K a multiple of 8, row stride >= K)");
  ROLA_CHECK(aligned16(x) && aligned16(xq), "quantize_rows_e4m3: 16-byte aligned rows required");
  return cuda_status(launch_quantize_rows_e4m3(BF(x), ld, (int)M, (int)K, reinterpret_cast<uint8_t*>(xq), scale,
                                               S(stream)),
                     "quantize_rows_e4m3");
}

int rola_b200_qkv_gemm_fp8(const void* xq, const float* x_scale, const void* wq, const float* w_scale,
                           const void* bias, void* out, float* ssq, int64_t M, int64_t N, int64_t K,
                           rola_stream_t stream) {
  ROLA_CHECK(xq && x_scale && wq && w_scale && out, "qkv_gemm_fp8: null pointer");
  ROLA_CHECK(M > 0 && M < (1ll << 31), "qkv_gemm_fp8: M out of range");
  ROLA_CHECK(N > 0 && N % 256 == 0 && N <= 65536, "qkv_gemm_fp8: N must be a positive multiple of 256");
  ROLA_CHECK(K > 0 && K % 128 == 0 && K <= 65536, "qkv_gemm_fp8: K must be a positive multiple of 128");
  ROLA_CHECK(aligned16(out), "qkv_gemm_fp8: out must be 16-byte aligned");
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {128, 128};
    ROLA_TRY(make_map(&ta, xq, 2, dims, strides, box, "qkv_gemm_fp8: xq", true));
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {128, 256};
    ROLA_TRY(make_map(&tb, wq, 2, dims, strides, box, "qkv_gemm_fp8: wq", true));
  }
  return cuda_status(launch_gemm_bf16(ta, tb, BF(bias), BFm(out), N, ssq, (int)M, (int)N, (int)K, nullptr, S(stream),
                                      x_scale, w_scale),
                     "qkv_gemm_fp8");
}

// Runs the streaming norm pass.  ssq: the QKV GEMM's per-256-column sums of
// squares (row stride ssq_ld), or nullptr, in which case the row statistics are
// computed first into stream-ordered scratch.
static int run_norm_pass(NormRopeParams& p, bool norm, bool rope, bool pool, const float* ssq, int ssq_ld,
                         cudaStream_t s, const char* what) {
  float* scratch = nullptr;
  if (norm && ssq == nullptr) {
    const int64_t rows = (int64_t)p.B * p.L;
    ROLA_TRY(cuda_status(cudaMallocAsync(reinterpret_cast<void**>(&scratch), rows * 2 * p.H * sizeof(float), s), what));
    const int rc = launch_row_ssq(p.q_in, p.k_in, p.ld_in, rows, p.H * 128, scratch, s);
    if (rc != 0) {
      cudaFreeAsync(scratch, s);
      return cuda_status(rc, what);
    }
    p.ssq = scratch;
    p.ssq_ld = 2 * p.H;
    p.ssq_tile = 128;
  } else {
    p.ssq = ssq;
    p.ssq_ld = ssq_ld;
    p.ssq_tile = 256;
  }
  const int rc = launch_norm_rope_pool(p, norm, rope, pool, s);
  if (scratch) cudaFreeAsync(scratch, s);
  if (rc == -1) return fail(ROLA_ERR_INVALID, "%s: unsupported configuration", what);
  return cuda_status(rc, what);
}

int rola_b200_qk_norm_rope(const void* q_raw, const void* k_raw, int64_t ld_raw, const float* ssq, int ssq_ld,
                           const void* x, const void* norm_wq, const void* norm_wk, const float* cos_sin,
                           const void* gate_w, const void* gate_b, int B, int L, int H, int blk, float eps,
                           void* q_rope, void* k_rope, void* q_normed, void* k_normed, void* gate_out, void* pooled_q,
                           float* ksum, rola_stream_t stream) {
  ROLA_CHECK(q_raw && k_raw && cos_sin, "qk_norm_rope: null input");
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && blk > 0 && blk <= 4096, "qk_norm_rope: bad sizes");
  ROLA_CHECK((norm_wq == nullptr) == (norm_wk == nullptr), "qk_norm_rope: give both norm weights or neither");
  ROLA_CHECK(ld_raw % 8 == 0 && aligned16(q_raw) && aligned16(k_raw), "qk_norm_rope: 16-byte aligned rows required");
  ROLA_CHECK((pooled_q == nullptr) == (ksum == nullptr), "qk_norm_rope: pooled_q and ksum go together");
  ROLA_CHECK(x == nullptr || (gate_w && gate_b && gate_out), "qk_norm_rope: the gate needs gate_w, gate_b, gate_out");
  ROLA_CHECK(x == nullptr || (aligned16(x) && aligned16(gate_w)), "qk_norm_rope: x and gate_w must be 16-byte aligned");
  ROLA_CHECK(ssq == nullptr || (H % 2 == 0 && ssq_ld >= H),
             "qk_norm_rope: sums of squares need an even head count and ssq_ld >= H");
  NormRopeParams p{};
  p.q_in = BF(q_raw);
  p.k_in = BF(k_raw);
  p.ld_in = ld_raw;
  p.x = BF(x);
  p.ld_x = (int64_t)H * 128;
  p.norm_wq = BF(norm_wq);
  p.norm_wk = BF(norm_wk);
  p.cos_sin = cos_sin;
  p.gate_w = BF(gate_w);
  p.gate_b = BF(gate_b);
  p.q_rope = BFm(q_rope);
  p.k_rope = BFm(k_rope);
  p.qn_dst[0] = BFm(q_normed);
  p.kn_dst[0] = BFm(k_normed);
  p.g_dst[0] = x ? BFm(gate_out) : nullptr;
  p.dst_sB = (int64_t)L * H * 128;
  p.pooled_q = BFm(pooled_q);
  p.ksum = ksum;
  p.B = B;
  p.L = L;
  p.H = H;
  p.blk = blk;
  p.NB = (L + blk - 1) / blk;
  p.heads_per_chunk = H;
  p.eps = eps;
  return run_norm_pass(p, norm_wq != nullptr, true, pooled_q != nullptr, ssq, ssq_ld, S(stream), "qk_norm_rope");
}

int rola_b200_qk_norm_pack(const void* q_raw, const void* k_raw, const void* v_raw, int64_t ld_raw, const float* ssq,
                           int ssq_ld, const void* x, const void* norm_wq, const void* norm_wk, const void* gate_w,
                           const void* gate_b, int B, int L, int H, int heads_per_chunk, float eps, void* q_send,
                           void* k_send, void* v_send, void* gate_out, rola_stream_t stream) {
  ROLA_CHECK(q_raw && k_raw && v_raw && norm_wq && norm_wk && q_send && k_send && v_send,
             "qk_norm_pack: null pointer");
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && heads_per_chunk > 0 && H % heads_per_chunk == 0 &&
                 H / heads_per_chunk <= kMaxChunks,
             "qk_norm_pack: bad sizes (at most 8 head chunks)");
  ROLA_CHECK(ld_raw % 8 == 0, "qk_norm_pack: 16-byte aligned rows required");
  ROLA_CHECK(x == nullptr || (gate_w && gate_b && gate_out), "qk_norm_pack: the gate needs gate_w, gate_b, gate_out");
  ROLA_CHECK(x == nullptr || (aligned16(x) && aligned16(gate_w)), "qk_norm_pack: x and gate_w must be 16-byte aligned");
  ROLA_CHECK(ssq == nullptr || (H % 2 == 0 && ssq_ld >= H), "qk_norm_pack: sums of squares need an even head count");
  NormRopeParams p{};
  p.q_in = BF(q_raw);
  p.k_in = BF(k_raw);
  p.v_in = BF(v_raw);
  p.ld_in = ld_raw;
  p.x = BF(x);
  p.ld_x = (int64_t)H * 128;
  p.norm_wq = BF(norm_wq);
  p.norm_wk = BF(norm_wk);
  p.gate_w = BF(gate_w);
  p.gate_b = BF(gate_b);
  // send block c of batch b: [B][H / heads_per_chunk][L][heads_per_chunk * D]
  for (int c = 0; c < H / heads_per_chunk && c < kMaxChunks; ++c) {
    const int64_t off = (int64_t)c * L * heads_per_chunk * 128;
    p.qn_dst[c] = BFm(q_send) + off;
    p.kn_dst[c] = BFm(k_send) + off;
    p.v_dst[c] = BFm(v_send) + off;
    p.g_dst[c] = x ? BFm(gate_out) + (int64_t)c * L * heads_per_chunk : nullptr;
  }
  p.dst_sB = (int64_t)L * H * 128;
  p.B = B;
  p.L = L;
  p.H = H;
  p.blk = 32;  // no pooling: short work items
  p.NB = (L + 31) / 32;
  p.heads_per_chunk = heads_per_chunk;
  p.eps = eps;
  return run_norm_pass(p, true, false, false, ssq, ssq_ld, S(stream), "qk_norm_pack");
}

// Validates a scatter description and turns it into norm-pass parameters.
static int scatter_params(const rola_scatter_args* a, bool compact, NormRopeParams* out, const char* what) {
  ROLA_CHECK(a, "%s: null arguments", what);
  ROLA_CHECK(a->q_raw && a->k_raw && a->v_raw && a->norm_wq && a->norm_wk && a->x && a->gate_w && a->gate_b,
             "%s: null pointer", what);
  ROLA_CHECK(a->world >= 1 && a->world <= kMaxChunks, "%s: bad world size (<= 8)", what);
  ROLA_CHECK(a->B > 0 && a->L > 0 && a->H > 0 && a->H % a->world == 0, "%s: world must divide the head count", what);
  ROLA_CHECK(a->dst_row0 >= 0 && a->dst_row0 + a->L <= a->dst_rows && a->dst_rows < (1ll << 31),
             "%s: rows [dst_row0, dst_row0 + L) outside the destination", what);
  ROLA_CHECK(a->ld_raw % 8 == 0 && aligned16(a->q_raw) && aligned16(a->k_raw) && aligned16(a->v_raw) &&
                 aligned16(a->x) && aligned16(a->gate_w),
             "%s: 16-byte aligned rows required", what);
  ROLA_CHECK(a->ssq == nullptr || (a->H % 2 == 0 && a->ssq_ld >= a->H),
             "%s: sums of squares need an even head count", what);
  for (int r = 0; r < a->world; ++r)
    ROLA_CHECK(a->q_dst[r] && a->k_dst[r] && a->v_dst[r] && a->g_dst[r] && aligned16(a->q_dst[r]) &&
                   aligned16(a->k_dst[r]) && aligned16(a->v_dst[r]),
               "%s: destination %d null or not 16-byte aligned", what, r);
  NormRopeParams p{};
  p.q_in = BF(a->q_raw);
  p.k_in = BF(a->k_raw);
  p.v_in = BF(a->v_raw);
  p.ld_in = a->ld_raw;
  p.x = BF(a->x);
  p.ld_x = (int64_t)a->H * 128;
  p.norm_wq = BF(a->norm_wq);
  p.norm_wk = BF(a->norm_wk);
  p.gate_w = BF(a->gate_w);
  p.gate_b = BF(a->gate_b);
  // destination r holds heads [r*Hl, (r+1)*Hl) of dst_rows tokens per batch;
  // this call's tokens start at row dst_row0 there
  for (int r = 0; r < a->world; ++r) {
    p.qn_dst[r] = BFm(a->q_dst[r]);
    p.kn_dst[r] = BFm(a->k_dst[r]);
    p.v_dst[r] = BFm(a->v_dst[r]);
    p.g_dst[r] = BFm(a->g_dst[r]);
  }
  p.dst_sB = a->dst_rows * (a->H / a->world) * 128;
  p.dst_t0 = (int)a->dst_row0;
  p.B = a->B;
  p.L = a->L;
  p.H = a->H;
  // no pooling here: short 32-token work items give the pass enough CTAs on small chunks
  p.blk = 32;
  p.NB = (a->L + 31) / 32;
  p.heads_per_chunk = a->H / a->world;
  p.compact = compact;
  p.eps = a->eps;
  p.ssq = a->ssq;
  p.ssq_ld = a->ssq_ld;
  p.ssq_tile = 256;
  *out = p;
  return ROLA_OK;
}

int rola_b200_qk_norm_scatter(const rola_scatter_args* args, int compact, rola_stream_t stream) {
  NormRopeParams p{};
  ROLA_TRY(scatter_params(args, compact != 0, &p, "qk_norm_scatter"));
  return run_norm_pass(p, true, false, false, args->ssq, args->ssq_ld, S(stream), "qk_norm_scatter");
}

int rola_b200_qkv_gemm_scatter(const void* x, const void* w, const void* bias, void* out, float* ssq, int64_t M,
                               int64_t N, int64_t K, const rola_scatter_args* side, rola_stream_t stream) {
  // no side job: the same single-SM persistent kernel without spare-warp work
  // (the first chunk of an overlapped exchange runs on the kernel of the others)
  if (side == nullptr) return qkv_gemm_impl(x, w, bias, out, ssq, M, N, K, nullptr, stream, false);
  NormRopeParams p{};
  ROLA_TRY(scatter_params(side, true, &p, "qkv_gemm_scatter"));
  ROLA_CHECK(side->B == 1 && side->ssq != nullptr, "qkv_gemm_scatter: the side job needs B == 1 and the GEMM sums");
  return qkv_gemm_impl(x, w, bias, out, ssq, M, N, K, &p, stream);
}

int rola_b200_rope_pool(const void* q_normed, const void* k_normed, int64_t ld, const float* cos_sin, int B, int L,
                        int H, int blk, void* q_rope, void* k_rope, void* pooled_q, float* ksum,
                        rola_stream_t stream) {
  ROLA_CHECK(q_normed && k_normed && cos_sin && q_rope && k_rope, "rope_pool: null pointer");
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && blk > 0 && blk <= 4096, "rope_pool: bad sizes");
  ROLA_CHECK((pooled_q == nullptr) == (ksum == nullptr), "rope_pool: pooled_q and ksum go together");
  ROLA_CHECK(ld % 8 == 0, "rope_pool: 16-byte aligned rows required");
  NormRopeParams p{};
  p.q_in = BF(q_normed);
  p.k_in = BF(k_normed);
  p.ld_in = ld;
  p.cos_sin = cos_sin;
  p.q_rope = BFm(q_rope);
  p.k_rope = BFm(k_rope);
  p.pooled_q = BFm(pooled_q);
  p.ksum = ksum;
  p.B = B;
  p.L = L;
  p.H = H;
  p.blk = blk;
  p.NB = (L + blk - 1) / blk;
  p.heads_per_chunk = H;
  return run_norm_pass(p, false, true, pooled_q != nullptr, nullptr, 0, S(stream), "rope_pool");
}

int rola_b200_mean_pool(const void* x, int64_t sB, int64_t sH, int64_t sT, int B, int H, int L, int blk,
                        const void* center, void* out, rola_stream_t stream) {
  ROLA_CHECK(x && out, "mean_pool: null pointer");
  ROLA_CHECK(B > 0 && H > 0 && L > 0 && blk > 0, "mean_pool: bad sizes");
  ROLA_CHECK(aligned16(x) && sB % 8 == 0 && sH % 8 == 0 && sT % 8 == 0, "mean_pool: 16-byte aligned rows required");
  return cuda_status(launch_block_pool(BF(x), sB, sH, sT, B, H, L, blk, BF(center), BFm(out), nullptr, S(stream)),
                     "mean_pool");
}

int rola_b200_smooth_k_center(const void* k, int64_t sB, int64_t sH, int64_t sT, int B, int H, int L, int blk,
                              float* ksum_ws, void* center, rola_stream_t stream) {
  ROLA_CHECK(k && ksum_ws && center, "smooth_k_center: null pointer");
  ROLA_CHECK(B > 0 && H > 0 && L > 0 && blk > 0, "smooth_k_center: bad sizes");
  ROLA_CHECK(aligned16(k) && sB % 8 == 0 && sH % 8 == 0 && sT % 8 == 0,
             "smooth_k_center: 16-byte aligned rows required");
  ROLA_TRY(cuda_status(launch_block_pool(BF(k), sB, sH, sT, B, H, L, blk, nullptr, nullptr, ksum_ws, S(stream)),
                       "smooth_k_center"));
  const int NB = (L + blk - 1) / blk;
  return cuda_status(launch_center(ksum_ws, B, NB, H * 128, L, BFm(center), S(stream)), "smooth_k_center");
}

int rola_b200_center_from_sums(const float* ksum, int B, int NB, int dim, int L, void* center,
                               rola_stream_t stream) {
  ROLA_CHECK(ksum && center, "center_from_sums: null pointer");
  ROLA_CHECK(B > 0 && NB > 0 && dim > 0 && L > 0, "center_from_sums: bad sizes");
  return cuda_status(launch_center(ksum, B, NB, dim, L, BFm(center), S(stream)), "center_from_sums");
}

int rola_b200_block_select(const void* pooled_q, const void* pooled_k, int BH, int NBq, int NBk, int topk,
                           float* scores_ws, int32_t* lut, rola_stream_t stream) {
  ROLA_CHECK(pooled_q && pooled_k && lut && (scores_ws || NBk <= 768), "block_select: null pointer");
  ROLA_CHECK(aligned16(pooled_q) && aligned16(pooled_k), "block_select: pooled tensors must be 16-byte aligned");
  ROLA_CHECK(BH > 0 && NBq > 0 && NBk > 0 && NBk <= 2048, "block_select: bad sizes (NBk <= 2048)");
  ROLA_CHECK(topk >= 1 && topk <= NBk, "block_select: topk must be in [1, NBk]");
  if (NBk <= 768) {
    // fused: the scores stay in registers (scores_ws is not written)
    return cuda_status(launch_select_fused(BF(pooled_q), BF(pooled_k), BH, NBq, NBk, topk, lut, S(stream)),
                       "block_select");
  }
  ROLA_TRY(cuda_status(launch_scores(BF(pooled_q), BF(pooled_k), BH, NBq, NBk, scores_ws, S(stream)),
                       "block_select/scores"));
  return cuda_status(launch_topk(scores_ws, BH * NBq, NBk, topk, lut, S(stream)), "block_select/topk");
}

int rola_b200_pair_blocks(const int32_t* lut, int BH, int NB, int topk, int32_t* paired, rola_stream_t stream) {
  ROLA_CHECK(lut && paired, "pair_blocks: null pointer");
  ROLA_CHECK(BH > 0 && NB > 0 && topk >= 1 && topk <= NB && topk < (1 << 20) && NB < (1 << 28),
             "pair_blocks: bad sizes");
  return cuda_status(launch_pair_blocks(lut, BH, NB, topk, NB, paired, S(stream)), "pair_blocks");
}

int rola_b200_lowrank_q(const void* q_normed, int64_t sB, int64_t sH, int64_t sT, const void* proj_q,
                        const void* lr_cos, const void* lr_sin, int rope_dim, int B, int L, int H, int R, void* q_lr,
                        rola_stream_t stream) {
  ROLA_CHECK(q_normed && proj_q && q_lr, "lowrank_q: null pointer");
  ROLA_CHECK(R == 64, "lowrank_q: rank must be 64");
  ROLA_CHECK(rope_dim >= 0 && rope_dim <= R / 2 && (rope_dim == 0 || (lr_cos && lr_sin)), "lowrank_q: bad rope_dim");
  ROLA_CHECK(B > 0 && L > 0 && H > 0, "lowrank_q: bad sizes");
  ROLA_CHECK(aligned16(q_normed) && sB % 8 == 0 && sH % 8 == 0 && sT % 8 == 0, "lowrank_q: 16-byte aligned rows required");
  LowrankParams p{};
  p.x = BF(q_normed);
  p.x_sB = sB;
  p.x_sH = sH;
  p.x_sT = sT;
  p.proj = BF(proj_q);
  p.cos = BF(lr_cos);
  p.sin = BF(lr_sin);
  p.lr_out = BFm(q_lr);
  p.B = B;
  p.L = L;
  p.H = H;
  p.R = R;
  p.rope_dim = rope_dim;
  return cuda_status(launch_lowrank_q(p, S(stream)), "lowrank_q");
}

int rola_b200_lowrank_kv(const void* k_normed, int64_t k_sB, int64_t k_sH, int64_t k_sT, const void* v, int64_t v_sB,
                         int64_t v_sH, int64_t v_sT, const void* proj_k, const void* lr_cos, const void* lr_sin,
                         int rope_dim, int B, int L, int H, int R, int splits, float* c_partial_ws, void* C, void* Ct,
                         rola_stream_t stream) {
  ROLA_CHECK(k_normed && v && proj_k && c_partial_ws && (C || Ct), "lowrank_kv: null pointer");
  ROLA_CHECK(R == 64, "lowrank_kv: rank must be 64");
  ROLA_CHECK(rope_dim >= 0 && rope_dim <= R / 2 && (rope_dim == 0 || (lr_cos && lr_sin)), "lowrank_kv: bad rope_dim");
  ROLA_CHECK(rope_dim == 0 || (aligned16(lr_cos) && aligned16(lr_sin)), "lowrank_kv: 16-byte aligned RoPE tables required");
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && splits > 0 && splits <= 4096, "lowrank_kv: bad sizes");
  ROLA_CHECK(aligned16(k_normed) && aligned16(v) && k_sB % 8 == 0 && k_sH % 8 == 0 && k_sT % 8 == 0 &&
                 v_sB % 8 == 0 && v_sH % 8 == 0 && v_sT % 8 == 0,
             "lowrank_kv: 16-byte aligned rows required");
  LowrankParams p{};
  p.x = BF(k_normed);
  p.x_sB = k_sB;
  p.x_sH = k_sH;
  p.x_sT = k_sT;
  p.v = BF(v);
  p.v_sB = v_sB;
  p.v_sH = v_sH;
  p.v_sT = v_sT;
  p.proj = BF(proj_k);
  p.cos = BF(lr_cos);
  p.sin = BF(lr_sin);
  p.c_partial = c_partial_ws;
  p.B = B;
  p.L = L;
  p.H = H;
  p.R = R;
  p.rope_dim = rope_dim;
  p.splits = splits;
  ROLA_TRY(cuda_status(launch_lowrank_kv(p, S(stream)), "lowrank_kv"));
  return cuda_status(launch_lowrank_reduce(c_partial_ws, lowrank_chunks(L), B * H, R, BFm(C), BFm(Ct), S(stream)),
                     "lowrank_kv/reduce");
}

// head-view 4-D map: dims (d = 128, t = L, h = H, b = B) with element strides (1, sT, sH, sB);
// boxes of 64 columns x `rows` tokens
static int make_head_map(CUtensorMap* m, const void* ptr, int cols, int64_t sB, int64_t sH, int64_t sT, int L, int H,
                         int B, const char* what, int rows = 128) {
  const uint64_t dims[4] = {(uint64_t)cols, (uint64_t)L, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)sT * 2, (uint64_t)sH * 2, (uint64_t)sB * 2};
  const uint32_t box[4] = {64, (uint32_t)rows, 1, 1};
  return make_map(m, ptr, 4, dims, strides, box, what);
}

// Output routing of the head->sequence exchange fused into the attention store.
struct PeerOut {
  void* const* dst;  // dst[r]: rank r's output buffer [B, L / world, H_total * D]
  int world, head_offset, H_total;
};

static int sparse_attn_impl(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT, const void* v,
                            int64_t v_sB, int64_t v_sH, int64_t v_sT, const int32_t* lut, int B, int L, int H, int blk,
                            int topk, const void* q_lr, const void* Ct, const void* gate, const void* x, int64_t x_sB,
                            int64_t x_sH, int64_t x_sT, const void* gate_w, const void* gate_b, float eps_lr,
                            void* out, void* o_sparse, int64_t o_sB, int64_t o_sH, int64_t o_sT, const PeerOut* peer,
                            rola_stream_t stream, float* lse = nullptr) {
  ROLA_CHECK(q && k && v && lut, "sparse_attn: null pointer");
  ROLA_CHECK(out || o_sparse || peer, "sparse_attn: no output requested");
  ROLA_CHECK(blk == 128 || blk == 64, "sparse_attn: block size must be 128 or 64");
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && (int64_t)B * H < 65536, "sparse_attn: bad sizes");
  const int NB = (L + blk - 1) / blk;
  ROLA_CHECK(topk >= 1 && topk <= NB, "sparse_attn: topk must be in [1, NB]");
  ROLA_CHECK((q_lr == nullptr) == (Ct == nullptr), "sparse_attn: q_lr and Ct go together");
  ROLA_CHECK(x == nullptr || (gate_w && gate_b && q_lr), "sparse_attn: the gate from x needs gate_w, gate_b and q_lr");
  ROLA_CHECK(x == nullptr || gate == nullptr, "sparse_attn: give gate values or x, not both");
  ROLA_CHECK(gate_w == nullptr || aligned16(gate_w), "sparse_attn: gate_w must be 16-byte aligned");
  ROLA_CHECK(o_sB % 8 == 0 && o_sH % 8 == 0 && o_sT % 8 == 0 && (out == nullptr || aligned16(out)) &&
                 (o_sparse == nullptr || aligned16(o_sparse)),
             "sparse_attn: 16-byte aligned output rows required");
  CUtensorMap tq, tk, tv, tqlr, tct, tx;
  memset(&tqlr, 0, sizeof(tqlr));
  memset(&tct, 0, sizeof(tct));
  memset(&tx, 0, sizeof(tx));
  if (x) ROLA_TRY(make_head_map(&tx, x, 128, x_sB, x_sH, x_sT, L, H, B, "sparse_attn: x"));
  ROLA_TRY(make_head_map(&tq, q, 128, qk_sB, qk_sH, qk_sT, L, H, B, "sparse_attn: q"));
  ROLA_TRY(make_head_map(&tk, k, 128, qk_sB, qk_sH, qk_sT, L, H, B, "sparse_attn: k", blk));
  ROLA_TRY(make_head_map(&tv, v, 128, v_sB, v_sH, v_sT, L, H, B, "sparse_attn: v", blk));
  if (q_lr) {
    ROLA_TRY(make_head_map(&tqlr, q_lr, 64, (int64_t)L * H * 64, 64, (int64_t)H * 64, L, H, B, "sparse_attn: q_lr"));
    const uint64_t dims[3] = {64, 128, (uint64_t)B * H};
    const uint64_t strides[2] = {64 * 2, 64 * 128 * 2};
    const uint32_t box[3] = {64, 128, 1};
    ROLA_TRY(make_map(&tct, Ct, 3, dims, strides, box, "sparse_attn: Ct"));
  }
  AttnParams p{};
  p.lut = lut;
  p.gate = BF(gate);
  p.gate_w = BF(gate_w);
  p.gate_b = BF(gate_b);
  p.has_x = x != nullptr;
  p.out = BFm(out);
  p.o_sB = o_sB;
  p.o_sH = o_sH;
  p.o_sT = o_sT;
  p.o_sparse = BFm(o_sparse);
  p.B = B;
  p.L = L;
  p.H = H;
  p.NBq = NB;
  p.NBk = NB;
  p.topk = topk;
  p.blk64 = blk == 64;
  p.has_lowrank = q_lr != nullptr;
  p.qk_scale = (float)(0.08838834764831845 * 1.4426950408889634);  // 128^-0.5 * log2(e)
  p.eps_lr = eps_lr;
  p.rescale_threshold = ROLA_RESCALE_THRESHOLD;
  p.lse = lse;
  p.lse_ld = 128 * ((L + 127) / 128);
  if (peer) {
    p.peer_n = peer->world;
    p.peer_Ls = L / peer->world;
    p.head_offset = peer->head_offset;
    p.peer_sT = (int64_t)peer->H_total * 128;
    p.peer_sB = p.peer_Ls * p.peer_sT;
    for (int r = 0; r < peer->world; ++r) p.out_peer[r] = BFm(peer->dst[r]);
  }
  return cuda_status(launch_sparse_attn(tq, tk, tv, tqlr, tct, tx, p, S(stream)), "sparse_attn");
}

int rola_b200_sparse_attn(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT, const void* v,
                          int64_t v_sB, int64_t v_sH, int64_t v_sT, const int32_t* lut, int B, int L, int H, int blk,
                          int topk, const void* q_lr, const void* Ct, const void* gate, const void* x, int64_t x_sB,
                          int64_t x_sH, int64_t x_sT, const void* gate_w, const void* gate_b, float eps_lr, void* out,
                          void* o_sparse, int64_t o_sB, int64_t o_sH, int64_t o_sT, rola_stream_t stream) {
  return sparse_attn_impl(q, k, qk_sB, qk_sH, qk_sT, v, v_sB, v_sH, v_sT, lut, B, L, H, blk, topk, q_lr, Ct, gate, x,
                          x_sB, x_sH, x_sT, gate_w, gate_b, eps_lr, out, o_sparse, o_sB, o_sH, o_sT, nullptr, stream);
}

int rola_b200_sparse_attn_scatter(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT,
                                  const void* v, int64_t v_sB, int64_t v_sH, int64_t v_sT, const int32_t* lut, int B,
                                  int L, int H, int blk, int topk, const void* q_lr, const void* Ct, const void* gate,
                                  float eps_lr, void* const* out_dst, int world, int head_offset, int H_total,
                                  rola_stream_t stream) {
  ROLA_CHECK(out_dst && q_lr && gate, "sparse_attn_scatter: null pointer");
  ROLA_CHECK(world >= 1 && world <= kMaxChunks && L % world == 0, "sparse_attn_scatter: world must divide L (<= 8 ranks)");
  ROLA_CHECK(head_offset >= 0 && head_offset + H <= H_total, "sparse_attn_scatter: head range outside H_total");
  for (int r = 0; r < world; ++r)
    ROLA_CHECK(out_dst[r] && aligned16(out_dst[r]), "sparse_attn_scatter: output %d null or not 16-byte aligned", r);
  const PeerOut peer{out_dst, world, head_offset, H_total};
  return sparse_attn_impl(q, k, qk_sB, qk_sH, qk_sT, v, v_sB, v_sH, v_sT, lut, B, L, H, blk, topk, q_lr, Ct, gate,
                          nullptr, 0, 0, 0, nullptr, nullptr, eps_lr, nullptr, nullptr, 0, 0, 0, &peer, stream);
}

// ---------------------------------------------------------------------------
// training: forward with the row log-sum-exp, backward
// ---------------------------------------------------------------------------
int rola_b200_sparse_attn_fwd_lse(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT,
                                  const void* v, int64_t v_sB, int64_t v_sH, int64_t v_sT, const int32_t* lut, int B,
                                  int L, int H, int blk, int topk, void* out, int64_t o_sB, int64_t o_sH, int64_t o_sT,
                                  float* lse, rola_stream_t stream) {
  ROLA_CHECK(out && lse, "sparse_attn_fwd_lse: null pointer");
  ROLA_CHECK(aligned16(lse), "sparse_attn_fwd_lse: lse must be 16-byte aligned");
  return sparse_attn_impl(q, k, qk_sB, qk_sH, qk_sT, v, v_sB, v_sH, v_sT, lut, B, L, H, blk, topk, nullptr, nullptr,
                          nullptr, nullptr, 0, 0, 0, nullptr, nullptr, 0.f, out, nullptr, o_sB, o_sH, o_sT, nullptr,
                          stream, lse);
}

struct BwdLayout {
  size_t delta, map, inv, total;
  int NB, NT, Lpad, width;
};

static BwdLayout bwd_layout(int B, int L, int H, int blk) {
  BwdLayout f{};
  f.NB = (L + blk - 1) / blk;
  f.NT = (L + 127) / 128;
  f.Lpad = 128 * f.NT;
  f.width = f.NB + 2;
  const size_t BH = (size_t)B * H;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  f.delta = take(BH * f.Lpad * 4);
  f.map = take(BH * f.NB * f.NB);
  f.inv = take(BH * f.NT * f.width * 4);
  f.total = off;
  return f;
}

size_t rola_b200_sparse_attn_bwd_workspace(int B, int L, int H, int blk) {
  if (B <= 0 || L <= 0 || H <= 0 || (blk != 64 && blk != 128)) return 0;
  return bwd_layout(B, L, H, blk).total;
}

int rola_b200_sparse_attn_bwd(const void* q, const void* k, int64_t qk_sB, int64_t qk_sH, int64_t qk_sT, const void* v,
                              int64_t v_sB, int64_t v_sH, int64_t v_sT, const void* out, const void* dout, int64_t o_sB,
                              int64_t o_sH, int64_t o_sT, const int32_t* lut, const int32_t* paired, const float* lse,
                              int B, int L, int H, int blk, int topk, void* dq, void* dk, void* dv, int64_t g_sB,
                              int64_t g_sH, int64_t g_sT, void* workspace, size_t workspace_bytes,
                              rola_stream_t stream) {
  ROLA_CHECK(q && k && v && out && dout && lut && lse && dq && dk && dv && workspace,
             "sparse_attn_bwd: null pointer");
  ROLA_CHECK(blk == 128 || blk == 64, "sparse_attn_bwd: block size must be 128 or 64");
  ROLA_CHECK(blk == 128 || paired, "sparse_attn_bwd: block 64 needs the paired table");
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && (int64_t)B * H < 65536, "sparse_attn_bwd: bad sizes");
  const BwdLayout f = bwd_layout(B, L, H, blk);
  ROLA_CHECK(f.NB < (1 << 28), "sparse_attn_bwd: too many blocks");
  ROLA_CHECK(topk >= 1 && topk <= f.NB, "sparse_attn_bwd: topk must be in [1, NB]");
  ROLA_CHECK(workspace_bytes >= f.total, "sparse_attn_bwd: workspace of %zu bytes < %zu", workspace_bytes, f.total);
  ROLA_CHECK(aligned16(workspace) && aligned16(lse), "sparse_attn_bwd: workspace and lse must be 16-byte aligned");
  ROLA_CHECK(aligned16(out) && aligned16(dout) && o_sB % 8 == 0 && o_sH % 8 == 0 && o_sT % 8 == 0,
             "sparse_attn_bwd: out / dout rows must be 16-byte aligned");
  ROLA_CHECK(aligned16(dq) && aligned16(dk) && aligned16(dv) && g_sB % 8 == 0 && g_sH % 8 == 0 && g_sT % 8 == 0,
             "sparse_attn_bwd: gradient rows must be 16-byte aligned");
  CUtensorMap tq, tk, tv, tdo;
  // 64-row boxes: the kernels stage 64-row steps and stack two boxes for the 128-row tiles
  ROLA_TRY(make_head_map(&tq, q, 128, qk_sB, qk_sH, qk_sT, L, H, B, "sparse_attn_bwd: q", 64));
  ROLA_TRY(make_head_map(&tk, k, 128, qk_sB, qk_sH, qk_sT, L, H, B, "sparse_attn_bwd: k", 64));
  ROLA_TRY(make_head_map(&tv, v, 128, v_sB, v_sH, v_sT, L, H, B, "sparse_attn_bwd: v", 64));
  ROLA_TRY(make_head_map(&tdo, dout, 128, o_sB, o_sH, o_sT, L, H, B, "sparse_attn_bwd: dout", 64));
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* delta = reinterpret_cast<float*>(ws + f.delta);
  int32_t* inv = reinterpret_cast<int32_t*>(ws + f.inv);
  cudaStream_t st = S(stream);
  ROLA_TRY(cuda_status(
      launch_attn_bwd_delta(BF(out), o_sB, o_sH, o_sT, BF(dout), o_sB, o_sH, o_sT, B, H, L, f.Lpad, delta, st),
      "sparse_attn_bwd/delta"));
  ROLA_TRY(cuda_status(launch_lut_invert(lut, B * H, f.NB, f.NB, topk, blk == 64, ws + f.map, inv, f.width, st),
                       "sparse_attn_bwd/lut_invert"));
  AttnBwdParams p{};
  p.lut = blk == 64 ? paired : lut;
  p.inv = inv;
  p.inv_width = f.width;
  p.lse = lse;
  p.delta = delta;
  p.dq = BFm(dq);
  p.dk = BFm(dk);
  p.dv = BFm(dv);
  p.g_sB = g_sB;
  p.g_sH = g_sH;
  p.g_sT = g_sT;
  p.B = B;
  p.L = L;
  p.H = H;
  p.NBq = f.NB;
  p.NBk = f.NB;
  p.NQT = f.NT;
  p.NKT = f.NT;
  p.Lpad = f.Lpad;
  p.topk = topk;
  p.blk64 = blk == 64;
  p.qk_scale = (float)(0.08838834764831845 * 1.4426950408889634);  // 128^-0.5 * log2(e)
  return cuda_status(launch_attn_bwd(tq, tk, tv, tdo, p, st), "sparse_attn_bwd");
}

// ---------------------------------------------------------------------------
// whole layer
// ---------------------------------------------------------------------------
struct FwdLayout {
  size_t qkv, ssq, q_rope, k_rope, q_normed, k_normed, gate, pooled_q, pooled_k, ksum, center, scores, lut, q_lr,
      c_partial, ct, total;
};

static FwdLayout fwd_layout(int B, int L, int H, int blk, int R, int splits, int topk) {
  const size_t BL = (size_t)B * L, dim = (size_t)H * 128, NB = (size_t)(L + blk - 1) / blk;
  FwdLayout f{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  f.qkv = take(BL * 3 * dim * 2);
  f.ssq = take(BL * (3 * dim / 256) * 4);
  f.q_rope = take(BL * dim * 2);
  f.k_rope = take(BL * dim * 2);
  f.q_normed = take(BL * dim * 2);
  f.k_normed = take(BL * dim * 2);
  f.gate = take(BL * H * 2);
  f.pooled_q = take((size_t)B * H * NB * 128 * 2);
  f.pooled_k = take((size_t)B * H * NB * 128 * 2);
  f.ksum = take((size_t)B * NB * dim * 4);
  f.center = take((size_t)B * dim * 2);
  f.scores = take((size_t)B * H * NB * NB * 4);
  f.lut = take((size_t)B * H * NB * (size_t)topk * 4);
  f.q_lr = take(BL * H * R * 2);
  f.c_partial = take((size_t)lowrank_chunks(L) * B * H * R * 128 * 4);
  f.ct = take((size_t)B * H * 128 * R * 2);
  f.total = off;
  return f;
}

size_t rola_b200_forward_workspace_bytes(int B, int L, int H, int blk, int R, int splits) {
  if (B <= 0 || L <= 0 || H <= 0 || blk <= 0 || R <= 0 || splits <= 0) return 0;
  const int NB = (L + blk - 1) / blk;
  return fwd_layout(B, L, H, blk, R, splits, NB).total;  // sized for the largest topk
}

int rola_b200_rola_forward(const void* x, const void* w_qkv, const void* b_qkv, const void* norm_wq,
                           const void* norm_wk, const float* cos_sin, const void* lr_cos, const void* lr_sin,
                           int rope_dim, const void* proj_q, const void* proj_k, const void* gate_w,
                           const void* gate_b, int B, int L, int H, int blk, int topk, int R, int splits, float eps,
                           void* workspace, size_t workspace_bytes, void* out, int32_t* lut_out,
                           rola_stream_t stream) {
  ROLA_CHECK(x && w_qkv && norm_wq && norm_wk && cos_sin && proj_q && proj_k && gate_w && gate_b && workspace && out,
             "rola_forward: null pointer");
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && H <= 40 && H % 2 == 0 && blk == 128 && R == 64 && splits > 0,
             "rola_forward: bad sizes (even H <= 40, blk 128, R 64)");
  const int NB = (L + blk - 1) / blk;
  ROLA_CHECK(topk >= 1 && topk <= NB, "rola_forward: topk must be in [1, NB]");
  const FwdLayout f = fwd_layout(B, L, H, blk, R, splits, NB);
  ROLA_CHECK(workspace_bytes >= f.total, "rola_forward: workspace too small (%zu < %zu)", workspace_bytes, f.total);
  ROLA_CHECK((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, "rola_forward: workspace must be 256-byte aligned");
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const int64_t dim = (int64_t)H * 128;
  const int64_t M = (int64_t)B * L;
  __nv_bfloat16* qkv = reinterpret_cast<__nv_bfloat16*>(ws + f.qkv);
  int32_t* lut = lut_out ? lut_out : reinterpret_cast<int32_t*>(ws + f.lut);
  float* ssq = reinterpret_cast<float*>(ws + f.ssq);
  const int ssq_ld = (int)(3 * dim / 256);
  ROLA_TRY(rola_b200_qkv_gemm(x, w_qkv, b_qkv, qkv, ssq, M, 3 * dim, dim, stream));
  ROLA_TRY(rola_b200_qk_norm_rope(qkv, qkv + dim, 3 * dim, ssq, ssq_ld, x, norm_wq, norm_wk, cos_sin, gate_w,
                                  gate_b, B, L, H, blk, eps, ws + f.q_rope, ws + f.k_rope, ws + f.q_normed,
                                  ws + f.k_normed, ws + f.gate, ws + f.pooled_q, reinterpret_cast<float*>(ws + f.ksum),
                                  stream));
  // fork: selection on the high-priority side stream (queued first), the
  // low-rank branches on the other two
  ForkJoin* fj = nullptr;
  ROLA_TRY(forkjoin_get(&fj));
  std::lock_guard<std::mutex> lock(fj->mu);
  cudaError_t ce = cudaEventRecord(fj->fork, S(stream));
  for (int i = 0; i < 3 && ce == cudaSuccess; ++i) ce = cudaStreamWaitEvent(fj->side[i], fj->fork, 0);
  if (ce != cudaSuccess) return fail(ROLA_ERR_CUDA, "rola_forward: %s", cudaGetErrorString(ce));
  const int64_t Ld = (int64_t)L * dim;
  ROLA_TRY(rola_b200_center_from_sums(reinterpret_cast<float*>(ws + f.ksum), B, NB, (int)dim, L, ws + f.center,
                                      fj->side[2]));
  ROLA_TRY(rola_b200_mean_pool(ws + f.k_rope, (int64_t)L * dim, 128, dim, B, H, L, blk, ws + f.center,
                               ws + f.pooled_k, fj->side[2]));
  ROLA_TRY(rola_b200_block_select(ws + f.pooled_q, ws + f.pooled_k, B * H, NB, NB, topk,
                                  reinterpret_cast<float*>(ws + f.scores), lut, fj->side[2]));
  ROLA_TRY(rola_b200_lowrank_kv(ws + f.k_normed, Ld, 128, dim, qkv + 2 * dim, 3 * Ld, 128, 3 * dim, proj_k, lr_cos,
                                lr_sin, rope_dim, B, L, H, R, splits, reinterpret_cast<float*>(ws + f.c_partial),
                                nullptr, ws + f.ct, fj->side[0]));
  ROLA_TRY(rola_b200_lowrank_q(ws + f.q_normed, Ld, 128, dim, proj_q, lr_cos, lr_sin, rope_dim, B, L, H, R,
                               ws + f.q_lr, fj->side[1]));
  // join before the attention
  for (int i = 0; i < 3 && ce == cudaSuccess; ++i) {
    ce = cudaEventRecord(fj->join[i], fj->side[i]);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(S(stream), fj->join[i], 0);
  }
  if (ce != cudaSuccess) return fail(ROLA_ERR_CUDA, "rola_forward: %s", cudaGetErrorString(ce));
  return rola_b200_sparse_attn(ws + f.q_rope, ws + f.k_rope, Ld, 128, dim, qkv + 2 * dim, 3 * Ld, 128, 3 * dim, lut,
                               B, L, H, blk, topk, ws + f.q_lr, ws + f.ct, ws + f.gate, nullptr, 0, 0, 0, nullptr,
                               nullptr, 0.0078125f, out, nullptr, Ld, 128, dim, stream);
}

}  // extern "C"
