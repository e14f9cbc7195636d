// Host-buffer pipeline around rola_b200_rola_forward: each call uploads one
// step's hidden states from pinned host memory, runs the forward and downloads
// the result, on three streams with double-buffered device copies of x and
// out, so that step s+1's upload and step s-1's download overlap step s's
// kernels (PCIe is full duplex; the copy engines do not take SMs).
//
// Included in the unity translation unit after capi.cu (shares its helpers).

struct rola_pipeline {
  int device;
  size_t x_bytes, out_bytes;
  void* x_dev[2];
  void* out_dev[2];
  cudaStream_t h2d, compute, d2h;
  cudaEvent_t x_ready[2], x_free[2], out_ready[2], out_free[2], caller, done;
  unsigned long long steps;
};

namespace {
void pipeline_release(rola_pipeline* p) {
  if (!p) return;
  for (int i = 0; i < 2; ++i) {
    if (p->x_dev[i]) cudaFree(p->x_dev[i]);
    if (p->out_dev[i]) cudaFree(p->out_dev[i]);
    for (cudaEvent_t e : {p->x_ready[i], p->x_free[i], p->out_ready[i], p->out_free[i]})
      if (e) cudaEventDestroy(e);
  }
  if (p->caller) cudaEventDestroy(p->caller);
  if (p->done) cudaEventDestroy(p->done);
  for (cudaStream_t s : {p->h2d, p->compute, p->d2h})
    if (s) cudaStreamDestroy(s);
  delete p;
}
}  // namespace

extern "C" {

int rola_b200_pipeline_create(size_t x_bytes, size_t out_bytes, rola_pipeline** out) {
  ROLA_CHECK(out && x_bytes > 0 && out_bytes > 0, "pipeline_create: null pointer or zero size");
  *out = nullptr;
  rola_pipeline* p = new rola_pipeline();
  cudaGetDevice(&p->device);
  p->x_bytes = x_bytes;
  p->out_bytes = out_bytes;
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
    e = cudaMalloc(&p->x_dev[i], x_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&p->out_dev[i], out_bytes);
    for (cudaEvent_t* ev : {&p->x_ready[i], &p->x_free[i], &p->out_ready[i], &p->out_free[i]})
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->caller, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming);
  for (cudaStream_t* s : {&p->h2d, &p->compute, &p->d2h})
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    pipeline_release(p);
    return fail(ROLA_ERR_CUDA, "pipeline_create: %s", cudaGetErrorString(e));
  }
  *out = p;
  return ROLA_OK;
}

int rola_b200_pipeline_forward(rola_pipeline* pl, const void* x_host, const void* w_qkv, const void* b_qkv,
                               const void* norm_wq, const void* norm_wk, const float* cos_sin, const void* lr_cos,
                               const void* lr_sin, int rope_dim, const void* proj_q, const void* proj_k,
                               const void* gate_w, const void* gate_b, int B, int L, int H, int blk, int topk, int R,
                               int splits, float eps, void* workspace, size_t workspace_bytes, void* out_host,
                               rola_stream_t stream) {
  ROLA_CHECK(pl && x_host && out_host, "pipeline_forward: null pointer");
  const size_t dim = (size_t)H * 128;
  ROLA_CHECK((size_t)B * L * dim * 2 <= pl->x_bytes && (size_t)B * L * dim * 2 <= pl->out_bytes,
             "pipeline_forward: sizes exceed the pipeline's device buffers");
  const size_t bytes = (size_t)B * L * dim * 2;
  const int i = (int)(pl->steps & 1);
  cudaError_t e = cudaSuccess;
  // the caller's earlier work (weights, tables) precedes this step's kernels
  e = cudaEventRecord(pl->caller, S(stream));
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->compute, pl->caller, 0);
  // upload into buffer i once the step that last read it (s-2) finished its kernels
  if (e == cudaSuccess && pl->steps >= 2) e = cudaStreamWaitEvent(pl->h2d, pl->x_free[i], 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(pl->x_dev[i], x_host, bytes, cudaMemcpyHostToDevice, pl->h2d);
  if (e == cudaSuccess) e = cudaEventRecord(pl->x_ready[i], pl->h2d);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->compute, pl->x_ready[i], 0);
  // out buffer i is free once step s-2's download finished
  if (e == cudaSuccess && pl->steps >= 2) e = cudaStreamWaitEvent(pl->compute, pl->out_free[i], 0);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "pipeline_forward: %s", cudaGetErrorString(e));
  ROLA_TRY(rola_b200_rola_forward(pl->x_dev[i], w_qkv, b_qkv, norm_wq, norm_wk, cos_sin, lr_cos, lr_sin, rope_dim,
                                  proj_q, proj_k, gate_w, gate_b, B, L, H, blk, topk, R, splits, eps, workspace,
                                  workspace_bytes, pl->out_dev[i], nullptr, pl->compute));
  e = cudaEventRecord(pl->x_free[i], pl->compute);
  if (e == cudaSuccess) e = cudaEventRecord(pl->out_ready[i], pl->compute);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->d2h, pl->out_ready[i], 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out_host, pl->out_dev[i], bytes, cudaMemcpyDeviceToHost, pl->d2h);
  if (e == cudaSuccess) e = cudaEventRecord(pl->out_free[i], pl->d2h);
  if (e == cudaSuccess) e = cudaEventRecord(pl->done, pl->d2h);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "pipeline_forward: %s", cudaGetErrorString(e));
  ++pl->steps;
  return ROLA_OK;
}

int rola_b200_pipeline_wait(rola_pipeline* pl, rola_stream_t stream) {
  ROLA_CHECK(pl, "pipeline_wait: null pointer");
  if (pl->steps == 0) return ROLA_OK;
  const cudaError_t e = cudaStreamWaitEvent(S(stream), pl->done, 0);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "pipeline_wait: %s", cudaGetErrorString(e));
  return ROLA_OK;
}

int rola_b200_pipeline_destroy(rola_pipeline* pl) {
  ROLA_CHECK(pl, "pipeline_destroy: null pointer");
  const cudaError_t e = cudaStreamSynchronize(pl->d2h);
  cudaStreamSynchronize(pl->compute);
  cudaStreamSynchronize(pl->h2d);
  pipeline_release(pl);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "pipeline_destroy: %s", cudaGetErrorString(e));
  return ROLA_OK;
}

}  // extern "C"
