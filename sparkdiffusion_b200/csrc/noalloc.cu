// Allocation-free variant of the low-rank C reduction (rola_b200_lowrank_kv).
//
// Some callers cannot hand this library a workspace or let it allocate one:
// an inference server or host framework that owns a fixed device-memory pool
// and forbids allocations outside it, or a latency-critical loop where
// cudaMalloc/cudaFree (which may synchronise the device) is not acceptable,
// or a foreign-language binding with no CUDA allocator at hand.  For them,
// rola_b200_lowrank_kv_noalloc keeps its fp32 partial sums in a fixed scratch
// array compiled into the library instead of a caller-provided buffer.
//
// The scratch is a file-scope __device__ array of kNoallocScratchFloats fp32
// values (16 MiB).  Every GPU that loads the library holds it until the
// process exits.  In host code the array's name is only a host-side handle,
// so its device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and passed to the kernels.
//
// Every call uses the same array and leaves its contents behind.  Nothing
// needs clearing: each CTA of the reduction overwrites every partial slot it
// owns before the final sum reads it.  Calls that overlap on the GPU (two
// streams, or two host threads on one device) race on the array; callers must
// serialise them.
#include <mutex>

#include "../../include/rola_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace rola {
namespace {

constexpr size_t kNoallocScratchFloats = size_t(4) << 20;  // 4 Mi floats = 16 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoallocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up on the
// first call for that device (so the first call on a device should not be
// issued while a stream on it is being captured).
int noalloc_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "lowrank_kv_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(ROLA_ERR_INVALID, "lowrank_kv_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(ROLA_ERR_CUDA, "lowrank_kv_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return ROLA_OK;
}

}  // namespace
}  // namespace rola

extern "C" int rola_b200_lowrank_kv_noalloc(const void* k_normed, int64_t k_sB, int64_t k_sH, int64_t k_sT,
                                            const void* v, int64_t v_sB, int64_t v_sH, int64_t v_sT,
                                            const void* proj_k, const void* lr_cos, const void* lr_sin, int rope_dim,
                                            int B, int L, int H, int R, int splits, void* C, void* Ct,
                                            rola_stream_t stream) {
  using namespace rola;
  ROLA_CHECK(B > 0 && L > 0 && H > 0 && R > 0 && splits > 0, "lowrank_kv_noalloc: bad sizes");
  const size_t need = (size_t)lowrank_chunks(L) * B * H * R * 128;
  ROLA_CHECK(need <= kNoallocScratchFloats,
             "lowrank_kv_noalloc: chunks*B*H*R*D = %zu fp32 partials (one per 1024 tokens) exceed the fixed "
             "scratch of %zu (16 MiB); use rola_b200_lowrank_kv with a workspace",
             need, kNoallocScratchFloats);
  float* scratch = nullptr;
  ROLA_TRY(noalloc_scratch(&scratch));
  return rola_b200_lowrank_kv(k_normed, k_sB, k_sH, k_sT, v, v_sB, v_sH, v_sT, proj_k, lr_cos, lr_sin, rope_dim, B,
                              L, H, R, splits, scratch, C, Ct, stream);
}
