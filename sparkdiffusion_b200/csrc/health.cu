// Self-test of the library's failure detection (no counterpart in the
// reference).  Every spin of the kernels on an mbarrier, a flag or a peer is a
// bounded wait that gives up after a wall-time limit, records a ROLA_DEV_*
// code in the device error flag and lets the kernel return, so that a lost
// hand-off ends as an error the host reads with rola_b200_device_status()
// instead of a hung GPU.  rola_b200_check_wait_timeout exercises exactly that
// path with a short limit: one thread waits on an mbarrier that nothing will
// ever complete, the wait expires, the flag is set and the kernel exits.  The
// context stays usable afterwards.
#include "../../include/rola_b200.h"
#include "common.cuh"

namespace rola {

__device__ int g_probe_gave_up = 0;

__global__ void wait_timeout_probe(uint64_t limit_ns) {
  __shared__ uint64_t bar_word;
  if (threadIdx.x != 0) return;
  const uint32_t bar = smem_u32(&bar_word);
  mbar_init(bar, 1);  // one arrival expected; none will come
  fence_barrier_init();
  const uint64_t t0 = globaltimer_ns();
  bool done = false;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, 0)) {
      done = true;
      break;
    }
    if ((it & 255u) == 255u && globaltimer_ns() - t0 > limit_ns) break;
  }
  if (!done) set_device_error(kDevTimeoutLoad);
  g_probe_gave_up = done ? 0 : 1;
}

}  // namespace rola

extern "C" int rola_b200_check_wait_timeout(unsigned limit_us, rola_stream_t stream) {
  using namespace rola;
  ROLA_CHECK(limit_us >= 1 && limit_us <= 1000000u, "check_wait_timeout: limit_us must be in [1, 1e6]");
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  wait_timeout_probe<<<1, 32, 0, st>>>((uint64_t)limit_us * 1000ull);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  int gave_up = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&gave_up, g_probe_gave_up, sizeof(int));
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "check_wait_timeout: %s", cudaGetErrorString(e));
  return gave_up == 1 ? ROLA_OK : fail(ROLA_ERR_DEVICE, "check_wait_timeout: the unfulfilled wait completed");
}
