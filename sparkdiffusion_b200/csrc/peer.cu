// Peer memory for the fused sequence<->head exchanges: device buffers that the
// other ranks of the node map through CUDA IPC, so that the norm pass and the
// attention epilogue store their rows straight into the rank that consumes
// them (plain peer stores over NVLink; no multicast objects are created).
//
// Included in the unity translation unit after capi.cu (shares its helpers).

extern "C" {

int rola_b200_peer_alloc(size_t bytes, void** ptr, unsigned char* handle) {
  ROLA_CHECK(ptr && handle && bytes > 0, "peer_alloc: null pointer or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(ROLA_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == ROLA_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return ROLA_OK;
}

int rola_b200_peer_open(const unsigned char* handle, void** ptr) {
  ROLA_CHECK(ptr && handle, "peer_open: null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "peer_open: %s", cudaGetErrorString(e));
  *ptr = p;
  return ROLA_OK;
}

int rola_b200_peer_close(void* ptr) {
  ROLA_CHECK(ptr, "peer_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "peer_close: %s", cudaGetErrorString(e));
  return ROLA_OK;
}

int rola_b200_peer_free(void* ptr) {
  ROLA_CHECK(ptr, "peer_free: null pointer");
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(ROLA_ERR_CUDA, "peer_free: %s", cudaGetErrorString(e));
  return ROLA_OK;
}

}  // extern "C"
