// Single translation unit of librola_b200.so: the kernels share one device
// error flag (defined in capi.cu), which needs them in one unit without
// relocatable device code.
#include "prologue.cu"
#include "select.cu"
#include "lowrank.cu"
#include "gemm.cu"
#include "attn.cu"
#include "attn_bwd.cu"
#include "capi.cu"
#include "peer.cu"
#include "pipeline.cu"
#include "noalloc.cu"
#include "health.cu"
