// libcie_attn.cu — single translation unit of libcie_attn.so. The kernels
// share one per-device status word (g_device_status), so they are compiled
// together instead of with relocatable device code.
#include "api.cu"
#include "kv_ops.cu"
#include "paged_attn.cu"
#include "paged_noalloc.cu"
#include "prefill_attn.cu"
#include "int8_gemm.cu"
#include "peer_barrier.cu"
