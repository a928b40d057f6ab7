// cie_common.cuh — shared host/device definitions of libcie_attn.so:
// the per-device status word, the thread-local error message and argument
// checking helpers used by every C-ABI entry point.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "../../include/cie_attn.h"

namespace cie {

// Per-device status word. Kernels OR CIE_DEV_* bits into it when they detect
// a bad block id, an out-of-table RoPE position or a wait that timed out;
// cie_device_status() reads and optionally clears it. The library is built as
// one translation unit (libcie_attn.cu), so this is its only definition.
__device__ unsigned int g_device_status = 0;

__device__ __forceinline__ void raise_status(unsigned int bits) {
  atomicOr(&g_device_status, bits);
}

// Upper bound for any single wait inside a kernel (nanoseconds). Pipeline
// waits (a role waiting for another role's data or a free stage) read the
// per-device value g_wait_limit_ns, which starts at this default and can be
// changed at run time (cie_set_wait_limit); the abort path's drain waits (work
// already in flight landing before shared memory or TMEM is released) always
// use the default.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ uint64_t g_wait_limit_ns = kWaitLimitNs;

// ---------------------------------------------------------------- host side
void set_error(const char* fmt, ...);

#define CIE_CHECK_ARG(cond, ...)        \
  do {                                  \
    if (!(cond)) {                      \
      ::cie::set_error(__VA_ARGS__);    \
      return CIE_ERR_INVALID;           \
    }                                   \
  } while (0)

#define CIE_CHECK_LAUNCH(what)                                                        \
  do {                                                                                \
    cudaError_t e__ = cudaGetLastError();                                             \
    if (e__ != cudaSuccess) {                                                         \
      ::cie::set_error("%s: launch failed: %s", what, cudaGetErrorString(e__));       \
      return CIE_ERR_LAUNCH;                                                          \
    }                                                                                 \
  } while (0)

inline int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n > 0 ? n : 148;
}

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                      const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                      const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion,
                                      CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver, resolved once through the runtime
// (no link-time dependency on libcuda); nullptr if unavailable.
PFN_encodeTiled_t tensor_map_encoder();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace cie
