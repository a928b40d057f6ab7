// api.cu — library-wide C-ABI entry points: error message retrieval, the
// per-device status word and the version string.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "cie_common.cuh"

namespace cie {

PFN_encodeTiled_t tensor_map_encoder() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(ptr);
  });
  return fn;
}

static thread_local char t_last_error[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

}  // namespace cie

using namespace cie;

extern "C" int cie_get_last_error(char* buf, int buf_len) {
  if (buf == nullptr || buf_len <= 0) return CIE_ERR_INVALID;
  std::strncpy(buf, t_last_error, static_cast<size_t>(buf_len) - 1);
  buf[buf_len - 1] = '\0';
  return CIE_OK;
}

extern "C" int cie_device_status(int* status_out, int clear, void* stream) {
  CIE_CHECK_ARG(status_out != nullptr, "cie_device_status: null output");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_device_status, sizeof(v), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_error("cie_device_status: %s", cudaGetErrorString(e));
    return CIE_ERR_LAUNCH;
  }
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice,
                                st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
      set_error("cie_device_status: %s", cudaGetErrorString(e));
      return CIE_ERR_LAUNCH;
    }
  }
  *status_out = static_cast<int>(v);
  return CIE_OK;
}

extern "C" int cie_set_wait_limit(uint64_t limit_ns, uint64_t* previous_ns) {
  uint64_t prev = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&prev, g_wait_limit_ns, sizeof(prev));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_wait_limit_ns, &limit_ns, sizeof(limit_ns));
  if (e != cudaSuccess) {
    set_error("cie_set_wait_limit: %s", cudaGetErrorString(e));
    return CIE_ERR_LAUNCH;
  }
  if (previous_ns) *previous_ns = prev;
  return CIE_OK;
}

extern "C" const char* cie_version(void) { return "cie_attn 0.1.0 sm_100a"; }
