// paged_noalloc.cu — cie_paged_attn_noalloc: the paged decode / verify kernel
// for callers that cannot allocate device memory.
//
// Some hosts cannot hand this library a workspace: an engine that owns every
// byte of device memory and gives its plugins no allocator, or a serving loop
// where a cudaMalloc (which synchronises the device) is not acceptable between
// steps. For them this entry point keeps the split-KV partial results in a
// fixed scratch array that lives in the library's own device image
// (kNoAllocScratchBytes per GPU, held from the moment the library's kernels are
// loaded on that GPU until the process exits). It never calls cudaMalloc,
// cudaFree or any allocating routine.
//
// The array is shared by every call on a device and keeps whatever the last
// call wrote. Nothing in it has to start at zero: every partial result the
// merge kernel reads was written by the same call. Calls whose kernels overlap
// on the GPU (different streams, or different host threads on one stream
// without ordering) race on the array and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "cie_common.cuh"

namespace cie {

// 32 MiB: enough for the split-KV partials of a 64-sequence decode batch
// (Llama-3.2-1B shape, 8K context) at the default partition size; larger
// batches get larger partitions automatically (see below).
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_paged_noalloc_scratch[kNoAllocScratchBytes];

typedef CUresult (*PFN_ctxGetCurrent_t)(CUcontext*);

// The driver's cuCtxGetCurrent, resolved once through the runtime (no
// link-time dependency on libcuda); nullptr if unavailable.
static PFN_ctxGetCurrent_t ctx_get_current() {
  static PFN_ctxGetCurrent_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_ctxGetCurrent_t>(ptr);
  });
  return fn;
}

// Device address of the scratch array for the current device. Resolved once
// per device, with that device current, on the first call made on it, and
// again whenever the device's current context is not the one the address was
// resolved in (after cudaDeviceReset the old address is gone; a program that
// makes its own context current gets that context's copy of the array).
static int noalloc_scratch(void** out) {
  constexpr int kMaxDevices = 64;
  static void* ptrs[kMaxDevices] = {};
  static CUcontext ctxs[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("cie_paged_attn_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return CIE_ERR_LAUNCH;
  }
  // No context yet (or no way to ask) means no cached address can be trusted;
  // cudaGetSymbolAddress then sets up the device's primary context itself.
  PFN_ctxGetCurrent_t get_ctx = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get_ctx != nullptr && get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr || ctx == nullptr || ctxs[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_paged_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("cie_paged_attn_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return CIE_ERR_LAUNCH;
    }
    if (get_ctx != nullptr && get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    ptrs[dev] = p;
    ctxs[dev] = ctx;
  }
  *out = ptrs[dev];
  return CIE_OK;
}

}  // namespace cie

using namespace cie;

extern "C" int cie_paged_attn_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                      const int32_t* block_tables, const int32_t* kv_lens,
                                      void* o, int B, int Hq, int Hkv, int M, int d,
                                      int num_blocks, int block_size, int max_blocks,
                                      const int64_t* q_strides, const int64_t* o_strides,
                                      float scale, int causal, int dtype, const float* rope_cos,
                                      const float* rope_sin, int rope_max_pos, int split_tokens,
                                      void* stream) {
  // Partition size: the caller's, which must fit the scratch array, or (0) the
  // library's default partition size, doubled until the partial results fit
  // (one partition per sequence needs no scratch at all).
  int split = split_tokens;
  size_t need = cie_paged_attn_workspace(B, Hq, Hkv, M, d, block_size, max_blocks, split);
  if (split_tokens == 0 && need > kNoAllocScratchBytes && Hkv > 0 && Hq % Hkv == 0) {
    const int max_len = max_blocks * block_size;
    split = make_plan(B, Hq, Hkv, M, d, max_len, 0).split_tokens;
    while (need > kNoAllocScratchBytes && split < max_len) {
      split *= 2;
      need = cie_paged_attn_workspace(B, Hq, Hkv, M, d, block_size, max_blocks, split);
    }
  }
  if (need > kNoAllocScratchBytes) {
    set_error("cie_paged_attn_noalloc: split-KV partials need %zu bytes but the fixed scratch "
              "holds %zu; pass a larger split_tokens (or 0)", need, kNoAllocScratchBytes);
    return CIE_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch(&scratch);
    if (rc != CIE_OK) return rc;
  }
  return cie_paged_attn(q, k_pool, v_pool, block_tables, kv_lens, o, B, Hq, Hkv, M, d,
                        num_blocks, block_size, max_blocks, q_strides, o_strides, scale, causal,
                        dtype, rope_cos, rope_sin, rope_max_pos, split, scratch,
                        need > 0 ? kNoAllocScratchBytes : 0, stream);
}
