// peer_barrier.cu — a stream-ordered barrier across the GPUs of a kv-head-group
// sharded attention (one process per GPU), through flags in peer memory.
//
// The fused prefill (cie_prefill_attn_peers) writes every output tile to the
// other GPUs' outputs with peer stores. Rank r's barrier launch, queued behind
// that kernel, publishes "epoch e reached" into every rank's flag array and
// then waits until all ranks published e into its own array: afterwards every
// GPU's output holds every rank's rows. The wait is bounded by the pipeline
// wait limit (cie_set_wait_limit); a rank that never arrives ends it with
// CIE_DEV_TIMEOUT in the status word instead of a hang.
#include <cuda_runtime.h>

#include <cstdint>

#include "cie_common.cuh"
#include "sm100_ptx.cuh"

namespace cie {

constexpr int kMaxRanks = 8;

struct PeerBarrierParams {
  uint32_t* flags[kMaxRanks];  // flags[r]: rank r's array of world counters, as mapped here
  int world, rank;
  uint32_t epoch;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(const PeerBarrierParams p) {
  const int i = threadIdx.x;
  if (i >= p.world) return;
  // everything this GPU wrote before this launch (the peer stores of the
  // preceding kernel included) is ordered before the flag
  __threadfence_system();
  st_release_sys(p.flags[i] + p.rank, p.epoch);
  const uint32_t* mine = p.flags[p.rank] + i;
  const uint64_t limit = *reinterpret_cast<const volatile uint64_t*>(&g_wait_limit_ns);
  const uint64_t t0 = globaltimer_ns();
  // counters only grow; compare modulo 2^32
  while (static_cast<int32_t>(ld_acquire_sys(mine) - p.epoch) < 0) {
    if (globaltimer_ns() - t0 > limit) {
      raise_status(CIE_DEV_TIMEOUT);
      break;
    }
  }
}

}  // namespace cie

using namespace cie;

extern "C" int cie_peer_barrier(uint32_t* const* flags, int world, int rank, uint32_t epoch,
                                void* stream) {
  CIE_CHECK_ARG(world >= 1 && world <= kMaxRanks, "cie_peer_barrier: world must be in [1, %d]",
                kMaxRanks);
  CIE_CHECK_ARG(rank >= 0 && rank < world, "cie_peer_barrier: rank %d outside [0, %d)", rank,
                world);
  CIE_CHECK_ARG(flags != nullptr, "cie_peer_barrier: null flags");
  PeerBarrierParams prm{};
  for (int r = 0; r < world; ++r) {
    CIE_CHECK_ARG(flags[r] != nullptr && (reinterpret_cast<uintptr_t>(flags[r]) & 3) == 0,
                  "cie_peer_barrier: flag array %d null or unaligned", r);
    prm.flags[r] = flags[r];
  }
  prm.world = world;
  prm.rank = rank;
  prm.epoch = epoch;
  peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(prm);
  CIE_CHECK_LAUNCH("peer_barrier_kernel");
  return CIE_OK;
}
