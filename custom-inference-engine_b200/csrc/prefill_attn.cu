// prefill_attn.cu — causal / non-causal grouped-query flash attention for
// prefill on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Semantics follow kernels/ref/flash_attention_ref.py:8-56 (fp32 reference)
// and the Triton entry kernels/flash_attention.py:136-209: out = softmax(
// q k^T * scale + bottom-right causal mask) v, with the kv head of q head h
// being h / (Hq / Hkv) (no K/V expansion), optional half-split RoPE of q
// applied to the Q tiles in shared memory (kernels/ref/rope_apply_ref.py:22-53).
//
// One CTA owns two 128-row query tiles (Q0, Q1) of one (batch, head) and
// streams 128-key K/V tiles through a TMA ring shared by both:
//   warp 0      TMA producer: Q0/Q1 once, then K_j into a ring of K stages
//   warp 2      TMA producer: V_j into a ring of V stages
//   warp 1      TMEM allocator and single-thread tcgen05.mma issuer
//   warps 4..7  softmax of tile 0, warps 8..11 softmax of tile 1: thread r owns
//               query row r == TMEM lane r (row max / sum need no shuffles),
//               writes P (16-bit) over its S columns in TMEM, rescales its O
//               rows in TMEM only when the running max grew by more than 2^8
//               (the stale max is exact because O and the row sum share it),
//               and stores O / l at the end.
// Tensor-core order per key tile j: PV0_j, S0_{j+1}, PV1_j, S1_{j+1}, so each
// softmax warpgroup works on its tile while the tensor core serves the other
// one. S_t accumulates in TMEM (fp32), P_t overwrites the first 64 columns of
// S_t, O_t accumulates in TMEM. MMAs of one CTA execute in issue order, so
// S_t{j+1} may be issued right behind PV_t_j that still reads P_t from the same
// columns, and the commit that signals S_t_j complete also covers PV_t_{j-1},
// which is what lets the softmax rescale O_t without a separate wait.
// The tensor core accepts about one MMA ahead of the one it executes, so any
// wait or commit in the issuing thread idles it. Per key tile the issuer
// therefore commits twice: after S0_{j+1} (softmax 0) and after S1_{j+1} on a
// ring of "step" barriers that tells softmax 1 its S is ready and tells both
// TMA producers which K and V stages are free. Readiness of the next K and V
// tiles is probed between MMAs, where the issuing thread stalls anyway.
// Causal tile pairs are ordered heaviest first across the grid.
//
// Paged variant (PAGED = true): K and V are read straight from the engine's
// paged pools (num_blocks, block_size, Hkv, d) through the block table, one
// 16-token TMA box per table lookup (block_size a multiple of 16), and each
// sequence b has its own history length kv_lens[b] (query i of the M new
// tokens sits at position kv_lens[b] - M + i). This serves prefill of a batch
// of sequences over non-empty histories (chunked prefill) in one launch, with
// no dense gather. Boxes wholly past a sequence's length (or with a refused
// block id) are fetched from outside the map and land as zeros.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "cie_common.cuh"
#include "sm100_ptx.cuh"

namespace cie {

constexpr int kPfThreads = 384;  // 3 warpgroups
// Launched at 168 registers per thread (3 warps per scheduler); warpgroup 0
// (producers, MMA issuer, an idle warp) gives registers to the two softmax
// warpgroups. The split (ctrl + 2 * softmax <= 3 * 168) is the one ptxas
// compiles without spills for each head dim.
template <int D>
constexpr int kRegsCtrl = D >= 128 ? 88 : 72;
template <int D>
constexpr int kRegsSoftmax = D >= 128 ? 208 : 216;
#ifndef CIE_KSTAGES_D128
#define CIE_KSTAGES_D128 3
#endif
#ifndef CIE_VSTAGES_D128
#define CIE_VSTAGES_D128 2
#endif
#ifndef CIE_KSTAGES_D64
#define CIE_KSTAGES_D64 4
#endif
#ifndef CIE_VSTAGES_D64
#define CIE_VSTAGES_D64 4
#endif
#ifndef CIE_MAX_CHAINS
#define CIE_MAX_CHAINS 8
#endif
constexpr int kMaxPeers = 7;     // other GPUs an output tile can be copied to
constexpr int kBM = 128;         // rows of one query tile; a CTA owns two
constexpr int kBN = 128;         // keys per K/V tile

template <int D>
struct PfCfg {
  static constexpr int KCH = D / 64;  // 128-byte swizzle chunks along d
  static constexpr int Q_BYTES = kBM * D * 2;
  static constexpr int KV_BYTES = kBN * D * 2;
  // K and V rings are sized separately: at d = 128 three K stages and two V
  // stages fill the 227 KB of shared memory next to the two Q tiles.
  static constexpr int KS = (D == 64) ? CIE_KSTAGES_D64 : CIE_KSTAGES_D128;
  static constexpr int VS = (D == 64) ? CIE_VSTAGES_D64 : CIE_VSTAGES_D128;
  // ring of per-key-tile completion barriers; deeper than either stage ring so
  // that no waiter can see a phase of the same slot one lap later
  static constexpr int R = 8;
  static_assert(R > KS && R > VS, "step ring must be deeper than the K/V rings");
  static constexpr int BAR_OFF = 2 * Q_BYTES + (KS + VS) * KV_BYTES;
  static constexpr int NBARS = 6 + KS + VS + 1 + R + 2 + 2 + 2 + 1;
  static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 /*tmem slot, abort flag, stored counters*/ + 1024 /*align*/;
  static constexpr uint32_t TM_S0 = 0, TM_S1 = 128;    // P_t aliases cols [0, 64) of S_t
  static constexpr uint32_t TM_O0 = 256, TM_O1 = 256 + D;
  static constexpr uint32_t TM_COLS = 512;
};

struct PrefillParams {
  int B, Hq, Hkv, M, N, G;
  int n_pairs;  // query tile pairs per (batch, head)
  int n_units;  // n_pairs * B * Hq: the work list the persistent grid walks
  float scale_log2;
  int causal;
  void* o;
  int64_t o_sb, o_sh, o_sm;
  const float* cos;
  const float* sin;
  int rope_max_pos;
  int rope_q_pos0;
  // paged variant
  const int32_t* kv_lens;   // (B,) history lengths including the M new tokens
  const int32_t* tables;    // (B, max_blocks) physical block ids
  int max_blocks, block_size, num_blocks;
  int pool_tokens;          // num_blocks * block_size: the map's token extent
  // output all-gather over peer memory: the same rows also go to n_peers other
  // GPUs' outputs (same layout as o, pointers already at this rank's heads)
  void* o_peers[kMaxPeers];
  int n_peers;
};

// Token coordinate of the 16-token box starting at logical position t of
// sequence b in the paged pool map; past the sequence (or for a refused block
// id) a coordinate outside the map, which TMA fills with zeros.
__device__ __forceinline__ int paged_box_coord(const PrefillParams& p, const int32_t* table,
                                               int t, int len) {
  if (t >= len) return p.pool_tokens;
  const int lb = t / p.block_size;
  const int blk = lb < p.max_blocks ? table[lb] : -1;
  if (blk < 0 || blk >= p.num_blocks) {
    raise_status(CIE_DEV_BAD_BLOCK_ID);
    return p.pool_tokens;
  }
  return blk * p.block_size + (t % p.block_size);
}

template <int D, bool BF16>
__device__ __forceinline__ void rope_q_row(uint8_t* sQt, int row, int pos, const float* cos,
                                           const float* sin) {
  constexpr int HALF = D / 2;
  const float* cr = cos + static_cast<int64_t>(pos) * HALF;
  const float* sr = sin + static_cast<int64_t>(pos) * HALF;
#pragma unroll
  for (int pc = 0; pc < HALF / 8; ++pc) {
    const int e_lo = pc * 8, e_hi = HALF + pc * 8;
    uint8_t* a_lo = sQt + (e_lo / 64) * kBM * 128 + row * 128 + ((((e_lo % 64) / 8) ^ (row & 7)) * 16);
    uint8_t* a_hi = sQt + (e_hi / 64) * kBM * 128 + row * 128 + ((((e_hi % 64) / 8) ^ (row & 7)) * 16);
    const uint4 x1 = *reinterpret_cast<uint4*>(a_lo);
    const uint4 x2 = *reinterpret_cast<uint4*>(a_hi);
    const float4 ca = *reinterpret_cast<const float4*>(cr + e_lo);
    const float4 cb = *reinterpret_cast<const float4*>(cr + e_lo + 4);
    const float4 sa = *reinterpret_cast<const float4*>(sr + e_lo);
    const float4 sb = *reinterpret_cast<const float4*>(sr + e_lo + 4);
    const float cc[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
    const float ss[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
    const uint32_t* u1 = reinterpret_cast<const uint32_t*>(&x1);
    const uint32_t* u2 = reinterpret_cast<const uint32_t*>(&x2);
    uint4 y1, y2;
    uint32_t* w1 = reinterpret_cast<uint32_t*>(&y1);
    uint32_t* w2 = reinterpret_cast<uint32_t*>(&y2);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f1 = unpack2<BF16>(u1[e]);
      const float2 f2 = unpack2<BF16>(u2[e]);
      const float c0 = cc[2 * e], c1 = cc[2 * e + 1];
      const float s0 = ss[2 * e], s1 = ss[2 * e + 1];
      // rot1 = x1*c - x2*s ; rot2 = x1*s + x2*c  (rope_apply_ref.py:49-53)
      w1[e] = pack2<BF16>(__fsub_rn(__fmul_rn(f1.x, c0), __fmul_rn(f2.x, s0)),
                          __fsub_rn(__fmul_rn(f1.y, c1), __fmul_rn(f2.y, s1)));
      w2[e] = pack2<BF16>(__fadd_rn(__fmul_rn(f1.x, s0), __fmul_rn(f2.x, c0)),
                          __fadd_rn(__fmul_rn(f1.y, s1), __fmul_rn(f2.y, c1)));
    }
    *reinterpret_cast<uint4*>(a_lo) = y1;
    *reinterpret_cast<uint4*>(a_hi) = y2;
  }
}

// One work unit: two 128-row query tiles (rows m0 .. m0 + 255) of one (batch,
// head) and the key tiles they see.
struct PfUnit {
  int b, h, kvh, m0, N;
  int n_kv[2];  // key tiles of query tile 0 / 1
  int n;        // max of the two: key steps of the unit
  const int32_t* table;
};

// Unit u of the grid's work list, heaviest first when causal (the causal work
// of a tile pair grows with its position).
template <bool PAGED>
__device__ __forceinline__ PfUnit pf_unit(const PrefillParams& p, int u) {
  PfUnit w;
  const int bh_count = p.B * p.Hq;
  const int pair_lin = u / bh_count;
  const int pr = p.causal ? (p.n_pairs - 1 - pair_lin) : pair_lin;
  const int bh = u % bh_count;
  w.b = bh / p.Hq;
  w.h = bh % p.Hq;
  w.kvh = w.h / p.G;
  w.m0 = pr * 2 * kBM;
  w.N = p.N;
  w.table = nullptr;
  if constexpr (PAGED) {
    int n = p.kv_lens[w.b];
    const int cap = p.max_blocks * p.block_size;
    if (n < 0) n = 0;
    if (n > cap) n = cap;  // the bad length is reported once, by softmax thread 0
    w.N = n;
    w.table = p.tables + static_cast<int64_t>(w.b) * p.max_blocks;
  }
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int mt0 = w.m0 + t * kBM;
    int n_end = p.causal ? min(w.N, w.N - p.M + mt0 + kBM) : w.N;
    if (n_end < 0) n_end = 0;
    w.n_kv[t] = (mt0 < p.M) ? (n_end + kBN - 1) / kBN : 0;
  }
  w.n = max(w.n_kv[0], w.n_kv[1]);
  return w;
}

// The CTA's units: round r takes unit r * G + c, and r * G + (G - 1 - c) on odd
// rounds (a snake over the heaviest-first list, so every CTA gets a similar mix
// of heavy and light units). -2: no more rounds; -1: nothing in this round.
__device__ __forceinline__ int pf_unit_index(int r, int n_units) {
  const int G = gridDim.x, c = blockIdx.x;
  const int base = r * G;
  if (base >= n_units) return -2;
  const int u = base + ((r & 1) ? (G - 1 - c) : c);
  return u < n_units ? u : -1;
}

template <int D, bool BF16, bool PAGED>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using C = PfCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // [2][KCH][128][128B]
  uint8_t* sK = sQ + 2 * C::Q_BYTES;       // [KS][KCH][128][128B]
  uint8_t* sV = sK + C::KS * C::KV_BYTES;  // [VS][KCH][128][128B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  // Per query tile t, counted over the units in which tile t has keys:
  uint64_t* bar_q_full = bars + 0;   // [2] Q_t of the unit landed
  uint64_t* bar_q_ready = bars + 2;  // [2] ... and rotated by softmax warpgroup t
  uint64_t* bar_q_free = bars + 4;   // [2] every S_t MMA of the unit complete: Q_t may go
  uint64_t* bar_k_full = bars + 6;
  uint64_t* bar_v_full = bar_k_full + C::KS;
  uint64_t* bar_s0_full = bar_v_full + C::VS;  // S0 of a key step complete (and PV0 before it)
  // bar_step[g % R], phase g / R, for the CTA's g-th key step (counted over all
  // its units): every MMA up to S1 of that step complete. Frees K_g's stage (S0_g,
  // S1_g done) and V_{g-1}'s stage (PV0_{g-1}, PV1_{g-1} done), and is softmax 1's
  // "S1 ready".
  uint64_t* bar_step = bar_s0_full + 1;
  uint64_t* bar_pa_full = bar_step + C::R;  // [2] per tile: P keys 0..63 written
  uint64_t* bar_p_full = bar_pa_full + 2;   // [2] per tile: all of P written
  uint64_t* bar_o_final = bar_p_full + 2;   // [2] per tile: last PV of the unit complete
  uint64_t* bar_drain = bar_o_final + 2;    // [1] abort path only
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [2] per tile: warps of the softmax warpgroup that stored a unit's rows to o
  // (4 per unit). A counter, not an mbarrier: the copy warp may fall several
  // units behind, and a counter cannot alias phases.
  volatile uint32_t* stored = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_units = p.n_units;

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar_q_full + t, 1);
      mbar_init(bar_q_ready + t, 4);  // one arrive per softmax warp
      mbar_init(bar_q_free + t, 1);
    }
    for (int s = 0; s < C::KS; ++s) mbar_init(bar_k_full + s, 1);
    for (int s = 0; s < C::VS; ++s) mbar_init(bar_v_full + s, 1);
    mbar_init(bar_s0_full, 1);
    for (int s = 0; s < C::R; ++s) mbar_init(bar_step + s, 1);
    for (int t = 0; t < 2; ++t) {
      // one arrive per softmax warp (after its lanes synchronised): four arrivals
      // complete a phase much sooner than 128 per-thread ones
      mbar_init(bar_pa_full + t, 4);
      mbar_init(bar_p_full + t, 4);
      mbar_init(bar_o_final + t, 1);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    stored[0] = 0;
    stored[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
   reg_dealloc<kRegsCtrl<D>>();
   if (warp == 3) {
    // -------------------------------------- output all-gather over peer memory
    // Each unit's output rows, once the softmax warpgroups stored them to o,
    // are copied to the other GPUs' outputs with 16-byte peer stores, while the
    // CTA computes its next unit: the NVLink transfer overlaps the math unit by
    // unit. Idle when there are no peers.
    if (p.n_peers > 0) {
      bool ok = true;
      uint32_t ui = 0;  // units of this CTA so far (every unit, with keys or not)
      using vec_t = uint4;
      constexpr int kVec = 8;  // 16-byte loads in flight per lane
      // wait (bounded, sleeping between polls so the softmax warps sharing this
      // scheduler keep their issue slots) until tile t's rows of unit ui are in o
      auto wait_stored = [&](int t, uint32_t target) -> bool {
        if (stored[t] >= target) return true;
        const uint64_t limit = *reinterpret_cast<const volatile uint64_t*>(&g_wait_limit_ns);
        if (limit == 0) {
          *abort_flag = 1;
          return false;
        }
        const uint64_t t0 = globaltimer_ns();
        while (stored[t] < target) {
          if (*abort_flag) return false;
          if (globaltimer_ns() - t0 > limit) {
            *abort_flag = 1;
            return false;
          }
          __nanosleep(128);
        }
        return true;
      };
      for (int r = 0; ok; ++r) {
        const int u = pf_unit_index(r, n_units);
        if (u == -2) break;
        if (u < 0) continue;
        const PfUnit w = pf_unit<PAGED>(p, u);
        for (int t = 0; t < 2 && ok; ++t) {
          ok = __all_sync(0xffffffffu, wait_stored(t, 4 * (ui + 1)));
          if (!ok) break;
          __threadfence_block();  // the softmax warps' stores of these rows are visible
          const int mt0 = w.m0 + t * kBM;
          const int rows = min(kBM, p.M - mt0);
          if (rows <= 0) continue;
          constexpr int CH = D * 2 / 16;  // 16-byte chunks per row
          const int64_t base = static_cast<int64_t>(w.b) * p.o_sb + w.h * p.o_sh;
          const uint8_t* src = reinterpret_cast<const uint8_t*>(p.o);
          for (int q0 = lane; q0 < rows * CH; q0 += 32 * kVec) {
            vec_t v[kVec];
            int64_t off[kVec];
#pragma unroll
            for (int i = 0; i < kVec; ++i) {
              const int q = q0 + 32 * i;
              off[i] = -1;
              if (q < rows * CH) {
                off[i] = (base + static_cast<int64_t>(mt0 + q / CH) * p.o_sm) * 2 + (q % CH) * 16;
                v[i] = *reinterpret_cast<const vec_t*>(src + off[i]);
              }
            }
            for (int pe = 0; pe < p.n_peers; ++pe) {
              uint8_t* dst = reinterpret_cast<uint8_t*>(p.o_peers[pe]);
#pragma unroll
              for (int i = 0; i < kVec; ++i)
                if (off[i] >= 0) *reinterpret_cast<vec_t*>(dst + off[i]) = v[i];
            }
          }
        }
        ++ui;
      }
      // make every peer store visible system-wide before the kernel ends; the
      // barrier that follows the kernel then publishes them
      __threadfence_system();
    }
   } else if (warp != 1) {
    // -------------------------------------- loaders (warp 0: Q and K, warp 2: V)
    // Lane 0 issues the TMA copies. Q_t of a unit is loaded once the previous
    // unit's last S_t MMA has completed (tile 0 finishes a key step before tile 1
    // under the causal mask, so its next Q comes in early); stage and step
    // counters run on across units.
    const bool kload = warp == 0, vload = warp == 2;
    if (lane == 0) {
      if (kload) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
      } else if (vload) {
        tma_prefetch_desc(&tm_v);
      }
    }
    int k_issued = 0, v_issued = 0;  // totals, for the drain on abort
    int q_issued[2] = {0, 0};
    // K tile g (the CTA's g-th key step) into its stage; j = tile within the unit
    auto load_k = [&](int g, const PfUnit& w, int j) -> bool {
      const int st = g % C::KS;
      // K_{g-KS} left this stage once S1_{g-KS} completed
      if (g >= C::KS && !mbar_wait_bounded(bar_step + (g - C::KS) % C::R,
                                           ((g - C::KS) / C::R) & 1, abort_flag,
                                           &g_wait_limit_ns))
        return false;
      mbar_arrive_expect_tx(bar_k_full + st, C::KV_BYTES);
      if constexpr (PAGED) {
        int tok[kBN / 16];
#pragma unroll
        for (int i = 0; i < kBN / 16; ++i) tok[i] = paged_box_coord(p, w.table, j * kBN + i * 16, w.N);
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
#pragma unroll
          for (int i = 0; i < kBN / 16; ++i)
            tma_load_4d(sK + st * C::KV_BYTES + c * kBN * 128 + i * 16 * 128, &tm_k,
                        bar_k_full + st, c * 64, w.kvh, tok[i], 0);
      } else {
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sK + st * C::KV_BYTES + c * kBN * 128, &tm_k, bar_k_full + st, c * 64,
                      j * kBN, w.kvh, w.b);
      }
      k_issued = g + 1;
      return true;
    };
    auto load_v = [&](int g, const PfUnit& w, int j) -> bool {
      const int st = g % C::VS;
      // V_{g-VS} left this stage once PV1_{g-VS} completed, i.e. by step g-VS+1
      if (g >= C::VS && !mbar_wait_bounded(bar_step + (g - C::VS + 1) % C::R,
                                           ((g - C::VS + 1) / C::R) & 1, abort_flag,
                                           &g_wait_limit_ns))
        return false;
      mbar_arrive_expect_tx(bar_v_full + st, C::KV_BYTES);
      if constexpr (PAGED) {
        int tok[kBN / 16];
#pragma unroll
        for (int i = 0; i < kBN / 16; ++i) tok[i] = paged_box_coord(p, w.table, j * kBN + i * 16, w.N);
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
#pragma unroll
          for (int i = 0; i < kBN / 16; ++i)
            tma_load_4d(sV + st * C::KV_BYTES + c * kBN * 128 + i * 16 * 128, &tm_v,
                        bar_v_full + st, c * 64, w.kvh, tok[i], 0);
      } else {
#pragma unroll
        for (int c = 0; c < C::KCH; ++c)
          tma_load_4d(sV + st * C::KV_BYTES + c * kBN * 128, &tm_v, bar_v_full + st, c * 64,
                      j * kBN, w.kvh, w.b);
      }
      v_issued = g + 1;
      return true;
    };
    int kt = 0;           // key steps before the current unit
    int qc[2] = {0, 0};   // units before the current one in which tile t had keys
    bool ok = true;
    if (lane == 0 && (kload || vload)) {
      for (int r = 0; ok; ++r) {
        const int u = pf_unit_index(r, n_units);
        if (u == -2) break;
        if (u < 0) continue;
        const PfUnit w = pf_unit<PAGED>(p, u);
        if (w.n == 0) continue;
        if (kload) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (w.n_kv[t] == 0) continue;
            if (qc[t] > 0 &&
                !(ok = mbar_wait_bounded(bar_q_free + t, (qc[t] - 1) & 1, abort_flag,
                                         &g_wait_limit_ns)))
              break;
            mbar_arrive_expect_tx(bar_q_full + t, C::Q_BYTES);
#pragma unroll
            for (int c = 0; c < C::KCH; ++c)
              tma_load_4d(sQ + t * C::Q_BYTES + c * kBM * 128, &tm_q, bar_q_full + t, c * 64,
                          w.m0 + t * kBM, w.h, w.b);
            q_issued[t] = qc[t] + 1;
          }
          for (int j = 0; ok && j < w.n; ++j) ok = load_k(kt + j, w, j);
        } else {
          for (int j = 0; ok && j < w.n; ++j) ok = load_v(kt + j, w, j);
        }
        kt += w.n;
        qc[0] += w.n_kv[0] > 0;
        qc[1] += w.n_kv[1] > 0;
      }
    }
    if (*abort_flag && lane == 0) {
      // let this CTA's copies still in flight land before its smem is released:
      // the newest load of each stage is the latest phase of that stage's barrier
      if (kload) {
        for (int t = 0; t < 2; ++t)
          if (q_issued[t] > 0) mbar_wait_timeout(bar_q_full + t, (q_issued[t] - 1) & 1, kWaitLimitNs);
        for (int g = k_issued - 1; g >= 0 && g >= k_issued - C::KS; --g)
          mbar_wait_timeout(bar_k_full + (g % C::KS), (g / C::KS) & 1, kWaitLimitNs);
      } else if (vload) {
        for (int g = v_issued - 1; g >= 0 && g >= v_issued - C::VS; --g)
          mbar_wait_timeout(bar_v_full + (g % C::VS), (g / C::VS) & 1, kWaitLimitNs);
      }
    }
   } else {
    // ------------------------------------------------ MMA issuer (warp 1)
    // The whole warp runs the issue loop (waits, probes, control flow) and one
    // elected lane issues each tcgen05 instruction. Measured on B200 with the
    // loop on a single lane instead, the per-group commits and waits cost ~40%
    // of the tensor core's throughput (91 instead of 64 cycles per MMA).
    constexpr int fmt = BF16 ? 1 : 0;
    constexpr uint32_t idesc_s = umma_idesc_f16(kBM, kBN, fmt, 0, 0);
    constexpr uint32_t idesc_o = umma_idesc_f16(kBM, D, fmt, 0, 1);
    // Descriptors are built once; each MMA only adds its byte offset (>> 4) to the
    // 14-bit start-address field.
    const uint64_t dq0 = umma_smem_desc(smem_u32(sQ), 16, 1024);
    const uint64_t dk0 = umma_smem_desc(smem_u32(sK), 16, 1024);
    const uint64_t dv0 = umma_smem_desc(smem_u32(sV), kBN * 128, 1024);
    auto commit = [](uint64_t* bar) {
      if (elect_one_sync()) umma_commit(bar);
    };
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu,
                        mbar_wait_bounded(bar, parity, abort_flag, &g_wait_limit_ns));
    };
    auto test = [](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_test(bar, parity));
    };
    // S_t = Q_t K_g^T for the CTA's g-th key tile
    auto issue_s = [&](int t, int g) {
      const int st = g % C::KS;
      const uint32_t s_col = t ? C::TM_S1 : C::TM_S0;
      const uint64_t aq = dq0 + static_cast<uint64_t>((t * C::Q_BYTES) >> 4);
      const uint64_t bk = dk0 + static_cast<uint64_t>((st * C::KV_BYTES) >> 4);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        constexpr int kRow = kBM * 128;
        const uint32_t off = ((kk >> 2) * kRow + (kk & 3) * 32) >> 4;
        if (elect_one_sync()) umma_ss(tmem + s_col, aq + off, bk + off, idesc_s, kk > 0 ? 1u : 0u);
      }
    };
    // O_t += P_t V_g in two halves of 64 keys, each behind its half of P; `pc`
    // counts the P tiles tile t published before this one, `last` marks the
    // unit's last PV of the tile. `probe` runs while the tensor core takes the
    // first half.
    auto issue_pv = [&](int t, int j, int g, int pc, bool last, auto&& probe) {
      const int st = g % C::VS;
      const uint32_t p_col = tmem + (t ? C::TM_S1 : C::TM_S0);
      const uint32_t o_col = tmem + (t ? C::TM_O1 : C::TM_O0);
      const uint64_t bv = dv0 + static_cast<uint64_t>((st * C::KV_BYTES) >> 4);
      const uint32_t acc0 = j > 0 ? 1u : 0u;
      if (!wait(bar_pa_full + t, pc & 1)) return false;
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kBN / 32; ++kk) {
        if (elect_one_sync())
          umma_ts(o_col, p_col + kk * 8, bv + ((kk * 16 * 128) >> 4), idesc_o,
                  kk > 0 ? 1u : acc0);
        if (kk == 2) probe();
      }
      if (!wait(bar_p_full + t, pc & 1)) return false;
      tc_fence_after();
#pragma unroll
      for (int kk = kBN / 32; kk < kBN / 16; ++kk) {
        if (elect_one_sync())
          umma_ts(o_col, p_col + kk * 8, bv + ((kk * 16 * 128) >> 4), idesc_o, 1u);
      }
      if (last) commit(bar_o_final + t);
      return true;
    };
    int kt = 0, pc0 = 0, pc1 = 0, qr0 = 0, qr1 = 0;
    bool ok = true;
    for (int r = 0; ok; ++r) {
      const int u = pf_unit_index(r, n_units);
      if (u == -2) break;
      if (u < 0) continue;
      const PfUnit w = pf_unit<PAGED>(p, u);
      if (w.n == 0) continue;
      const int n = w.n;
      // qr_t: earlier units in which tile t had keys (one Q_t each)
      ok = wait(bar_k_full + kt % C::KS, (kt / C::KS) & 1);
      if (!ok) break;
      if (w.n_kv[0] > 0) {
        if (!(ok = wait(bar_q_ready + 0, qr0 & 1))) break;
        tc_fence_after();
        issue_s(0, kt);
        commit(bar_s0_full);
        if (w.n_kv[0] == 1) commit(bar_q_free + 0);
      }
      if (w.n_kv[1] > 0) {
        if (!(ok = wait(bar_q_ready + 1, qr1 & 1))) break;
        tc_fence_after();
        issue_s(1, kt);
        if (w.n_kv[1] == 1) commit(bar_q_free + 1);
      }
      commit(bar_step + kt % C::R);
      bool v_seen = false;  // V_g's barrier already observed complete
      for (int j = 0; j < n; ++j) {
        const int g = kt + j, gn = g + 1, jn = j + 1;
        const int stn = gn % C::KS;  // K stage of the next key tile
        const uint32_t phn = (gn / C::KS) & 1;
        bool k_seen = false;
        if (!v_seen && !(ok = wait(bar_v_full + g % C::VS, (g / C::VS) & 1))) break;
        if (j < w.n_kv[0] &&
            !(ok = issue_pv(0, j, g, pc0 + j, j == w.n_kv[0] - 1, [&] {
                if (jn < n) k_seen = test(bar_k_full + stn, phn);
              })))
          break;
        if (jn < n) {
          if (!k_seen && !(ok = wait(bar_k_full + stn, phn))) break;
          if (jn < w.n_kv[0]) {
            issue_s(0, gn);
            commit(bar_s0_full);
            if (jn == w.n_kv[0] - 1) commit(bar_q_free + 0);  // tile 0's last S
          }
        }
        v_seen = false;
        auto probe_v = [&] {
          if (jn < n) v_seen = test(bar_v_full + gn % C::VS, (gn / C::VS) & 1);
        };
        if (j < w.n_kv[1] && !(ok = issue_pv(1, j, g, pc1 + j, j == w.n_kv[1] - 1, probe_v)))
          break;
        if (jn < n) {
          if (jn < w.n_kv[1]) {
            issue_s(1, gn);
            if (jn == w.n_kv[1] - 1) commit(bar_q_free + 1);  // tile 1's last S
          }
          commit(bar_step + gn % C::R);
        }
      }
      kt += n;
      pc0 += w.n_kv[0];
      pc1 += w.n_kv[1];
      qr0 += w.n_kv[0] > 0;
      qr1 += w.n_kv[1] > 0;
    }
    if (!ok) {
      if (lane == 0) raise_status(CIE_DEV_TIMEOUT);
      commit(bar_drain);  // all MMAs issued so far must finish before TMEM is freed
      mbar_wait_timeout(bar_drain, 0, kWaitLimitNs);
    }
   }
  } else {
    reg_alloc<kRegsSoftmax<D>>();
    // ------------------------------------------------ softmax warpgroups
    const int t = (warp - 4) >> 2;       // query tile of this warpgroup
    const int wq = warp & 3;             // TMEM lane quarter this warp may access
    const int row = wq * 32 + lane;      // query row within the tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t s_col = t ? C::TM_S1 : C::TM_S0;
    const uint32_t o_col = t ? C::TM_O1 : C::TM_O0;
    using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    if constexpr (PAGED) {
      if (threadIdx.x == 128) {
        for (int b = 0; b < p.B; ++b)
          if (p.kv_lens[b] > p.max_blocks * p.block_size) raise_status(CIE_DEV_BAD_BLOCK_ID);
      }
    }
    int kt = 0, sc = 0, of = 0;  // key steps, S tiles of this tile, units with keys before
    bool ok = true;
    for (int r = 0; ok; ++r) {
      const int u = pf_unit_index(r, n_units);
      if (u == -2) break;
      if (u < 0) continue;
      const PfUnit w = pf_unit<PAGED>(p, u);
      const int gm = w.m0 + t * kBM + row;   // global query index
      const int nkv = w.n_kv[t];
      if (nkv == 0) {
        // no visible keys: N == 0 -> zeros (matches the fp32 reference), else NaN rows
        if (gm < p.M) {
          elem_t* o = reinterpret_cast<elem_t*>(p.o) + w.b * p.o_sb + w.h * p.o_sh + gm * p.o_sm;
          const float fill = (w.N == 0) ? 0.f : __int_as_float(0x7fc00000);
          for (int d = 0; d < D; ++d) {
            if constexpr (BF16) o[d] = __float2bfloat16_rn(fill);
            else o[d] = __float2half_rn(fill);
          }
        }
        if (p.n_peers > 0) {
          __threadfence_block();
          __syncwarp();
          if (lane == 0) atomicAdd(const_cast<uint32_t*>(stored + t), 1u);
        }
        kt += w.n;
        continue;
      }
      // Q_t of this unit: rotate this thread's row in shared memory, then hand the
      // tile to the MMA warp
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_q_full + t, of & 1, abort_flag,
                                                     &g_wait_limit_ns));
      if (!ok) break;
      if (p.cos != nullptr && gm < p.M) {
        int pos = (PAGED ? w.N - p.M : p.rope_q_pos0) + gm;
        if (pos < 0 || pos >= p.rope_max_pos) {
          raise_status(CIE_DEV_BAD_POSITION);
          pos = pos < 0 ? 0 : p.rope_max_pos - 1;
        }
        rope_q_row<D, BF16>(sQ + t * C::Q_BYTES, row, pos, p.cos, p.sin);
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_q_ready + t);
      const int lim = p.causal ? (w.N - p.M + gm) : (w.N - 1);  // keys <= lim are visible
      float m_run = -INFINITY;  // running max, log2 domain, scaled
      float l_run = 0.f;
      float sv[kBN];
      for (int j = 0; ok && j < nkv; ++j) {
        const int g = kt + j;
        ok = t ? mbar_wait_bounded(bar_step + g % C::R, (g / C::R) & 1, abort_flag,
                                   &g_wait_limit_ns)
               : mbar_wait_bounded(bar_s0_full, (sc + j) & 1, abort_flag, &g_wait_limit_ns);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const int n0 = j * kBN;
        // a tile that reaches past some row's last visible key takes the masked path
        const bool masked = __any_sync(0xffffffffu, n0 + kBN - 1 > lim);
        // Row max in CIE_MAX_CHAINS independent fmax3 chains.
        float mx[CIE_MAX_CHAINS];
#pragma unroll
        for (int i = 0; i < CIE_MAX_CHAINS; ++i) mx[i] = -INFINITY;
        auto mask_cols = [&](int c0, int c1) {
          if (masked) {
#pragma unroll
            for (int c = c0; c < c1; ++c)
              if (n0 + c > lim) sv[c] = -INFINITY;
          }
        };
        auto reduce_cols = [&](int c0, int c1) {
#pragma unroll
          for (int c = c0; c < c1; c += 2) {
            const int i = ((c - c0) / 2) % CIE_MAX_CHAINS;
            mx[i] = fmax3(mx[i], sv[c], sv[c + 1]);
          }
        };
        auto row_max_scaled = [&]() {
#pragma unroll
          for (int wv = CIE_MAX_CHAINS / 2; wv >= 1; wv /= 2)
#pragma unroll
            for (int i = 0; i < wv; ++i) mx[i] = fmaxf(mx[i], mx[i + wv]);
          return mx[0] * p.scale_log2;
        };
        // Lazy rescale: only rows whose max grew by more than 2^8 move their
        // reference; S_t_j complete implies PV_t_{j-1} complete, so O_t may be
        // rescaled in TMEM here.
        auto rescale = [&](float m_new) {
          const bool need = m_new > m_run + 8.0f;
          if (__any_sync(0xffffffffu, need)) {
            const float alpha = need ? ex2(m_run - m_new) : 1.0f;
#pragma unroll
            for (int c = 0; c < D / 16; ++c) {
              uint32_t ov[16];
              tmem_ld16(tmem + lane_addr + o_col + c * 16, ov);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e)
                ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
              tmem_st16(tmem + lane_addr + o_col + c * 16, ov);
            }
            if (need) {
              l_run *= alpha;
              m_run = m_new;
            }
          }
        };
        // p = 2^(s * scale - m): packed FFMA, MUFU ex2, packed row sum, bf16/fp16
        // pack. Staged in groups of 8 pairs (8 FFMA2, then 16 ex2, then sums and
        // packs): measured on B200 with the softmax register budget this keeps the
        // MUFU unit busier than the per-pair chain (1255 vs 1385 cycles per row of
        // 128, against a 1024-cycle MUFU floor).
        uint64_t sum2a = f2_pack(0.f, 0.f), sum2b = sum2a;
        // P goes to TMEM 16 columns (32 keys) at a time, which keeps only 16 packed
        // registers live next to the row of S.
        auto exp_half = [&](int hb, float m) {
          const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
          const uint64_t nm2 = f2_pack(-m, -m);
          uint32_t pk[16];
#pragma unroll
          for (int g0 = 0; g0 < 32; g0 += 8) {
            float e[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int c = hb * 64 + 2 * (g0 + i);
              f2_unpack(ffma2(f2_pack(sv[c], sv[c + 1]), sc2, nm2), e[2 * i], e[2 * i + 1]);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) e[i] = ex2(e[i]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint64_t p2 = f2_pack(e[2 * i], e[2 * i + 1]);
              if (i & 1) sum2b = fadd2(sum2b, p2);
              else sum2a = fadd2(sum2a, p2);
              pk[(g0 + i) & 15] = pack2<BF16>(e[2 * i], e[2 * i + 1]);
            }
            if (g0 & 8) tmem_st16(tmem + lane_addr + s_col + hb * 32 + (g0 & 16), pk);
          }
        };
        // P is written and announced in two halves of 64 keys so that the tensor
        // core starts on the first half while the second is exponentiated.
        auto publish = [&](int hb) {
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive((hb ? bar_p_full : bar_pa_full) + t);
        };

        // first half of S; the second half's load goes out right behind it and
        // lands while the first half is reduced
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tmem_ld32(tmem + lane_addr + s_col + c * 32, reinterpret_cast<uint32_t*>(sv) + c * 32);
        tmem_wait_ld();
        mask_cols(0, 64);
#pragma unroll
        for (int c = 2; c < 4; ++c)
          tmem_ld32(tmem + lane_addr + s_col + c * 32, reinterpret_cast<uint32_t*>(sv) + c * 32);
        reduce_cols(0, 64);
        tmem_wait_ld();
        mask_cols(64, 128);
        reduce_cols(64, 128);
        const float m_new = fmaxf(m_run, row_max_scaled());
        if (j == 0) m_run = m_new;  // PV of tile t starts O from zero
        else rescale(m_new);
        const float m_use = m_run == -INFINITY ? 0.f : m_run;
        exp_half(0, m_use);
        publish(0);
        exp_half(1, m_use);
        publish(1);
        float lsum0, lsum1;
        f2_unpack(fadd2(sum2a, sum2b), lsum0, lsum1);
        l_run += lsum0 + lsum1;
      }

      if (ok) {
        ok = mbar_wait_bounded(bar_o_final + t, of & 1, abort_flag, &g_wait_limit_ns);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        // O_t of this unit out of TMEM; the next unit's first PV_t, which
        // overwrites it, waits for this warpgroup's next P
        tc_fence_after();
        const float inv_l = (l_run > 0.f) ? 1.0f / l_run : __int_as_float(0x7fc00000);
        elem_t* o = reinterpret_cast<elem_t*>(p.o) + w.b * p.o_sb + w.h * p.o_sh + gm * p.o_sm;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          tmem_ld32(tmem + lane_addr + o_col + c * 32, ov);
          tmem_wait_ld();
          if (gm < p.M) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              pk[e] = pack2<BF16>(__uint_as_float(ov[2 * e]) * inv_l,
                                  __uint_as_float(ov[2 * e + 1]) * inv_l);
            uint4* dst = reinterpret_cast<uint4*>(o + c * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              dst[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
          }
        }
        tc_fence_before();
        if (p.n_peers > 0) {
          // the rows are in o: hand them to the copy warp
          __threadfence_block();
          __syncwarp();
          if (lane == 0) atomicAdd(const_cast<uint32_t*>(stored + t), 1u);
        }
      }
      kt += w.n;
      sc += nkv;
      ++of;
    }
    if (!ok) raise_status(CIE_DEV_TIMEOUT);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

// ------------------------------------------------------------------ host
// 4-D map over (d, seq, head, batch) with a (64, 128, 1, 1) box, 128B swizzle.
static int make_map(CUtensorMap* map, const void* base, int d, int seq, int heads, int batch,
                    const int64_t* strides, bool bf16, const char* what) {
  PFN_encodeTiled_t enc = tensor_map_encoder();
  if (!enc) {
    set_error("%s: cuTensorMapEncodeTiled unavailable", what);
    return CIE_ERR_LAUNCH;
  }
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)seq, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2,
                        (cuuint64_t)strides[0] * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void*>(base), dims, gstr, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
    return CIE_ERR_INVALID;
  }
  return CIE_OK;
}

template <int D, bool BF16, bool PAGED = false>
static int launch_prefill(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                          const PrefillParams& prm, cudaStream_t st) {
  constexpr int smem = PfCfg<D>::SMEM;
  auto kern = prefill_attn_kernel<D, BF16, PAGED>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  // persistent: one CTA per SM (225 KB of shared memory each) walks the work list
  // (CIE_PF_ONE_UNIT_PER_CTA builds the one-unit-per-CTA grid instead, for comparison)
#ifdef CIE_PF_ONE_UNIT_PER_CTA
  const int grid = prm.n_units;
#else
  const int grid = prm.n_units < num_sms() ? prm.n_units : num_sms();
#endif
  kern<<<grid, kPfThreads, smem, st>>>(mq, mk, mv, prm);
  CIE_CHECK_LAUNCH("prefill_attn_kernel");
  return CIE_OK;
}

int rope_launch(const void* x, void* y, int B, int H, int L, int d, const int64_t* xs,
                const int64_t* ys, int pos0, bool bf16, const float* cos, const float* sin,
                int max_pos, cudaStream_t st);
size_t dense_mma_workspace(int B, int Hq, int Hkv, int M, int N, int d);
int dense_mma_attn(const void* q, const void* k, const void* v, void* o, int B, int Hq, int Hkv,
                   int M, int N, int d, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                   const int64_t* os, float scale, int causal, bool bf16, const float* cos,
                   const float* sin, int max_pos, int q_pos0, void* workspace,
                   size_t workspace_bytes, cudaStream_t st);

// The tcgen05 kernel takes head dims 64 / 128 with at least one full query
// tile's worth of rows per kv head; short query blocks (decode-like, G*M <= 64)
// and other head dims go to the split-KV mma.sync kernel over dense K/V.
static bool use_tcgen05(int Hq, int Hkv, int M, int d) {
  return (d == 64 || d == 128) && static_cast<int64_t>(Hq / Hkv) * M > 64;
}

// Paged prefill on the tcgen05 kernel: q (B, Hq, M, d) dense, K/V from the
// paged pools through the block table. Called by cie_paged_attn when the query
// block is long enough for the tensor-core kernel (paged_uses_tcgen05).
bool paged_uses_tcgen05(int Hq, int Hkv, int M, int d, int block_size) {
  return use_tcgen05(Hq, Hkv, M, d) && block_size % 16 == 0;
}

int paged_prefill_tcgen05(const void* q, const void* k_pool, const void* v_pool,
                          const int32_t* block_tables, const int32_t* kv_lens, void* o, int B,
                          int Hq, int Hkv, int M, int d, int num_blocks, int block_size,
                          int max_blocks, const int64_t* q_strides, const int64_t* o_strides,
                          float scale, int causal, bool bf16, const float* rope_cos,
                          const float* rope_sin, int rope_max_pos, cudaStream_t st) {
  CIE_CHECK_ARG(aligned16(o) && o_strides[0] % 8 == 0 && o_strides[1] % 8 == 0 &&
                    o_strides[2] % 8 == 0,
                "cie_paged_attn: o must be 16-byte aligned with strides multiple of 8");
  CIE_CHECK_ARG(rope_cos == nullptr || (aligned16(rope_cos) && aligned16(rope_sin)),
                "cie_paged_attn: rope tables must be 16-byte aligned");
  const int64_t pool_tokens = static_cast<int64_t>(num_blocks) * block_size;
  CIE_CHECK_ARG(pool_tokens < (int64_t(1) << 31) - 16, "cie_paged_attn: pool too large");
  PrefillParams prm{};
  prm.B = B;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.M = M;
  prm.N = 0;
  prm.G = Hq / Hkv;
  prm.n_pairs = (M + 2 * kBM - 1) / (2 * kBM);
  prm.n_units = prm.n_pairs * B * Hq;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal ? 1 : 0;
  prm.o = o;
  prm.o_sb = o_strides[0];
  prm.o_sh = o_strides[1];
  prm.o_sm = o_strides[2];
  prm.cos = rope_cos;
  prm.sin = rope_sin;
  prm.rope_max_pos = rope_max_pos;
  prm.kv_lens = kv_lens;
  prm.tables = block_tables;
  prm.max_blocks = max_blocks;
  prm.block_size = block_size;
  prm.num_blocks = num_blocks;
  prm.pool_tokens = static_cast<int>(pool_tokens);
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, q, d, M, Hq, B, q_strides, bf16, "cie_paged_attn(q)");
  if (rc != CIE_OK) return rc;
  // (d, head, pool token, 1) with a (64, 1, 16, 1) box: one 16-token slice of
  // one head per table lookup, 128-byte swizzle as the dense tiles
  const cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)Hkv, (cuuint64_t)pool_tokens, 1};
  const cuuint64_t strides[3] = {(cuuint64_t)d * 2, (cuuint64_t)Hkv * d * 2,
                                 (cuuint64_t)pool_tokens * Hkv * d * 2};
  const cuuint32_t box[4] = {64, 1, 16, 1};
  if (!make_kv_map(&mk, k_pool, d, dims, strides, box, bf16) ||
      !make_kv_map(&mv, v_pool, d, dims, strides, box, bf16)) {
    set_error("cie_paged_attn: cuTensorMapEncodeTiled failed for the pools");
    return CIE_ERR_LAUNCH;
  }
  if (d == 64)
    return bf16 ? launch_prefill<64, true, true>(mq, mk, mv, prm, st)
                : launch_prefill<64, false, true>(mq, mk, mv, prm, st);
  return bf16 ? launch_prefill<128, true, true>(mq, mk, mv, prm, st)
              : launch_prefill<128, false, true>(mq, mk, mv, prm, st);
}

static size_t rope_k_bytes(int B, int Hkv, int N, int d) {
  return (static_cast<size_t>(B) * Hkv * N * d * 2 + 255) & ~size_t(255);
}

}  // namespace cie

using namespace cie;

extern "C" size_t cie_prefill_attn_workspace(int B, int Hq, int Hkv, int M, int N, int d,
                                             int dtype, int rope_k) {
  (void)dtype;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || M <= 0 || N < 0 || d <= 0) return 0;
  size_t bytes = (rope_k && N > 0) ? rope_k_bytes(B, Hkv, N, d) : 0;
  if (!use_tcgen05(Hq, Hkv, M, d)) bytes += dense_mma_workspace(B, Hq, Hkv, M, N, d);
  return bytes > 0 ? bytes + 256 : 0;
}

static int prefill_impl(const void* q, const void* k, const void* v, void* o, int B, int Hq,
                        int Hkv, int M, int N, int d, const int64_t* q_strides,
                        const int64_t* k_strides, const int64_t* v_strides,
                        const int64_t* o_strides, float scale, int causal, int dtype,
                        const float* rope_cos, const float* rope_sin, int rope_max_pos,
                        int rope_q_pos0, int rope_k, void* workspace, size_t workspace_bytes,
                        void* const* o_peers, int n_peers, void* stream) {
  CIE_CHECK_ARG(q && o && (N == 0 || (k && v)), "cie_prefill_attn: null tensor pointer");
  CIE_CHECK_ARG(q_strides && k_strides && v_strides && o_strides,
                "cie_prefill_attn: null strides");
  CIE_CHECK_ARG(B >= 0 && Hq > 0 && Hkv > 0 && M >= 0 && N >= 0, "cie_prefill_attn: bad shape");
  CIE_CHECK_ARG(Hq % Hkv == 0, "cie_prefill_attn: Hq (%d) must be a multiple of Hkv (%d)", Hq,
                Hkv);
  CIE_CHECK_ARG(dtype == CIE_DTYPE_BF16 || dtype == CIE_DTYPE_FP16,
                "cie_prefill_attn: bad dtype %d", dtype);
  CIE_CHECK_ARG((rope_cos == nullptr) == (rope_sin == nullptr),
                "cie_prefill_attn: rope_cos and rope_sin must both be given or both NULL");
  CIE_CHECK_ARG(rope_cos == nullptr || rope_max_pos > 0, "cie_prefill_attn: rope_max_pos <= 0");
  CIE_CHECK_ARG(!(rope_k && rope_cos == nullptr), "cie_prefill_attn: rope_k needs rope tables");
  if (d != 16 && d != 32 && d != 64 && d != 128 && d != 256) {
    set_error("cie_prefill_attn: head_dim %d unsupported (16, 32, 64, 128 or 256)", d);
    return CIE_ERR_UNSUPPORTED;
  }
  if (B == 0 || M == 0) return CIE_OK;
  CIE_CHECK_ARG(rope_cos == nullptr || (aligned16(rope_cos) && aligned16(rope_sin)),
                "cie_prefill_attn: rope tables must be 16-byte aligned");
  const int64_t* all[4] = {q_strides, k_strides, v_strides, o_strides};
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 3; ++j)
      CIE_CHECK_ARG(all[i][j] % 8 == 0 && all[i][j] >= 0,
                    "cie_prefill_attn: strides must be non-negative multiples of 8 elements");
  CIE_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o),
                "cie_prefill_attn: tensors must be 16-byte aligned");
  const bool bf16 = dtype == CIE_DTYPE_BF16;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  const void* kk = k;
  int64_t kws[3];
  const int64_t* ks = k_strides;
  const size_t need = cie_prefill_attn_workspace(B, Hq, Hkv, M, N, d, dtype, rope_k);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) {
    set_error("cie_prefill_attn: workspace of %zu bytes required, got %zu", need,
              workspace_bytes);
    return CIE_ERR_WORKSPACE;
  }
  uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) &
                                           ~uintptr_t(255));
  size_t ws_left = need > 256 ? need - 256 : 0;
  if (rope_k && N > 0) {
    void* kr = ws;
    ws += rope_k_bytes(B, Hkv, N, d);
    ws_left -= rope_k_bytes(B, Hkv, N, d);
    kws[0] = static_cast<int64_t>(Hkv) * N * d;
    kws[1] = static_cast<int64_t>(N) * d;
    kws[2] = d;
    int rc = rope_launch(k, kr, B, Hkv, N, d, k_strides, kws, 0, bf16, rope_cos, rope_sin,
                         rope_max_pos, st);
    if (rc != CIE_OK) return rc;
    kk = kr;
    ks = kws;
  }

  const int q_pos0_eff = rope_q_pos0;
  if (N == 0) {
    // no keys: the short-query kernel writes zeros and never reads K/V
    kk = q;
    v = q;
    ks = q_strides;
    v_strides = q_strides;
  }
  if (n_peers > 0 && (N == 0 || !use_tcgen05(Hq, Hkv, M, d))) {
    set_error("cie_prefill_attn_peers: the peer all-gather needs the tcgen05 path (d 64 or 128, "
              "more than 64 query rows per kv head, N > 0)");
    return CIE_ERR_UNSUPPORTED;
  }
  if (N == 0 || !use_tcgen05(Hq, Hkv, M, d))
    return dense_mma_attn(q, kk, v, o, B, Hq, Hkv, M, N, d, q_strides, ks, v_strides, o_strides,
                          scale, causal, bf16, rope_cos, rope_sin, rope_max_pos, q_pos0_eff, ws,
                          ws_left, st);

  PrefillParams prm{};
  prm.B = B;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.M = M;
  prm.N = N;
  prm.G = Hq / Hkv;
  prm.n_pairs = (M + 2 * kBM - 1) / (2 * kBM);
  prm.n_units = prm.n_pairs * B * Hq;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal ? 1 : 0;
  prm.o = o;
  prm.o_sb = o_strides[0];
  prm.o_sh = o_strides[1];
  prm.o_sm = o_strides[2];
  prm.cos = rope_cos;
  prm.sin = rope_sin;
  prm.rope_max_pos = rope_max_pos;
  prm.rope_q_pos0 = rope_q_pos0;
  prm.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i) prm.o_peers[i] = o_peers[i];

  CUtensorMap mq, mk, mv;
  int rc;
  // a zero-length key axis still needs a valid map; it is never read (n_kv == 0)
  const int n_map = N > 0 ? N : 1;
  if ((rc = make_map(&mq, q, d, M, Hq, B, q_strides, bf16, "cie_prefill_attn(q)")) != CIE_OK)
    return rc;
  if ((rc = make_map(&mk, kk, d, n_map, Hkv, B, ks, bf16, "cie_prefill_attn(k)")) != CIE_OK)
    return rc;
  if ((rc = make_map(&mv, v, d, n_map, Hkv, B, v_strides, bf16, "cie_prefill_attn(v)")) !=
      CIE_OK)
    return rc;
  if (d == 64)
    return bf16 ? launch_prefill<64, true>(mq, mk, mv, prm, st)
                : launch_prefill<64, false>(mq, mk, mv, prm, st);
  return bf16 ? launch_prefill<128, true>(mq, mk, mv, prm, st)
              : launch_prefill<128, false>(mq, mk, mv, prm, st);
}

extern "C" int cie_prefill_attn(const void* q, const void* k, const void* v, void* o, int B,
                                int Hq, int Hkv, int M, int N, int d, const int64_t* q_strides,
                                const int64_t* k_strides, const int64_t* v_strides,
                                const int64_t* o_strides, float scale, int causal, int dtype,
                                const float* rope_cos, const float* rope_sin, int rope_max_pos,
                                int rope_q_pos0, int rope_k, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return prefill_impl(q, k, v, o, B, Hq, Hkv, M, N, d, q_strides, k_strides, v_strides,
                      o_strides, scale, causal, dtype, rope_cos, rope_sin, rope_max_pos,
                      rope_q_pos0, rope_k, workspace, workspace_bytes, nullptr, 0, stream);
}

extern "C" int cie_prefill_attn_peers(const void* q, const void* k, const void* v, void* o,
                                      void* const* o_peers, int n_peers, int B, int Hq, int Hkv,
                                      int M, int N, int d, const int64_t* q_strides,
                                      const int64_t* k_strides, const int64_t* v_strides,
                                      const int64_t* o_strides, float scale, int causal,
                                      int dtype, const float* rope_cos, const float* rope_sin,
                                      int rope_max_pos, int rope_q_pos0, int rope_k,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  CIE_CHECK_ARG(n_peers >= 0 && n_peers <= kMaxPeers,
                "cie_prefill_attn_peers: n_peers must be in [0, %d]", kMaxPeers);
  CIE_CHECK_ARG(n_peers == 0 || o_peers != nullptr, "cie_prefill_attn_peers: null o_peers");
  for (int i = 0; i < n_peers; ++i)
    CIE_CHECK_ARG(o_peers[i] != nullptr && aligned16(o_peers[i]) && o_peers[i] != o,
                  "cie_prefill_attn_peers: peer output %d null, unaligned or the local one", i);
  return prefill_impl(q, k, v, o, B, Hq, Hkv, M, N, d, q_strides, k_strides, v_strides,
                      o_strides, scale, causal, dtype, rope_cos, rope_sin, rope_max_pos,
                      rope_q_pos0, rope_k, workspace, workspace_bytes, o_peers, n_peers, stream);
}
