// int8_gemm.cu — weight-only INT8 GEMM (W8A16) on sm_100a tensor cores.
//
// Semantics follow kernels/int8_matmul.py:17-110 and its reference
// kernels/ref/int8_matmul_ref.py:7-47: y = x @ (w_int8 * scales[:, None]).T
// (+ bias), x (M, K) in bf16/fp16, w_int8 (N, K) with one fp32 scale per output
// channel, fp32 accumulation, y (M, N) in x's dtype.
//
// One CTA computes a 128 x 128 tile of y over a range of K (split-K when the
// tile grid alone cannot fill the GPU, e.g. decode-sized M):
//   warp 0      TMA producer: x tile (128 x 64, 128-byte swizzle) and the int8
//               w tile (128 x 64 bytes) into a ring of stages
//   warp 1      TMEM allocator and MMA issuer (whole warp runs the loop, one
//               elected lane issues): D(TMEM) += x_tile * w_tile^T, kind::f16
//   warps 4..7  converters: int8 w tile -> bf16/fp16 in the 128-byte swizzled
//               K-major layout the MMA reads (exact: |w| <= 128), then the
//               epilogue: D * scale[n] (+ bias[n]) -> y, or fp32 partials of
//               this K range for the split-K reduce.
// The per-channel scale factors out of the K sum, so it is applied once to the
// fp32 accumulator instead of to every weight.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "cie_common.cuh"
#include "sm100_ptx.cuh"

namespace cie {

constexpr int kQBM = 128;   // rows of x (and y) per tile
constexpr int kQBN = 128;   // output channels per tile
constexpr int kQBK = 64;    // K per stage (128 bytes of bf16 per row)
constexpr int kQStages = 5;
constexpr int kQThreads = 256;
constexpr int kQX = kQBM * kQBK * 2;    // x stage bytes (16 KB)
constexpr int kQW8 = kQBN * kQBK;       // int8 w stage bytes (8 KB)
constexpr int kQW16 = kQBN * kQBK * 2;  // converted w stage bytes (16 KB)
constexpr int kQStageBytes = kQX + kQW8 + kQW16;
constexpr int kQBarOff = kQStages * kQStageBytes;
constexpr int kQNBars = 3 * kQStages + 2;  // full, conv, empty per stage; acc_full; drain
constexpr int kQSmem = kQBarOff + kQNBars * 8 + 16 + 1024;

struct Int8Params {
  void* y;          // (M, N), x's dtype (split_k == 1)
  float* part;      // (split_k, M, N) fp32 partials (split_k > 1)
  const float* scales;
  const float* bias;  // may be null
  int M, N, K;
  int64_t y_sm;     // row stride of y in elements
  int k_tiles;      // ceil(K / 64)
  int split_k;
  int tiles_per_split;
};

// int8 -> two packed 16-bit floats, exact. The byte b is placed in the
// mantissa of 2^23 (fp32 0x4B000000 | (b ^ 0x80)), which is 2^23 + b + 128;
// subtracting 2^23 + 128 leaves b, then a round-to-nearest pack (exact here).
template <bool BF16>
__device__ __forceinline__ uint32_t i8x2_to_f16x2(uint32_t word, int sel) {
  // sel picks bytes (2*sel, 2*sel+1) of word
  const uint32_t flipped = word ^ 0x80808080u;
  const uint32_t lo = __byte_perm(flipped, 0x4B000000u, sel ? 0x7652 : 0x7650);
  const uint32_t hi = __byte_perm(flipped, 0x4B000000u, sel ? 0x7653 : 0x7651);
  const float a = __uint_as_float(lo) - 8388736.0f;  // 2^23 + 128
  const float b = __uint_as_float(hi) - 8388736.0f;
  return pack2<BF16>(a, b);
}


// int8 -> fp16x2 in two instructions: with u = b ^ 0x80, the fp16 bit pattern
// 0x6400 | u is 1024 + u (exact: 10-bit mantissa, one binade), so one byte
// permute builds two of them and one packed subtract of 1152 leaves b.
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t flipped, int sel) {
  const uint32_t h = __byte_perm(flipped, 0x64646464u, sel ? 0x7372 : 0x7170);
  uint32_t r;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
  return r;
}

// 16 int8 -> 16 bf16/fp16 as two 16-byte chunks.
template <bool BF16>
__device__ __forceinline__ void i8x16_to_f16x16(const uint4 v, uint4& lo, uint4& hi) {
  if constexpr (!BF16) {
    const uint4 f = make_uint4(v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u,
                               v.w ^ 0x80808080u);
    lo = make_uint4(i8x2_to_h2(f.x, 0), i8x2_to_h2(f.x, 1), i8x2_to_h2(f.y, 0),
                    i8x2_to_h2(f.y, 1));
    hi = make_uint4(i8x2_to_h2(f.z, 0), i8x2_to_h2(f.z, 1), i8x2_to_h2(f.w, 0),
                    i8x2_to_h2(f.w, 1));
    return;
  }
  lo.x = i8x2_to_f16x2<BF16>(v.x, 0);
  lo.y = i8x2_to_f16x2<BF16>(v.x, 1);
  lo.z = i8x2_to_f16x2<BF16>(v.y, 0);
  lo.w = i8x2_to_f16x2<BF16>(v.y, 1);
  hi.x = i8x2_to_f16x2<BF16>(v.z, 0);
  hi.y = i8x2_to_f16x2<BF16>(v.z, 1);
  hi.z = i8x2_to_f16x2<BF16>(v.w, 0);
  hi.w = i8x2_to_f16x2<BF16>(v.w, 1);
}

template <bool BF16>
__global__ void __launch_bounds__(kQThreads, 1)
    int8_matmul_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_w, const Int8Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQBarOff);
  uint64_t* bar_full = bars;                   // [S] x and int8 w landed
  uint64_t* bar_conv = bars + kQStages;        // [S] w converted (4 warps)
  uint64_t* bar_empty = bars + 2 * kQStages;   // [S] MMAs of the stage done
  uint64_t* bar_acc = bars + 3 * kQStages;     // accumulator complete
  uint64_t* bar_drain = bar_acc + 1;           // abort path only
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto sx = [&](int st) { return smem + st * kQStageBytes; };
  auto sw8 = [&](int st) { return smem + st * kQStageBytes + kQX; };
  auto sw16 = [&](int st) { return smem + st * kQStageBytes + kQX + kQW8; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kQBM;
  const int n0 = blockIdx.y * kQBN;
  const int split = blockIdx.z;
  const int kt0 = split * p.tiles_per_split;
  const int kt1 = min(p.k_tiles, kt0 + p.tiles_per_split);
  const int nk = kt1 > kt0 ? kt1 - kt0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(bar_full + s, 1);
      mbar_init(bar_conv + s, 4);
      mbar_init(bar_empty + s, 1);
    }
    mbar_init(bar_acc, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kQBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0 && nk > 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int st = i % kQStages;
        if (i >= kQStages &&
            !mbar_wait_bounded(bar_empty + st, ((i / kQStages) - 1) & 1, abort_flag,
                               kWaitLimitNs))
          break;
        mbar_arrive_expect_tx(bar_full + st, kQX + kQW8);
        const int k = (kt0 + i) * kQBK;
        tma_load_4d(sx(st), &tm_x, bar_full + st, k, m0, 0, 0);
        tma_load_4d(sw8(st), &tm_w, bar_full + st, k, n0, 0, 0);
        issued = i + 1;
      }
      if (*abort_flag) {
        for (int i = issued - 1; i >= 0 && i >= issued - kQStages; --i)
          mbar_wait_timeout(bar_full + (i % kQStages), (i / kQStages) & 1, kWaitLimitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (nk > 0) {
      constexpr uint32_t idesc = umma_idesc_f16(kQBM, kQBN, BF16 ? 1 : 0, 0, 0);
      const uint64_t dx0 = umma_smem_desc(smem_u32(sx(0)), 16, 1024);
      const uint64_t dw0 = umma_smem_desc(smem_u32(sw16(0)), 16, 1024);
      for (int i = 0; i < nk && ok; ++i) {
        const int st = i % kQStages;
        // x landed (TMA) and the converted w is in place
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(bar_full + st, (i / kQStages) & 1, abort_flag,
                                          kWaitLimitNs) &&
                            mbar_wait_bounded(bar_conv + st, (i / kQStages) & 1, abort_flag,
                                              kWaitLimitNs));
        if (!ok) break;
        tc_fence_after();
        const uint64_t ax = dx0 + static_cast<uint64_t>((st * kQStageBytes) >> 4);
        const uint64_t bw = dw0 + static_cast<uint64_t>((st * kQStageBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kQBK / 16; ++kk) {
          const uint32_t off = (kk * 32) >> 4;
          if (elect_one_sync()) umma_ss(tmem, ax + off, bw + off, idesc, (i | kk) ? 1u : 0u);
        }
        if (elect_one_sync()) umma_commit(bar_empty + st);
      }
      if (ok) {
        if (elect_one_sync()) umma_commit(bar_acc);
      } else {
        if (lane == 0) raise_status(CIE_DEV_TIMEOUT);
        if (elect_one_sync()) umma_commit(bar_drain);
        mbar_wait_timeout(bar_drain, 0, kWaitLimitNs);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ converters + epilogue
    const int ct = threadIdx.x - 128;  // 0..127
    for (int i = 0; i < nk; ++i) {
      const int st = i % kQStages;
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_full + st, (i / kQStages) & 1,
                                                     abort_flag, kWaitLimitNs));
      if (!ok) break;
      const uint8_t* src = sw8(st);
      uint8_t* dst = sw16(st);
      // 128 rows x 64 int8: per pass a warp reads 8 rows x 4 chunks of 16 bytes
      // (conflict-free) and writes each chunk as 2 swizzled 16-byte chunks
      // all loads first (independent), then convert and store: the converter
      // warps are latency-bound otherwise
      constexpr int kPass = kQW8 / (128 * 16);
      uint4 vin[kPass];
#pragma unroll
      for (int pass = 0; pass < kPass; ++pass) {
        const int idx = pass * 128 + ct;
        vin[pass] = *reinterpret_cast<const uint4*>(src + (idx >> 2) * kQBK + (idx & 3) * 16);
      }
#pragma unroll
      for (int pass = 0; pass < kPass; ++pass) {
        const int idx = pass * 128 + ct;
        const int row = idx >> 2, c = idx & 3;
        uint4 lo, hi;
        i8x16_to_f16x16<BF16>(vin[pass], lo, hi);
        uint8_t* drow = dst + row * 128;
        *reinterpret_cast<uint4*>(drow + (((2 * c) ^ (row & 7)) * 16)) = lo;
        *reinterpret_cast<uint4*>(drow + (((2 * c + 1) ^ (row & 7)) * 16)) = hi;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_conv + st);
    }
    if (ok && nk > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_acc, 0, abort_flag, kWaitLimitNs));
    }
    const int wq = warp & 3;
    const int m = m0 + wq * 32 + lane;  // TMEM lane == tile row
    const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
    if (ok) {
      tc_fence_after();
      using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
#pragma unroll 1
      for (int c0 = 0; c0 < kQBN; c0 += 32) {
        uint32_t acc[32];
        if (nk > 0) {
          tmem_ld32(tmem + lane_addr + c0, acc);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0u;  // empty K range: zero partial
        }
        const int nb = n0 + c0;
        if (m < p.M) {
        if (p.split_k > 1) {
          float* dst = p.part + (static_cast<int64_t>(split) * p.M + m) * p.N + nb;
          if (nb + 32 <= p.N && (p.N & 3) == 0) {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<float4*>(dst + e) =
                  make_float4(__uint_as_float(acc[e]), __uint_as_float(acc[e + 1]),
                              __uint_as_float(acc[e + 2]), __uint_as_float(acc[e + 3]));
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (nb + e < p.N) dst[e] = __uint_as_float(acc[e]);
          }
        } else {
          elem_t* dst = reinterpret_cast<elem_t*>(p.y) + m * p.y_sm + nb;
          float vals[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int n = nb + e < p.N ? nb + e : p.N - 1;
            float v = __uint_as_float(acc[e]) * __ldg(p.scales + n);
            if (p.bias) v += __ldg(p.bias + n);
            vals[e] = v;
          }
          if (nb + 32 <= p.N && (p.y_sm & 7) == 0 && (p.N & 7) == 0) {
#pragma unroll
            for (int e = 0; e < 32; e += 8)
              *reinterpret_cast<uint4*>(dst + e) =
                  make_uint4(pack2<BF16>(vals[e], vals[e + 1]), pack2<BF16>(vals[e + 2], vals[e + 3]),
                             pack2<BF16>(vals[e + 4], vals[e + 5]),
                             pack2<BF16>(vals[e + 6], vals[e + 7]));
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (nb + e >= p.N) continue;
              if constexpr (BF16) dst[e] = __float2bfloat16_rn(vals[e]);
              else dst[e] = __float2half_rn(vals[e]);
            }
          }
        }
        }
      }
    }
    if (!ok) raise_status(CIE_DEV_TIMEOUT);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kQBN);
}

// Decode-sized M (<= 64 rows of x): the roles are swapped, y^T = W x^T, so the
// 128 weight rows of a tile are the MMA's M side and the few tokens its N side
// (NT = 16 / 32 / 64). A stage then carries 2-8 KB of x instead of a 128-row
// tile, leaving room for 6-8 stages of weights in flight, which is what an
// HBM-bound GEMV needs; each epilogue thread owns one output channel (its
// scale and bias are per-thread constants) and writes it for every token.
// K per stage of the GEMV path: 128 int8 (one 128-byte row per output channel,
// which TMA streams far faster than 64-byte rows at a 4 KB row pitch).
constexpr int kGBK = 128;
// 12 warps: TMA producer, MMA issuer, two idle, eight converters (two per
// scheduler: the widening is the GEMV's critical path); warps 4..7 also run
// the epilogue.
constexpr int kGConvWarps = 8;
constexpr int kGThreads = 128 + 32 * kGConvWarps;

template <int NT>
struct GemvCfg {
  // ring of (int8 w tile, x tile) stages; converted bf16/fp16 w in 2 buffers.
  // 16-bit tiles are two 64-column blocks with the 128-byte swizzle.
  static constexpr int W8 = kQBN * kGBK;         // int8 weights, 16 KB
  static constexpr int W16 = kQBN * kGBK * 2;    // converted weights (A operand), 32 KB
  static constexpr int XBLK = NT * 128;          // one 64-column block of x
  static constexpr int XB = 2 * XBLK;            // x rows (B operand)
  static constexpr int STAGE = XB + W8;
  static constexpr int STAGES = (192 * 1024 - 2 * W16) / STAGE > 16 ? 16
                                : (192 * 1024 - 2 * W16) / STAGE;
  static constexpr int BAR_OFF = 2 * W16 + STAGES * STAGE;
  static constexpr int NBARS = 2 * STAGES + 4 + 2;
  static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;
  static constexpr int TM_COLS = NT < 32 ? 32 : NT;
};

template <bool BF16, int NT>
__global__ void __launch_bounds__(kGThreads, 1)
    int8_gemv_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_w, const Int8Params p) {
  using C = GemvCfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* bar_full = bars;                     // [S] x and int8 w landed
  uint64_t* bar_empty = bars + C::STAGES;        // [S] MMAs of the stage done
  uint64_t* bar_conv = bars + 2 * C::STAGES;     // [2] converted buffer ready
  uint64_t* bar_free = bar_conv + 2;             // [2] converted buffer consumed
  uint64_t* bar_acc = bar_free + 2;
  uint64_t* bar_drain = bar_acc + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto sw16 = [&](int buf) { return smem + buf * C::W16; };
  auto sx = [&](int st) { return smem + 2 * C::W16 + st * C::STAGE; };
  auto sw8 = [&](int st) { return smem + 2 * C::W16 + st * C::STAGE + C::XB; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kQBN;
  const int split = blockIdx.y;
  const int kt0 = split * p.tiles_per_split;
  const int kt1 = min(p.k_tiles, kt0 + p.tiles_per_split);
  const int nk = kt1 > kt0 ? kt1 - kt0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + s, 1);
      mbar_init(bar_empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_conv + b, kGConvWarps);
      mbar_init(bar_free + b, 1);
    }
    mbar_init(bar_acc, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
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
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0 && nk > 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::STAGES;
        if (i >= C::STAGES &&
            !mbar_wait_bounded(bar_empty + st, ((i / C::STAGES) - 1) & 1, abort_flag,
                               kWaitLimitNs))
          break;
        mbar_arrive_expect_tx(bar_full + st, C::XB + C::W8);
        const int k = (kt0 + i) * kGBK;
        tma_load_4d(sx(st), &tm_x, bar_full + st, k, 0, 0, 0);
        tma_load_4d(sx(st) + C::XBLK, &tm_x, bar_full + st, k + 64, 0, 0, 0);
        tma_load_4d(sw8(st), &tm_w, bar_full + st, k, n0, 0, 0);
        issued = i + 1;
      }
      if (*abort_flag) {
        for (int i = issued - 1; i >= 0 && i >= issued - C::STAGES; --i)
          mbar_wait_timeout(bar_full + (i % C::STAGES), (i / C::STAGES) & 1, kWaitLimitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (nk > 0) {
      constexpr uint32_t idesc = umma_idesc_f16(kQBN, NT, BF16 ? 1 : 0, 0, 0);
      const uint64_t dw0 = umma_smem_desc(smem_u32(sw16(0)), 16, 1024);
      const uint64_t dx0 = umma_smem_desc(smem_u32(sx(0)), 16, 1024);
      for (int i = 0; i < nk && ok; ++i) {
        const int st = i % C::STAGES, buf = i & 1;
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(bar_full + st, (i / C::STAGES) & 1, abort_flag,
                                          kWaitLimitNs) &&
                            mbar_wait_bounded(bar_conv + buf, (i >> 1) & 1, abort_flag,
                                              kWaitLimitNs));
        if (!ok) break;
        tc_fence_after();
        const uint64_t aw = dw0 + static_cast<uint64_t>((buf * C::W16) >> 4);
        const uint64_t bx = dx0 + static_cast<uint64_t>((st * C::STAGE) >> 4);
#pragma unroll
        for (int kk = 0; kk < kGBK / 16; ++kk) {
          const uint32_t offa = ((kk >> 2) * (kQBN * 128) + (kk & 3) * 32) >> 4;
          const uint32_t offb = ((kk >> 2) * C::XBLK + (kk & 3) * 32) >> 4;
          if (elect_one_sync()) umma_ss(tmem, aw + offa, bx + offb, idesc, (i | kk) ? 1u : 0u);
        }
        if (elect_one_sync()) {
          umma_commit(bar_empty + st);
          umma_commit(bar_free + buf);
        }
      }
      if (ok) {
        if (elect_one_sync()) umma_commit(bar_acc);
      } else {
        if (lane == 0) raise_status(CIE_DEV_TIMEOUT);
        if (elect_one_sync()) umma_commit(bar_drain);
        mbar_wait_timeout(bar_drain, 0, kWaitLimitNs);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ converters + epilogue
    const int ct = threadIdx.x - 128;  // 0 .. 32 * kGConvWarps - 1
    for (int i = 0; i < nk; ++i) {
      const int st = i % C::STAGES, buf = i & 1;
      ok = __all_sync(0xffffffffu,
                      mbar_wait_bounded(bar_full + st, (i / C::STAGES) & 1, abort_flag,
                                        kWaitLimitNs) &&
                          (i < 2 || mbar_wait_bounded(bar_free + buf, ((i >> 1) - 1) & 1,
                                                      abort_flag, kWaitLimitNs)));
      if (!ok) break;
      const uint8_t* src = sw8(st);
      uint8_t* dst = sw16(buf);
      // 128 rows x 128 int8: a warp reads 4 rows x 8 chunks of 16 bytes per pass
      constexpr int kCT = 32 * kGConvWarps;
      constexpr int kPass = C::W8 / (kCT * 16);
      uint4 vin[kPass];
#pragma unroll
      for (int pass = 0; pass < kPass; ++pass) {
        const int idx = pass * kCT + ct;
        vin[pass] = *reinterpret_cast<const uint4*>(src + (idx >> 3) * kGBK + (idx & 7) * 16);
      }
#pragma unroll
      for (int pass = 0; pass < kPass; ++pass) {
        const int idx = pass * kCT + ct;
        const int row = idx >> 3, c = idx & 7;
        uint4 lo, hi;
        i8x16_to_f16x16<BF16>(vin[pass], lo, hi);
        // 16-bit chunks 2c, 2c+1 of the row: block (chunk >> 3), swizzled in it
        uint8_t* drow = dst + (c >> 2) * (kQBN * 128) + row * 128;
        *reinterpret_cast<uint4*>(drow + ((((2 * c) & 7) ^ (row & 7)) * 16)) = lo;
        *reinterpret_cast<uint4*>(drow + ((((2 * c + 1) & 7) ^ (row & 7)) * 16)) = hi;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_conv + buf);
    }
    if (ok && nk > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_acc, 0, abort_flag, kWaitLimitNs));
    }
    if (ok && warp < 8) {
      tc_fence_after();
      const int wq = warp & 3;
      const int n = n0 + wq * 32 + lane;  // TMEM lane == output channel
      const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
      uint32_t acc[NT];
      if (nk > 0) {
        if constexpr (NT == 16) {
          uint32_t (&a16)[16] = reinterpret_cast<uint32_t (&)[16]>(acc);
          tmem_ld16(tmem + lane_addr, a16);
        } else {
#pragma unroll
          for (int c = 0; c < NT; c += 32) tmem_ld32(tmem + lane_addr + c, acc + c);
        }
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < NT; ++e) acc[e] = 0u;
      }
      if (n < p.N) {
        using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        const float sc = p.scales[n];
        const float bi = p.bias ? p.bias[n] : 0.f;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= p.M) break;
          const float v = __uint_as_float(acc[t]);
          if (p.split_k > 1) {
            p.part[(static_cast<int64_t>(split) * p.M + t) * p.N + n] = v;
          } else {
            elem_t* y = reinterpret_cast<elem_t*>(p.y) + t * p.y_sm + n;
            if constexpr (BF16) *y = __float2bfloat16_rn(v * sc + bi);
            else *y = __float2half_rn(v * sc + bi);
          }
        }
      }
    }
    if (!ok) raise_status(CIE_DEV_TIMEOUT);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TM_COLS);
}

// Sum of the split-K partials, then scale / bias and the cast to x's dtype.
template <bool BF16>
__global__ void __launch_bounds__(256) int8_splitk_reduce_kernel(const Int8Params p) {
  const int64_t total = static_cast<int64_t>(p.M) * p.N;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int m = static_cast<int>(i / p.N), n = static_cast<int>(i % p.N);
  float acc = 0.f;
  for (int s = 0; s < p.split_k; ++s) acc += p.part[s * total + i];
  float v = acc * p.scales[n];
  if (p.bias) v += p.bias[n];
  using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  elem_t* y = reinterpret_cast<elem_t*>(p.y) + m * p.y_sm + n;
  if constexpr (BF16) *y = __float2bfloat16_rn(v);
  else *y = __float2half_rn(v);
}

}  // namespace cie

namespace cie {

struct Int8Plan {
  int m_tiles, n_tiles, k_tiles, split_k, tiles_per_split;
  int gemv_nt;  // 16 / 32 / 64: decode-sized M, swapped roles; 0: 128 x 128 tiles
};

// Split K only when the output tiles alone leave SMs idle (decode-sized M),
// keeping at least 4 K tiles per split so each CTA's pipeline fills.
static Int8Plan int8_plan(int M, int N, int K) {
  Int8Plan pl{};
  pl.gemv_nt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 0;
  if (pl.gemv_nt) {
    // one CTA per SM (~200 KB of stages): split K so the channel tiles times the
    // splits come close to the SM count without a second wave
    pl.m_tiles = 1;
    pl.n_tiles = (N + kQBN - 1) / kQBN;
    pl.k_tiles = (K + kGBK - 1) / kGBK;
    int split = num_sms() / pl.n_tiles;
    const int cap = pl.k_tiles / 2 > 1 ? pl.k_tiles / 2 : 1;
    if (split > cap) split = cap;
    if (split < 1) split = 1;
    pl.tiles_per_split = (pl.k_tiles + split - 1) / split;
    pl.split_k = (pl.k_tiles + pl.tiles_per_split - 1) / pl.tiles_per_split;
    return pl;
  }
  pl.m_tiles = (M + kQBM - 1) / kQBM;
  pl.n_tiles = (N + kQBN - 1) / kQBN;
  pl.k_tiles = (K + kQBK - 1) / kQBK;
  const int tiles = pl.m_tiles * pl.n_tiles;
  const int sms = num_sms();
  int split = 1;
  if (tiles < sms) {
    split = (sms + tiles - 1) / tiles;
    const int cap = pl.k_tiles / 4 > 1 ? pl.k_tiles / 4 : 1;
    if (split > cap) split = cap;
  }
  pl.tiles_per_split = (pl.k_tiles + split - 1) / split;
  pl.split_k = (pl.k_tiles + pl.tiles_per_split - 1) / pl.tiles_per_split;
  return pl;
}

static size_t int8_part_bytes(const Int8Plan& pl, int M, int N) {
  return pl.split_k > 1 ? static_cast<size_t>(pl.split_k) * M * N * sizeof(float) : 0;
}

// 2-D (K innermost) map over `rows` rows, box 64 x box_rows.
static int make_rows_map(CUtensorMap* map, const void* base, CUtensorMapDataType type,
                         int elem_bytes, int K, int rows, int64_t row_stride_elems,
                         CUtensorMapSwizzle sw, const char* what, int box_rows = 128,
                         int box_k = kQBK) {
  PFN_encodeTiled_t enc = tensor_map_encoder();
  if (!enc) {
    set_error("%s: cuTensorMapEncodeTiled unavailable", what);
    return CIE_ERR_LAUNCH;
  }
  cuuint64_t dims[4] = {(cuuint64_t)K, (cuuint64_t)rows, 1, 1};
  const cuuint64_t rs = static_cast<cuuint64_t>(row_stride_elems) * elem_bytes;
  cuuint64_t gstr[3] = {rs, rs * rows, rs * rows};
  cuuint32_t box[4] = {(cuuint32_t)box_k, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, type, 4, const_cast<void*>(base), dims, gstr, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
    return CIE_ERR_INVALID;
  }
  return CIE_OK;
}

template <bool BF16, int NT>
static void launch_gemv(const CUtensorMap& mx, const CUtensorMap& mw, const Int8Params& prm,
                        const Int8Plan& pl, cudaStream_t st) {
  constexpr int smem = GemvCfg<NT>::SMEM;
  auto kern = int8_gemv_kernel<BF16, NT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  kern<<<dim3(pl.n_tiles, pl.split_k), kGThreads, smem, st>>>(mx, mw, prm);
}

template <bool BF16>
static int launch_int8(const CUtensorMap& mx, const CUtensorMap& mw, const Int8Params& prm,
                       const Int8Plan& pl, cudaStream_t st) {
  if (pl.gemv_nt == 16) launch_gemv<BF16, 16>(mx, mw, prm, pl, st);
  else if (pl.gemv_nt == 32) launch_gemv<BF16, 32>(mx, mw, prm, pl, st);
  else if (pl.gemv_nt == 64) launch_gemv<BF16, 64>(mx, mw, prm, pl, st);
  else {
    auto kern = int8_matmul_kernel<BF16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kQSmem);
    dim3 grid(pl.m_tiles, pl.n_tiles, pl.split_k);
    kern<<<grid, kQThreads, kQSmem, st>>>(mx, mw, prm);
  }
  CIE_CHECK_LAUNCH("int8_matmul_kernel");
  if (pl.split_k > 1) {
    const int64_t total = static_cast<int64_t>(prm.M) * prm.N;
    const int blocks = static_cast<int>((total + 255) / 256);
    int8_splitk_reduce_kernel<BF16><<<blocks, 256, 0, st>>>(prm);
    CIE_CHECK_LAUNCH("int8_splitk_reduce_kernel");
  }
  return CIE_OK;
}

}  // namespace cie

using namespace cie;

extern "C" size_t cie_int8_matmul_workspace(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const Int8Plan pl = int8_plan(M, N, K);
  const size_t b = int8_part_bytes(pl, M, N);
  return b > 0 ? b + 256 : 0;
}

extern "C" int cie_int8_matmul(const void* x, const void* w, const float* scales,
                               const float* bias, void* y, int M, int N, int K,
                               int64_t x_stride_m, int64_t w_stride_n, int64_t y_stride_m,
                               int dtype, void* workspace, size_t workspace_bytes,
                               void* stream) {
  CIE_CHECK_ARG(x && w && scales && y, "cie_int8_matmul: null pointer");
  CIE_CHECK_ARG(M >= 0 && N > 0 && K > 0, "cie_int8_matmul: bad shape (M=%d, N=%d, K=%d)", M, N,
                K);
  CIE_CHECK_ARG(dtype == CIE_DTYPE_BF16 || dtype == CIE_DTYPE_FP16,
                "cie_int8_matmul: bad dtype %d", dtype);
  if (M == 0) return CIE_OK;
  CIE_CHECK_ARG(x_stride_m >= K && x_stride_m % 8 == 0,
                "cie_int8_matmul: x row stride must be >= K and a multiple of 8 elements");
  CIE_CHECK_ARG(w_stride_n >= K && w_stride_n % 16 == 0,
                "cie_int8_matmul: w row stride must be >= K and a multiple of 16 bytes");
  CIE_CHECK_ARG(y_stride_m >= N, "cie_int8_matmul: y row stride must be >= N");
  CIE_CHECK_ARG(aligned16(x) && aligned16(w) && aligned16(y),
                "cie_int8_matmul: x, w and y must be 16-byte aligned");
  const Int8Plan pl = int8_plan(M, N, K);
  const size_t need = cie_int8_matmul_workspace(M, N, K);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) {
    set_error("cie_int8_matmul: workspace of %zu bytes required, got %zu", need, workspace_bytes);
    return CIE_ERR_WORKSPACE;
  }
  const bool bf16 = dtype == CIE_DTYPE_BF16;
  CUtensorMap mx, mw;
  int rc = make_rows_map(&mx, x, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, K, M, x_stride_m, CU_TENSOR_MAP_SWIZZLE_128B, "cie_int8_matmul(x)",
                         pl.gemv_nt ? pl.gemv_nt : 128);
  if (rc != CIE_OK) return rc;
  rc = make_rows_map(&mw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, w_stride_n,
                     CU_TENSOR_MAP_SWIZZLE_NONE, "cie_int8_matmul(w)", 128,
                     pl.gemv_nt ? kGBK : kQBK);
  if (rc != CIE_OK) return rc;
  Int8Params prm{};
  prm.y = y;
  prm.part = need > 0 ? reinterpret_cast<float*>(
                            (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255))
                      : nullptr;
  prm.scales = scales;
  prm.bias = bias;
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.y_sm = y_stride_m;
  prm.k_tiles = pl.k_tiles;
  prm.split_k = pl.split_k;
  prm.tiles_per_split = pl.tiles_per_split;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return bf16 ? launch_int8<true>(mx, mw, prm, pl, st) : launch_int8<false>(mx, mw, prm, pl, st);
}
