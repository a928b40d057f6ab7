// int8_gemm.cu — weight-only INT8 GEMM (W8A16) on sm_100a tensor cores.
//
// Semantics follow kernels/int8_matmul.py:17-110 and its reference
// kernels/ref/int8_matmul_ref.py:7-47: y = x @ (w_int8 * scales[:, None]).T
// (+ bias), x (M, K) in bf16/fp16, w_int8 (N, K) with one fp32 scale per output
// channel, fp32 accumulation, y (M, N) in x's dtype.
//
// The tcgen05 kernels compute y^T = W x^T: 128 weight rows (output channels)
// per tile are the MMA's M side and the tokens its N side (16-64 for decode,
// 128 or 256 otherwise), with split-K when the tile grid alone cannot fill the
// GPU (decode-sized M):
//   warp 0       TMA producer: int8 w tile (128 rows, swizzled) and the x tile
//                (tokens x 64 columns, 128-byte swizzle) into a ring of stages
//   warp 1       TMEM allocator and MMA issuer (whole warp runs the loop, one
//                elected lane issues): D(TMEM) += W(TMEM) * x_tile^T, kind::f16
//                with the A operand read from tensor memory
//   warps 4..11  converters: int8 w rows -> bf16/fp16 in registers (exact:
//                |w| <= 128), stored into tensor memory with tcgen05.st, so the
//                widened weights never pass through shared memory; then the
//                epilogue (one thread per output channel): D * scale[n]
//                (+ bias[n]) -> y, or fp32 partials of this K range for the
//                split-K reduce.
// For at most 16 tokens an mma.sync GEMV without staging or split-K is used.
// The per-channel scale factors out of the K sum, so it is applied once to the
// fp32 accumulator instead of to every weight.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "cie_common.cuh"
#include "sm100_ptx.cuh"

namespace cie {

constexpr int kQBN = 128;   // output channels per tile (the MMA's M side)
constexpr int kQBK = 64;    // K per stage: 64-byte int8 rows, 128-byte x rows
// 12 warps: TMA producer, MMA issuer, two idle, eight converters (two per
// TMEM lane quadrant, one per 32-column half of a stage) that also run the
// epilogue (one per lane quadrant and half of the token columns).
constexpr int kQConvWarps = 8;
constexpr int kQThreads = 128 + 32 * kQConvWarps;

template <int NT>
struct GemmCfg {
  static constexpr int XS = NT * kQBK * 2;      // x stage (B operand), 128-byte swizzle
  static constexpr int W8 = kQBN * kQBK;        // int8 w stage, 64-byte swizzle (8 KB)
  static constexpr int STAGE = XS + W8;
  static constexpr int STAGES = (200 * 1024) / STAGE > 8 ? 8 : (200 * 1024) / STAGE;
  static constexpr int NA = 4;                  // widened weight buffers in TMEM
  static constexpr int BAR_OFF = STAGES * STAGE;
  static constexpr int NBARS = 2 * STAGES + 2 * NA + 2;
  static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;
  // columns 0..NT-1: fp32 accumulator (channel x token); A_COL + 32 b: widened
  // buffer b (128 lanes x 64 16-bit values = 32 columns)
  static constexpr int A_COL = NT;
  static constexpr int TM_COLS = NT + 32 * NA <= 256 ? 256 : 512;
};

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

// M > 16: y^T = W x^T with 128 weight rows per tile as the MMA's M side (A
// operand, widened by the converter warps straight into tensor memory) and
// NT = 128 or 256 tokens as its N side (B operand, x by TMA). Per 64-column
// stage shared memory carries the int8 tile twice (TMA write, converter read)
// and the x tile twice (TMA write, MMA read).
template <bool BF16, int NT>
__global__ void __launch_bounds__(kQThreads, 1)
    int8_matmul_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_w, const Int8Params p) {
  using C = GemmCfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* bar_full = bars;                     // [S] x and int8 w landed
  uint64_t* bar_empty = bars + C::STAGES;        // [S] MMAs of the stage done
  uint64_t* bar_aready = bars + 2 * C::STAGES;   // [NA] widened buffer stored
  uint64_t* bar_afree = bar_aready + C::NA;      // [NA] widened buffer consumed
  uint64_t* bar_acc = bar_afree + C::NA;         // accumulator complete
  uint64_t* bar_drain = bar_acc + 1;             // abort path only
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto sx = [&](int st) { return smem + st * C::STAGE; };
  auto sw8 = [&](int st) { return smem + st * C::STAGE + C::XS; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * NT;
  const int n0 = blockIdx.y * kQBN;
  const int split = blockIdx.z;
  const int kt0 = split * p.tiles_per_split;
  const int kt1 = min(p.k_tiles, kt0 + p.tiles_per_split);
  const int nk = kt1 > kt0 ? kt1 - kt0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + s, 1);
      mbar_init(bar_empty + s, 1);
    }
    for (int b = 0; b < C::NA; ++b) {
      mbar_init(bar_aready + b, kQConvWarps);
      mbar_init(bar_afree + b, 1);
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
                               &g_wait_limit_ns))
          break;
        mbar_arrive_expect_tx(bar_full + st, C::STAGE);
        const int k = (kt0 + i) * kQBK;
        tma_load_4d(sw8(st), &tm_w, bar_full + st, k, n0, 0, 0);
        tma_load_4d(sx(st), &tm_x, bar_full + st, k, m0, 0, 0);
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
      const uint64_t dx0 = umma_smem_desc(smem_u32(sx(0)), 16, 1024);
      for (int i = 0; i < nk && ok; ++i) {
        const int st = i % C::STAGES, b = i % C::NA;
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(bar_full + st, (i / C::STAGES) & 1, abort_flag,
                                          &g_wait_limit_ns) &&
                            mbar_wait_bounded(bar_aready + b, (i / C::NA) & 1, abort_flag,
                                              &g_wait_limit_ns));
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_col = tmem + C::A_COL + b * 32;
        const uint64_t bx = dx0 + static_cast<uint64_t>((st * C::STAGE) >> 4);
#pragma unroll
        for (int kk = 0; kk < kQBK / 16; ++kk) {
          if (elect_one_sync())
            umma_ts(tmem, a_col + kk * 8, bx + ((kk * 32) >> 4), idesc, (i | kk) ? 1u : 0u);
        }
        if (elect_one_sync()) {
          umma_commit(bar_empty + st);
          umma_commit(bar_afree + b);
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
    const int quad = warp & 3, kh = (warp - 4) >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    for (int i = 0; i < nk; ++i) {
      const int st = i % C::STAGES, b = i % C::NA;
      ok = __all_sync(0xffffffffu,
                      mbar_wait_bounded(bar_full + st, (i / C::STAGES) & 1, abort_flag,
                                        &g_wait_limit_ns) &&
                          (i < C::NA || mbar_wait_bounded(bar_afree + b, ((i / C::NA) - 1) & 1,
                                                          abort_flag, &g_wait_limit_ns)));
      if (!ok) break;
      tc_fence_after();
      // 64-byte swizzle: chunk c of row r sits at chunk c ^ ((r >> 1) & 3); a
      // warp's 32 rows read one chunk each, conflict-free
      const uint8_t* src = sw8(st) + row * kQBK;
      uint4 vin[2];
#pragma unroll
      for (int c = 0; c < 2; ++c)
        vin[c] = *reinterpret_cast<const uint4*>(src + (((kh * 2 + c) ^ ((row >> 1) & 3)) * 16));
      uint32_t w16[16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint4 lo, hi;
        i8x16_to_f16x16<BF16>(vin[c], lo, hi);
        w16[8 * c + 0] = lo.x;
        w16[8 * c + 1] = lo.y;
        w16[8 * c + 2] = lo.z;
        w16[8 * c + 3] = lo.w;
        w16[8 * c + 4] = hi.x;
        w16[8 * c + 5] = hi.y;
        w16[8 * c + 6] = hi.z;
        w16[8 * c + 7] = hi.w;
      }
      tmem_st16(tmem + lane_addr + C::A_COL + b * 32 + kh * 16, w16);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_aready + b);
    }
    if (ok && nk > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_acc, 0, abort_flag, &g_wait_limit_ns));
    }
    if (ok) {
      tc_fence_after();
      using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      const int n = n0 + row;  // TMEM lane == output channel
      const float sc = n < p.N ? p.scales[n] : 0.f;
      const float bi = (n < p.N && p.bias) ? p.bias[n] : 0.f;
#pragma unroll 1
      for (int c0 = kh * (NT / 2); c0 < (kh + 1) * (NT / 2); c0 += 32) {
        uint32_t acc[32];
        if (nk > 0) {
          tmem_ld32(tmem + lane_addr + c0, acc);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0u;  // empty K range: zero partial
        }
        if (n < p.N) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int m = m0 + c0 + e;
            if (m >= p.M) break;
            const float v = __uint_as_float(acc[e]);
            if (p.split_k > 1) {
              p.part[(static_cast<int64_t>(split) * p.M + m) * p.N + n] = v;
            } else {
              elem_t* y = reinterpret_cast<elem_t*>(p.y) + m * p.y_sm + n;
              if constexpr (BF16) *y = __float2bfloat16_rn(v * sc + bi);
              else *y = __float2half_rn(v * sc + bi);
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
  if (warp == 1) tmem_dealloc(tmem, C::TM_COLS);
}

// Decode-sized M (17..64 rows of x): the roles are swapped, y^T = W x^T, so the
// 128 weight rows of a tile are the MMA's M side and the few tokens its N side
// (NT = 32 / 64). A stage carries 128 int8 columns of 128 weight rows (16 KB,
// 128-byte swizzle) and 8-16 KB of x. The converter warps widen the weights in
// registers and store them straight into tensor memory, where the MMA reads
// its A operand (tcgen05.mma with A in TMEM): shared memory then carries each
// weight byte twice (TMA write, converter read) instead of five times through
// a widened shared-memory copy. Each epilogue thread owns one output channel
// (its scale and bias are per-thread constants) and writes it for every token.
constexpr int kGBK = 128;
// Warps: TMA producer, MMA issuer, (two idle,) eight converters (two per TMEM
// lane quadrant, one per 64-column half of a stage), the first four of which
// also run the epilogue. PER_SM CTAs share an SM: 1 normally (a ~200 KB ring,
// 12 warps), 2 when the channel tiles alone exceed the SM count (a ~100 KB
// ring each and 10 warps, so that a wide layer runs in one wave instead of
// 1.5). The idle pair of the 12-warp form measured ~4 % faster than 10 warps.
constexpr int kGConvWarps = 8;
template <int PER_SM>
constexpr int kGConv0 = PER_SM == 1 ? 4 : 2;  // first converter warp
template <int PER_SM>
constexpr int kGThreads = 32 * (kGConv0<PER_SM> + kGConvWarps);

template <int NT, int PER_SM>
struct GemvCfg {
  static constexpr int W8 = kQBN * kGBK;         // int8 weights, 16 KB, 128-byte swizzle
  static constexpr int XBLK = NT * 128;          // one 64-column block of x
  static constexpr int XB = 2 * XBLK;            // x rows (B operand)
  static constexpr int STAGE = W8 + XB;
  static constexpr int RING = (PER_SM == 1 ? 200 : 100) * 1024;
  static constexpr int STAGES = RING / STAGE > 16 ? 16 : RING / STAGE;
  static constexpr int NA = 3;                   // widened weight buffers in TMEM
  static constexpr int BAR_OFF = STAGES * STAGE;
  static constexpr int NBARS = 2 * STAGES + 2 * NA + 2;
  static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;
  // columns 0..NT-1: fp32 accumulator; A_COL + 64 b: widened buffer b
  // (128 lanes x 128 16-bit values = 64 columns)
  static constexpr int A_COL = 64;
  static constexpr int TM_COLS = 256;
};

template <bool BF16, int NT, int PER_SM>
__global__ void __launch_bounds__(kGThreads<PER_SM>, PER_SM)
    int8_gemv_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_w, const Int8Params p) {
  using C = GemvCfg<NT, PER_SM>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* bar_full = bars;                     // [S] x and int8 w landed
  uint64_t* bar_empty = bars + C::STAGES;        // [S] MMAs of the stage done
  uint64_t* bar_aready = bars + 2 * C::STAGES;   // [NA] widened buffer stored
  uint64_t* bar_afree = bar_aready + C::NA;      // [NA] widened buffer consumed
  uint64_t* bar_acc = bar_afree + C::NA;
  uint64_t* bar_drain = bar_acc + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto sw8 = [&](int st) { return smem + st * C::STAGE; };
  auto sx = [&](int st) { return smem + st * C::STAGE + C::W8; };

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
    for (int b = 0; b < C::NA; ++b) {
      mbar_init(bar_aready + b, kGConvWarps);
      mbar_init(bar_afree + b, 1);
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
                               &g_wait_limit_ns))
          break;
        mbar_arrive_expect_tx(bar_full + st, C::XB + C::W8);
        const int k = (kt0 + i) * kGBK;
        tma_load_4d(sw8(st), &tm_w, bar_full + st, k, n0, 0, 0);
        tma_load_4d(sx(st), &tm_x, bar_full + st, k, 0, 0, 0);
        tma_load_4d(sx(st) + C::XBLK, &tm_x, bar_full + st, k + 64, 0, 0, 0);
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
      const uint64_t dx0 = umma_smem_desc(smem_u32(sx(0)), 16, 1024);
      for (int i = 0; i < nk && ok; ++i) {
        const int st = i % C::STAGES, b = i % C::NA;
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(bar_full + st, (i / C::STAGES) & 1, abort_flag,
                                          &g_wait_limit_ns) &&
                            mbar_wait_bounded(bar_aready + b, (i / C::NA) & 1, abort_flag,
                                              &g_wait_limit_ns));
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_col = tmem + C::A_COL + b * 64;
        const uint64_t bx = dx0 + static_cast<uint64_t>((st * C::STAGE) >> 4);
#pragma unroll
        for (int kk = 0; kk < kGBK / 16; ++kk) {
          const uint32_t offb = ((kk >> 2) * C::XBLK + (kk & 3) * 32) >> 4;
          if (elect_one_sync()) umma_ts(tmem, a_col + kk * 8, bx + offb, idesc, (i | kk) ? 1u : 0u);
        }
        if (elect_one_sync()) {
          umma_commit(bar_empty + st);
          umma_commit(bar_afree + b);
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
  } else if (warp >= kGConv0<PER_SM>) {
    // ------------------------------------------------ converters + epilogue
    // TMEM lane quadrant (warp % 4) = 32 weight rows; kh = which 64 columns
    const int quad = warp & 3, kh = (warp - kGConv0<PER_SM>) >> 2;
    const int row = quad * 32 + lane;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quad * 32) << 16) + C::A_COL + kh * 32;
    for (int i = 0; i < nk; ++i) {
      const int st = i % C::STAGES, b = i % C::NA;
      ok = __all_sync(0xffffffffu,
                      mbar_wait_bounded(bar_full + st, (i / C::STAGES) & 1, abort_flag,
                                        &g_wait_limit_ns) &&
                          (i < C::NA || mbar_wait_bounded(bar_afree + b, ((i / C::NA) - 1) & 1,
                                                          abort_flag, &g_wait_limit_ns)));
      if (!ok) break;
      tc_fence_after();
      // the 16-byte chunk c of row r sits at chunk c ^ (r & 7) (128-byte swizzle):
      // a warp's 32 rows read one chunk each, conflict-free
      const uint8_t* src = sw8(st) + row * kGBK;
      uint4 vin[4];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        vin[c] = *reinterpret_cast<const uint4*>(src + (((kh * 4 + c) ^ (row & 7)) * 16));
      uint32_t w16[32];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 lo, hi;
        i8x16_to_f16x16<BF16>(vin[c], lo, hi);
        w16[8 * c + 0] = lo.x;
        w16[8 * c + 1] = lo.y;
        w16[8 * c + 2] = lo.z;
        w16[8 * c + 3] = lo.w;
        w16[8 * c + 4] = hi.x;
        w16[8 * c + 5] = hi.y;
        w16[8 * c + 6] = hi.z;
        w16[8 * c + 7] = hi.w;
      }
      tmem_st32(t_row + b * 64, w16);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_aready + b);
    }
    if (ok && nk > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_acc, 0, abort_flag, &g_wait_limit_ns));
    }
    if (ok && kh == 0) {
      tc_fence_after();
      const int n = n0 + quad * 32 + lane;  // TMEM lane == output channel
      const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
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

// Small M (<= 16 tokens, K a multiple of 64): a tensor-core GEMV on mma.sync
// m16n8k16 with no tensor memory and no second kernel. A CTA owns 16 output
// channels over all of K; its 8 warps split K into 8 contiguous slices and add
// their 16 x 8NB accumulators in shared memory at the end. Each thread streams
// 16 bytes of two weight rows per 64-column chunk straight into registers
// (kMAhead chunks in flight), widens them there and feeds them as the A
// fragment; the K order inside a chunk is permuted identically for A and B
// (the MMA sums over k, so any common permutation gives the same result):
// fragment slots {2q, 2q+1, 2q+8, 2q+9} of step s hold columns 16q + 4s + 0..3,
// which makes a thread's A operand one 32-bit word of its 16-byte weight load
// and its B operand two consecutive words of its 16 x-values.
constexpr int kMWarps = 8;
constexpr int kMChunk = 64;
constexpr int kMAhead = 3;
constexpr int kMXBytes = 32 * 1024;  // x staged in shared memory up to this size (measured:
                                     // 64 KB staging is slower than per-chunk loads)

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t u4_word(const uint4& v, int s) {
  return s == 0 ? v.x : s == 1 ? v.y : s == 2 ? v.z : v.w;
}

template <bool BF16>
__device__ __forceinline__ uint32_t i8pair(uint32_t word, int sel) {
  if constexpr (BF16) return i8x2_to_f16x2<true>(word, sel);
  else return i8x2_to_h2(word ^ 0x80808080u, sel);
}

// XS: x (M x K, M <= 8, at most kMXBytes) is copied once into shared memory
// at launch (one bulk copy per token row, rows padded by 16 bytes so a warp's
// 16-byte reads of two tokens fall in disjoint banks) while the first weight
// chunks are in flight; otherwise each chunk's x-values are loaded from L2
// next to its weights.
template <bool BF16, int NB, bool XS>
// three CTAs per SM (<= 85 registers) so a 6144-channel layer fits in one wave
__global__ void __launch_bounds__(kMWarps * 32, 3) int8_gemv_mma_kernel(
    const int8_t* __restrict__ w, const uint16_t* __restrict__ x, const Int8Params p,
    int64_t w_sn, int64_t x_sm) {
  __shared__ float red[kMWarps][NB][4][32];
  __shared__ __align__(8) uint64_t x_bar;
  extern __shared__ __align__(16) uint8_t x_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = lane & 3, r = lane >> 2;
  const int n0 = blockIdx.x * 16;
  const int K = p.K;
  const int kc = K / kMChunk;
  const int cpw = (kc + kMWarps - 1) / kMWarps;
  const int c_begin = warp * cpw;
  const int c_end = min(kc, c_begin + cpw);
  const bool row0_ok = n0 + r < p.N, row1_ok = n0 + r + 8 < p.N;
  const int8_t* w0p = w + static_cast<int64_t>(row0_ok ? n0 + r : 0) * w_sn + 16 * q;
  const int8_t* w1p = w + static_cast<int64_t>(row1_ok ? n0 + r + 8 : 0) * w_sn + 16 * q;
  const uint32_t x_pitch = static_cast<uint32_t>(K) * 2u + 16u;

  if constexpr (XS) {
    if (threadIdx.x == 0) {
      mbar_init(&x_bar, 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(&x_bar, static_cast<uint32_t>(p.M) * K * 2u);
      for (int t = 0; t < p.M; ++t)
        bulk_load(x_smem + t * x_pitch, x + static_cast<int64_t>(t) * x_sm,
                  static_cast<uint32_t>(K) * 2u, &x_bar);
    }
  }

  auto load_w = [&](const int8_t* rowp, bool ok, int c) -> uint4 {
    return ok ? ld_stream16(rowp + c * kMChunk) : make_uint4(0u, 0u, 0u, 0u);
  };
  // 16 x values of token t at chunk c (zero for t >= M)
  auto load_x = [&](int t, int c, uint4& lo, uint4& hi) {
    if (t >= p.M) {
      lo = hi = make_uint4(0u, 0u, 0u, 0u);
      return;
    }
    if constexpr (XS) {
      const uint4* xp = reinterpret_cast<const uint4*>(x_smem + t * x_pitch +
                                                       (c * kMChunk + 16 * q) * 2);
      lo = xp[0];
      hi = xp[1];
    } else {
      const uint4* xp = reinterpret_cast<const uint4*>(
          x + static_cast<int64_t>(t) * x_sm + c * kMChunk + 16 * q);
      lo = __ldg(xp);
      hi = __ldg(xp + 1);
    }
  };

  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nb][e] = 0.f;

  uint4 wb[kMAhead][2];
#pragma unroll
  for (int u = 0; u < kMAhead; ++u) {
    const int c = c_begin + u;
    wb[u][0] = c < c_end ? load_w(w0p, row0_ok, c) : make_uint4(0u, 0u, 0u, 0u);
    wb[u][1] = c < c_end ? load_w(w1p, row1_ok, c) : make_uint4(0u, 0u, 0u, 0u);
  }
  bool ok = true;
  if constexpr (XS) {
    __syncthreads();  // x_bar initialised before anyone waits on it
    ok = mbar_wait_timeout(&x_bar, 0, kWaitLimitNs);
    if (!ok) raise_status(CIE_DEV_TIMEOUT);
  }
  for (int c0 = c_begin; ok && c0 < c_end; c0 += kMAhead) {
#pragma unroll
    for (int u = 0; u < kMAhead; ++u) {
      const int c = c0 + u;
      if (c >= c_end) break;
      uint4 xl[NB], xh[NB];
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) load_x(nb * 8 + r, c, xl[nb], xh[nb]);
      const uint4 wa = wb[u][0], wc = wb[u][1];
      if (c + kMAhead < c_end) {
        wb[u][0] = load_w(w0p, row0_ok, c + kMAhead);
        wb[u][1] = load_w(w1p, row1_ok, c + kMAhead);
      }
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint32_t w0s = u4_word(wa, s), w1s = u4_word(wc, s);
        const uint32_t a[4] = {i8pair<BF16>(w0s, 0), i8pair<BF16>(w1s, 0), i8pair<BF16>(w0s, 1),
                               i8pair<BF16>(w1s, 1)};
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const uint4& xv = s < 2 ? xl[nb] : xh[nb];
          mma_16816<BF16>(acc[nb], a, u4_word(xv, (2 * s) & 3), u4_word(xv, (2 * s + 1) & 3));
        }
      }
    }
  }
  if constexpr (XS) {
    // on a timeout the copies may still be landing: give them the same bound
    if (!ok) mbar_wait_timeout(&x_bar, 0, kWaitLimitNs);
  }

#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e) red[warp][nb][e][lane] = acc[nb][e];
  __syncthreads();
  using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  for (int o = threadIdx.x; ok && o < NB * 4 * 32; o += kMWarps * 32) {
    const int l = o & 31, e = (o >> 5) & 3, nb = o >> 7;
    float sum = 0.f;
#pragma unroll
    for (int wi = 0; wi < kMWarps; ++wi) sum += red[wi][nb][e][l];
    const int n = n0 + (l >> 2) + (e >= 2 ? 8 : 0);
    const int t = nb * 8 + 2 * (l & 3) + (e & 1);
    if (n < p.N && t < p.M) {
      float v = sum * p.scales[n];
      if (p.bias) v += p.bias[n];
      elem_t* y = reinterpret_cast<elem_t*>(p.y) + t * p.y_sm + n;
      if constexpr (BF16) *y = __float2bfloat16_rn(v);
      else *y = __float2half_rn(v);
    }
  }
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
  int tile_m;   // M > 64: tokens per tile (128 / 256)
  int gemv_nt;  // 16 / 32 / 64: decode-sized M on the tcgen05 GEMV
  int gemv_per_sm;  // tcgen05 GEMV CTAs per SM (1 / 2)
  int mma_nb;   // 1 / 2: M <= CIE_INT8_MMA_MAX_M on the mma.sync GEMV (8 tokens per block)
};

#ifndef CIE_INT8_MMA_MAX_M
#define CIE_INT8_MMA_MAX_M 16
#endif

// Split K only when the output tiles alone leave SMs idle (decode-sized M),
// keeping at least 4 K tiles per split so each CTA's pipeline fills.
static Int8Plan int8_plan(int M, int N, int K) {
  Int8Plan pl{};
  if (M <= CIE_INT8_MMA_MAX_M && K % kMChunk == 0) {
    // one CTA per 16 output channels over all of K: no split, no workspace
    pl.mma_nb = M <= 8 ? 1 : 2;
    pl.m_tiles = 1;
    pl.n_tiles = (N + 15) / 16;
    pl.k_tiles = K / kMChunk;
    pl.split_k = 1;
    pl.tiles_per_split = pl.k_tiles;
    return pl;
  }
  pl.gemv_nt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 0;
  if (pl.gemv_nt) {
    // one CTA per SM (~200 KB of stages): split K so the channel tiles times the
    // splits come close to the SM count without a second wave
    pl.m_tiles = 1;
    pl.n_tiles = (N + kQBN - 1) / kQBN;
    pl.k_tiles = (K + kGBK - 1) / kGBK;
    pl.gemv_per_sm = pl.n_tiles > num_sms() ? 2 : 1;
    int split = pl.gemv_per_sm * num_sms() / pl.n_tiles;
    const int cap = pl.k_tiles / 2 > 1 ? pl.k_tiles / 2 : 1;
    if (split > cap) split = cap;
    if (split < 1) split = 1;
    pl.tiles_per_split = (pl.k_tiles + split - 1) / split;
    pl.split_k = (pl.k_tiles + pl.tiles_per_split - 1) / pl.tiles_per_split;
    return pl;
  }
  pl.tile_m = M <= 128 ? 128 : 256;
  pl.m_tiles = (M + pl.tile_m - 1) / pl.tile_m;
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

template <bool BF16, int NT, int PER_SM>
static void launch_gemv_k(const CUtensorMap& mx, const CUtensorMap& mw, const Int8Params& prm,
                          const Int8Plan& pl, cudaStream_t st) {
  constexpr int smem = GemvCfg<NT, PER_SM>::SMEM;
  auto kern = int8_gemv_kernel<BF16, NT, PER_SM>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  kern<<<dim3(pl.n_tiles, pl.split_k), kGThreads<PER_SM>, smem, st>>>(mx, mw, prm);
}

template <bool BF16, int NT>
static void launch_gemv(const CUtensorMap& mx, const CUtensorMap& mw, const Int8Params& prm,
                        const Int8Plan& pl, cudaStream_t st) {
  if (pl.gemv_per_sm == 2) launch_gemv_k<BF16, NT, 2>(mx, mw, prm, pl, st);
  else launch_gemv_k<BF16, NT, 1>(mx, mw, prm, pl, st);
}

template <bool BF16, int NB>
static void launch_gemv_mma(const int8_t* w, const uint16_t* x, const Int8Params& prm,
                            const Int8Plan& pl, int64_t w_sn, int64_t x_sm, cudaStream_t st) {
  const size_t x_bytes = static_cast<size_t>(prm.M) * prm.K * 2;
  if (NB == 1 && x_bytes <= static_cast<size_t>(kMXBytes)) {
    const int smem = prm.M * (prm.K * 2 + 16);
    auto kern = int8_gemv_mma_kernel<BF16, 1, true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kMXBytes + 8 * 16);
    kern<<<pl.n_tiles, kMWarps * 32, smem, st>>>(w, x, prm, w_sn, x_sm);
  } else {
    int8_gemv_mma_kernel<BF16, NB, false><<<pl.n_tiles, kMWarps * 32, 0, st>>>(w, x, prm, w_sn,
                                                                              x_sm);
  }
}

template <bool BF16>
static int launch_int8(const CUtensorMap& mx, const CUtensorMap& mw, const Int8Params& prm,
                       const Int8Plan& pl, cudaStream_t st) {
  if (pl.gemv_nt == 16) launch_gemv<BF16, 16>(mx, mw, prm, pl, st);
  else if (pl.gemv_nt == 32) launch_gemv<BF16, 32>(mx, mw, prm, pl, st);
  else if (pl.gemv_nt == 64) launch_gemv<BF16, 64>(mx, mw, prm, pl, st);
  else {
    dim3 grid(pl.m_tiles, pl.n_tiles, pl.split_k);
    if (pl.tile_m == 128) {
      auto kern = int8_matmul_kernel<BF16, 128>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<128>::SMEM);
      kern<<<grid, kQThreads, GemmCfg<128>::SMEM, st>>>(mx, mw, prm);
    } else {
      auto kern = int8_matmul_kernel<BF16, 256>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<256>::SMEM);
      kern<<<grid, kQThreads, GemmCfg<256>::SMEM, st>>>(mx, mw, prm);
    }
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
  Int8Params prm{};
  prm.y = y;
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
  if (pl.mma_nb) {
    const auto* wi = static_cast<const int8_t*>(w);
    const auto* xi = static_cast<const uint16_t*>(x);
    if (bf16) {
      if (pl.mma_nb == 1) launch_gemv_mma<true, 1>(wi, xi, prm, pl, w_stride_n, x_stride_m, st);
      else launch_gemv_mma<true, 2>(wi, xi, prm, pl, w_stride_n, x_stride_m, st);
    } else {
      if (pl.mma_nb == 1) launch_gemv_mma<false, 1>(wi, xi, prm, pl, w_stride_n, x_stride_m, st);
      else launch_gemv_mma<false, 2>(wi, xi, prm, pl, w_stride_n, x_stride_m, st);
    }
    CIE_CHECK_LAUNCH("int8_gemv_mma_kernel");
    return CIE_OK;
  }
  CUtensorMap mx, mw;
  int rc = make_rows_map(&mx, x, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, K, M, x_stride_m, CU_TENSOR_MAP_SWIZZLE_128B, "cie_int8_matmul(x)",
                         pl.gemv_nt ? pl.gemv_nt : pl.tile_m);
  if (rc != CIE_OK) return rc;
  rc = make_rows_map(&mw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, w_stride_n,
                     pl.gemv_nt ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     "cie_int8_matmul(w)", 128, pl.gemv_nt ? kGBK : kQBK);
  if (rc != CIE_OK) return rc;
  prm.part = need > 0 ? reinterpret_cast<float*>(
                            (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255))
                      : nullptr;
  return bf16 ? launch_int8<true>(mx, mw, prm, pl, st) : launch_int8<false>(mx, mw, prm, pl, st);
}
