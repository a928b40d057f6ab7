// paged_attn.cu — paged-KV attention for single-token decode and speculative
// verify on sm_100a (and the same kernel over dense K/V for short query
// blocks and head dims the tcgen05 prefill kernel does not take).
//
// What it computes (per sequence b, query head h, query row i < M):
//   out[b,h,i,:] = softmax_j(q_rot[b,h,i,:] . K[b,kvh,j,:] * scale) V[b,kvh,j,:]
// over keys j < kv_len[b] (and j <= kv_len[b] - M + i when causal), where
// K/V rows are fetched through the block table exactly as
// PagedKVCache.gather does (engine/cache/kv_cache.py:141-165) and the
// attention matches kernels/ref/flash_attention_ref.py:8-56 with GQA
// (kv head = h / (Hq / Hkv)).
//
// How: one CTA per (split-KV partition, kv head, row group, sequence). The
// query rows of all heads sharing a kv head (G = Hq/Hkv heads x M rows) form
// the M side of m16n8k16 tensor-core MMAs, so K/V bytes are read from HBM once
// per kv head. Each of the 4 warps streams its own 16-token K/V tiles through
// a private ring of shared-memory stages:
//   * TMA path (block size a multiple of 16, or dense K/V): one elected lane
//     issues one 2-D box per 64-column slice of a 16-token block, completion
//     tracked by an mbarrier per stage; no per-row address arithmetic.
//   * cp.async path (any other block size): 16-byte cp.async per row chunk
//     with a block-table lookup per row.
// Both land tiles in the 16-byte-chunk XOR-swizzled layout TMA produces for
// 32/64/128-byte rows, which ldmatrix reads without bank conflicts. Each warp
// runs an online softmax (quad shuffles) over its tiles; the 4 warps are
// merged in shared memory, and split-KV partitions of one sequence by a
// log-sum-exp merge kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <type_traits>

#include "cie_common.cuh"
#include "sm100_ptx.cuh"

namespace cie {

struct PagedParams {
  const void* q;
  const void* k_pool;
  const void* v_pool;
  const int32_t* block_tables;
  const int32_t* kv_lens;
  void* o;
  float* part_o;    // [units][max_splits][RG][D]
  float* part_lse;  // [units][max_splits][RG]
  const float* cos;
  const float* sin;
  int rope_max_pos;
  int B, Hq, Hkv, M, G;
  int num_blocks, block_size, max_blocks;
  int bs_log2;  // log2(block_size) when it is a power of two, else -1
  int64_t q_sb, q_sh, q_sm;
  int64_t o_sb, o_sh, o_sm;
  int split_tokens;
  int max_splits;
  int row_groups;  // ceil(G*M / RG)
  float scale_log2;
  int causal;
  // dense mode (K/V as (B, Hkv, N, d) tensors instead of paged pools)
  int dense_n;
  int64_t k_sb, k_sh, k_sn;
  int64_t v_sb, v_sh, v_sn;
  int rope_q_pos0;  // dense mode: q row i rotated at rope_q_pos0 + i
};

constexpr int kPagedWarps = 4;
constexpr int kTileTok = 16;

template <int D>
struct PagedCfg {
  static constexpr int ROWB = (D * 2 < 128) ? D * 2 : 128;  // bytes per swizzled sub-row
  static constexpr int KCS = ROWB / 16;                     // 16B chunks per sub-row
  static constexpr int SUBS = (D * 2) / ROWB;               // 64-column slices per row
  static constexpr int kStages = (D <= 64) ? 3 : (D == 128 ? 3 : 2);
  static constexpr int kTileBytes = kTileTok * D * 2;  // K or V tile
  static constexpr int kStageBytes = 2 * kTileBytes;   // K + V
  static constexpr int kWarpBytes = kStages * kStageBytes;
  static constexpr int kPipeBytes = kPagedWarps * kWarpBytes;
};

// 16-byte-chunk XOR swizzle of rows of KC chunks: the layout TMA writes for
// 32/64/128-byte swizzle modes, so the 8 rows an ldmatrix phase reads land in
// 8 distinct 16-byte bank groups.
template <int KC>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  if constexpr (KC >= 8) return static_cast<uint32_t>(chunk ^ (row & 7));
  else return static_cast<uint32_t>(chunk ^ ((row / (8 / KC)) & (KC - 1)));
}

// Byte offset of 16-byte chunk `ch` of tile row `row` in a K/V tile:
// [SUBS][16 rows][ROWB], each slice swizzled.
template <int D>
__device__ __forceinline__ uint32_t kv_off(int row, int ch) {
  using C = PagedCfg<D>;
  const int sub = ch / C::KCS, w = ch % C::KCS;
  return sub * (kTileTok * C::ROWB) + row * C::ROWB + swz<C::KCS>(row, w) * 16;
}

template <int D, int MT>
__host__ __device__ constexpr int paged_pipe_or_merge() {
  constexpr int RG = 16 * MT;
  constexpr int pipe = PagedCfg<D>::kPipeBytes;
  constexpr int merge = kPagedWarps * RG * (D + 6) * 4;
  return pipe > merge ? pipe : merge;
}

template <int D, int MT>
__host__ __device__ constexpr int paged_smem_bytes() {
  // pipeline ring (reused for the cross-warp merge) + rotated Q tile + barriers
  return paged_pipe_or_merge<D, MT>() + 16 * MT * D * 2 +
         kPagedWarps * PagedCfg<D>::kStages * 8 + 16 + kPagedWarps * PagedCfg<D>::kStages * 4 +
         1024;
}

template <int D, int MT, bool BF16, bool PAGED, bool TMA>
__global__ void __launch_bounds__(kPagedWarps * 32)
    paged_attn_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const PagedParams p) {
  using Cfg = PagedCfg<D>;
  constexpr int RG = 16 * MT;
  constexpr int KC = D / 8;
  constexpr int STAGES = Cfg::kStages;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* pipe = smem;
  uint8_t* qs = smem + paged_pipe_or_merge<D, MT>();
  uint64_t* full_bars = reinterpret_cast<uint64_t*>(qs + RG * D * 2);  // [warps][STAGES]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full_bars + kPagedWarps * STAGES);
  int* stage_bad = const_cast<int*>(abort_flag) + 4;  // [warps][STAGES]

  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.row_groups;
  const int rg = blockIdx.y % p.row_groups;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  int kv_len = PAGED ? p.kv_lens[b] : p.dense_n;
  if (kv_len < 0) kv_len = 0;
  if (PAGED && kv_len > p.max_blocks * p.block_size) {
    // a length beyond the table's capacity cannot be served: flag it and clamp
    if (split == 0 && blockIdx.y == 0 && tid == 0) raise_status(CIE_DEV_BAD_BLOCK_ID);
    kv_len = p.max_blocks * p.block_size;
  }
  const int nsplit = kv_len > 0 ? (kv_len + p.split_tokens - 1) / p.split_tokens : 1;
  if (split >= nsplit) return;
  const int R = p.G * p.M;   // rows of this kv-head group
  const int row0 = rg * RG;  // first row of this CTA
  // keys past the last visible key of this CTA's rows are never loaded
  int key_cap = kv_len;
  if (p.causal) {
    const int last = min(row0 + RG, R) - 1;
    const int max_m = (row0 / p.M != last / p.M) ? p.M - 1 : last % p.M;
    key_cap = max(0, min(kv_len, kv_len - p.M + max_m + 1));
  }
  const int tok_begin = split * p.split_tokens;
  const int tok_end = min(key_cap, tok_begin + p.split_tokens);
  const int n_tiles = tok_end > tok_begin ? (tok_end - tok_begin + kTileTok - 1) / kTileTok : 0;
  const int q_pos_base = PAGED ? kv_len - p.M : p.rope_q_pos0;

  if constexpr (TMA) {
    if (tid == 0) {
      for (int i = 0; i < kPagedWarps * STAGES; ++i) mbar_init(full_bars + i, 1);
      *abort_flag = 0;
      fence_mbar_init();
    }
  }

  __syncthreads();  // barrier init visible before the first TMA is issued

  // ---- per-warp streaming of K/V tiles ----
  const int g = lane >> 2;  // row within an 8-row group
  const int t4 = lane & 3;

  float o_acc[MT][D / 8][4];
  float m_run[MT][2], l_run[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o_acc[mt][nt][e] = 0.f;
    m_run[mt][0] = m_run[mt][1] = -INFINITY;
    l_run[mt][0] = l_run[mt][1] = 0.f;
  }

  uint8_t* wpipe = pipe + warp * Cfg::kWarpBytes;
  uint64_t* wbars = full_bars + warp * STAGES;
  const int32_t* table = PAGED ? p.block_tables + static_cast<int64_t>(b) * p.max_blocks : nullptr;
  const uint8_t* kpool = reinterpret_cast<const uint8_t*>(p.k_pool);
  const uint8_t* vpool = reinterpret_cast<const uint8_t*>(p.v_pool);
  const int64_t tok_stride = static_cast<int64_t>(p.Hkv) * D * 2;  // bytes per token row
  const int64_t head_off = static_cast<int64_t>(kvh) * D * 2;

  // physical block of the 16-token tile starting at t0 (TMA path: one block
  // holds the whole tile); -1 when the table entry is invalid
  auto tile_block = [&](int t0) -> int {
    const int lb = p.bs_log2 >= 0 ? (t0 >> p.bs_log2) : t0 / p.block_size;
    const int blk = lb < p.max_blocks ? table[lb] : -1;
    return (blk < 0 || blk >= p.num_blocks) ? -1 : blk;
  };

  auto issue_tile = [&](int tile, int stage) {
    uint8_t* ks = wpipe + stage * Cfg::kStageBytes;
    uint8_t* vs = ks + Cfg::kTileBytes;
    const int t0 = tok_begin + tile * kTileTok;
    if constexpr (TMA) {
      if (lane == 0) {
        fence_proxy_async_smem();  // this warp's reads of the stage precede the overwrite
        int c2 = 0, c3 = 0;
        bool ok = true;
        if constexpr (PAGED) {
          const int blk = tile_block(t0);
          ok = blk >= 0;
          c2 = blk * p.block_size +
               (p.bs_log2 >= 0 ? (t0 & (p.block_size - 1)) : t0 % p.block_size);
          // record a refused block id for the consumer lanes (read after the wait)
          stage_bad[warp * STAGES + stage] = ok ? 0 : 1;
        } else {
          c2 = kvh;
          c3 = b;
        }
        if (ok) {
          mbar_arrive_expect_tx(wbars + stage, 2 * Cfg::kTileBytes);
#pragma unroll
          for (int sub = 0; sub < Cfg::SUBS; ++sub) {
            if constexpr (PAGED) {
              tma_load_4d(ks + sub * kTileTok * Cfg::ROWB, &tm_k, wbars + stage, sub * 64, kvh,
                          c2, 0);
              tma_load_4d(vs + sub * kTileTok * Cfg::ROWB, &tm_v, wbars + stage, sub * 64, kvh,
                          c2, 0);
            } else {
              tma_load_4d(ks + sub * kTileTok * Cfg::ROWB, &tm_k, wbars + stage, sub * 64, t0,
                          c2, c3);
              tma_load_4d(vs + sub * kTileTok * Cfg::ROWB, &tm_v, wbars + stage, sub * 64, t0,
                          c2, c3);
            }
          }
        } else {
          raise_status(CIE_DEV_BAD_BLOCK_ID);
          mbar_arrive(wbars + stage);  // completes the phase; the stage is zeroed on use
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < (kTileTok * KC) / 32; ++i) {
        const int q = lane + 32 * i;
        const int row = q / KC;
        const int ch = q % KC;
        const int tok = t0 + row;
        bool valid = tok < tok_end;
        int64_t koff = 0, voff = 0;
        if (valid) {
          if constexpr (PAGED) {
            const int lb = tok / p.block_size;
            const int blk = lb < p.max_blocks ? table[lb] : -1;
            if (blk < 0 || blk >= p.num_blocks) {
              raise_status(CIE_DEV_BAD_BLOCK_ID);
              valid = false;
            } else {
              koff = (static_cast<int64_t>(blk) * p.block_size + (tok % p.block_size)) *
                         tok_stride + head_off + ch * 16;
              voff = koff;
            }
          } else {
            koff = (b * p.k_sb + kvh * p.k_sh + tok * p.k_sn) * 2 + ch * 16;
            voff = (b * p.v_sb + kvh * p.v_sh + tok * p.v_sn) * 2 + ch * 16;
          }
        }
        const uint32_t so = kv_off<D>(row, ch);
        cp_async_16(ks + so, kpool + koff, valid);
        cp_async_16(vs + so, vpool + voff, valid);
      }
    }
  };

  // K/V prologue first: the copies are in flight while Q is rotated below
  const int my_tiles = n_tiles > warp ? (n_tiles - warp + kPagedWarps - 1) / kPagedWarps : 0;
  int issued = 0;
  const uint64_t wait_ns = g_wait_limit_ns;  // pipeline wait limit of this launch
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < my_tiles) {
      issue_tile(warp + kPagedWarps * s, s);
      ++issued;
    }
    if constexpr (!TMA) cp_async_commit();
  }

  // ---- rotated Q tile -> shared memory (16B-chunk swizzle) ----
  {
    using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    const elem_t* q = reinterpret_cast<const elem_t*>(p.q);
    constexpr int HALF = D / 2;
    constexpr int PAIR_CHUNKS = HALF / 8;  // 8 rotation pairs per work item
    for (int w = tid; w < RG * PAIR_CHUNKS; w += blockDim.x) {
      const int r = w / PAIR_CHUNKS;
      const int pc = w % PAIR_CHUNKS;
      const int gr = row0 + r;
      uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
      if (gr < R) {
        const int gh = gr / p.M, m = gr % p.M;
        const int h = kvh * p.G + gh;
        const elem_t* src = q + b * p.q_sb + h * p.q_sh + m * p.q_sm;
        const uint4 x1 = *reinterpret_cast<const uint4*>(src + pc * 8);
        const uint4 x2 = *reinterpret_cast<const uint4*>(src + HALF + pc * 8);
        if (p.cos != nullptr) {
          int pos = q_pos_base + m;
          if (pos < 0 || pos >= p.rope_max_pos) {
            raise_status(CIE_DEV_BAD_POSITION);
            pos = pos < 0 ? 0 : p.rope_max_pos - 1;
          }
          const float* cr = p.cos + static_cast<int64_t>(pos) * HALF + pc * 8;
          const float* sr = p.sin + static_cast<int64_t>(pos) * HALF + pc * 8;
          const uint32_t* a = reinterpret_cast<const uint32_t*>(&x1);
          const uint32_t* c = reinterpret_cast<const uint32_t*>(&x2);
          uint32_t* lo_w = reinterpret_cast<uint32_t*>(&lo);
          uint32_t* hi_w = reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 u1 = unpack2<BF16>(a[e]);
            const float2 u2 = unpack2<BF16>(c[e]);
            const float c0 = cr[2 * e], c1 = cr[2 * e + 1];
            const float s0 = sr[2 * e], s1 = sr[2 * e + 1];
            // rot1 = x1*c - x2*s ; rot2 = x1*s + x2*c  (rope_apply_ref.py:49-53)
            lo_w[e] = pack2<BF16>(__fsub_rn(__fmul_rn(u1.x, c0), __fmul_rn(u2.x, s0)),
                                  __fsub_rn(__fmul_rn(u1.y, c1), __fmul_rn(u2.y, s1)));
            hi_w[e] = pack2<BF16>(__fadd_rn(__fmul_rn(u1.x, s0), __fmul_rn(u2.x, c0)),
                                  __fadd_rn(__fmul_rn(u1.y, s1), __fmul_rn(u2.y, c1)));
          }
        } else {
          lo = x1;
          hi = x2;
        }
      }
      const int c_lo = pc, c_hi = HALF / 8 + pc;
      *reinterpret_cast<uint4*>(qs + r * (D * 2) + swz<KC>(r, c_lo) * 16) = lo;
      *reinterpret_cast<uint4*>(qs + r * (D * 2) + swz<KC>(r, c_hi) * 16) = hi;
    }
  }
  __syncthreads();

  // Q A-fragments (held in registers when small).
  constexpr bool kQReg = (MT * D) <= 128;
  uint32_t qa[kQReg ? MT : 1][kQReg ? D / 16 : 1][4];
  auto load_qfrag = [&](int mt, int kk, uint32_t (&a)[4]) {
    const int row = mt * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
    const int ch = 2 * kk + (lane >> 4);
    ldmatrix_x4(smem_u32(qs + row * (D * 2) + swz<KC>(row, ch) * 16), a[0], a[1], a[2], a[3]);
  };
  if constexpr (kQReg) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) load_qfrag(mt, kk, qa[mt][kk]);
  }

  // Key limit of each row this thread owns: (mt, half) -> keys <= lim are visible
  int lim[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int gr = row0 + mt * 16 + g + 8 * hf;
      const int m = gr % p.M;
      lim[mt][hf] = p.causal ? (kv_len - p.M + m) : (kv_len - 1);
    }
  const int lim_min = p.causal ? (kv_len - p.M) : (kv_len - 1);

  for (int it = 0; it < my_tiles; ++it) {
    {
      const int nx = it + STAGES - 1;
      if (nx < my_tiles) {
        issue_tile(warp + kPagedWarps * nx, nx % STAGES);
        ++issued;
      }
      if constexpr (!TMA) cp_async_commit();
    }
    const int stage = it % STAGES;
    uint8_t* ks = wpipe + stage * Cfg::kStageBytes;
    uint8_t* vs = ks + Cfg::kTileBytes;
    const int t0 = tok_begin + (warp + kPagedWarps * it) * kTileTok;
    if constexpr (TMA) {
      const bool ok = mbar_wait_bounded(wbars + stage, (it / STAGES) & 1, abort_flag, wait_ns);
      if (!__all_sync(0xffffffffu, ok)) {
        raise_status(CIE_DEV_TIMEOUT);
        break;
      }
      // rows past the valid keys of a paged tile hold whatever the block holds:
      // zero them in V (P is 0 there, but 0 * NaN would not be); a tile whose
      // block id was refused is zeroed entirely
      int valid_rows = kTileTok;
      if constexpr (PAGED) {
        if (stage_bad[warp * STAGES + stage]) valid_rows = 0;
        else if (t0 + kTileTok > kv_len) valid_rows = kv_len - t0;
      }
      if (valid_rows < kTileTok) {
        for (int q = lane; q < kTileTok * KC; q += 32) {
          const int row = q / KC, ch = q % KC;
          if (row >= valid_rows) {
            *reinterpret_cast<uint4*>(vs + kv_off<D>(row, ch)) = make_uint4(0, 0, 0, 0);
            if (valid_rows == 0)
              *reinterpret_cast<uint4*>(ks + kv_off<D>(row, ch)) = make_uint4(0, 0, 0, 0);
          }
        }
      }
    } else {
      cp_async_wait<STAGES - 1>();
    }
    __syncwarp();

    // S = Q K^T over 16 tokens (2 n-tiles of 8)
    float s[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[mt][nt][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t b0, b1, b2, b3;
      {
        const int row = (lane & 7) + ((lane >> 4) << 3);
        const int ch = 2 * kk + ((lane >> 3) & 1);
        ldmatrix_x4(smem_u32(ks + kv_off<D>(row, ch)), b0, b1, b2, b3);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t a[4];
        if constexpr (kQReg) {
#pragma unroll
          for (int e = 0; e < 4; ++e) a[e] = qa[mt][kk][e];
        } else {
          load_qfrag(mt, kk, a);
        }
        mma_16816<BF16>(s[mt][0], a, b0, b1);
        mma_16816<BF16>(s[mt][1], a, b2, b3);
      }
    }

    // online softmax (log2 domain); O is rescaled only when a row's max grew by > 2^8
    const bool need_mask = (t0 + kTileTok - 1) > lim_min;
    // fp16: P = p_hi + p_lo, both fp16, so the PV product sees P to about 2^-22
    // relative instead of one rounding's 2^-12 and the output matches the fp32
    // reference to within one fp16 rounding (the reference's own fp16 kernel
    // test asks for 1e-3 where outputs reach |2|, i.e. half an ulp). bf16 keeps a
    // single rounding: its output ulp (2^-8) dwarfs the P error, and the second
    // PV MMA measured 10% slower on the verify workload.
    constexpr bool kSplitP = !BF16;
    uint32_t pa[MT][4];
    uint32_t pl[kSplitP ? MT : 1][4];
    float alpha[MT][2];
    bool any_rescale = false;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float v[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float x = s[mt][nt][2 * hf + e] * p.scale_log2;
            if (need_mask) {
              const int tok = t0 + nt * 8 + 2 * t4 + e;
              if (tok > lim[mt][hf]) x = -INFINITY;
            }
            v[nt * 2 + e] = x;
          }
        float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        // keep a stale max until the row max grows by more than 2^8: O and l
        // share it, so the result is exact and p stays <= 256
        const float m_new = fmaxf(m_run[mt][hf], mx);
        const bool need = m_new > m_run[mt][hf] + 8.0f;
        alpha[mt][hf] = need ? ex2(m_run[mt][hf] - m_new) : 1.0f;
        any_rescale |= need;
        if (need) m_run[mt][hf] = m_new;
        const float m_use = m_run[mt][hf] == -INFINITY ? 0.f : m_run[mt][hf];
        float ps = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[j] = ex2(v[j] - m_use);
          ps += v[j];
        }
        l_run[mt][hf] = l_run[mt][hf] * alpha[mt][hf] + ps;
        // A fragment of P: a0/a1 = rows g/g+8, tokens 2t..2t+1; a2/a3 = tokens 8+2t..
        pa[mt][hf] = pack2<BF16>(v[0], v[1]);
        pa[mt][2 + hf] = pack2<BF16>(v[2], v[3]);
        if constexpr (kSplitP) {
          const float2 h01 = unpack2<BF16>(pa[mt][hf]);
          const float2 h23 = unpack2<BF16>(pa[mt][2 + hf]);
          pl[mt][hf] = pack2<BF16>(v[0] - h01.x, v[1] - h01.y);
          pl[mt][2 + hf] = pack2<BF16>(v[2] - h23.x, v[3] - h23.y);
        }
      }
    }
    if (__any_sync(0xffffffffu, any_rescale)) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt) {
          o_acc[mt][nt][0] *= alpha[mt][0];
          o_acc[mt][nt][1] *= alpha[mt][0];
          o_acc[mt][nt][2] *= alpha[mt][1];
          o_acc[mt][nt][3] *= alpha[mt][1];
        }
    }

    // O += P V
#pragma unroll
    for (int nd = 0; nd < D / 16; ++nd) {
      uint32_t b0, b1, b2, b3;
      {
        const int row = (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = 2 * nd + (lane >> 4);
        ldmatrix_x4_trans(smem_u32(vs + kv_off<D>(row, ch)), b0, b1, b2, b3);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma_16816<BF16>(o_acc[mt][2 * nd], pa[mt], b0, b1);
        mma_16816<BF16>(o_acc[mt][2 * nd + 1], pa[mt], b2, b3);
        if constexpr (kSplitP) {
          mma_16816<BF16>(o_acc[mt][2 * nd], pl[mt], b0, b1);
          mma_16816<BF16>(o_acc[mt][2 * nd + 1], pl[mt], b2, b3);
        }
      }
    }
    __syncwarp();
  }
  if constexpr (TMA) {
    if (*abort_flag && lane == 0) {
      // drain this warp's copies still in flight before the stages are reused
      for (int j = issued - 1; j >= 0 && j >= issued - STAGES; --j)
        mbar_wait_timeout(wbars + (j % STAGES), (j / STAGES) & 1, kWaitLimitNs);
    }
  } else {
    cp_async_wait<0>();
  }
  __syncthreads();  // pipeline ring is reused below

  // ---- merge the 4 warps in shared memory ----
  constexpr int OS = D + 4;                       // padded row: conflict-free float2 stores
  float* sm_o = reinterpret_cast<float*>(pipe);   // [W][RG][OS]
  float* sm_m = sm_o + kPagedWarps * RG * OS;     // [W][RG]
  float* sm_l = sm_m + kPagedWarps * RG;          // [W][RG]
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float l = l_run[mt][hf];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      const int r = mt * 16 + g + 8 * hf;
      if (t4 == 0) {
        sm_m[warp * RG + r] = m_run[mt][hf];
        sm_l[warp * RG + r] = l;
      }
#pragma unroll
      for (int nt = 0; nt < D / 8; ++nt) {
        float2 v2 = make_float2(o_acc[mt][nt][2 * hf], o_acc[mt][nt][2 * hf + 1]);
        *reinterpret_cast<float2*>(sm_o + (warp * RG + r) * OS + nt * 8 + 2 * t4) = v2;
      }
    }
  __syncthreads();

  using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const bool direct = (nsplit == 1);
  const int unit = (b * p.Hkv + kvh) * p.row_groups + rg;
  for (int idx = tid; idx < RG * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D;
    const int gr = row0 + r;
    if (gr >= R) continue;
    float mt_ = -INFINITY;
#pragma unroll
    for (int w = 0; w < kPagedWarps; ++w) mt_ = fmaxf(mt_, sm_m[w * RG + r]);
    const float mu = mt_ == -INFINITY ? 0.f : mt_;
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kPagedWarps; ++w) {
      const float wt = ex2(sm_m[w * RG + r] - mu);
      acc += wt * sm_o[(w * RG + r) * OS + d];
      l += wt * sm_l[w * RG + r];
    }
    if (direct) {
      float out;
      if (l > 0.f) out = acc / l;
      else out = (kv_len == 0) ? 0.f : __int_as_float(0x7fc00000);  // NaN: fully masked row
      const int gh = gr / p.M, m = gr % p.M;
      const int h = kvh * p.G + gh;
      elem_t* o = reinterpret_cast<elem_t*>(p.o);
      if constexpr (BF16) o[b * p.o_sb + h * p.o_sh + m * p.o_sm + d] = __float2bfloat16_rn(out);
      else o[b * p.o_sb + h * p.o_sh + m * p.o_sm + d] = __float2half_rn(out);
    } else {
      const int64_t base = (static_cast<int64_t>(unit) * p.max_splits + split) * RG;
      p.part_o[(base + r) * D + d] = l > 0.f ? acc / l : 0.f;
      if (d == 0) p.part_lse[base + r] = l > 0.f ? mu + __log2f(l) : -INFINITY;
    }
  }
}

// Log-sum-exp merge of split-KV partitions (sequences with >1 split only).
// One CTA per (sequence, kv head, row group) and slice of kMergeRows<D> rows,
// one thread per float4 column of a row: the CTA stages its rows' partition
// log-sum-exps in shared memory with all threads at once, then every thread
// walks the partitions with its loads unrolled, so the merge costs a few L2
// round trips however many partitions there are (a per-row serial walk over
// the log-sum-exps cost ~15 us at 17 partitions). CTAs whose rows are all
// padding (row >= G*M) return at once. Partitions past kMergeCap read their
// log-sum-exp from global memory.
constexpr int kMergeCap = 32;
constexpr int kMergeThreads = 128;

template <int D, int RG>
__host__ __device__ constexpr int merge_rows() {
  return (kMergeThreads / (D / 4)) < RG ? kMergeThreads / (D / 4) : RG;
}

template <int D, int RG, bool BF16, bool PAGED>
__global__ void __launch_bounds__(kMergeThreads) paged_merge_kernel(const PagedParams p) {
  constexpr int D4 = D / 4;
  constexpr int RPC = merge_rows<D, RG>();
  __shared__ float s_lse[RPC][kMergeCap];
  const int unit = blockIdx.x;
  const int r0 = blockIdx.y * RPC;  // first row (within the row group) of this CTA
  const int rg = unit % p.row_groups;
  const int kvh = (unit / p.row_groups) % p.Hkv;
  const int b = unit / (p.row_groups * p.Hkv);
  const int R = p.G * p.M;
  if (rg * RG + r0 >= R) return;
  int kv_len = PAGED ? p.kv_lens[b] : p.dense_n;
  if (kv_len < 0) kv_len = 0;
  if (PAGED && kv_len > p.max_blocks * p.block_size) kv_len = p.max_blocks * p.block_size;
  const int nsplit = kv_len > 0 ? (kv_len + p.split_tokens - 1) / p.split_tokens : 1;
  if (nsplit <= 1) return;
  const int64_t base = static_cast<int64_t>(unit) * p.max_splits * RG;
  const int ns_c = nsplit < kMergeCap ? nsplit : kMergeCap;
  for (int i = threadIdx.x; i < RPC * ns_c; i += kMergeThreads) {
    const int r = i / ns_c, s = i % ns_c;
    s_lse[r][s] = __ldg(p.part_lse + base + s * RG + r0 + r);
  }
  __syncthreads();
  const int lr = threadIdx.x / D4, c = threadIdx.x % D4;
  const int r = r0 + lr;
  if (lr >= RPC || r >= RG || rg * RG + r >= R) return;
  const float* lse_g = p.part_lse + base + r;  // partition s at lse_g[s * RG]
  float mx = -INFINITY;
  for (int s = 0; s < ns_c; ++s) mx = fmaxf(mx, s_lse[lr][s]);
  for (int s = ns_c; s < nsplit; ++s) mx = fmaxf(mx, __ldg(lse_g + s * RG));
  // weights, their sum and the weighted rows in partition order
  float sum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const float* po = p.part_o + (base + r) * D + c * 4;  // partition s at po[s * RG * D]
  auto add = [&](float lse, int s) {
    const float w = mx == -INFINITY ? 0.f : ex2(lse - mx);
    sum += w;
    const float4 v = __ldg(reinterpret_cast<const float4*>(po + static_cast<int64_t>(s) * RG * D));
    acc.x += w * v.x;
    acc.y += w * v.y;
    acc.z += w * v.z;
    acc.w += w * v.w;
  };
#pragma unroll 8
  for (int s = 0; s < ns_c; ++s) add(s_lse[lr][s], s);
  for (int s = ns_c; s < nsplit; ++s) add(__ldg(lse_g + s * RG), s);
  const float inv = sum > 0.f ? 1.0f / sum : __int_as_float(0x7fc00000);
  const int gr = rg * RG + r;
  const int gh = gr / p.M, m = gr % p.M;
  const int h = kvh * p.G + gh;
  using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  elem_t* dst = reinterpret_cast<elem_t*>(p.o) + b * p.o_sb + h * p.o_sh + m * p.o_sm + c * 4;
  if constexpr (BF16) {
    dst[0] = __float2bfloat16_rn(acc.x * inv);
    dst[1] = __float2bfloat16_rn(acc.y * inv);
    dst[2] = __float2bfloat16_rn(acc.z * inv);
    dst[3] = __float2bfloat16_rn(acc.w * inv);
  } else {
    dst[0] = __float2half_rn(acc.x * inv);
    dst[1] = __float2half_rn(acc.y * inv);
    dst[2] = __float2half_rn(acc.z * inv);
    dst[3] = __float2half_rn(acc.w * inv);
  }
}

// ------------------------------------------------------------------ host
static int pick_mt(int R, int d) {
  // rows per CTA = 16 * MT; MT * d <= 256 keeps the O accumulator in registers
  if (R <= 16 || d >= 256) return 1;
  if (R <= 32 || d == 128) return 2;
  return 4;
}

static int auto_split_tokens(int64_t units, int max_len, int d) {
  // Lengths are only known on the device, so partitions are sized from the
  // table width: about 7 partitions per SM over the batch if every sequence
  // were full (14 once there are more than two (sequence, kv head, row group)
  // units per SM), never below 512 tokens at d <= 64 / 2048 at d >= 128, at
  // most 4096. Measured on B200 (decode d=64 and verify d=128, full batch and
  // one rank's head slice at 2, 4 and 8 GPUs): shorter partitions lose more to
  // each CTA's pipeline start and to the merge than they gain in parallelism.
  const int sms = num_sms();
  const int per_sm = units > 2 * sms ? 14 : 7;
  int64_t want = (static_cast<int64_t>(max_len) * units) / (static_cast<int64_t>(sms) * per_sm);
  const int lo = (d >= 128) ? 2048 : 512;
  if (want < lo) want = lo;
  if (want > 4096) want = 4096;
  want = ((want + 63) / 64) * 64;
  return static_cast<int>(want);
}

struct MmaPlan {
  int mt, rg_rows, row_groups, split_tokens, max_splits;
  size_t part_o_bytes, part_lse_bytes;
  size_t workspace() const {
    return max_splits > 1 ? part_o_bytes + part_lse_bytes + 256 : 0;
  }
};

static MmaPlan make_plan(int B, int Hq, int Hkv, int M, int d, int max_len, int split_tokens) {
  MmaPlan pl{};
  const int G = Hq / Hkv;
  const int R = G * M;
  pl.mt = pick_mt(R, d);
  pl.rg_rows = 16 * pl.mt;
  pl.row_groups = (R + pl.rg_rows - 1) / pl.rg_rows;
  const int64_t units = static_cast<int64_t>(B) * Hkv * pl.row_groups;
  pl.split_tokens = split_tokens > 0 ? split_tokens : auto_split_tokens(units, max_len, d);
  pl.max_splits = max_len > 0 ? (max_len + pl.split_tokens - 1) / pl.split_tokens : 1;
  if (pl.max_splits < 1) pl.max_splits = 1;
  pl.part_o_bytes = static_cast<size_t>(units) * pl.max_splits * pl.rg_rows * d * sizeof(float);
  pl.part_lse_bytes = static_cast<size_t>(units) * pl.max_splits * pl.rg_rows * sizeof(float);
  pl.part_o_bytes = (pl.part_o_bytes + 255) & ~size_t(255);
  return pl;
}

static bool mma_head_dim_ok(int d) { return d == 16 || d == 32 || d == 64 || d == 128 || d == 256; }

// 4-D map whose box is one 16-token, min(d, 64)-column K or V slice, swizzled
// as kv_off<> expects. dims / strides innermost first, strides in bytes.
static bool make_kv_map(CUtensorMap* map, const void* base, int d, const cuuint64_t* dims,
                        const cuuint64_t* strides, const cuuint32_t* box, bool bf16) {
  PFN_encodeTiled_t enc = tensor_map_encoder();
  if (!enc) return false;
  const int rowb = d * 2 < 128 ? d * 2 : 128;
  const CUtensorMapSwizzle sw = rowb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : rowb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                             : CU_TENSOR_MAP_SWIZZLE_32B;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
             const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, int MT, bool BF16, bool PAGED, bool TMA>
static int launch_mma_t(const CUtensorMap& mk, const CUtensorMap& mv, const PagedParams& prm,
                        cudaStream_t st) {
  constexpr int smem = paged_smem_bytes<D, MT>();
  auto kern = paged_attn_kernel<D, MT, BF16, PAGED, TMA>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(prm.max_splits, prm.Hkv * prm.row_groups, prm.B);
  kern<<<grid, kPagedWarps * 32, smem, st>>>(mk, mv, prm);
  CIE_CHECK_LAUNCH("paged_attn_kernel");
  if (prm.max_splits > 1) {
    constexpr int RG = 16 * MT;
    const dim3 mgrid(prm.B * prm.Hkv * prm.row_groups,
                     (RG + merge_rows<D, RG>() - 1) / merge_rows<D, RG>());
    paged_merge_kernel<D, RG, BF16, PAGED><<<mgrid, kMergeThreads, 0, st>>>(prm);
    CIE_CHECK_LAUNCH("paged_merge_kernel");
  }
  return CIE_OK;
}

template <int D, int MT, bool BF16, bool PAGED>
static int launch_mma(const PagedParams& prm, cudaStream_t st) {
  // TMA feeds need a 16-token tile inside one block (paged) and 16-byte
  // aligned rows; otherwise the cp.async path serves the call.
  using C = PagedCfg<D>;
  CUtensorMap mk{}, mv{};
  bool tma = false;
  const bool bf16 = BF16;
  if constexpr (PAGED) {
    if (prm.block_size % kTileTok == 0) {
      const cuuint64_t tokens = static_cast<cuuint64_t>(prm.num_blocks) * prm.block_size;
      const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)prm.Hkv, tokens, 1};
      const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)prm.Hkv * D * 2,
                                     tokens * prm.Hkv * D * 2};
      const cuuint32_t box[4] = {(cuuint32_t)(C::ROWB / 2), 1, kTileTok, 1};
      tma = make_kv_map(&mk, prm.k_pool, D, dims, strides, box, bf16) &&
            make_kv_map(&mv, prm.v_pool, D, dims, strides, box, bf16);
    }
  } else {
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)(prm.dense_n > 0 ? prm.dense_n : 1),
                                (cuuint64_t)prm.Hkv, (cuuint64_t)prm.B};
    const cuuint64_t ks[3] = {(cuuint64_t)prm.k_sn * 2, (cuuint64_t)prm.k_sh * 2,
                              (cuuint64_t)prm.k_sb * 2};
    const cuuint64_t vs[3] = {(cuuint64_t)prm.v_sn * 2, (cuuint64_t)prm.v_sh * 2,
                              (cuuint64_t)prm.v_sb * 2};
    const cuuint32_t box[4] = {(cuuint32_t)(C::ROWB / 2), kTileTok, 1, 1};
    const bool ok_strides = prm.k_sn > 0 && prm.k_sh > 0 && prm.k_sb > 0 && prm.v_sn > 0 &&
                            prm.v_sh > 0 && prm.v_sb > 0;
    tma = ok_strides && make_kv_map(&mk, prm.k_pool, D, dims, ks, box, bf16) &&
          make_kv_map(&mv, prm.v_pool, D, dims, vs, box, bf16);
  }
  if (tma) return launch_mma_t<D, MT, BF16, PAGED, true>(mk, mv, prm, st);
  return launch_mma_t<D, MT, BF16, PAGED, false>(mk, mv, prm, st);
}

template <int D, bool BF16, bool PAGED>
static int dispatch_mt(const PagedParams& prm, int mt, cudaStream_t st) {
  if constexpr (D >= 256) {
    return launch_mma<D, 1, BF16, PAGED>(prm, st);
  } else if constexpr (D == 128) {
    return mt == 1 ? launch_mma<D, 1, BF16, PAGED>(prm, st)
                   : launch_mma<D, 2, BF16, PAGED>(prm, st);
  } else {
    switch (mt) {
      case 1: return launch_mma<D, 1, BF16, PAGED>(prm, st);
      case 2: return launch_mma<D, 2, BF16, PAGED>(prm, st);
      default: return launch_mma<D, 4, BF16, PAGED>(prm, st);
    }
  }
}

template <bool PAGED>
static int dispatch_d(const PagedParams& prm, int d, int mt, bool bf16, cudaStream_t st) {
  switch (d) {
    case 16: return bf16 ? dispatch_mt<16, true, PAGED>(prm, mt, st)
                         : dispatch_mt<16, false, PAGED>(prm, mt, st);
    case 32: return bf16 ? dispatch_mt<32, true, PAGED>(prm, mt, st)
                         : dispatch_mt<32, false, PAGED>(prm, mt, st);
    case 64: return bf16 ? dispatch_mt<64, true, PAGED>(prm, mt, st)
                         : dispatch_mt<64, false, PAGED>(prm, mt, st);
    case 128: return bf16 ? dispatch_mt<128, true, PAGED>(prm, mt, st)
                          : dispatch_mt<128, false, PAGED>(prm, mt, st);
    case 256: return bf16 ? dispatch_mt<256, true, PAGED>(prm, mt, st)
                          : dispatch_mt<256, false, PAGED>(prm, mt, st);
    default:
      set_error("attention: head_dim %d unsupported", d);
      return CIE_ERR_UNSUPPORTED;
  }
}

static void fill_common(PagedParams& prm, const MmaPlan& pl, const void* q, void* o, int B, int Hq,
                        int Hkv, int M, const int64_t* qs, const int64_t* os, float scale,
                        int causal, const float* cos, const float* sin, int max_pos,
                        void* workspace) {
  prm.q = q;
  prm.o = o;
  if (pl.max_splits > 1) {
    uintptr_t w = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255);
    prm.part_o = reinterpret_cast<float*>(w);
    prm.part_lse = reinterpret_cast<float*>(w + pl.part_o_bytes);
  }
  prm.cos = cos;
  prm.sin = sin;
  prm.rope_max_pos = max_pos;
  prm.B = B;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.M = M;
  prm.G = Hq / Hkv;
  prm.q_sb = qs[0];
  prm.q_sh = qs[1];
  prm.q_sm = qs[2];
  prm.o_sb = os[0];
  prm.o_sh = os[1];
  prm.o_sm = os[2];
  prm.split_tokens = pl.split_tokens;
  prm.max_splits = pl.max_splits;
  prm.row_groups = pl.row_groups;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal ? 1 : 0;
}

// Dense-K/V variant of the same kernel, used by cie_prefill_attn for short
// query blocks and for head dims the tcgen05 kernel does not cover.
size_t dense_mma_workspace(int B, int Hq, int Hkv, int M, int N, int d) {
  return make_plan(B, Hq, Hkv, M, d, N, 0).workspace();
}

int dense_mma_attn(const void* q, const void* k, const void* v, void* o, int B, int Hq, int Hkv,
                   int M, int N, int d, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                   const int64_t* os, float scale, int causal, bool bf16, const float* cos,
                   const float* sin, int max_pos, int q_pos0, void* workspace,
                   size_t workspace_bytes, cudaStream_t st) {
  if (!mma_head_dim_ok(d)) {
    set_error("attention: head_dim %d unsupported", d);
    return CIE_ERR_UNSUPPORTED;
  }
  MmaPlan pl = make_plan(B, Hq, Hkv, M, d, N, 0);
  if (pl.workspace() > 0 && (workspace == nullptr || workspace_bytes < pl.workspace())) {
    set_error("attention: workspace of %zu bytes required, got %zu", pl.workspace(),
              workspace_bytes);
    return CIE_ERR_WORKSPACE;
  }
  if (B > 65535 || static_cast<int64_t>(Hkv) * pl.row_groups > 65535) {
    set_error("attention: grid too large (B=%d, Hkv*row_groups=%d)", B, Hkv * pl.row_groups);
    return CIE_ERR_UNSUPPORTED;
  }
  PagedParams prm{};
  fill_common(prm, pl, q, o, B, Hq, Hkv, M, qs, os, scale, causal, cos, sin, max_pos, workspace);
  prm.k_pool = k;
  prm.v_pool = v;
  prm.dense_n = N;
  prm.k_sb = ks[0];
  prm.k_sh = ks[1];
  prm.k_sn = ks[2];
  prm.v_sb = vs[0];
  prm.v_sh = vs[1];
  prm.v_sn = vs[2];
  prm.rope_q_pos0 = q_pos0;
  return dispatch_d<false>(prm, d, pl.mt, bf16, st);
}

// Defined in prefill_attn.cu: the tcgen05 kernel reading the paged pools,
// for query blocks of more than 64 rows per kv head (chunked prefill).
bool paged_uses_tcgen05(int Hq, int Hkv, int M, int d, int block_size);
int paged_prefill_tcgen05(const void* q, const void* k_pool, const void* v_pool,
                          const int32_t* block_tables, const int32_t* kv_lens, void* o, int B,
                          int Hq, int Hkv, int M, int d, int num_blocks, int block_size,
                          int max_blocks, const int64_t* q_strides, const int64_t* o_strides,
                          float scale, int causal, bool bf16, const float* rope_cos,
                          const float* rope_sin, int rope_max_pos, cudaStream_t st);

}  // namespace cie

using namespace cie;

extern "C" size_t cie_paged_attn_workspace(int B, int Hq, int Hkv, int M, int d,
                                           int block_size, int max_blocks, int split_tokens) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || M <= 0 || Hq % Hkv != 0 || !mma_head_dim_ok(d) ||
      block_size <= 0 || max_blocks < 0)
    return 0;
  if (paged_uses_tcgen05(Hq, Hkv, M, d, block_size)) return 0;
  return make_plan(B, Hq, Hkv, M, d, max_blocks * block_size, split_tokens).workspace();
}

extern "C" int cie_paged_attn(const void* q, const void* k_pool, const void* v_pool,
                              const int32_t* block_tables, const int32_t* kv_lens, void* o, int B,
                              int Hq, int Hkv, int M, int d, int num_blocks, int block_size,
                              int max_blocks, const int64_t* q_strides, const int64_t* o_strides,
                              float scale, int causal, int dtype, const float* rope_cos,
                              const float* rope_sin, int rope_max_pos, int split_tokens,
                              void* workspace, size_t workspace_bytes, void* stream) {
  CIE_CHECK_ARG(q && k_pool && v_pool && block_tables && kv_lens && o,
                "cie_paged_attn: null tensor pointer");
  CIE_CHECK_ARG(B >= 0 && Hq > 0 && Hkv > 0 && M >= 0, "cie_paged_attn: bad shape");
  CIE_CHECK_ARG(Hq % Hkv == 0, "cie_paged_attn: Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
  CIE_CHECK_ARG(dtype == CIE_DTYPE_BF16 || dtype == CIE_DTYPE_FP16, "cie_paged_attn: bad dtype %d",
                dtype);
  CIE_CHECK_ARG(num_blocks > 0 && block_size > 0 && max_blocks > 0,
                "cie_paged_attn: bad pool geometry");
  CIE_CHECK_ARG(q_strides && o_strides, "cie_paged_attn: null strides");
  CIE_CHECK_ARG(aligned16(q) && aligned16(k_pool) && aligned16(v_pool),
                "cie_paged_attn: q/k_pool/v_pool must be 16-byte aligned");
  CIE_CHECK_ARG(q_strides[0] % 8 == 0 && q_strides[1] % 8 == 0 && q_strides[2] % 8 == 0,
                "cie_paged_attn: q strides must be multiples of 8 elements");
  CIE_CHECK_ARG(split_tokens == 0 || (split_tokens > 0 && split_tokens % 16 == 0),
                "cie_paged_attn: split_tokens must be 0 or a positive multiple of 16");
  CIE_CHECK_ARG((rope_cos == nullptr) == (rope_sin == nullptr),
                "cie_paged_attn: rope_cos and rope_sin must both be given or both NULL");
  CIE_CHECK_ARG(rope_cos == nullptr || rope_max_pos > 0, "cie_paged_attn: rope_max_pos <= 0");
  if (!mma_head_dim_ok(d)) {
    set_error("cie_paged_attn: head_dim %d unsupported (16, 32, 64, 128 or 256)", d);
    return CIE_ERR_UNSUPPORTED;
  }
  if (B == 0 || M == 0) return CIE_OK;
  if (paged_uses_tcgen05(Hq, Hkv, M, d, block_size)) {
    CIE_CHECK_ARG(B <= 65535, "cie_paged_attn: B must be <= 65535");
    return paged_prefill_tcgen05(q, k_pool, v_pool, block_tables, kv_lens, o, B, Hq, Hkv, M, d,
                                 num_blocks, block_size, max_blocks, q_strides, o_strides, scale,
                                 causal, dtype == CIE_DTYPE_BF16, rope_cos, rope_sin,
                                 rope_max_pos, reinterpret_cast<cudaStream_t>(stream));
  }
  MmaPlan pl = make_plan(B, Hq, Hkv, M, d, max_blocks * block_size, split_tokens);
  if (pl.workspace() > 0 && (workspace == nullptr || workspace_bytes < pl.workspace())) {
    set_error("cie_paged_attn: workspace of %zu bytes required, got %zu", pl.workspace(),
              workspace_bytes);
    return CIE_ERR_WORKSPACE;
  }
  if (B > 65535 || static_cast<int64_t>(Hkv) * pl.row_groups > 65535) {
    set_error("cie_paged_attn: grid too large (B=%d, Hkv*row_groups=%d)", B,
              Hkv * pl.row_groups);
    return CIE_ERR_UNSUPPORTED;
  }
  PagedParams prm{};
  fill_common(prm, pl, q, o, B, Hq, Hkv, M, q_strides, o_strides, scale, causal, rope_cos,
              rope_sin, rope_max_pos, workspace);
  prm.k_pool = k_pool;
  prm.v_pool = v_pool;
  prm.block_tables = block_tables;
  prm.kv_lens = kv_lens;
  prm.num_blocks = num_blocks;
  prm.block_size = block_size;
  prm.max_blocks = max_blocks;
  prm.bs_log2 = (block_size & (block_size - 1)) == 0 ? __builtin_ctz(block_size) : -1;
  return dispatch_d<true>(prm, d, pl.mt, dtype == CIE_DTYPE_BF16,
                          reinterpret_cast<cudaStream_t>(stream));
}
