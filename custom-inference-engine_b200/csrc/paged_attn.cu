// paged_attn.cu — paged-KV attention for single-token decode and speculative
// verify on sm_100a.
//
// What it computes (per sequence b, query head h, query row i < M):
//   out[b,h,i,:] = softmax_j(q_rot[b,h,i,:] . K[b,kvh,j,:] * scale) V[b,kvh,j,:]
// over keys j < kv_len[b] (and j <= kv_len[b] - M + i when causal), where
// K/V rows are fetched through the block table exactly as
// PagedKVCache.gather does (engine/cache/kv_cache.py:141-165) and the
// attention matches kernels/ref/flash_attention_ref.py:8-56 with GQA
// (kv head = h / (Hq / Hkv)).
//
// How: one CTA per (split-KV partition, kv head, row group, sequence).
// The query rows of all heads sharing a kv head (G = Hq/Hkv heads x M rows)
// form the M side of m16n8k16 tensor-core MMAs, so K/V bytes are read from
// HBM exactly once per kv head. Each of the 4 warps streams its own 16-token
// K/V tiles with 16-byte cp.async (block-table lookup per row) through a
// private multi-stage shared-memory ring, runs an online softmax with quad
// shuffles, and the warps are merged in shared memory at the end. Partitions
// of one sequence are merged by a log-sum-exp kernel.
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
  int64_t q_sb, q_sh, q_sm;
  int64_t o_sb, o_sh, o_sm;
  int split_tokens;
  int max_splits;
  int row_groups;  // ceil(G*M / RG)
  float scale_log2;
  int causal;
  // dense mode (K/V as (B, Hkv, N, d) tensors instead of paged pools)
  int dense_n;                       // N (keys per sequence)
  int64_t k_sb, k_sh, k_sn;          // element strides of K
  int64_t v_sb, v_sh, v_sn;          // element strides of V
  int rope_q_pos0;                   // dense mode: q row i rotated at rope_q_pos0 + i
};

constexpr int kPagedWarps = 4;
constexpr int kTileTok = 16;

template <int D>
struct PagedCfg {
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
  static constexpr int kStages = (D <= 64) ? 4 : (D == 128 ? 3 : 2);
  static constexpr int kTileBytes = kTileTok * D * 2;           // K or V tile
  static constexpr int kStageBytes = 2 * kTileBytes;            // K + V
  static constexpr int kWarpBytes = kStages * kStageBytes;
  static constexpr int kPipeBytes = kPagedWarps * kWarpBytes;
};

// 16-byte-chunk XOR swizzle of a [rows][KC chunks] tile so that the 8 rows
// an ldmatrix phase reads land in 8 distinct 16-byte bank groups.
template <int KC>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  if constexpr (KC >= 8) return static_cast<uint32_t>(chunk ^ (row & 7));
  else return static_cast<uint32_t>(chunk ^ ((row / (8 / KC)) & (KC - 1)));
}

template <int D, int MT>
__host__ __device__ constexpr int paged_smem_bytes() {
  // pipeline ring, reused for the cross-warp merge, plus the rotated Q tile
  constexpr int RG = 16 * MT;
  constexpr int pipe = PagedCfg<D>::kPipeBytes;
  constexpr int merge = kPagedWarps * RG * (D + 2) * 4;
  return (pipe > merge ? pipe : merge) + RG * D * 2;
}

template <int D, int MT, bool BF16, bool PAGED>
__global__ void __launch_bounds__(kPagedWarps * 32)
    paged_attn_kernel(const PagedParams p) {
  using Cfg = PagedCfg<D>;
  constexpr int RG = 16 * MT;
  constexpr int KC = Cfg::kChunks;
  constexpr int STAGES = Cfg::kStages;

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* pipe = smem;
  const int pipe_or_merge = paged_smem_bytes<D, MT>() - RG * D * 2;
  uint8_t* qs = smem + pipe_or_merge;

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
    if (split == 0 && blockIdx.y == 0 && threadIdx.x == 0) raise_status(CIE_DEV_BAD_BLOCK_ID);
    kv_len = p.max_blocks * p.block_size;
  }
  const int nsplit = kv_len > 0 ? (kv_len + p.split_tokens - 1) / p.split_tokens : 1;
  if (split >= nsplit) return;
  const int R = p.G * p.M;            // rows of this kv-head group
  const int row0 = rg * RG;           // first row of this CTA
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

  // ---- rotated Q tile -> shared memory (bf16/fp16, 16B-chunk swizzle) ----
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
        uint4 x1 = *reinterpret_cast<const uint4*>(src + pc * 8);
        uint4 x2 = *reinterpret_cast<const uint4*>(src + HALF + pc * 8);
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
            const float r10 = __fsub_rn(__fmul_rn(u1.x, c0), __fmul_rn(u2.x, s0));
            const float r11 = __fsub_rn(__fmul_rn(u1.y, c1), __fmul_rn(u2.y, s1));
            const float r20 = __fadd_rn(__fmul_rn(u1.x, s0), __fmul_rn(u2.x, c0));
            const float r21 = __fadd_rn(__fmul_rn(u1.y, s1), __fmul_rn(u2.y, c1));
            lo_w[e] = pack2<BF16>(r10, r11);
            hi_w[e] = pack2<BF16>(r20, r21);
          }
        } else {
          lo = x1;
          hi = x2;
        }
      }
      const int c_lo = pc, c_hi = HALF / 8 + pc;
      *reinterpret_cast<uint4*>(qs + r * (D * 2) + swz<D / 8>(r, c_lo) * 16) = lo;
      *reinterpret_cast<uint4*>(qs + r * (D * 2) + swz<D / 8>(r, c_hi) * 16) = hi;
    }
  }
  __syncthreads();

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
  const int32_t* table = PAGED ? p.block_tables + static_cast<int64_t>(b) * p.max_blocks : nullptr;
  const uint8_t* kpool = reinterpret_cast<const uint8_t*>(p.k_pool);
  const uint8_t* vpool = reinterpret_cast<const uint8_t*>(p.v_pool);
  const int64_t tok_stride = static_cast<int64_t>(p.Hkv) * D * 2;  // bytes per token row
  const int64_t head_off = static_cast<int64_t>(kvh) * D * 2;

  auto issue_tile = [&](int tile, int stage) {
    uint8_t* ks = wpipe + stage * Cfg::kStageBytes;
    uint8_t* vs = ks + Cfg::kTileBytes;
    const int t0 = tok_begin + tile * kTileTok;
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
            koff = (static_cast<int64_t>(blk) * p.block_size + (tok % p.block_size)) * tok_stride +
                   head_off + ch * 16;
            voff = koff;
          }
        } else {
          koff = (b * p.k_sb + kvh * p.k_sh + tok * p.k_sn) * 2 + ch * 16;
          voff = (b * p.v_sb + kvh * p.v_sh + tok * p.v_sn) * 2 + ch * 16;
        }
      }
      const uint32_t so = row * (D * 2) + swz<KC>(row, ch) * 16;
      cp_async_16(ks + so, kpool + koff, valid);
      cp_async_16(vs + so, vpool + voff, valid);
    }
  };

  // Q A-fragments (held in registers when small).
  constexpr bool kQReg = (MT * D) <= 128;
  uint32_t qa[kQReg ? MT : 1][kQReg ? D / 16 : 1][4];
  auto load_qfrag = [&](int mt, int ks, uint32_t (&a)[4]) {
    const int row = mt * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
    const int ch = 2 * ks + (lane >> 4);
    ldmatrix_x4(smem_u32(qs + row * (D * 2) + swz<KC>(row, ch) * 16), a[0], a[1], a[2], a[3]);
  };
  if constexpr (kQReg) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) load_qfrag(mt, ks, qa[mt][ks]);
  }

  // Rows owned by this thread: (mt, half) -> global row / query index / key limit
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

  const int my_tiles = n_tiles > warp ? (n_tiles - warp + kPagedWarps - 1) / kPagedWarps : 0;
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < my_tiles) issue_tile(warp + kPagedWarps * s, s);
    cp_async_commit();
  }

  for (int it = 0; it < my_tiles; ++it) {
    {
      const int nx = it + STAGES - 1;
      if (nx < my_tiles) issue_tile(warp + kPagedWarps * nx, nx % STAGES);
      cp_async_commit();
    }
    cp_async_wait<STAGES - 1>();
    __syncwarp();

    const uint8_t* ks = wpipe + (it % STAGES) * Cfg::kStageBytes;
    const uint8_t* vs = ks + Cfg::kTileBytes;
    const int t0 = tok_begin + (warp + kPagedWarps * it) * kTileTok;

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
        ldmatrix_x4(smem_u32(ks + row * (D * 2) + swz<KC>(row, ch) * 16), b0, b1, b2, b3);
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

    // online softmax (log2 domain)
    const bool need_mask = (t0 + kTileTok - 1) > lim_min;
    uint32_t pa[MT][4];
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
        const float m_new = fmaxf(m_run[mt][hf], mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = ex2(m_run[mt][hf] - m_use);
        m_run[mt][hf] = m_new;
        float ps = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[j] = ex2(v[j] - m_use);
          ps += v[j];
        }
        l_run[mt][hf] = l_run[mt][hf] * alpha + ps;
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt) {
          o_acc[mt][nt][2 * hf] *= alpha;
          o_acc[mt][nt][2 * hf + 1] *= alpha;
        }
        // A fragment of P: a0/a1 = rows g/g+8, tokens 2t..2t+1; a2/a3 = tokens 8+2t..
        pa[mt][hf] = pack2<BF16>(v[0], v[1]);
        pa[mt][2 + hf] = pack2<BF16>(v[2], v[3]);
      }
    }

    // O += P V
#pragma unroll
    for (int nd = 0; nd < D / 16; ++nd) {
      uint32_t b0, b1, b2, b3;
      {
        const int row = (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = 2 * nd + (lane >> 4);
        ldmatrix_x4_trans(smem_u32(vs + row * (D * 2) + swz<KC>(row, ch) * 16), b0, b1, b2, b3);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma_16816<BF16>(o_acc[mt][2 * nd], pa[mt], b0, b1);
        mma_16816<BF16>(o_acc[mt][2 * nd + 1], pa[mt], b2, b3);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  __syncthreads();  // pipeline ring is reused below

  // ---- merge the 4 warps in shared memory ----
  float* sm_o = reinterpret_cast<float*>(pipe);                   // [W][RG][D]
  float* sm_m = sm_o + kPagedWarps * RG * D;                      // [W][RG]
  float* sm_l = sm_m + kPagedWarps * RG;                          // [W][RG]
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
        *reinterpret_cast<float2*>(sm_o + (warp * RG + r) * D + nt * 8 + 2 * t4) = v2;
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
      acc += wt * sm_o[(w * RG + r) * D + d];
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

// Log-sum-exp merge of split-KV partitions (only sequences with >1 split).
template <int D, int RG, bool BF16, bool PAGED>
__global__ void __launch_bounds__(128) paged_merge_kernel(const PagedParams p) {
  const int kvh = blockIdx.x / p.row_groups;
  const int rg = blockIdx.x % p.row_groups;
  const int b = blockIdx.y;
  int kv_len = PAGED ? p.kv_lens[b] : p.dense_n;
  if (kv_len < 0) kv_len = 0;
  if (PAGED && kv_len > p.max_blocks * p.block_size) kv_len = p.max_blocks * p.block_size;
  const int nsplit = kv_len > 0 ? (kv_len + p.split_tokens - 1) / p.split_tokens : 1;
  if (nsplit <= 1) return;
  const int R = p.G * p.M;
  const int unit = (b * p.Hkv + kvh) * p.row_groups + rg;
  const int64_t base = static_cast<int64_t>(unit) * p.max_splits * RG;
  using elem_t = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  elem_t* o = reinterpret_cast<elem_t*>(p.o);
  for (int idx = threadIdx.x; idx < RG * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D;
    const int gr = rg * RG + r;
    if (gr >= R) continue;
    float mx = -INFINITY;
    for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, p.part_lse[base + s * RG + r]);
    float out;
    if (mx == -INFINITY) {
      out = __int_as_float(0x7fc00000);
    } else {
      float acc = 0.f, wsum = 0.f;
      for (int s = 0; s < nsplit; ++s) {
        const float w = ex2(p.part_lse[base + s * RG + r] - mx);
        wsum += w;
        acc += w * p.part_o[(base + s * RG + r) * D + d];
      }
      out = acc / wsum;
    }
    const int gh = gr / p.M, m = gr % p.M;
    const int h = kvh * p.G + gh;
    if constexpr (BF16) o[b * p.o_sb + h * p.o_sh + m * p.o_sm + d] = __float2bfloat16_rn(out);
    else o[b * p.o_sb + h * p.o_sh + m * p.o_sm + d] = __float2half_rn(out);
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
  // aim for ~8 partitions of work per SM over the whole batch, each at least
  // 256 tokens (512 for d >= 128), at most 4096, a multiple of 64 (one
  // 16-token tile per warp)
  const int sms = num_sms();
  int64_t want = (static_cast<int64_t>(max_len) * units) / (static_cast<int64_t>(sms) * 8);
  const int lo = (d >= 128) ? 512 : 256;
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

template <int D, int MT, bool BF16, bool PAGED>
static int launch_mma(const PagedParams& prm, cudaStream_t st) {
  constexpr int smem = paged_smem_bytes<D, MT>();
  auto kern = paged_attn_kernel<D, MT, BF16, PAGED>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(prm.max_splits, prm.Hkv * prm.row_groups, prm.B);
  kern<<<grid, kPagedWarps * 32, smem, st>>>(prm);
  CIE_CHECK_LAUNCH("paged_attn_kernel");
  if (prm.max_splits > 1) {
    dim3 mg(prm.Hkv * prm.row_groups, prm.B);
    paged_merge_kernel<D, 16 * MT, BF16, PAGED><<<mg, 128, 0, st>>>(prm);
    CIE_CHECK_LAUNCH("paged_merge_kernel");
  }
  return CIE_OK;
}

template <int D, bool BF16, bool PAGED>
static int dispatch_mt(const PagedParams& prm, int mt, cudaStream_t st) {
  if constexpr (D >= 256) {
    return launch_mma<D, 1, BF16, PAGED>(prm, st);
  } else if constexpr (D == 128) {
    return mt == 1 ? launch_mma<D, 1, BF16, PAGED>(prm, st) : launch_mma<D, 2, BF16, PAGED>(prm, st);
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
    case 16: return bf16 ? dispatch_mt<16, true, PAGED>(prm, mt, st) : dispatch_mt<16, false, PAGED>(prm, mt, st);
    case 32: return bf16 ? dispatch_mt<32, true, PAGED>(prm, mt, st) : dispatch_mt<32, false, PAGED>(prm, mt, st);
    case 64: return bf16 ? dispatch_mt<64, true, PAGED>(prm, mt, st) : dispatch_mt<64, false, PAGED>(prm, mt, st);
    case 128: return bf16 ? dispatch_mt<128, true, PAGED>(prm, mt, st) : dispatch_mt<128, false, PAGED>(prm, mt, st);
    case 256: return bf16 ? dispatch_mt<256, true, PAGED>(prm, mt, st) : dispatch_mt<256, false, PAGED>(prm, mt, st);
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

// Dense-K/V variant of the same kernel, used by cie_prefill_attn for head
// dims the tcgen05 kernel does not cover (16, 32, 256).
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

}  // namespace cie

using namespace cie;

extern "C" size_t cie_paged_attn_workspace(int B, int Hq, int Hkv, int M, int d,
                                           int block_size, int max_blocks, int split_tokens) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || M <= 0 || Hq % Hkv != 0 || !mma_head_dim_ok(d) ||
      block_size <= 0 || max_blocks < 0)
    return 0;
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
  MmaPlan pl = make_plan(B, Hq, Hkv, M, d, max_blocks * block_size, split_tokens);
  if (pl.workspace() > 0 && (workspace == nullptr || workspace_bytes < pl.workspace())) {
    set_error("cie_paged_attn: workspace of %zu bytes required, got %zu", pl.workspace(),
              workspace_bytes);
    return CIE_ERR_WORKSPACE;
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
  return dispatch_d<true>(prm, d, pl.mt, dtype == CIE_DTYPE_BF16,
                          reinterpret_cast<cudaStream_t>(stream));
}
