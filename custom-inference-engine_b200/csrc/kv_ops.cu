// kv_ops.cu — the byte-moving kernels around the attention hot path:
//   * gather_kv   bit-exact dense gather of the paged history
//                 (PagedKVCache.gather, engine/cache/kv_cache.py:141-165)
//   * rope        half-split RoPE of a (B, H, L, d) tensor
//                 (apply_rotary_ref, kernels/ref/rope_apply_ref.py:22-53)
//   * rope_append RoPE of new K rows fused with the scatter of K and V into
//                 the paged pools (PagedKVCache.append, kv_cache.py:102-139,
//                 after rope.apply at engine/model/block.py:53-54)
//   * copy_blocks whole-block copies inside a pool (PagedKVCache.fork,
//                 kv_cache.py:169-185)
// All four are HBM-bound: each thread moves 16-byte vectors, consecutive
// threads touch consecutive 16-byte chunks of one head row, and grids are
// sized as a multiple of the SM count.
#include <cuda_runtime.h>

#include <cstdint>

#include "cie_common.cuh"
#include "sm100_ptx.cuh"

namespace cie {

// ------------------------------------------------------------------ gather
__global__ void __launch_bounds__(256) gather_kv_kernel(const uint8_t* __restrict__ pool,
                                                        const int32_t* __restrict__ tables,
                                                        const int32_t* __restrict__ kv_lens,
                                                        uint8_t* __restrict__ out, int out_len,
                                                        int row_bytes, int num_blocks,
                                                        int block_size, int max_blocks) {
  // grid.y = sequence; each thread copies 16-byte chunks of token rows (all
  // heads of a token are contiguous in both the pool and the output)
  const int b = blockIdx.y;
  const int chunks = row_bytes / 16;
  const int len = min(kv_lens[b], out_len);
  const int total = len * chunks;
  const int32_t* table = tables + static_cast<int64_t>(b) * max_blocks;
  uint8_t* ob = out + static_cast<int64_t>(b) * out_len * row_bytes;
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < total; w += gridDim.x * blockDim.x) {
    const int t = w / chunks, c = w % chunks;
    const int lb = t / block_size;
    const int blk = lb < max_blocks ? table[lb] : -1;
    if (blk < 0 || blk >= num_blocks) {
      raise_status(CIE_DEV_BAD_BLOCK_ID);
      continue;
    }
    const uint4 v = *reinterpret_cast<const uint4*>(
        pool + (static_cast<int64_t>(blk) * block_size + t % block_size) * row_bytes + c * 16);
    *reinterpret_cast<uint4*>(ob + static_cast<int64_t>(t) * row_bytes + c * 16) = v;
  }
}

// ------------------------------------------------------------------ rope
// One work item = 8 rotation pairs (16 bytes of each half) of one row.
template <bool BF16>
__device__ __forceinline__ void rotate8(const uint4& x1, const uint4& x2, const float* cr,
                                        const float* sr, uint4& y1, uint4& y2) {
  const uint32_t* u1 = reinterpret_cast<const uint32_t*>(&x1);
  const uint32_t* u2 = reinterpret_cast<const uint32_t*>(&x2);
  uint32_t* w1 = reinterpret_cast<uint32_t*>(&y1);
  uint32_t* w2 = reinterpret_cast<uint32_t*>(&y2);
  const float4 c0 = *reinterpret_cast<const float4*>(cr);
  const float4 c1 = *reinterpret_cast<const float4*>(cr + 4);
  const float4 s0 = *reinterpret_cast<const float4*>(sr);
  const float4 s1 = *reinterpret_cast<const float4*>(sr + 4);
  const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 a = unpack2<BF16>(u1[e]);
    const float2 b = unpack2<BF16>(u2[e]);
    // rot1 = x1*c - x2*s ; rot2 = x1*s + x2*c, each product rounded to fp32
    // before the add as in the fp32 reference
    w1[e] = pack2<BF16>(__fsub_rn(__fmul_rn(a.x, cc[2 * e]), __fmul_rn(b.x, ss[2 * e])),
                        __fsub_rn(__fmul_rn(a.y, cc[2 * e + 1]), __fmul_rn(b.y, ss[2 * e + 1])));
    w2[e] = pack2<BF16>(__fadd_rn(__fmul_rn(a.x, ss[2 * e]), __fmul_rn(b.x, cc[2 * e])),
                        __fadd_rn(__fmul_rn(a.y, ss[2 * e + 1]), __fmul_rn(b.y, cc[2 * e + 1])));
  }
}

__device__ __forceinline__ int clamp_pos(int pos, int max_pos) {
  if (pos < 0 || pos >= max_pos) {
    raise_status(CIE_DEV_BAD_POSITION);
    return pos < 0 ? 0 : max_pos - 1;
  }
  return pos;
}

template <bool BF16>
__global__ void __launch_bounds__(256) rope_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                                   int H, int L, int d, int64_t xs_b, int64_t xs_h,
                                                   int64_t xs_l, int64_t ys_b, int64_t ys_h,
                                                   int64_t ys_l, int pos0,
                                                   const float* __restrict__ cos,
                                                   const float* __restrict__ sin, int max_pos,
                                                   int rows_per_block) {
  // block = rows_per_block consecutive sequence rows of one (b, h); thread =
  // one 8-pair group of one row. Only 32-bit index math in the hot loop.
  const int half = d / 2;
  const int groups = half / 8;
  const int bh = blockIdx.y;
  const int b = bh / H, hh = bh % H;
  const int l = blockIdx.x * rows_per_block + threadIdx.x / groups;
  const int gi = threadIdx.x % groups;
  if (l >= L || threadIdx.x >= rows_per_block * groups) return;
  const int pos = clamp_pos(pos0 + l, max_pos);
  const uint8_t* src = x + (b * xs_b + hh * xs_h + l * xs_l) * 2;
  uint8_t* dst = y + (b * ys_b + hh * ys_h + l * ys_l) * 2;
  const uint4 x1 = *reinterpret_cast<const uint4*>(src + gi * 16);
  const uint4 x2 = *reinterpret_cast<const uint4*>(src + half * 2 + gi * 16);
  uint4 y1, y2;
  rotate8<BF16>(x1, x2, cos + static_cast<int64_t>(pos) * half + gi * 8,
                sin + static_cast<int64_t>(pos) * half + gi * 8, y1, y2);
  *reinterpret_cast<uint4*>(dst + gi * 16) = y1;
  *reinterpret_cast<uint4*>(dst + half * 2 + gi * 16) = y2;
}

// ------------------------------------------------------------------ append
template <bool BF16>
__global__ void __launch_bounds__(256) rope_append_kernel(
    const uint8_t* __restrict__ k_new, const uint8_t* __restrict__ v_new,
    uint8_t* __restrict__ k_pool, uint8_t* __restrict__ v_pool,
    const int32_t* __restrict__ tables, const int32_t* __restrict__ start_pos, int L, int Hkv,
    int d, int num_blocks, int block_size, int max_blocks, int64_t s_b, int64_t s_l, int64_t s_h,
    const float* __restrict__ cos, const float* __restrict__ sin, int max_pos) {
  // grid.y = sequence; one thread = one 8-pair group of one (token, head) row
  const int half = d / 2;
  const int groups = half / 8;
  const int b = blockIdx.y;
  const int per_tok = Hkv * groups;
  const int total = L * per_tok;
  const int start = start_pos[b];
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < total; w += gridDim.x * blockDim.x) {
    const int i = w / per_tok;
    const int rem = w % per_tok;
    const int hh = rem / groups, gi = rem % groups;
    const int pos = start + i;
    const int lb = pos / block_size;
    const int blk =
        (pos >= 0 && lb < max_blocks) ? tables[static_cast<int64_t>(b) * max_blocks + lb] : -1;
    if (blk < 0 || blk >= num_blocks) {
      raise_status(CIE_DEV_BAD_BLOCK_ID);
      continue;
    }
    const int64_t src_off = (b * s_b + i * s_l + hh * s_h) * 2;
    const int64_t dst_off =
        ((static_cast<int64_t>(blk) * block_size + pos % block_size) * Hkv + hh) * d * 2;
    const uint4 x1 = *reinterpret_cast<const uint4*>(k_new + src_off + gi * 16);
    const uint4 x2 = *reinterpret_cast<const uint4*>(k_new + src_off + half * 2 + gi * 16);
    uint4 y1 = x1, y2 = x2;
    if (cos != nullptr) {
      const int rp = clamp_pos(pos, max_pos);
      rotate8<BF16>(x1, x2, cos + static_cast<int64_t>(rp) * half + gi * 8,
                    sin + static_cast<int64_t>(rp) * half + gi * 8, y1, y2);
    }
    *reinterpret_cast<uint4*>(k_pool + dst_off + gi * 16) = y1;
    *reinterpret_cast<uint4*>(k_pool + dst_off + half * 2 + gi * 16) = y2;
    *reinterpret_cast<uint4*>(v_pool + dst_off + gi * 16) =
        *reinterpret_cast<const uint4*>(v_new + src_off + gi * 16);
    *reinterpret_cast<uint4*>(v_pool + dst_off + half * 2 + gi * 16) =
        *reinterpret_cast<const uint4*>(v_new + src_off + half * 2 + gi * 16);
  }
}

// ------------------------------------------------------------------ block copy
// grid.x = block pair, grid.y = slices of the block; each thread moves 16-byte
// vectors of one physical block of the pool into another.
__global__ void __launch_bounds__(256) copy_blocks_kernel(uint8_t* __restrict__ pool,
                                                          const int32_t* __restrict__ src,
                                                          const int32_t* __restrict__ dst,
                                                          int num_blocks, int64_t block_bytes) {
  const int i = blockIdx.x;
  const int s = src[i], t = dst[i];
  if (s < 0 || s >= num_blocks || t < 0 || t >= num_blocks) {
    if (blockIdx.y == 0 && threadIdx.x == 0) raise_status(CIE_DEV_BAD_BLOCK_ID);
    return;
  }
  const uint4* from = reinterpret_cast<const uint4*>(pool + s * block_bytes);
  uint4* to = reinterpret_cast<uint4*>(pool + t * block_bytes);
  const int64_t n = block_bytes / 16;
  for (int64_t w = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x; w < n;
       w += static_cast<int64_t>(gridDim.y) * blockDim.x)
    to[w] = from[w];
}

int rope_launch(const void* x, void* y, int B, int H, int L, int d, const int64_t* xs,
                const int64_t* ys, int pos0, bool bf16, const float* cos, const float* sin,
                int max_pos, cudaStream_t st) {
  if (static_cast<int64_t>(B) * H * L == 0) return CIE_OK;
  const int groups = d / 16;
  const int rows_per_block = 256 / groups;
  dim3 grid((L + rows_per_block - 1) / rows_per_block, B * H);
  if (grid.y > 65535u) {
    set_error("rope: B*H = %d exceeds 65535", B * H);
    return CIE_ERR_UNSUPPORTED;
  }
  if (bf16)
    rope_kernel<true><<<grid, rows_per_block * groups, 0, st>>>(
        reinterpret_cast<const uint8_t*>(x), reinterpret_cast<uint8_t*>(y), H, L, d, xs[0], xs[1],
        xs[2], ys[0], ys[1], ys[2], pos0, cos, sin, max_pos, rows_per_block);
  else
    rope_kernel<false><<<grid, rows_per_block * groups, 0, st>>>(
        reinterpret_cast<const uint8_t*>(x), reinterpret_cast<uint8_t*>(y), H, L, d, xs[0], xs[1],
        xs[2], ys[0], ys[1], ys[2], pos0, cos, sin, max_pos, rows_per_block);
  CIE_CHECK_LAUNCH("rope_kernel");
  return CIE_OK;
}

}  // namespace cie

using namespace cie;

extern "C" int cie_gather_kv(const void* pool, const int32_t* block_tables,
                             const int32_t* kv_lens, void* out, int B, int out_len, int Hkv,
                             int d, int num_blocks, int block_size, int max_blocks, int dtype,
                             void* stream) {
  CIE_CHECK_ARG(pool && block_tables && kv_lens && out, "cie_gather_kv: null pointer");
  CIE_CHECK_ARG(B >= 0 && out_len >= 0 && Hkv > 0 && d > 0, "cie_gather_kv: bad shape");
  CIE_CHECK_ARG(num_blocks > 0 && block_size > 0 && max_blocks > 0,
                "cie_gather_kv: bad pool geometry");
  CIE_CHECK_ARG(dtype == CIE_DTYPE_BF16 || dtype == CIE_DTYPE_FP16, "cie_gather_kv: bad dtype");
  CIE_CHECK_ARG((Hkv * d * 2) % 16 == 0, "cie_gather_kv: token row must be a multiple of 16 B");
  CIE_CHECK_ARG(aligned16(pool) && aligned16(out), "cie_gather_kv: pointers must be 16B aligned");
  const int row_bytes = Hkv * d * 2;
  if (B == 0 || out_len == 0) return CIE_OK;
  CIE_CHECK_ARG(B <= 65535, "cie_gather_kv: B must be <= 65535");
  const int64_t per_seq = static_cast<int64_t>(out_len) * (row_bytes / 16);
  CIE_CHECK_ARG(per_seq < (int64_t(1) << 31), "cie_gather_kv: sequence too long");
  const int threads = 256;
  int gx = static_cast<int>((per_seq + threads - 1) / threads);
  const int cap = (num_sms() * 16 + B - 1) / B;
  if (gx > cap) gx = cap < 1 ? 1 : cap;
  gather_kv_kernel<<<dim3(gx, B), threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint8_t*>(pool), block_tables, kv_lens,
      reinterpret_cast<uint8_t*>(out), out_len, row_bytes, num_blocks, block_size, max_blocks);
  CIE_CHECK_LAUNCH("gather_kv_kernel");
  return CIE_OK;
}

extern "C" int cie_rope(const void* x, void* y, int B, int H, int L, int d,
                        const int64_t* x_strides, const int64_t* y_strides, int pos0, int dtype,
                        const float* rope_cos, const float* rope_sin, int rope_max_pos,
                        void* stream) {
  CIE_CHECK_ARG(x && y && x_strides && y_strides && rope_cos && rope_sin,
                "cie_rope: null pointer");
  CIE_CHECK_ARG(B >= 0 && H >= 0 && L >= 0, "cie_rope: bad shape");
  CIE_CHECK_ARG(d > 0 && d % 16 == 0, "cie_rope: head_dim must be a multiple of 16");
  CIE_CHECK_ARG(dtype == CIE_DTYPE_BF16 || dtype == CIE_DTYPE_FP16, "cie_rope: bad dtype");
  CIE_CHECK_ARG(rope_max_pos > 0, "cie_rope: rope_max_pos <= 0");
  for (int i = 0; i < 3; ++i)
    CIE_CHECK_ARG(x_strides[i] % 8 == 0 && y_strides[i] % 8 == 0,
                  "cie_rope: strides must be multiples of 8 elements");
  CIE_CHECK_ARG(aligned16(x) && aligned16(y), "cie_rope: pointers must be 16B aligned");
  CIE_CHECK_ARG(aligned16(rope_cos) && aligned16(rope_sin),
                "cie_rope: rope tables must be 16B aligned");
  return rope_launch(x, y, B, H, L, d, x_strides, y_strides, pos0, dtype == CIE_DTYPE_BF16,
                     rope_cos, rope_sin, rope_max_pos, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int cie_rope_append(const void* k_new, const void* v_new, void* k_pool, void* v_pool,
                               const int32_t* block_tables, const int32_t* start_pos, int B, int L,
                               int Hkv, int d, int num_blocks, int block_size, int max_blocks,
                               const int64_t* kv_strides, int dtype, const float* rope_cos,
                               const float* rope_sin, int rope_max_pos, void* stream) {
  CIE_CHECK_ARG(k_new && v_new && k_pool && v_pool && block_tables && start_pos && kv_strides,
                "cie_rope_append: null pointer");
  CIE_CHECK_ARG(B >= 0 && L >= 0 && Hkv > 0, "cie_rope_append: bad shape");
  CIE_CHECK_ARG(d > 0 && d % 16 == 0, "cie_rope_append: head_dim must be a multiple of 16");
  CIE_CHECK_ARG(num_blocks > 0 && block_size > 0 && max_blocks > 0,
                "cie_rope_append: bad pool geometry");
  CIE_CHECK_ARG(dtype == CIE_DTYPE_BF16 || dtype == CIE_DTYPE_FP16, "cie_rope_append: bad dtype");
  CIE_CHECK_ARG((rope_cos == nullptr) == (rope_sin == nullptr),
                "cie_rope_append: rope_cos and rope_sin must both be given or both NULL");
  CIE_CHECK_ARG(rope_cos == nullptr || rope_max_pos > 0, "cie_rope_append: rope_max_pos <= 0");
  for (int i = 0; i < 3; ++i)
    CIE_CHECK_ARG(kv_strides[i] % 8 == 0, "cie_rope_append: strides must be multiples of 8");
  CIE_CHECK_ARG(aligned16(k_new) && aligned16(v_new) && aligned16(k_pool) && aligned16(v_pool),
                "cie_rope_append: pointers must be 16B aligned");
  if (B == 0 || L == 0) return CIE_OK;
  CIE_CHECK_ARG(B <= 65535, "cie_rope_append: B must be <= 65535");
  CIE_CHECK_ARG(static_cast<int64_t>(L) * Hkv * (d / 16) < (int64_t(1) << 31),
                "cie_rope_append: too many rows");
  CIE_CHECK_ARG(rope_cos == nullptr || (aligned16(rope_cos) && aligned16(rope_sin)),
                "cie_rope_append: rope tables must be 16B aligned");
  const int threads = 256;
  const int64_t per_seq = static_cast<int64_t>(L) * Hkv * (d / 16);
  int gx = static_cast<int>((per_seq + threads - 1) / threads);
  const int cap = (num_sms() * 16 + B - 1) / B;
  if (gx > cap) gx = cap < 1 ? 1 : cap;
  dim3 grid(gx, B);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CIE_DTYPE_BF16)
    rope_append_kernel<true><<<grid, threads, 0, st>>>(
        reinterpret_cast<const uint8_t*>(k_new), reinterpret_cast<const uint8_t*>(v_new),
        reinterpret_cast<uint8_t*>(k_pool), reinterpret_cast<uint8_t*>(v_pool), block_tables,
        start_pos, L, Hkv, d, num_blocks, block_size, max_blocks, kv_strides[0], kv_strides[1],
        kv_strides[2], rope_cos, rope_sin, rope_max_pos);
  else
    rope_append_kernel<false><<<grid, threads, 0, st>>>(
        reinterpret_cast<const uint8_t*>(k_new), reinterpret_cast<const uint8_t*>(v_new),
        reinterpret_cast<uint8_t*>(k_pool), reinterpret_cast<uint8_t*>(v_pool), block_tables,
        start_pos, L, Hkv, d, num_blocks, block_size, max_blocks, kv_strides[0], kv_strides[1],
        kv_strides[2], rope_cos, rope_sin, rope_max_pos);
  CIE_CHECK_LAUNCH("rope_append_kernel");
  return CIE_OK;
}

extern "C" int cie_copy_blocks(void* const* pools, int n_pools, const int32_t* src_blocks,
                               const int32_t* dst_blocks, int n, int num_blocks,
                               size_t block_bytes, void* stream) {
  CIE_CHECK_ARG(n >= 0 && n_pools >= 0, "cie_copy_blocks: negative count");
  if (n == 0 || n_pools == 0) return CIE_OK;
  CIE_CHECK_ARG(pools && src_blocks && dst_blocks, "cie_copy_blocks: null pointer");
  CIE_CHECK_ARG(num_blocks > 0 && block_bytes > 0 && block_bytes % 16 == 0,
                "cie_copy_blocks: block size must be a positive multiple of 16 bytes");
  for (int i = 0; i < n_pools; ++i)
    CIE_CHECK_ARG(pools[i] && aligned16(pools[i]), "cie_copy_blocks: pool %d null or unaligned",
                  i);
  const int threads = 256;
  const int64_t vec = static_cast<int64_t>(block_bytes / 16);
  int gy = static_cast<int>((vec + threads - 1) / threads);
  const int cap = (num_sms() * 8 + n - 1) / n;
  if (gy > cap) gy = cap < 1 ? 1 : cap;
  if (gy > 65535) gy = 65535;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int i = 0; i < n_pools; ++i) {
    copy_blocks_kernel<<<dim3(n, gy), threads, 0, st>>>(reinterpret_cast<uint8_t*>(pools[i]),
                                                        src_blocks, dst_blocks, num_blocks,
                                                        static_cast<int64_t>(block_bytes));
    CIE_CHECK_LAUNCH("copy_blocks_kernel");
  }
  return CIE_OK;
}
