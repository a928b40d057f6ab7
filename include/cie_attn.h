/*
 * cie_attn.h — C ABI of libcie_attn.so, the B200 (sm_100a) attention hot path
 * of the Custom-Inference-Engine LLM engine.
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are CUDA device pointers owned by the caller.
 *     The library never allocates device memory; scratch space is passed in
 *     through `workspace` with a size obtained from the matching *_workspace()
 *     query (cie_paged_attn_noalloc instead uses a fixed array of its own).
 *   - Work is enqueued asynchronously on `stream` (a cudaStream_t, NULL = the
 *     legacy default stream). A return value of CIE_OK means the launch was
 *     accepted; device-side faults that the kernels detect themselves (bad
 *     block ids, a pipeline wait that ran out of time) are recorded in a
 *     per-device status word read by cie_device_status().
 *   - Element type codes: CIE_DTYPE_BF16 or CIE_DTYPE_FP16 (Q, K, V, O and the
 *     paged pools share one type). RoPE tables are fp32.
 *   - Strides are in elements; the innermost (head_dim) stride must be 1.
 *   - Every call is thread-safe: TMA descriptors are built per call on the
 *     host stack and the only shared host state is a once-initialised driver
 *     entry point.
 */
#ifndef CIE_ATTN_H_
#define CIE_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum cie_status {
  CIE_OK = 0,
  CIE_ERR_INVALID = -1,      /* bad argument (shape, stride, alignment, dtype) */
  CIE_ERR_UNSUPPORTED = -2,  /* valid but not implemented (e.g. head_dim 96)   */
  CIE_ERR_WORKSPACE = -3,    /* workspace NULL or smaller than required        */
  CIE_ERR_LAUNCH = -4,       /* CUDA launch / driver error                     */
  CIE_ERR_DEVICE = -5        /* device-side status word is non-zero            */
};

enum cie_dtype { CIE_DTYPE_BF16 = 0, CIE_DTYPE_FP16 = 1 };

/* Device status bits (cie_device_status). */
#define CIE_DEV_BAD_BLOCK_ID 0x1  /* a block-table entry was < 0 or >= num_blocks */
#define CIE_DEV_TIMEOUT 0x2       /* a bounded pipeline wait expired               */
#define CIE_DEV_BAD_POSITION 0x4  /* a RoPE position fell outside the cos/sin table */

/*
 * Dense causal / non-causal grouped-query attention (prefill).
 *
 * Replaces the Triton launch in kernels/flash_attention.py:136-209
 * (`flash_attention(q, k, v, causal, scale)`, grid at :175-208) and the GQA
 * expansion at :152-155, which this kernel does not need (kv head = q head /
 * (Hq / Hkv)).
 *
 *   q: (B, Hq, M, d)   k, v: (B, Hkv, N, d)   o: (B, Hq, M, d)
 *   *_strides[0..2] = strides of the B, H and sequence dims (elements).
 *   causal: bottom-right aligned, query i sees keys j <= N - M + i
 *           (kernels/ref/flash_attention_ref.py:44-49).
 *   rope_cos / rope_sin: optional fp32 (rope_max_pos, d/2) tables built as in
 *           kernels/ref/rope_apply_ref.py:6-19. When non-NULL, q row i is
 *           rotated at position rope_q_pos0 + i inside the kernel, and when
 *           rope_k != 0, K row j is rotated at position j (half-split rotation,
 *           kernels/ref/rope_apply_ref.py:49-53) into the workspace first.
 *   d: 16, 32, 64, 128 or 256 (the reference accepts powers of two >= 16,
 *      kernels/flash_attention.py:160-163). d in {64, 128} with more than 64
 *      query rows per kv head runs on the tcgen05 kernel; everything else on
 *      the split-KV mma.sync kernel over dense K/V.
 */
int cie_prefill_attn(const void* q, const void* k, const void* v, void* o,
                     int B, int Hq, int Hkv, int M, int N, int d,
                     const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides,
                     float scale, int causal, int dtype,
                     const float* rope_cos, const float* rope_sin,
                     int rope_max_pos, int rope_q_pos0, int rope_k,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * cie_prefill_attn fused with the all-gather of its output across the GPUs of
 * a kv-head-group sharded prefill (one process per GPU, NVLink peer memory).
 * Replaces the launch of kernels/flash_attention.py:136-209 on each shard plus
 * the collective that reassembles [B, S, Hq * d] (the reference is one GPU;
 * this is the multi-GPU layer).
 *
 * Same arguments as cie_prefill_attn; o is this rank's slice of the full
 * output (its heads), and o_peers[0 .. n_peers) are the same slice in the other
 * ranks' full outputs, as mapped into this process (e.g. symmetric memory).
 * Every output tile is written to o and, while the kernel goes on computing,
 * copied to each peer with 16-byte peer stores. 1 <= n_peers <= 7. Only the
 * tcgen05 path (d 64 / 128, more than 64 query rows per kv head, N > 0) takes
 * peers. The peers' rows are complete once every rank's cie_peer_barrier that
 * follows this call on its stream has returned.
 */
int cie_prefill_attn_peers(const void* q, const void* k, const void* v, void* o,
                           void* const* o_peers, int n_peers,
                           int B, int Hq, int Hkv, int M, int N, int d,
                           const int64_t* q_strides, const int64_t* k_strides,
                           const int64_t* v_strides, const int64_t* o_strides,
                           float scale, int causal, int dtype,
                           const float* rope_cos, const float* rope_sin,
                           int rope_max_pos, int rope_q_pos0, int rope_k,
                           void* workspace, size_t workspace_bytes, void* stream);

/*
 * Stream-ordered barrier across `world` GPUs (one process each) through
 * counters in peer memory: flags[r] is rank r's array of `world` uint32
 * counters (zero-initialised, all ranks' arrays mapped into this process);
 * `epoch` grows by one per call. Publishes epoch into slot `rank` of every
 * array, then waits (bounded by cie_set_wait_limit; CIE_DEV_TIMEOUT when a
 * rank does not arrive) until its own array holds epoch in every slot. Work
 * queued after it on `stream` sees everything the other ranks wrote before
 * their call. No counterpart in the reference (single GPU).
 */
int cie_peer_barrier(uint32_t* const* flags, int world, int rank, uint32_t epoch,
                     void* stream);

/* Bytes of workspace cie_prefill_attn needs for these arguments: the
 * rotated copy of K when rope_k is set, plus split-KV partials when the call
 * is served by the short-query kernel (G*M <= 64, or d not 64/128). */
size_t cie_prefill_attn_workspace(int B, int Hq, int Hkv, int M, int N, int d,
                                  int dtype, int rope_k);

/*
 * Paged-KV attention for single-token decode (M = 1) and speculative verify
 * (M = gamma + 1), reading K/V straight from the paged pools through the
 * block table. Replaces the dense history gather of
 * engine/cache/kv_cache.py:141-165 followed by flash_attention() at
 * engine/model/block.py:65-71, for every sequence of a batch at once.
 *
 *   q:            (B, Hq, M, d) with q_strides (B, H, M dims, elements)
 *   k_pool/v_pool:(num_blocks, block_size, Hkv, d) contiguous
 *                 (engine/cache/kv_cache.py:34-64 layout)
 *   block_tables: int32 (B, max_blocks); row b lists physical block ids in
 *                 logical order (engine/cache/block_table.py:6-36)
 *   kv_lens:      int32 (B,); kv_lens[b] tokens of history including the M
 *                 query tokens, so query i sits at position kv_lens[b]-M+i.
 *   o:            (B, Hq, M, d) with o_strides.
 *   causal:       bottom-right aligned as above.
 *   rope_cos/sin: optional; when non-NULL q row i is rotated at position
 *                 kv_lens[b] - M + i (K is stored pre-rotated in the pool).
 *   split_tokens: 0 = automatic; else tokens per split-KV partition (multiple
 *                 of 16). Partitions are merged by a log-sum-exp kernel.
 * Query blocks of more than 64 rows per kv head ((Hq / Hkv) * M > 64, i.e.
 * chunked prefill of a batch over non-empty histories) with d 64 or 128 and a
 * block size that is a multiple of 16 run on the tcgen05 prefill kernel
 * instead, which reads the pools through the table in 16-token TMA boxes (no
 * gather, no workspace, split_tokens ignored); o must then be 16-byte aligned
 * with strides multiples of 8 elements. This replaces the gather + dense
 * attention of a chunked prefill (engine/model/block.py:65-71 with L > 1).
 */
int cie_paged_attn(const void* q, const void* k_pool, const void* v_pool,
                   const int32_t* block_tables, const int32_t* kv_lens,
                   void* o, int B, int Hq, int Hkv, int M, int d,
                   int num_blocks, int block_size, int max_blocks,
                   const int64_t* q_strides, const int64_t* o_strides,
                   float scale, int causal, int dtype,
                   const float* rope_cos, const float* rope_sin,
                   int rope_max_pos, int split_tokens,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace cie_paged_attn needs for these arguments. */
size_t cie_paged_attn_workspace(int B, int Hq, int Hkv, int M, int d,
                                int block_size, int max_blocks,
                                int split_tokens);

/*
 * cie_paged_attn for callers that cannot allocate device memory — hosts that
 * own all device memory and give plugins no allocator, or serving loops that
 * cannot afford cudaMalloc's device synchronisation between steps. It has no
 * counterpart in the reference (the reference allocates with torch).
 *
 * Same arguments and results as cie_paged_attn, without workspace. Split-KV
 * partial results go to a fixed 32 MiB scratch array inside the library's
 * device image, held on every GPU that loads the library until the process
 * exits. With split_tokens = 0 the partition size is grown until the
 * partials fit; an explicit split_tokens whose partials exceed 32 MiB is
 * rejected with CIE_ERR_WORKSPACE and a message. The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture. The address is
 * kept per device and context and looked up again when the current context
 * changes (e.g. after cudaDeviceReset); make the first call after such a
 * change outside stream capture too. The array is
 * shared by all calls on a device and keeps the last call's contents (nothing
 * in it needs to start at zero); calls that overlap on the GPU race on it and
 * must be serialised by the caller. It never calls cudaMalloc or cudaFree.
 */
int cie_paged_attn_noalloc(const void* q, const void* k_pool, const void* v_pool,
                           const int32_t* block_tables, const int32_t* kv_lens,
                           void* o, int B, int Hq, int Hkv, int M, int d,
                           int num_blocks, int block_size, int max_blocks,
                           const int64_t* q_strides, const int64_t* o_strides,
                           float scale, int causal, int dtype,
                           const float* rope_cos, const float* rope_sin,
                           int rope_max_pos, int split_tokens, void* stream);

/*
 * Bit-exact gather of the paged history into a dense buffer:
 *   out[b, t, h, :] = pool[block_tables[b, t / block_size], t % block_size, h, :]
 * for t < kv_lens[b]; rows t >= kv_lens[b] (up to out_len) are left as they
 * are. Mirrors PagedKVCache.gather (engine/cache/kv_cache.py:141-165) for a
 * batch of sequences. out: (B, out_len, Hkv, d) contiguous.
 */
int cie_gather_kv(const void* pool, const int32_t* block_tables,
                  const int32_t* kv_lens, void* out, int B, int out_len,
                  int Hkv, int d, int num_blocks, int block_size,
                  int max_blocks, int dtype, void* stream);

/*
 * Fused RoPE-on-K + paged append. For every new token (b, i), i < L:
 *   pos = start_pos[b] + i
 *   k_pool[blk, off, h, :] = rope(k_new[b, i, h, :], pos)   (if rope_cos)
 *   v_pool[blk, off, h, :] = v_new[b, i, h, :]
 * with (blk, off) = (block_tables[b, pos / block_size], pos % block_size).
 * Replaces rope.apply(k) (engine/model/block.py:53-54) and the block-walked
 * slice copies of PagedKVCache.append (engine/cache/kv_cache.py:102-139).
 * k_new / v_new: (B, L, Hkv, d) with strides (elements) for the B, L, H dims.
 */
int cie_rope_append(const void* k_new, const void* v_new, void* k_pool,
                    void* v_pool, const int32_t* block_tables,
                    const int32_t* start_pos, int B, int L, int Hkv, int d,
                    int num_blocks, int block_size, int max_blocks,
                    const int64_t* kv_strides, int dtype,
                    const float* rope_cos, const float* rope_sin,
                    int rope_max_pos, void* stream);

/*
 * Whole-block copies inside paged pools, the data movement of
 * PagedKVCache.fork (engine/cache/kv_cache.py:169-185, where it is an
 * index_select + index_copy_ per layer):
 *   pools[p][dst_blocks[i]] = pools[p][src_blocks[i]]  for i < n, p < n_pools
 * pools: host array of n_pools device pointers (e.g. the K and V pool of every
 * layer), each holding num_blocks blocks of block_bytes bytes (a multiple of
 * 16). src_blocks / dst_blocks: int32 device arrays of n block ids; ids
 * outside [0, num_blocks) set CIE_DEV_BAD_BLOCK_ID and are skipped. Source
 * and destination blocks must not overlap. One launch per pool.
 */
int cie_copy_blocks(void* const* pools, int n_pools, const int32_t* src_blocks,
                    const int32_t* dst_blocks, int n, int num_blocks,
                    size_t block_bytes, void* stream);

/*
 * Standalone half-split RoPE: y[b, h, i, :] = rope(x[b, h, i, :], pos0 + i),
 * computed in fp32 and rounded to the element type
 * (kernels/ref/rope_apply_ref.py:22-53). x, y: (B, H, L, d) with strides.
 */
int cie_rope(const void* x, void* y, int B, int H, int L, int d,
             const int64_t* x_strides, const int64_t* y_strides, int pos0,
             int dtype, const float* rope_cos, const float* rope_sin,
             int rope_max_pos, void* stream);

/* Weight-only INT8 GEMM (replaces the Triton kernel of kernels/int8_matmul.py:
 * 17-110, semantics of kernels/ref/int8_matmul_ref.py:31-47):
 *   y[m, n] = sum_k x[m, k] * w[n, k] * scales[n] (+ bias[n])
 * x: (M, K) bf16/fp16 (dtype), row stride x_stride_m elements (multiple of 8);
 * w: (N, K) int8, row stride w_stride_n bytes (multiple of 16);
 * scales, bias: fp32 (N,) (bias may be NULL); y: (M, N) in x's dtype, row
 * stride y_stride_m. fp32 accumulation on the tensor cores. A workspace of
 * cie_int8_matmul_workspace(M, N, K) bytes holds split-K partials (0 when the
 * output tiles alone fill the GPU). */
int cie_int8_matmul(const void* x, const void* w, const float* scales,
                    const float* bias, void* y, int M, int N, int K,
                    int64_t x_stride_m, int64_t w_stride_n, int64_t y_stride_m,
                    int dtype, void* workspace, size_t workspace_bytes,
                    void* stream);
size_t cie_int8_matmul_workspace(int M, int N, int K);

/* Per-device status word (CIE_DEV_* bits) of the current device. Synchronizes
 * `stream`. If clear != 0 the word is reset to 0 afterwards. */
int cie_device_status(int* status_out, int clear, void* stream);

/* Sets the time limit (nanoseconds) of every pipeline wait inside the kernels
 * on the current device, for kernels launched after this call; the previous
 * value is stored in *previous_ns when it is non-NULL. The default is
 * 2 000 000 000 (2 s). A wait that runs out sets CIE_DEV_TIMEOUT, makes the
 * kernel's other roles leave their loops, lets copies and MMAs already in
 * flight land (waits that always use the 2 s default), releases tensor memory
 * and returns; the outputs of that launch are undefined, the context stays
 * usable. A limit of 0 makes every wait that is not satisfied at once run
 * out, which is how the tests reach that path. No counterpart in the
 * reference (its Triton kernels have no device-side waits). Synchronous. */
int cie_set_wait_limit(uint64_t limit_ns, uint64_t* previous_ns);

/* Copies the last host-side error message of the calling thread into buf. */
int cie_get_last_error(char* buf, int buf_len);

/* Library version string, e.g. "cie_attn 0.1.0 sm_100a". */
const char* cie_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CIE_ATTN_H_ */
