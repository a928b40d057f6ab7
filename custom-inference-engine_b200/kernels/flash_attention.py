"""Flash attention, paged attention and the K/V byte movers on B200 (sm_100a).

``flash_attention`` is the drop-in for the reference's Triton entry
(kernels/flash_attention.py:136-209): same positional signature, same
bottom-right causal alignment, same default scale and the same exception types
for bad input (kernels/flash_attention.py:147-165), with bf16 accepted besides
fp16. GQA is handled inside the kernel (kv head = q head // (Hq // Hkv)) instead
of by ``repeat_interleave`` (kernels/flash_attention.py:152-155).

The remaining functions cover the paged-KV side of the engine
(engine/cache/kv_cache.py) for batches of sequences:

* ``paged_attention``  decode (M=1) / speculative verify (M=gamma+1) straight
                        from the block table, split-KV + log-sum-exp merge.
* ``gather_kv``        bit-exact dense gather (PagedKVCache.gather).
* ``rope_append``      RoPE of the new K rows fused with the paged append.
* ``apply_rotary``     standalone half-split RoPE (apply_rotary_ref).

Every call is asynchronous on the current CUDA stream and allocates its output
(and scratch workspace, when the kernel needs one) with torch.
"""

from __future__ import annotations

import ctypes
import math

import torch

from kernels import _lib

_DTYPES = {torch.bfloat16: _lib.CIE_DTYPE_BF16, torch.float16: _lib.CIE_DTYPE_FP16}
_TABLE_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _require() -> ctypes.CDLL:
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required but not available")
    try:
        return _lib.load()
    except _lib.ExtensionNotBuiltError as e:
        raise RuntimeError(str(e)) from e


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _vp(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _kernel_ready(t: torch.Tensor) -> torch.Tensor:
    """Innermost dim contiguous, other strides multiples of 8 elements, 16B-aligned."""
    if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16:
        # a fresh copy: .contiguous() would return a contiguous view at an
        # unaligned offset unchanged
        t = t.clone(memory_format=torch.contiguous_format)
    return t


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _rope_tables(rope, device) -> tuple[torch.Tensor | None, torch.Tensor | None, int]:
    if rope is None:
        return None, None, 0
    cos, sin = rope
    if cos.dtype not in _TABLE_DTYPES or sin.dtype not in _TABLE_DTYPES:
        raise ValueError("rope tables must be float32, float16 or bfloat16 (max_pos, head_dim/2)")
    # the kernels read fp32 tables; widening a 16-bit table (e.g. the engine's
    # RotaryEmbedding buffers after the runtime's cast) is exact
    cos, sin = cos.float(), sin.float()
    if cos.device != device or sin.device != device:
        raise ValueError("rope tables must live on the same device as q")
    cos = cos.contiguous()
    sin = sin.contiguous()
    if cos.shape != sin.shape or cos.ndim != 2:
        raise ValueError("rope cos/sin must both be (max_pos, head_dim/2)")
    return cos, sin, int(cos.shape[0])


def flash_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    scale: float | None = None,
    *,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    rope_q_pos0: int | None = None,
    rope_k: bool = True,
    out: torch.Tensor | None = None,
    out_peers: list[int] | None = None,
) -> torch.Tensor:
    """Flash attention on CUDA (tcgen05 tensor cores for d in {64, 128}).

    q: (B, H, M, D), k/v: (B, Hk, N, D), H a multiple of Hk. Returns (B, H, M, D)
    in q's dtype. ``causal`` masks key j for query i when j > N - M + i.

    rope: optional fp32 ``(cos, sin)`` tables of shape (max_pos, D/2). When given,
    query row i is rotated at position ``rope_q_pos0 + i`` (default N - M + i)
    inside the kernel, and keys are rotated at positions 0..N-1 unless
    ``rope_k=False`` (K already rotated, e.g. read from the cache).

    out: optional (B, H, M, D) tensor (any strides, 16-byte aligned rows) to
    write into instead of a new one. out_peers: device addresses of the same
    slice in other GPUs' outputs (peer memory mapped into this process); every
    output tile is then also copied to each of them inside the kernel
    (``cie_prefill_attn_peers``) and is complete there once every rank has run
    :func:`peer_barrier` after this call.
    """
    if not q.is_cuda:
        raise RuntimeError("flash_attention requires CUDA tensors")
    B, H, M, D = q.shape
    if k.ndim != 4 or v.ndim != 4 or k.shape != v.shape:
        raise ValueError(f"k/v must both be (B, Hk, N, D), got {tuple(k.shape)} / {tuple(v.shape)}")
    _, Hk, N, _ = k.shape
    if k.shape[0] != B or k.shape[3] != D:
        raise ValueError(f"k/v shape {tuple(k.shape)} does not match q {tuple(q.shape)}")
    if H % Hk:
        raise ValueError(f"num_heads {H} must be a multiple of num_kv_heads {Hk}")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if D & (D - 1):
        raise ValueError(f"head_dim must be a power of 2, got {D}")
    if D < 16:
        raise ValueError(f"head_dim must be >= 16, got {D}")
    if D > 256:
        raise ValueError(f"head_dim must be <= 256, got {D}")
    if q.dtype not in _DTYPES:
        raise ValueError(f"flash_attention expects FP16 or BF16 Q/K/V, got {q.dtype}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"q/k/v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    if not (k.is_cuda and v.is_cuda) or k.device != q.device or v.device != q.device:
        raise RuntimeError("flash_attention requires CUDA tensors on one device")
    lib = _require()

    q = _kernel_ready(q)
    k = _kernel_ready(k)
    v = _kernel_ready(v)
    if out is None:
        if out_peers:
            raise ValueError("out_peers needs an explicit out (the local slice of the output)")
        out = torch.empty((B, H, M, D), dtype=q.dtype, device=q.device)
    elif out.shape != (B, H, M, D) or out.dtype != q.dtype or out.device != q.device:
        raise ValueError(f"out must be a ({B}, {H}, {M}, {D}) {q.dtype} tensor on {q.device}")
    if B == 0 or M == 0 or H == 0:
        return out
    cos, sin, max_pos = _rope_tables(rope, q.device)
    if rope is not None and cos.shape[1] * 2 != D:
        raise ValueError(f"rope tables are for head_dim {cos.shape[1] * 2}, q has {D}")
    q_pos0 = (N - M) if rope_q_pos0 is None else int(rope_q_pos0)
    do_rope_k = 1 if (rope is not None and rope_k) else 0
    dt = _DTYPES[q.dtype]
    ws_bytes = lib.cie_prefill_attn_workspace(B, H, Hk, M, N, D, dt, do_rope_k)
    ws = _workspace(ws_bytes, q.device)
    strides = (_lib.strides3(q.stride()[:3]), _lib.strides3(k.stride()[:3]),
               _lib.strides3(v.stride()[:3]), _lib.strides3(out.stride()[:3]))
    tail = (float(scale), 1 if causal else 0, dt, _vp(cos), _vp(sin), max_pos, q_pos0, do_rope_k,
            _vp(ws), ws_bytes, _stream(q))
    if out_peers:
        peers = (ctypes.c_void_p * len(out_peers))(*[int(x) for x in out_peers])
        rc = lib.cie_prefill_attn_peers(_vp(q), _vp(k), _vp(v), _vp(out), peers, len(out_peers),
                                        B, H, Hk, M, N, D, *strides, *tail)
    else:
        rc = lib.cie_prefill_attn(_vp(q), _vp(k), _vp(v), _vp(out), B, H, Hk, M, N, D, *strides,
                                  *tail)
    _lib.check(rc, "flash_attention")
    return out


def peer_barrier(flag_ptrs: list[int], rank: int, epoch: int, device: torch.device) -> None:
    """Stream-ordered barrier over the GPUs whose counter arrays ``flag_ptrs`` (one
    per rank, uint32[world] each, zero-initialised, mapped into this process) name;
    ``epoch`` grows by one per call. See ``cie_peer_barrier``."""
    lib = _require()
    arr = (ctypes.c_void_p * len(flag_ptrs))(*[int(x) for x in flag_ptrs])
    rc = lib.cie_peer_barrier(arr, len(flag_ptrs), int(rank), ctypes.c_uint32(epoch & 0xFFFFFFFF),
                              ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    _lib.check(rc, "peer_barrier")


def paged_attention(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    kv_lens: torch.Tensor,
    causal: bool = True,
    scale: float | None = None,
    *,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    split_tokens: int = 0,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Attention of q against each sequence's paged K/V history.

    Decode (M = 1) and verify (M = gamma + 1) run on the split-KV kernel; query
    blocks of more than 64 rows per kv head (chunked prefill of a batch) run on
    the tcgen05 prefill kernel, which reads the pools through the block table
    (block sizes multiple of 16, D 64 / 128; ``split_tokens`` does not apply).

    q: (B, Hq, M, D); k_pool/v_pool: (num_blocks, block_size, Hkv, D) contiguous;
    block_tables: int32 (B, max_blocks) of physical block ids in logical order;
    kv_lens: int32 (B,) history length including the M query tokens, so query i
    sits at position kv_lens[b] - M + i. Rows attend bottom-right causally
    (``causal``) as in the reference. ``rope``: rotate q at those positions (K is
    stored rotated). Returns (B, Hq, M, D).
    """
    if not q.is_cuda:
        raise RuntimeError("paged_attention requires CUDA tensors")
    if q.ndim != 4:
        raise ValueError(f"q must be (B, Hq, M, D), got {tuple(q.shape)}")
    B, Hq, M, D = q.shape
    if k_pool.ndim != 4 or k_pool.shape != v_pool.shape:
        raise ValueError("k_pool/v_pool must both be (num_blocks, block_size, Hkv, D)")
    nb, bs, Hkv, Dk = k_pool.shape
    if Dk != D:
        raise ValueError(f"pool head_dim {Dk} != q head_dim {D}")
    if Hq % Hkv:
        raise ValueError(f"num_heads {Hq} must be a multiple of num_kv_heads {Hkv}")
    if q.dtype not in _DTYPES or k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError(f"paged_attention expects matching FP16/BF16 q and pools, got "
                         f"{q.dtype}/{k_pool.dtype}/{v_pool.dtype}")
    if block_tables.dtype != torch.int32 or kv_lens.dtype != torch.int32:
        raise ValueError("block_tables and kv_lens must be int32")
    if block_tables.ndim != 2 or block_tables.shape[0] != B or kv_lens.shape != (B,):
        raise ValueError("block_tables must be (B, max_blocks) and kv_lens (B,)")
    for t in (k_pool, v_pool, block_tables, kv_lens):
        if not t.is_cuda or t.device != q.device:
            raise RuntimeError("paged_attention requires all tensors on q's CUDA device")
    if not (k_pool.is_contiguous() and v_pool.is_contiguous()):
        raise ValueError("k_pool/v_pool must be contiguous")
    lib = _require()
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    q = _kernel_ready(q)
    block_tables = block_tables.contiguous()
    kv_lens = kv_lens.contiguous()
    if out is None:
        out = torch.empty((B, Hq, M, D), dtype=q.dtype, device=q.device)
    if B == 0 or M == 0:
        return out
    cos, sin, max_pos = _rope_tables(rope, q.device)
    max_blocks = block_tables.shape[1]
    ws_bytes = lib.cie_paged_attn_workspace(B, Hq, Hkv, M, D, bs, max_blocks, int(split_tokens))
    ws = _workspace(ws_bytes, q.device)
    rc = lib.cie_paged_attn(
        _vp(q), _vp(k_pool), _vp(v_pool), _vp(block_tables), _vp(kv_lens), _vp(out),
        B, Hq, Hkv, M, D, nb, bs, max_blocks,
        _lib.strides3(q.stride()[:3]), _lib.strides3(out.stride()[:3]),
        float(scale), 1 if causal else 0, _DTYPES[q.dtype], _vp(cos), _vp(sin), max_pos,
        int(split_tokens), _vp(ws), ws_bytes, _stream(q))
    _lib.check(rc, "paged_attention")
    return out


def gather_kv(
    pool: torch.Tensor,
    block_tables: torch.Tensor,
    kv_lens: torch.Tensor,
    out_len: int | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Dense copy of the paged history: (B, out_len, Hkv, D), rows >= kv_lens[b] untouched.

    Bit-exact with PagedKVCache.gather (reference engine/cache/kv_cache.py:141-165).
    ``out_len`` defaults to max_blocks * block_size. Note: reading kv_lens would need a
    host sync, so the default output is over-allocated rather than trimmed.
    """
    if not pool.is_cuda:
        raise RuntimeError("gather_kv requires CUDA tensors")
    nb, bs, Hkv, D = pool.shape
    B, max_blocks = block_tables.shape
    if block_tables.dtype != torch.int32 or kv_lens.dtype != torch.int32:
        raise ValueError("block_tables and kv_lens must be int32")
    if pool.dtype not in _DTYPES:
        raise ValueError(f"gather_kv expects an FP16/BF16 pool, got {pool.dtype}")
    lib = _require()
    if out_len is None:
        out_len = max_blocks * bs
    if out is None:
        out = torch.empty((B, out_len, Hkv, D), dtype=pool.dtype, device=pool.device)
    if not out.is_contiguous() or out.shape != (B, out_len, Hkv, D):
        raise ValueError("out must be a contiguous (B, out_len, Hkv, D) tensor")
    rc = lib.cie_gather_kv(_vp(pool.contiguous()), _vp(block_tables.contiguous()),
                           _vp(kv_lens.contiguous()), _vp(out), B, out_len, Hkv, D, nb, bs,
                           max_blocks, _DTYPES[pool.dtype], _stream(pool))
    _lib.check(rc, "gather_kv")
    return out


def rope_append(
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    start_pos: torch.Tensor,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> None:
    """Write k_new/v_new (B, L, Hkv, D) into the pools at positions start_pos[b] + i.

    K rows are rotated at their positions when ``rope`` is given (the cache stores
    rotated K, as the reference does at engine/model/block.py:53-64). Blocks must
    already be assigned in ``block_tables``.
    """
    if not k_new.is_cuda:
        raise RuntimeError("rope_append requires CUDA tensors")
    B, L, Hkv, D = k_new.shape
    if v_new.shape != k_new.shape:
        raise ValueError("k_new and v_new must have the same shape")
    nb, bs, Hp, Dp = k_pool.shape
    if (Hp, Dp) != (Hkv, D) or v_pool.shape != k_pool.shape:
        raise ValueError("pool geometry does not match k_new")
    if k_new.dtype not in _DTYPES or {v_new.dtype, k_pool.dtype, v_pool.dtype} != {k_new.dtype}:
        raise ValueError("rope_append expects one FP16/BF16 dtype for all tensors")
    if block_tables.dtype != torch.int32 or start_pos.dtype != torch.int32:
        raise ValueError("block_tables and start_pos must be int32")
    lib = _require()
    k_new = _kernel_ready(k_new)
    v_new = _kernel_ready(v_new)
    if k_new.stride() != v_new.stride():
        k_new = k_new.contiguous()
        v_new = v_new.contiguous()
    cos, sin, max_pos = _rope_tables(rope, k_new.device)
    rc = lib.cie_rope_append(
        _vp(k_new), _vp(v_new), _vp(k_pool), _vp(v_pool), _vp(block_tables.contiguous()),
        _vp(start_pos.contiguous()), B, L, Hkv, D, nb, bs, block_tables.shape[1],
        _lib.strides3(k_new.stride()[:3]), _DTYPES[k_new.dtype], _vp(cos), _vp(sin), max_pos,
        _stream(k_new))
    _lib.check(rc, "rope_append")


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos0: int = 0) -> torch.Tensor:
    """Half-split RoPE of x (B, H, L, D) at positions pos0 .. pos0 + L - 1 (fp32 math)."""
    if not x.is_cuda:
        raise RuntimeError("apply_rotary requires CUDA tensors")
    if x.dtype not in _DTYPES:
        raise ValueError(f"apply_rotary expects FP16/BF16, got {x.dtype}")
    lib = _require()
    x = _kernel_ready(x)
    cos, sin, max_pos = _rope_tables((cos, sin), x.device)
    B, H, L, D = x.shape
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    rc = lib.cie_rope(_vp(x), _vp(y), B, H, L, D, _lib.strides3(x.stride()[:3]),
                      _lib.strides3(y.stride()[:3]), int(pos0), _DTYPES[x.dtype], _vp(cos),
                      _vp(sin), max_pos, _stream(x))
    _lib.check(rc, "apply_rotary")
    return y
