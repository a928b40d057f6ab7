"""ctypes binding of libcie_attn.so (declared in include/cie_attn.h).

This is the only place Python touches the native library. Every entry point
takes raw device pointers, element strides and a cudaStream_t; the wrappers in
kernels/flash_attention.py and engine/ turn torch tensors into those.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

# The in-tree build; CIE_ATTN_LIB names another build of the same library
# (e.g. one compiled with different tuning macros) to load instead.
LIB_PATH = Path(os.environ.get("CIE_ATTN_LIB") or
                Path(__file__).resolve().parent / "libcie_attn.so")

CIE_OK = 0
CIE_ERR_INVALID = -1
CIE_ERR_UNSUPPORTED = -2
CIE_ERR_WORKSPACE = -3
CIE_ERR_LAUNCH = -4
CIE_ERR_DEVICE = -5

CIE_DTYPE_BF16 = 0
CIE_DTYPE_FP16 = 1

CIE_DEV_BAD_BLOCK_ID = 0x1
CIE_DEV_TIMEOUT = 0x2
CIE_DEV_BAD_POSITION = 0x4

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t
_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); must match include/cie_attn.h
SIGNATURES: dict[str, tuple] = {
    "cie_prefill_attn": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i64p, _i64p, _i64p,
                              _i64p, _f, _i, _i, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "cie_prefill_attn_peers": (_i, [_vp, _vp, _vp, _vp, ctypes.POINTER(_vp), _i, _i, _i, _i, _i,
                                    _i, _i, _i64p, _i64p, _i64p, _i64p, _f, _i, _i, _vp, _vp, _i,
                                    _i, _i, _vp, _sz, _vp]),
    "cie_peer_barrier": (_i, [ctypes.POINTER(_vp), _i, _i, ctypes.c_uint32, _vp]),
    "cie_prefill_attn_workspace": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "cie_paged_attn": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i64p,
                            _i64p, _f, _i, _i, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    "cie_paged_attn_workspace": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "cie_paged_attn_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i,
                                    _i64p, _i64p, _f, _i, _i, _vp, _vp, _i, _i, _vp]),
    "cie_gather_kv": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "cie_rope_append": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i64p,
                             _i, _vp, _vp, _i, _vp]),
    "cie_copy_blocks": (_i, [ctypes.POINTER(_vp), _i, _vp, _vp, _i, _i, _sz, _vp]),
    "cie_rope": (_i, [_vp, _vp, _i, _i, _i, _i, _i64p, _i64p, _i, _i, _vp, _vp, _i, _vp]),
    "cie_int8_matmul": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, ctypes.c_int64,
                             ctypes.c_int64, ctypes.c_int64, _i, _vp, _sz, _vp]),
    "cie_int8_matmul_workspace": (_sz, [_i, _i, _i]),
    "cie_device_status": (_i, [ctypes.POINTER(ctypes.c_int), _i, _vp]),
    "cie_set_wait_limit": (_i, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "cie_get_last_error": (_i, [ctypes.c_char_p, _i]),
    "cie_version": (ctypes.c_char_p, []),
}

_LIB: ctypes.CDLL | None = None


class ExtensionNotBuiltError(RuntimeError):
    """libcie_attn.so is missing: run build_ext.py (or __graft_entry__.build())."""


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load the library once and attach the C signatures."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ExtensionNotBuiltError(
            f"CUDA extension not built: {p} is missing "
            "(run `python custom-inference-engine_b200/build_ext.py`)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def last_error(lib: ctypes.CDLL | None = None) -> str:
    lib = lib or load()
    buf = ctypes.create_string_buffer(512)
    lib.cie_get_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def strides3(strides) -> ctypes.Array:
    arr = (ctypes.c_int64 * 3)(*[int(s) for s in strides])
    return arr


def check(rc: int, what: str) -> None:
    """Map a cie_status to the exception types of the reference entry points."""
    if rc == CIE_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (CIE_ERR_INVALID, CIE_ERR_WORKSPACE):
        raise ValueError(msg)
    if rc == CIE_ERR_UNSUPPORTED:
        raise ValueError(msg)
    raise RuntimeError(msg)


DEFAULT_WAIT_LIMIT_NS = 2_000_000_000


def set_wait_limit(limit_ns: int) -> int:
    """Set the in-kernel pipeline wait limit on the current device; returns the old one."""
    lib = load()
    prev = ctypes.c_uint64(0)
    check(lib.cie_set_wait_limit(ctypes.c_uint64(int(limit_ns)), ctypes.byref(prev)),
          "cie_set_wait_limit")
    return int(prev.value)


def device_status(stream: int = 0, clear: bool = True) -> int:
    """Read (and by default clear) the per-device status word; synchronizes."""
    lib = load()
    out = ctypes.c_int(0)
    rc = lib.cie_device_status(ctypes.byref(out), 1 if clear else 0, ctypes.c_void_p(stream))
    check(rc, "cie_device_status")
    return out.value
