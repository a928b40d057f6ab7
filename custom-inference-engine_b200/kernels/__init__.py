"""B200 (sm_100a) attention kernels behind the reference's kernel entry points.

Mirrors the reference package layout (kernels/__init__.py, kernels/flash_attention.py):
``flash_attention`` keeps its signature and error behaviour; the Triton JIT is
replaced by hand-written CUDA in libcie_attn.so, loaded through ctypes. There is
no CPU or Triton fallback: every entry point raises when CUDA or the built
library is missing.
"""

from __future__ import annotations

import torch

from kernels import _lib


def require_extension() -> None:
    """Verify CUDA and the native library are available before running a kernel.

    Counterpart of ``require_triton`` (reference kernels/__init__.py:14-22).
    """
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required but not available")
    try:
        _lib.load()
    except _lib.ExtensionNotBuiltError as e:
        raise RuntimeError(str(e)) from e


# The entry points live in kernels.flash_attention, as in the reference
# (``from kernels.flash_attention import flash_attention``); the package does not
# re-export them so that ``kernels.flash_attention`` stays the module.
from kernels.rope import build_rope_cache  # noqa: E402

__all__ = ["require_extension", "build_rope_cache"]
