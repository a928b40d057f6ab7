"""Build libcie_attn.so in-tree with nvcc for sm_100a.

The library is one translation unit (csrc/libcie_attn.cu) and is written to
kernels/libcie_attn.so next to the ctypes loader, so it travels with the
source tree. Run as ``python build_ext.py`` or call ``build()``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
OUT = PKG_ROOT / "kernels" / "libcie_attn.so"
REPO_ROOT = PKG_ROOT.parent

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    f"-I{REPO_ROOT / 'include'}",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) +
                  [REPO_ROOT / "include" / "cie_attn.h"])


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    mtime = OUT.stat().st_mtime
    return all(src.stat().st_mtime <= mtime for src in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than the built .so."""
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "libcie_attn.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
