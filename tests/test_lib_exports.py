"""CPU checks of the C-ABI boundary: the library builds, loads without a GPU,
exports every function include/cie_attn.h declares, and the ctypes table in
kernels/_lib.py agrees with the header. No kernel is launched."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from tests.conftest import PKG, REPO


def _header_functions() -> dict[str, int]:
    text = (REPO / "include" / "cie_attn.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"^\s*(?:const\s+)?\w+\s*\*?\s*(cie_\w+)\s*\((.*?)\);", text, re.S | re.M):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else len(args.split(","))
    return out


@pytest.fixture(scope="module")
def lib():
    import build_ext

    build_ext.build()
    from kernels import _lib

    return _lib.load()


def test_header_declares_the_boundary():
    fns = _header_functions()
    for name in ("cie_prefill_attn", "cie_paged_attn", "cie_gather_kv", "cie_rope_append",
                 "cie_rope", "cie_device_status", "cie_get_last_error", "cie_version"):
        assert name in fns


def test_library_exports_every_header_symbol(lib):
    for name in _header_functions():
        assert hasattr(lib, name), name


def test_ctypes_signatures_match_header(lib):
    from kernels import _lib

    fns = _header_functions()
    assert set(fns) == set(_lib.SIGNATURES)
    for name, nargs in fns.items():
        assert len(_lib.SIGNATURES[name][1]) == nargs, name


def test_host_only_calls_work_without_gpu(lib):
    from kernels import _lib

    assert lib.cie_version().decode().startswith("cie_attn")
    # workspace queries are pure host arithmetic
    ws = lib.cie_paged_attn_workspace(64, 32, 8, 1, 64, 16, 513, 0)
    assert ws > 0
    assert lib.cie_paged_attn_workspace(1, 32, 8, 1, 64, 16, 1, 0) == 0
    assert lib.cie_prefill_attn_workspace(4, 32, 8, 8192, 8192, 128, 0, 0) == 0
    assert lib.cie_prefill_attn_workspace(4, 32, 8, 8192, 8192, 128, 0, 1) >= 4 * 8 * 8192 * 128 * 2
    # argument validation happens before any CUDA call and reports a message
    s = (ctypes.c_int64 * 3)(0, 0, 0)
    rc = lib.cie_paged_attn(None, None, None, None, None, None, 1, 32, 8, 1, 64, 1, 16, 1, s, s,
                            1.0, 1, 0, None, None, 0, 0, None, 0, None)
    assert rc == _lib.CIE_ERR_INVALID
    assert "null" in _lib.last_error(lib)
    p = ctypes.c_void_p(16)
    rc = lib.cie_prefill_attn(p, p, p, p, 1, 6, 4, 8, 8, 64, s, s, s, s, 1.0, 1, 0, None, None, 0,
                              0, 0, None, 0, None)
    assert rc == _lib.CIE_ERR_INVALID and "multiple" in _lib.last_error(lib)
    rc = lib.cie_prefill_attn(p, p, p, p, 1, 4, 4, 8, 8, 96, s, s, s, s, 1.0, 1, 0, None, None, 0,
                              0, 0, None, 0, None)
    assert rc == _lib.CIE_ERR_UNSUPPORTED


def test_built_for_sm100a_only():
    src = (PKG / "build_ext.py").read_text()
    assert "arch=compute_100a,code=sm_100a" in src
