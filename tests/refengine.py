"""Test scaffolding: the reference engine, unmodified, on top of this repo's kernels.

The reference (yuvvantalreja/Custom-Inference-Engine) is a Python package whose
``engine`` and ``kernels`` packages share their names with this repo's. Its
installed copy (``python -m pip install --no-deps --target baseline/_ref <ref>``,
or any directory named by ``CIE_REFERENCE_ENGINE``) is composed *behind* this
repo's packages: its directories are appended to the ``__path__`` of this repo's
``engine`` and ``kernels`` packages, so

* ``engine.attention``, ``engine.cache.*``, ``kernels.flash_attention`` and
  ``kernels.int8_matmul`` resolve to this repo (they exist here and come first);
* ``engine.model.*``, ``engine.decode.*``, ``engine.quant.*``, ``engine.config``,
  ``engine.runtime``, ``engine.dtype`` and ``kernels.ref`` resolve to the
  reference, byte for byte as it ships.

That is exactly the drop-in claim: the reference's ``TransformerLM``,
``Attention.forward`` (engine/model/block.py:39-75), ``generate``
(engine/decode/base_loop.py:12) and ``speculative_generate``
(engine/decode/speculative.py:47) import this repo's attention and cache by
their own import statements. Nothing from the reference is copied into the repo.
"""

from __future__ import annotations

import os
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "custom-inference-engine_b200"
ENV = "CIE_REFERENCE_ENGINE"


def reference_root() -> Path | None:
    """Directory holding the reference's ``engine`` and ``kernels`` packages, or None."""
    cands = []
    if os.environ.get(ENV):
        cands.append(Path(os.environ[ENV]))
    cands.append(REPO / "baseline" / "_ref")
    for c in cands:
        if (c / "engine" / "model" / "block.py").is_file() and (c / "kernels" / "ref").is_dir():
            return c
    return None


def compose(root: Path) -> None:
    """Put the reference's packages behind this repo's (idempotent)."""
    import engine
    import kernels

    for pkg, sub in ((engine, "engine"), (kernels, "kernels")):
        d = str(root / sub)
        if d not in pkg.__path__:
            pkg.__path__.append(d)


def origin(module) -> str:
    """'repo' or 'reference' for an imported module."""
    f = Path(module.__file__).resolve()
    return "repo" if PKG in f.parents else "reference"
