"""Where the tests find the reference engine (XVX-016/vLLM-inference-engine).

Every test that runs the reference's own Python code (its allocator, its
runner, its scheduler, its test modules) locates it here and nowhere else:

1. the directory named by the environment variable ``PAGEDKV_REFERENCE`` (a
   checkout of the reference, or a ``pip install --target`` of it), else
2. ``baseline/_ref`` at the repository root: the reference installed with
   ``pip install --target baseline/_ref``. That directory is git-ignored but
   travels with the working tree to a GPU box, so these tests run there too.

A checkout keeps the reference's test modules in ``tests/``; the install
keeps them in the package ``reference_tests``. Tests that need the reference
are skipped when neither location holds it.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO_ROOT = Path(__file__).resolve().parent.parent
ENV_VAR = "PAGEDKV_REFERENCE"


def root() -> Path | None:
    """The directory the reference's ``engine`` package is imported from."""
    env = os.environ.get(ENV_VAR)
    cands = [Path(env)] if env else []
    cands.append(REPO_ROOT / "baseline" / "_ref")
    for c in cands:
        if (c / "engine" / "kernels" / "paged_attention.py").exists():
            return c.resolve()
    return None


def available() -> bool:
    return root() is not None


def ensure_on_path() -> Path | None:
    """Put the reference's root on ``sys.path`` (first) and return it."""
    r = root()
    if r is not None and str(r) not in sys.path:
        sys.path.insert(0, str(r))
    return r


def reference_test_file(name: str) -> Path | None:
    """Path of the reference test module ``name`` (e.g.
    ``test_block_allocator.py``) in a checkout or in the install."""
    r = root()
    if r is None:
        return None
    for sub in ("tests", "reference_tests"):
        p = r / sub / name
        if p.exists():
            return p
    return None


requires_reference = pytest.mark.skipif(
    not available(), reason=f"reference not found (set {ENV_VAR} or install it into baseline/_ref)"
)
