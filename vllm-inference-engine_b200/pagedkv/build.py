"""Build the pagedkv C-ABI shared library for sm_100a with nvcc.

The library is built in-tree (``pagedkv/libpagedkv_b200.so``) from the CUDA
sources in ``../csrc`` so that it travels with the source tree; nothing is
installed into site-packages and no JIT cache is used.

    python -m pagedkv.build          # or pagedkv.build.build()
"""
from __future__ import annotations

import concurrent.futures as _cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC_DIR = PKG_DIR.parent / "csrc"
INCLUDE_DIR = PKG_DIR.parent.parent / "include"
BUILD_DIR = PKG_DIR.parent / "_build"
LIB_NAME = "libpagedkv_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-warn-spills",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the pagedkv CUDA library cannot be built")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC_DIR.glob("*.h")) + list(CSRC_DIR.glob("*.cuh")) + list(INCLUDE_DIR.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool, extra: list[str]) -> None:
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout, res.stderr, sep="\n", flush=True)


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libpagedkv_b200.so in-tree."""
    extra = list(extra_flags or [])
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    objs: list[Path] = []
    jobs = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or extra or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    if jobs:
        with _cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, verbose, extra) for s, o in jobs]
            for f in futs:
                f.result()
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def ptxas_report(src_name: str) -> str:
    """Registers / spills / shared memory of one source file (``-Xptxas -v``)."""
    src = CSRC_DIR / src_name
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-Xptxas", "-v", "-I", str(INCLUDE_DIR), "-c", str(src), "-o", os.devnull]
    res = subprocess.run(cmd, capture_output=True, text=True)
    return res.stdout + res.stderr


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "--ptxas":
        print(ptxas_report(sys.argv[2]))
    else:
        print(build(verbose=True, force="--force" in sys.argv))
