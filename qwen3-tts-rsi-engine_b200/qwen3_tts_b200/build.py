"""Compile the sm_100a kernels into the in-tree shared library ``libq3t_b200.so``.

The library is plain CUDA C++ with a C ABI (``include/q3t.h``); it does not link
against torch. Each ``csrc/*.cu`` compiles to an object under ``_build/`` (only
when the source or a header changed), then everything links into one ``.so``
next to this file so it travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent                 # qwen3-tts-rsi-engine_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"     # repository-level C headers
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libq3t_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the kernels")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def _compile(source: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (source.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(source), "-o", str(obj)]
    if ptxas_verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Build (incrementally) and return the path of the shared library."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    todo = [s for s in sources if force or ptxas_verbose or _stale(BUILD / (s.stem + ".o"), [s, *headers])]
    if todo:
        workers = min(len(todo), os.cpu_count() or 1)
        with concurrent.futures.ThreadPoolExecutor(workers) as pool:
            for obj, log in pool.map(lambda s: _compile(s, ptxas_verbose), todo):
                if verbose or ptxas_verbose:
                    print(f"[q3t] compiled {obj.name}", file=sys.stderr)
                    if log.strip():
                        print(log, file=sys.stderr)
    objects = [BUILD / (s.stem + ".o") for s in sources]
    if force or todo or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-cudart", "static"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
        os.replace(tmp, LIBRARY)
        if verbose:
            print(f"[q3t] linked {LIBRARY}", file=sys.stderr)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="--ptxas" in sys.argv)
