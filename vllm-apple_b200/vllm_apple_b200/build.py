"""Build the sm_100a C-ABI library ``libvllm_apple_b200.so`` in-tree.

``python -m vllm_apple_b200.build`` (or ``build()``) compiles every
``csrc/*.cu`` with nvcc for ``sm_100a`` into ``<pkg>/_lib/``.  Object files go
to ``vllm-apple_b200/_build/``.  The library links the CUDA runtime
statically, so it loads in any process (with or without torch) and exports
only the ``va_*`` symbols declared in ``include/vllm_apple_b200.h``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
PROJ_DIR = PKG_DIR.parent                      # vllm-apple_b200/
REPO_DIR = PROJ_DIR.parent
CSRC = PROJ_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
OBJ_DIR = PROJ_DIR / "_build"
LIB_DIR = PKG_DIR / "_lib"
LIB_NAME = "libvllm_apple_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile (incrementally) and return the path of the shared library."""
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
             "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]

    def compile_one(src: Path):
        obj = OBJ_DIR / (src.stem + ".o")
        if not force and not ptxas_verbose and not _stale(obj, [src, *headers]):
            return obj, ""
        cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources))
    objs = [o for o, _ in results]
    if verbose or ptxas_verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    lib = LIB_DIR / LIB_NAME
    if force or _stale(lib, objs):
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv, ptxas_verbose="-v" in sys.argv))
