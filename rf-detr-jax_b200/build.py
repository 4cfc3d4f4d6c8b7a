"""Build recipe for the native library ``librfdetr_b200.so`` (sm_100a only).

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` and links one shared library next to this
file, so it travels with the source tree.  Objects go to ``_build/``.  Run as
``python rf-detr-jax_b200/build.py`` or through ``__graft_entry__.build()``.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "librfdetr_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and os.path.exists(candidate):
            return candidate
    raise RuntimeError("nvcc not found")


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    mtime = os.path.getmtime(target)
    return any(os.path.getmtime(s) > mtime for s in sources)


def build(verbose: bool = False, force: bool = False) -> str:
    """Compile (incrementally) and link the library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = []
    objects = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            jobs.append([nvcc, *ARCH, *FLAGS, "-c", src, "-o", obj])
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as pool:
        results = list(pool.map(lambda cmd: subprocess.run(cmd, capture_output=True, text=True), jobs))
    for cmd, res in zip(jobs, results):
        if verbose or res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {cmd[-3]}")
    if force or jobs or _stale(LIB, objects):
        link = [nvcc, *ARCH, "-shared", "-o", LIB, *objects, "-lcudart"]
        res = subprocess.run(link, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
