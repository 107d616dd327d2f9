"""Build ``libmoe_b200.so`` from ``csrc/*.cu`` with nvcc for sm_100a.

Each translation unit compiles to ``_build/*.o`` in parallel; the shared
library links the CUDA runtime statically and exports only the ``extern "C"``
entry points of ``include/moe_b200.h`` (every other symbol, the runtime's
included, stays local so it cannot interpose with another CUDA runtime in the
same process, such as PyTorch's).
"""
from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
ROOT = PKG.parent.parent
INCLUDE = ROOT / "include"
BUILD = PKG.parent / "_build"
LIB = PKG / "libmoe_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the B200 library cannot be built")
    return cand


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + \
        sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build_library(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile and link the library if any source is newer than it."""
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    exe = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = BUILD / (src.stem + ".o")
        cmd = [exe, *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stdout + r.stderr

    workers = max(1, min(len(_sources()), os.cpu_count() or 1))
    with ThreadPoolExecutor(workers) as pool:
        results = list(pool.map(compile_one, _sources()))
    if verbose or ptxas_info:
        for obj, log in results:
            if log.strip():
                print(f"--- {obj.name}\n{log}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [exe, *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--exclude-libs,ALL",
           "-o", str(tmp), *[str(o) for o, _ in results]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys
    print(build_library(force="--force" in sys.argv, verbose=True,
                        ptxas_info="--ptxas" in sys.argv))
