"""Build ``fracture_b200/libfracture_b200.so`` in place (sm_100a).

``python -m fracture_b200.build`` (or ``__graft_entry__.build()``) compiles every
CUDA source for ``sm_100a`` with nvcc and the host C++ with g++, and links one
shared library with the CUDA runtime linked statically. Objects are cached
under ``fracture_b200/_build/`` and rebuilt when a source or header changes.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libfracture_b200.so"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = shutil.which("nvcc") or os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"] + ARCH
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", f"-I{INCLUDE}",
             f"-I{CSRC}", f"-I{CUDA_HOME}/include"]


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def _compile(src: Path, deps: list[Path], verbose: bool) -> Path:
    obj = BUILD / (src.name + ".o")
    if not _stale(obj, src, deps):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    deps = _headers()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, deps, verbose), sources))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(LIB), *map(str, objs), "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
        _check_defined(LIB)
    return LIB


def _check_defined(lib: Path) -> None:
    """A shared library links with undefined symbols; fail the build if one of this library's own
    (namespace fb or an fb_/launch_ entry point) is left undefined, instead of at first call."""
    r = subprocess.run(["nm", "-D", "--undefined-only", str(lib)], capture_output=True, text=True)
    if r.returncode != 0:
        return  # no nm: nothing to check with
    missing = [ln.split()[-1] for ln in r.stdout.splitlines()
               if ln.split() and ln.split()[-1].startswith(("_ZN2fb", "fb_", "launch_"))]
    if missing:
        lib.unlink()
        raise RuntimeError("undefined library symbols: " + ", ".join(missing))


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
