"""Build ``libnf4b200.so`` in-tree with nvcc for sm_100a.

Each ``csrc/*.cu`` is compiled separately (in parallel) with
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared library
next to this file, so it travels with the source tree. The CUDA runtime is
linked statically: the library carries its own runtime and shares only the
driver (and therefore the current context and streams) with the PyTorch that
calls it. ``python -m ttspipe_b200.build`` rebuilds when a source is newer
than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libnf4b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-O3"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise FileNotFoundError("nvcc not found (set NVCC or install CUDA 12.9)")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every kernel source and link the shared library. Returns its path."""
    if not force and up_to_date() and not ptxas_info:
        return LIB
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    env = dict(os.environ, TMPDIR=str(BUILD))  # nvcc's intermediate files stay in the build folder

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = BUILD / (src.stem + ".o")
        cmd = [cc, *ARCH, *NVCC_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True, env=env)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources()))
    if ptxas_info:
        for _, err in results:
            sys.stdout.write(err)
    objs = [str(o) for o, _ in results]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                ptxas_info="--ptxas" in sys.argv))
