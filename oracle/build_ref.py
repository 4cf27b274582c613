"""Build the reference's own CPU NF4 kernels into ``oracle/_ref/`` - TEST INFRASTRUCTURE.

The reference ships its CPU NF4 path as a C++ source string inside
``app/engine/nf4cpu.py`` (``_SOURCE``, lines 51-781: ``nf4_gemv``, ``nf4_amx``,
``decode_block``, ``prefill_block``). This recipe reads that string from the
read-only reference checkout, compiles it with ``g++`` through
``torch.utils.cpp_extension.load_inline`` into a scratch directory inside
``oracle/_ref/`` (removed afterwards; the compilers' temporary files go there too),
and copies only the resulting extension module into ``oracle/_ref/``. Nothing
from the reference is written into the repository's tracked files.

The extension is used (a) by ``tests/golden/make_golden.py`` to produce the
golden fixtures that pin ``oracle/nf4_oracle.py``, and (b) by ``bench.py`` as
the timed CPU baseline (``cpu_baseline.kind == "reference"``) on hosts whose
CPU has AVX512-BF16.

``build_gpu()`` does the same for the reference's GPU kernel: the NVRTC
source string of ``nf4_mma`` in ``app/engine/nf4gemv.py`` is read in place,
instantiated as the reference's own build does, and compiled with nvcc for
sm_100a (with a small launcher of this repository's) into
``oracle/_ref/nf4mma_ref.so``, which ``bench.py`` times on the B200 beside this
build's kernels.

The image's default ``/opt/gcc`` g++ cannot link ``-fopenmp`` (no
libgomp.spec), so ``/usr/bin/g++`` is used.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import shutil
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
MODULE = "nf4cpu_ref"
FUNCTIONS = ["nf4_gemv", "nf4_amx", "amx_available", "decode_block", "prefill_block"]


class _scratch:
    """A temporary build directory inside oracle/_ref/ that is also TMPDIR
    while it lives, so neither the build nor the compilers write outside the
    repository."""

    def __init__(self, prefix: str):
        REF_DIR.mkdir(parents=True, exist_ok=True)
        self._dir = tempfile.TemporaryDirectory(prefix=prefix, dir=REF_DIR)
        self._old = None

    def __enter__(self) -> str:
        path = self._dir.__enter__()
        self._old = os.environ.get("TMPDIR")
        os.environ["TMPDIR"] = path
        return path

    def __exit__(self, *exc):
        if self._old is None:
            os.environ.pop("TMPDIR", None)
        else:
            os.environ["TMPDIR"] = self._old
        return self._dir.__exit__(*exc)


def so_path() -> Path | None:
    """The built extension, if present."""
    hits = sorted(REF_DIR.glob(f"{MODULE}*.so"))
    return hits[0] if hits else None


def cpu_supported() -> bool:
    """The reference kernels need AVX512-BW and AVX512-BF16 (nf4cpu.py:793-795)."""
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        return False
    return " avx512_bf16 " in flags and " avx512bw " in flags


def load():
    """Import the prebuilt reference extension (torch must be importable)."""
    import torch  # noqa: F401 - the extension links against libtorch

    path = so_path()
    if path is None:
        raise FileNotFoundError(f"no reference build under {REF_DIR}; run oracle/build_ref.py")
    if not cpu_supported():
        raise RuntimeError("this CPU lacks AVX512-BF16/BW; the reference kernels cannot run")
    loader = importlib.machinery.ExtensionFileLoader(MODULE, str(path))
    spec = importlib.util.spec_from_file_location(MODULE, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def reference_root() -> Path:
    """The read-only reference checkout: ``$TTSPIPE_REFERENCE`` when set, else a
    directory named ``reference`` beside this repository."""
    env = os.environ.get("TTSPIPE_REFERENCE")
    return Path(env) if env else HERE.parent.parent / "reference"


def reference_source(reference_root_dir: str | None = None) -> str:
    """The C++ source string of the reference's nf4cpu module, read in place."""
    root = Path(reference_root_dir) if reference_root_dir else reference_root()
    if not (root / "app" / "engine" / "nf4cpu.py").exists():
        raise FileNotFoundError(f"reference checkout not found at {root}")
    sys.path.insert(0, str(root))
    try:
        from app.engine import nf4cpu  # imports only logging/os/threading/pathlib
        return nf4cpu._SOURCE
    finally:
        sys.path.remove(str(root))


def build(reference_root_dir: str | None = None, verbose: bool = False) -> Path:
    """Compile the reference's nf4cpu source into oracle/_ref/. Returns the .so path."""
    from torch.utils.cpp_extension import load_inline

    source = reference_source(reference_root_dir)
    os.environ["CXX"] = "/usr/bin/g++"
    REF_DIR.mkdir(parents=True, exist_ok=True)
    with _scratch("nf4cpu_ref_") as tmp:
        ext = load_inline(
            name=MODULE,
            cpp_sources=source,
            functions=FUNCTIONS,
            extra_cflags=["-O3", "-mavx512f", "-mavx512bw", "-mavx512bf16",
                          "-mamx-tile", "-mamx-bf16", "-fopenmp"],
            extra_ldflags=["-fopenmp"],
            build_directory=tmp,
            verbose=verbose,
        )
        built = Path(ext.__file__)
        for old in REF_DIR.glob(f"{MODULE}*.so"):
            old.unlink()
        dest = REF_DIR / built.name
        shutil.copy2(built, dest)
    return dest


# --------------------------------------------------------------------------
# the reference's GPU kernel (nf4_mma), for timing beside this build's on a B200
# --------------------------------------------------------------------------

GPU_MODULE = "nf4mma_ref"
#: Instantiations the launcher serves: (inputs per launch, nested scales).
GPU_ROWS = (1, 8, 16, 32)

# A launcher of my own for the reference's kernels: one C entry point that
# picks the instantiation for (rows, nested) and launches it with the grid and
# block the reference's matmul uses (app/engine/nf4gemv.py:460-478:
# ceil(M / (16 * MT)) blocks of 32 * WARPS threads, MT and WARPS from its
# `_config`). The kernel declarations restate the argument list of the
# reference's nf4_mma (app/engine/nf4gemv.py:108-117) - the interface it is
# launched through.
_LAUNCHER = r"""
#include <cuda_runtime.h>
#define DECL(name) extern "C" __global__ void name(const half_t*, const uint4*, const unsigned char*, \
    const float*, const float*, half_t*, const float*, float, int, int, int, int, int, int, const half_t*, int);
@DECLS@
extern "C" int nf4mma_ref_launch(int rows, int nested, const void* X, const void* W, const void* A8,
                                 const void* AMAX, const void* CODE2, void* Y, const void* LUT, float offset,
                                 int M, int K, int nblk, int bs_shift, int bs2_shift, const void* R, int epi,
                                 void* stream) {
  @DISPATCH@
  return -1;
}
"""


def gpu_so_path() -> Path | None:
    hits = sorted(REF_DIR.glob(f"{GPU_MODULE}*.so"))
    return hits[-1] if hits else None


def build_gpu(reference_root_dir: str | None = None, verbose: bool = False) -> Path:
    """Compile the reference's NVRTC kernel nf4_mma (app/engine/nf4gemv.py:94-231,
    with nvrtc.PRELUDE) for sm_100a with nvcc, using the options its own build
    passes NVRTC (app/engine/nvrtc.py: --use_fast_math, default device
    functions), one instantiation per (rows, nested) as its `_config` picks,
    plus the launcher above, into oracle/_ref/nf4mma_ref.so."""
    import subprocess

    root = Path(reference_root_dir) if reference_root_dir else reference_root()
    sys.path.insert(0, str(root))
    try:
        from app.engine import nf4gemv as ref  # imports only ctypes/logging/threading and its nvrtc module
        source, config = ref._SOURCE, ref._config
    finally:
        sys.path.remove(str(root))
    parts, decls, dispatch = [], [], []
    for rows in GPU_ROWS:
        nt, mt, warps = config(rows)
        for nested in (0, 1):
            name = f"nf4_mma_r{rows}_n{nested}"
            body = (source.replace("__NT__", str(nt)).replace("__MT__", str(mt))
                    .replace("__WARPS__", str(warps)).replace("__NESTED__", str(nested))
                    .replace("void nf4_mma(", f"void {name}("))
            if parts:  # the prelude and helper functions once
                body = body[body.index("#define NT"):]
                body = body.replace("__device__ __forceinline__ uint pack2", f"__device__ __forceinline__ uint pack2_{name}")
                body = body.replace("pack2(", f"pack2_{name}(").replace(f"pack2_{name}_{name}", f"pack2_{name}")
            body = body.replace("#define NT", "#undef NT\n#undef MT\n#undef WARPS\n#undef NESTED\n#define NT")
            parts.append(body)
            decls.append(f"DECL({name})")
            dispatch.append(f"if (rows == {rows} && nested == {nested}) {{ {name}<<<(M + {16 * mt - 1}) / {16 * mt}, "
                            f"{32 * warps}, 0, (cudaStream_t)stream>>>((const half_t*)X, (const uint4*)W, "
                            f"(const unsigned char*)A8, (const float*)AMAX, (const float*)CODE2, (half_t*)Y, "
                            f"(const float*)LUT, offset, M, K, rows, nblk, bs_shift, bs2_shift, (const half_t*)R, epi); "
                            f"return (int)cudaGetLastError(); }}")
    launcher = _LAUNCHER.replace("@DECLS@", "\n".join(decls)).replace("@DISPATCH@", "\n  ".join(dispatch))
    REF_DIR.mkdir(parents=True, exist_ok=True)
    with _scratch("nf4mma_ref_") as tmp:
        cu = Path(tmp) / "nf4mma_ref.cu"
        cu.write_text("\n".join(parts) + launcher)
        out = REF_DIR / f"{GPU_MODULE}.so"
        cmd = [os.environ.get("NVCC", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3",
               "--use_fast_math", "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", str(cu), "-o", str(out)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on the reference kernel:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(r.stderr)
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    print(build_gpu(verbose="-v" in sys.argv))
