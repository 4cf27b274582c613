"""Build the reference's own CPU NF4 kernels into ``oracle/_ref/`` - TEST INFRASTRUCTURE.

The reference ships its CPU NF4 path as a C++ source string inside
``app/engine/nf4cpu.py`` (``_SOURCE``, lines 51-781: ``nf4_gemv``, ``nf4_amx``,
``decode_block``, ``prefill_block``). This recipe reads that string from the
read-only reference checkout, compiles it with ``g++`` through
``torch.utils.cpp_extension.load_inline`` into a scratch directory under /tmp,
and copies only the resulting extension module into ``oracle/_ref/``. Nothing
from the reference is written into the repository's tracked files.

The extension is used (a) by ``tests/golden/make_golden.py`` to produce the
golden fixtures that pin ``oracle/nf4_oracle.py``, and (b) by ``bench.py`` as
the timed CPU baseline (``cpu_baseline.kind == "reference"``) on hosts whose
CPU has AVX512-BF16.

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
    with tempfile.TemporaryDirectory(prefix="nf4cpu_ref_") as tmp:
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


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
