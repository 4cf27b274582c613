"""A plain C99 host builds against ``include/nf4b200.h`` and links
``libnf4b200.so`` with no Python or torch in its process: the C ABI is usable
the way a cgo, JNI or N-API binding would use it. The library carries its own
CUDA runtime (linked statically), so nothing else needs to be on the loader's
path. Every call made is answered on the host (the version, argument and
alignment refusals), so the test needs no GPU."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

from ttspipe_b200 import _lib

INCLUDE = Path(__file__).resolve().parent.parent / "include"

C_HOST = r"""
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "nf4b200.h"

int main(void) {
  static char buf[256];
  char* p = (char*)(((uintptr_t)buf + 15) & ~(uintptr_t)15);
  nf4b_weight w;
  if (nf4b_version() < 100) return 1;
  if (nf4b_rms_norm(NULL, p, p, 1, 8, 1e-6f, NULL) != NF4B_ERR_ARG) return 2;
  if (strlen(nf4b_last_error()) == 0) return 3;
  if (nf4b_rms_norm(p + 1, p, p, 1, 8, 1e-6f, NULL) != NF4B_ERR_ALIGN) return 4;
  memset(&w, 0, sizeof w);
  if (nf4b_gemm(&w, p, p, 1, NF4B_EPI_NONE, NULL, NULL, 0, NULL) != NF4B_ERR_ARG) return 5;
  if (nf4b_gemm_workspace_size(NULL, 1) != 0) return 6;
  printf("ok %d\n", nf4b_version());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_a_plain_c_host_builds_links_and_calls_the_library(tmp_path):
    _lib.lib()  # the library is built (a clear error otherwise)
    lib_dir = _lib.LIB_PATH.resolve().parent
    src = tmp_path / "host.c"
    exe = tmp_path / "host"
    src.write_text(C_HOST)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", f"-I{INCLUDE}", str(src),
                    f"-L{lib_dir}", f"-l:{_lib.LIB_PATH.name}", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    assert run.stdout.strip() == f"ok {_lib.lib().nf4b_version()}"
