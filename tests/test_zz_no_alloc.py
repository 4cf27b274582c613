"""nf4b_gemm_noalloc: the decode GEMV for callers that cannot allocate.

Some hosts of this library cannot hand the GEMV a workspace: an audio
callback that must never enter an allocator, a cgo or JNI host that only holds
raw device pointers owned by another runtime, a recording CUDA graph. For
them the library carries its own fixed scratch array on every device, and
nf4b_gemm_noalloc uses it instead of a caller-provided workspace. This file
checks, through the C ABI as such a caller would use it, that two calls in a
row give what nf4b_gemm gives with a workspace, and that a call too large for
the built-in scratch is refused with a clear error instead of overrunning it.

It is collected last on purpose (a run that stops at the first failure has
then already run everything else), and it must pass both on its own in a fresh
process and after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import make_linear, randn_bf16
from tests.test_gpu_kernels import check_matmul
from ttspipe_b200 import _lib, nf4gemv

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 4 << 20   # NF4B_NOALLOC_SCRATCH_BYTES in include/nf4b200.h


def _with_workspace(desc, x, rows, n):
    """The existing entry point, with a workspace this test allocates."""
    L = _lib.lib()
    need = int(L.nf4b_gemm_workspace_size(ctypes.byref(desc), rows))
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    y = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    st = L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), rows, 0, None,
                     ws.data_ptr(), need, None)
    assert st == 0, _lib.last_error()
    return y


def _noalloc(desc, x, rows, n, epi=0, operand=None):
    y = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    st = _lib.lib().nf4b_gemm_noalloc(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), rows, epi,
                                      None if operand is None else operand.data_ptr(), None)
    return st, y


@pytest.mark.parametrize("shape,rows", [((9728, 2560), 1), ((6144, 2560), 3), ((2560, 9728), 1),
                                        ((1544, 2560), 9)])
def test_noalloc_gives_what_the_workspace_entry_point_gives(shape, rows):
    assert nf4gemv.available()
    layer = make_linear(*shape, seed=4242 + rows)
    desc = layer._nf4_fast["desc"]
    x = randn_bf16((rows, shape[1]), seed=4343 + rows, device="cuda")
    want = _with_workspace(desc, x, rows, shape[0])
    for _ in range(2):   # two calls in a row share, and must re-clear, the scratch
        st, got = _noalloc(desc, x, rows, shape[0])
        assert st == 0, _lib.last_error()
        torch.cuda.synchronize()
        check_matmul(got, x, layer)                     # the suite's tolerance
        assert torch.equal(got, want)                   # and the same bits
    assert _lib.lib().nf4b_device_error(0) == 0


def test_noalloc_residual_epilogue():
    layer = make_linear(2560, 4096, seed=11)
    desc = layer._nf4_fast["desc"]
    x = randn_bf16((1, 4096), seed=12, device="cuda")
    r = randn_bf16((1, 2560), seed=13, device="cuda")
    want = nf4gemv.matmul(layer, x, epi=nf4gemv.EPI_RESIDUAL, operand=r)
    for _ in range(2):
        st, got = _noalloc(desc, x, 1, 2560, nf4gemv.EPI_RESIDUAL, r)
        assert st == 0, _lib.last_error()
        assert torch.equal(got, want)


def test_noalloc_refuses_a_call_larger_than_its_scratch():
    """A decode GEMV (1..8 rows) whose partial sums exceed the scratch: 32768
    output features at 8 rows (~6.4 MB of slots)."""
    layer = make_linear(32768, 4096, seed=5)
    desc = layer._nf4_fast["desc"]
    rows = 8
    assert _lib.lib().nf4b_gemm_workspace_size(ctypes.byref(desc), rows) > NOALLOC_SCRATCH_BYTES
    x = randn_bf16((rows, 4096), seed=6, device="cuda")
    y = torch.full((rows, 32768), 7.0, dtype=torch.bfloat16, device="cuda")
    st = _lib.lib().nf4b_gemm_noalloc(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), rows, 0,
                                      None, None)
    assert st == -5
    assert "scratch" in _lib.last_error()
    torch.cuda.synchronize()
    assert torch.all(y == 7.0)   # nothing was launched


def test_noalloc_gemm_splits_its_k_range_in_the_scratch():
    """More than 8 rows run the tensor-core GEMM. Where its split-K partial
    sums fit the built-in scratch (1024x2560 at 64 rows splits the k range
    across CTAs), it splits exactly as nf4b_gemm does with a workspace, so the
    two give the same bits - twice in a row on the shared scratch."""
    layer = make_linear(1024, 2560, seed=21)
    desc = layer._nf4_fast["desc"]
    rows = 64
    need = int(_lib.lib().nf4b_gemm_workspace_size(ctypes.byref(desc), rows))
    assert 0 < need <= NOALLOC_SCRATCH_BYTES, "this call must take the split path"
    x = randn_bf16((rows, 2560), seed=22, device="cuda")
    want = _with_workspace(desc, x, rows, 1024)
    for _ in range(2):
        st, got = _noalloc(desc, x, rows, 1024)
        assert st == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    check_matmul(got, x, layer)
    assert np.isfinite(got.float().cpu().numpy()).all()


def test_noalloc_gemm_too_large_for_the_scratch_runs_unsplit():
    """A GEMM whose split-K sums would not fit the scratch (2560x9728 at 256
    rows splits three ways, ~7.9 MB) is not refused: it runs unsplit, which is
    what nf4b_gemm does when it is given no workspace."""
    layer = make_linear(2560, 9728, seed=31)
    desc = layer._nf4_fast["desc"]
    rows = 256
    L = _lib.lib()
    assert int(L.nf4b_gemm_workspace_size(ctypes.byref(desc), rows)) > NOALLOC_SCRATCH_BYTES
    x = randn_bf16((rows, 9728), seed=32, device="cuda")
    want = torch.empty((rows, 2560), dtype=torch.bfloat16, device="cuda")
    assert L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), want.data_ptr(), rows, 0, None, None, 0, None) == 0
    for _ in range(2):
        st, got = _noalloc(desc, x, rows, 2560)
        assert st == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    check_matmul(got, x, layer)
    assert L.nf4b_device_error(0) == 0
