"""Failure detection on the device (B200 only), without faulting anything.

Every wait in the library's kernels is bounded and reports through
nf4b_device_error instead of hanging or trapping. This makes one such wait run
out on purpose in the allowed way - a flag that nothing sets, with a short
limit - through the test hook nf4b_debug_decode_step: the boundary before
`stall_job` waits for a flag no launch writes. The test then checks that the
launch returned, that the error word says which wait gave up, that the CUDA
context is still usable, and that the next launch on the same workspace gives
the same bits as before the failure (the step's launch counter gives every
launch a new flag space, so nothing the abandoned launch wrote is read). The
tcgen05 GEMM's waits are made to run out the same way through
nf4b_debug_gemm_hook: an activation-tile copy that is never requested.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.helpers import make_linear, randn_bf16
from ttspipe_b200 import _lib, nf4gemv

pytestmark = pytest.mark.gpu

STEP_HANDOFF_BIT = 8   # bit 3 of nf4b_device_error


def _steps():
    g = torch.Generator().manual_seed(3)
    nw = (1.0 + 0.1 * torch.randn(2560, generator=g)).to(torch.bfloat16).cuda()
    wo, w1, w3, w2 = (make_linear(2560, 4096, seed=11), make_linear(9728, 2560, seed=12),
                      make_linear(9728, 2560, seed=13), make_linear(2560, 9728, seed=14))
    attn = randn_bf16((1, 4096), seed=15, device="cuda")
    h = randn_bf16((1, 2560), seed=16, device="cuda")
    return [dict(w=wo, x=attn, epi=nf4gemv.EPI_RESIDUAL, operand=h),
            dict(w=w1, w3=w3, x=0, norm=(nw, 1e-6)),
            dict(w=w2, x=1, epi=nf4gemv.EPI_RESIDUAL, operand=0)]


@pytest.mark.parametrize("stall_job", [1, 2])
def test_a_stalled_decode_step_boundary_gives_up_and_the_next_launch_is_clean(stall_job):
    L = _lib.lib()
    assert nf4gemv.available() and L.nf4b_device_error(1) == 0
    steps = _steps()
    want = [o.clone() for o in nf4gemv.decode_step(steps)]
    torch.cuda.synchronize()

    arr, outs, keep, rows, dev = nf4gemv._chain_jobs(steps, 152)
    need = int(L.nf4b_decode_step_workspace_size(arr, len(steps), rows))
    ws = nf4gemv.step_workspace(dev, need)
    st = L.nf4b_debug_decode_step(arr, len(steps), rows, ws.data_ptr(), ws.numel(), stall_job, 200_000,
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, _lib.last_error()
    torch.cuda.synchronize()                      # the launch ended by itself
    err = L.nf4b_device_error(1)                  # reads and clears the error word
    assert err == STEP_HANDOFF_BIT, err
    assert L.nf4b_device_error(0) == 0

    # the context still works, and the next launch on the same workspace is exact
    again = nf4gemv.decode_step(steps)
    torch.cuda.synchronize()
    for a, b in zip(again, want):
        assert torch.equal(a, b)
    assert L.nf4b_device_error(0) == 0
    del keep


def test_the_hook_rejects_a_limit_outside_its_range():
    L = _lib.lib()
    steps = _steps()
    arr, outs, keep, rows, dev = nf4gemv._chain_jobs(steps, 152)
    ws = nf4gemv.step_workspace(dev, int(L.nf4b_decode_step_workspace_size(arr, len(steps), rows)))
    assert L.nf4b_debug_decode_step(arr, len(steps), rows, ws.data_ptr(), ws.numel(), 1, 0, None) == _lib.NF4B_ERR_ARG
    assert L.nf4b_debug_decode_step(arr, len(steps), rows, ws.data_ptr(), ws.numel(), 1, 3_000_000_000,
                                    None) == _lib.NF4B_ERR_ARG
    del keep


GEMM_BIT = 1   # bit 0 of nf4b_device_error


@pytest.mark.parametrize("n,k,rows", [(1024, 2560, 64), (9728, 2560, 256)])
def test_a_gemm_whose_activation_copy_never_lands_gives_up_and_the_next_call_is_exact(n, k, rows):
    """The tcgen05 GEMM (64-row tiles with split-K, two MMA issuers and the
    staged epilogue; 256-row tiles, one issuer, direct stores) through the test
    hook nf4b_debug_gemm_hook: the first k block's activation tile is never
    requested, so the barrier it would complete never does, and with a 200 us
    limit the waits on it run out. The launch returns by itself with bit 0 of
    the error word set, the context stays usable, and after the workspace is
    zeroed again (as the header asks after a non-zero error word) the next call
    gives the same bits as before the failure."""
    L = _lib.lib()
    assert nf4gemv.available() and L.nf4b_device_error(1) == 0
    lin = make_linear(n, k, seed=n + rows)
    desc = lin._nf4_fast["desc"]
    x = randn_bf16((rows, k), seed=rows, device="cuda")
    need = int(L.nf4b_gemm_workspace_size(ctypes.byref(desc), rows))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call():
        y = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
        st = L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), rows, 0, None,
                         ws.data_ptr() if need else None, need, stream)
        assert st == 0, _lib.last_error()
        return y

    want = call()
    torch.cuda.synchronize()
    try:
        assert L.nf4b_debug_gemm_hook(1, 200_000) == 0
        call()
        torch.cuda.synchronize()                  # the launch ended by itself
    finally:
        assert L.nf4b_debug_gemm_hook(0, 2_000_000_000) == 0
    err = L.nf4b_device_error(1)                  # reads and clears the error word
    assert err == GEMM_BIT, err
    assert L.nf4b_device_error(0) == 0
    ws.zero_()
    again = call()
    torch.cuda.synchronize()
    assert torch.equal(again, want)
    assert L.nf4b_device_error(0) == 0


def test_the_gemm_hook_rejects_arguments_outside_their_range():
    L = _lib.lib()
    assert L.nf4b_debug_gemm_hook(1, 0) == _lib.NF4B_ERR_ARG
    assert L.nf4b_debug_gemm_hook(1, 3_000_000_000) == _lib.NF4B_ERR_ARG
    assert L.nf4b_debug_gemm_hook(2, 1_000_000) == _lib.NF4B_ERR_ARG
