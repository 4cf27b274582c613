"""Failure detection on the device (B200 only), without faulting anything.

Every wait in the library's kernels is bounded and reports through
nf4b_device_error instead of hanging or trapping. This makes one such wait run
out on purpose in the allowed way - a flag that nothing sets, with a short
limit - through the test hook nf4b_debug_decode_step: the boundary before
`stall_job` waits for a flag no launch writes. The test then checks that the
launch returned, that the error word says which wait gave up, that the CUDA
context is still usable, and that the next launch on the same workspace gives
the same bits as before the failure (the step's launch counter gives every
launch a new flag space, so nothing the abandoned launch wrote is read).
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
