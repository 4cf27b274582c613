"""RMSNorm fused into the decode GEMV (nf4b_gemm_opts.norm_weight; B200 only).

The fused launch stages x in shared memory, normalises it there with
nf4b_rms_norm's arithmetic and multiplies the normalised x, so it must equal
``fusedops.rms_norm`` followed by the plain (or gated) GEMV bit for bit; those
two are checked against the oracle in test_gpu_kernels / test_gpu_gated.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.helpers import make_linear, randn_bf16
from ttspipe_b200 import _lib, fusedops, nf4gemv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available() and nf4gemv.install()


def norm_weight(k, seed):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("n,k,nested", [(6144, 2560, True), (9728, 2560, False), (2560, 4096, True),
                                        (2560, 9728, True), (200, 384, True)])
@pytest.mark.parametrize("rows", [1, 2, 4])
def test_fused_norm_equals_norm_then_matmul(n, k, nested, rows):
    if rows * k * 2 > nf4gemv.NORM_X_MAX:
        pytest.skip("x larger than the staging limit")
    lin = make_linear(n, k, seed=n + k + rows, nested=nested)
    nw = norm_weight(k, seed=rows)
    x = randn_bf16((rows, k), seed=7 * rows + k, device="cuda") * 3
    for eps in (1e-6, 1e-5):
        want = nf4gemv.matmul(lin, fusedops.rms_norm(x, nw, eps))
        got = nf4gemv.matmul(lin, x, norm=(nw, eps))
        assert got is not None
        assert torch.equal(got, want)


@pytest.mark.parametrize("rows", [1, 3])
def test_fused_norm_with_residual_epilogue(rows):
    lin = make_linear(2560, 2560, seed=5)
    nw = norm_weight(2560, seed=6)
    x = randn_bf16((rows, 2560), seed=8, device="cuda")
    res = randn_bf16((rows, 2560), seed=9, device="cuda")
    want = nf4gemv.matmul(lin, fusedops.rms_norm(x, nw, 1e-6), epi=nf4gemv.EPI_RESIDUAL, operand=res)
    got = nf4gemv.matmul(lin, x, epi=nf4gemv.EPI_RESIDUAL, operand=res, norm=(nw, 1e-6))
    assert torch.equal(got, want)


@pytest.mark.parametrize("rows", [1, 2, 4])
def test_fused_norm_gated(rows):
    w1, w3 = make_linear(9728, 2560, seed=11), make_linear(9728, 2560, seed=12)
    nw = norm_weight(2560, seed=13)
    h = randn_bf16((rows, 2560), seed=14 + rows, device="cuda") * 5
    want = nf4gemv.matmul_gated(w1, w3, fusedops.rms_norm(h, nw, 1e-6))
    got = nf4gemv.matmul_gated(w1, w3, h, norm=(nw, 1e-6))
    assert torch.equal(got, want)


def test_fused_norm_repeated_launches_are_identical():
    lin = make_linear(6144, 2560, seed=21)
    nw = norm_weight(2560, seed=22)
    x = randn_bf16((1, 2560), seed=23, device="cuda")
    first = nf4gemv.matmul(lin, x, norm=(nw, 1e-6))
    for _ in range(5):
        assert torch.equal(nf4gemv.matmul(lin, x, norm=(nw, 1e-6)), first)


def test_fused_norm_outside_the_staging_limit_is_declined():
    nw = norm_weight(2560, seed=32)
    lin = make_linear(256, 2560, seed=31)
    x9 = randn_bf16((9, 2560), seed=33, device="cuda")
    assert nf4gemv.matmul(lin, x9, norm=(nw, 1e-6)) is None       # 9 rows: the GEMM
    lin_big = make_linear(256, 12288, seed=34)
    x_big = randn_bf16((8, 12288), seed=35, device="cuda")           # 192 KB of x
    assert nf4gemv.matmul(lin_big, x_big, norm=(norm_weight(12288, 36), 1e-6)) is None
    lin_odd = make_linear(256, 2688, seed=37)                        # k_in % 256 != 0: no register-fed kernel
    x5 = randn_bf16((5, 2688), seed=38, device="cuda")               # 5 rows: the block kernel
    assert nf4gemv.matmul(lin_odd, x5, norm=(norm_weight(2688, 39), 1e-6)) is None
    # the C ABI itself refuses rather than computing without the norm
    L = _lib.lib()
    desc = lin._nf4_fast["desc"]
    need = int(L.nf4b_gemm_workspace_size(ctypes.byref(desc), 9))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    y = torch.empty(9, 256, dtype=torch.bfloat16, device="cuda")
    opts = _lib.GemmOpts(None, None, nw.data_ptr(), 1e-6)
    st = L.nf4b_gemm_ex(ctypes.byref(desc), x9.data_ptr(), y.data_ptr(), 9, 0, None, ws.data_ptr(), ws.numel(),
                        ctypes.byref(opts), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.NF4B_ERR_SHAPE
