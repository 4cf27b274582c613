"""The tcgen05 GEMM (every call of more than 8 activation rows; here 33..1024
rows: batched decode M=64 and prefill M=256..1024, BASELINE config 3, and
ragged counts) against the oracle (B200 only). 9-32 rows through the same
GEMM are in test_gpu_kernels.py::test_rows_match_the_oracle.

Its dequantised tiles are bit-exact bf16(NF4[q] * scale), so its outputs
differ from the oracle's exactly-accumulated product only by fp32
accumulation order and the final bf16 rounding.
"""

from __future__ import annotations

import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import make_linear, oracle_dequant, randn_bf16, to_bits
from tests.test_gpu_kernels import S2PRO, check_epilogue, check_matmul
from ttspipe_b200 import _lib, fusedops, nf4gemv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available() and nf4gemv.install() and fusedops.install()


@pytest.mark.parametrize("rows", [33, 64, 70, 100, 256])
@pytest.mark.parametrize("shape", [(6144, 2560), (2560, 9728), (1544, 2560)])
def test_rows_match_the_oracle(shape, rows):
    layer = make_linear(*shape, seed=shape[0] + rows)
    x = randn_bf16((1, rows, shape[1]), seed=6000 + rows, device="cuda")
    y = layer(x)
    assert y.shape == (1, rows, shape[0])
    check_matmul(y, x, layer)
    assert _lib.lib().nf4b_device_error(0) == 0


@pytest.mark.parametrize("rows", [64, 256, 512, 1024])
@pytest.mark.parametrize("idx", [0, 1, 2, 3, 4, 5, 6])
def test_config3_projections(idx, rows):
    """All seven S2-Pro projections (q, k, v, o, gate, up, down) at BASELINE
    config 3's batched-decode and prefill row counts; the narrow k and v
    (1024x2560) take their own tile height at M >= 128."""
    out_f, in_f = S2PRO[idx]
    layer = make_linear(out_f, in_f, seed=100 + idx)
    x = randn_bf16((rows, in_f), seed=1000 + rows, device="cuda")
    y = nf4gemv.matmul(layer, x)
    check_matmul(y, x, layer)


@pytest.mark.parametrize("shape", [(13, 64), (48, 128), (16, 64), (100, 192), (17, 256)])
@pytest.mark.parametrize("rows", [40, 130])
def test_tiny_and_ragged_shapes(shape, rows):
    layer = make_linear(*shape, seed=3 * shape[0] + rows)
    x = randn_bf16((rows, shape[1]), seed=7000 + rows, device="cuda")
    y = nf4gemv.matmul(layer, x)
    check_matmul(y, x, layer)


@pytest.mark.parametrize("rows", [40, 300])
@pytest.mark.parametrize("epi", ["residual", "gate"])
def test_fused_epilogues(epi, rows):
    layer = make_linear(2560, 9728, seed=11 + rows)
    x = randn_bf16((rows, 9728), seed=5000 + rows, device="cuda")
    check_epilogue(layer, x, epi)


@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("bs", [64, 128, 256])
def test_blocksizes_and_plain_scales(nested, bs):
    layer = make_linear(1024, 2560, seed=bs, nested=nested, blocksize=bs)
    x = randn_bf16((96, 2560), seed=9000 + bs, device="cuda")
    y = nf4gemv.matmul(layer, x)
    check_matmul(y, x, layer)


def test_repeated_calls_are_deterministic():
    layer = make_linear(9728, 2560, seed=5)
    x = randn_bf16((300, 2560), seed=6, device="cuda")
    a = nf4gemv.matmul(layer, x)
    b = nf4gemv.matmul(layer, x)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("n,k,rows", [(2560, 4096, 64), (2560, 9728, 64), (6144, 2560, 64), (1024, 2560, 64),
                                      (1024, 2560, 40), (2560, 4096, 33)])
def test_split_k_matches_the_unsplit_gemm(n, k, rows):
    """Given a workspace the GEMM splits the k range across CTAs when its 64-row
    tiles cannot fill the GPU (batched decode, M <= 64); the splits' sums (in
    split order, so repeatable) equal the one-pass GEMM up to fp32 summation
    order, and the workspace's tile counters are left at zero."""
    import ctypes

    lin = make_linear(n, k, seed=n + k + rows)
    x = randn_bf16((rows, k), seed=7000 + rows, device="cuda")
    L = _lib.lib()
    desc = lin._nf4_fast["desc"]
    need = int(L.nf4b_gemm_workspace_size(ctypes.byref(desc), rows))
    assert need > 0, "a 148-SM B200 splits this shape"
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    y_split = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    y_again = torch.empty_like(y_split)
    y_one = torch.empty_like(y_split)
    assert L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), y_split.data_ptr(), rows, 0, None, ws.data_ptr(), need, st) == 0
    assert L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), y_again.data_ptr(), rows, 0, None, ws.data_ptr(), need, st) == 0
    assert L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), y_one.data_ptr(), rows, 0, None, None, 0, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(y_split, y_again)
    assert int(ws[:4096].count_nonzero()) == 0
    got, one = orc.bf16_to_f32(to_bits(y_split)), orc.bf16_to_f32(to_bits(y_one))
    # the fp32 sums differ only in order (~1e-5 absolute here): after the bf16
    # rounding at most one ulp apart, or a hair apart near zero
    import numpy as np
    rms = float(np.sqrt((one.astype(np.float64) ** 2).mean()))
    assert np.all(np.abs(got - one) <= np.maximum(np.abs(got), np.abs(one)) * 2.0 ** -7 + 1e-4 * rms)
    check_matmul(y_split.view(1, rows, n), x.view(1, rows, k), lin)
    check_matmul(y_one.view(1, rows, n), x.view(1, rows, k), lin)
    assert L.nf4b_device_error(0) == 0
