"""The tcgen05 GEMM (more than 32 activation rows: batched decode M=64 and
prefill M=256..1024) against the oracle (B200 only).

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
@pytest.mark.parametrize("idx", [0, 3, 4, 6])
def test_config3_projections(idx, rows):
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
