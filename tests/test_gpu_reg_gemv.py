"""The register-fed pair GEMV (B200 only).

Decode calls with 1 or 2 activation rows, blocksize-64 weights, k_in % 256 == 0
and 32-byte aligned packed weights run `nf4_gemv_reg_kernel`: weights loaded
straight into registers, MMA columns of (activation row, 64-block), x staged
with padding. These cases complement test_gpu_kernels / test_gpu_gated with
the variants that kernel adds: plain fp32 scales (one 8-byte pair per lane),
the gated pair with plain scales, row counts that do not fill a tile at one
activation row, and the fall-back to the TMA-ring pair kernel when the packed
weight is 16- but not 32-byte aligned.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import make_linear, oracle_dequant, randn_bf16, to_bits
from tests.test_gpu_gated import exact_gate
from ttspipe_b200 import nf4gemv
from ttspipe_b200.quant import Linear4bit, Params4bit

pytestmark = pytest.mark.gpu

GEMM_TOL = 0.02


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available() and nf4gemv.install()


def check_matmul(got, x, layer):
    w = orc.matmul_exact(to_bits(x).reshape(-1, layer.in_features), oracle_dequant(layer))
    g = orc.bf16_to_f32(to_bits(got)).reshape(w.shape)
    assert np.isfinite(g).all()
    assert orc.rms_relative_max_error(g, w) <= GEMM_TOL
    assert orc.norm_relative_error(g, w) < 5e-3


@pytest.mark.parametrize("shape", [(9728, 2560), (2560, 4096), (1544, 2560), (2560, 9728)])
@pytest.mark.parametrize("rows", [1, 2])
def test_plain_fp32_scales(shape, rows):
    layer = make_linear(*shape, seed=7 * shape[0] + rows, nested=False)
    x = randn_bf16((rows, shape[1]), seed=31 + rows, device="cuda")
    check_matmul(nf4gemv.matmul(layer, x), x, layer)


@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("rows", [1, 2])
def test_gated_pair(nested, rows):
    """Against the exact gate (each product rounded once to bf16): the gated
    launch sums W1 and W3 in its own split, so near-zero outputs with heavy
    cancellation may sit several ulps from the plain GEMV's; the error is
    bounded relative to the outputs' scale instead."""
    w1 = make_linear(9728, 2560, seed=41, nested=nested)
    w3 = make_linear(9728, 2560, seed=42, nested=nested)
    x = randn_bf16((rows, 2560), seed=43 + rows, device="cuda") * 3
    got = orc.bf16_to_f32(to_bits(nf4gemv.matmul_gated(w1, w3, x))).reshape(rows, 9728)
    want = exact_gate(x, w1, w3)
    assert np.isfinite(got).all()
    assert orc.norm_relative_error(got, want) < 1e-2
    assert orc.rms_relative_max_error(got, want) <= 4 * GEMM_TOL


@pytest.mark.parametrize("shape", [(13, 256), (100, 512), (1544, 2560), (17, 768)])
@pytest.mark.parametrize("nested", [True, False])
def test_rows_that_do_not_fill_a_tile(shape, nested):
    """n_out % 16 != 0: the last tile's missing rows re-read row n_out - 1 and
    are never stored."""
    layer = make_linear(*shape, seed=shape[0] + 5, nested=nested)
    x = randn_bf16((1, shape[1]), seed=shape[1], device="cuda")
    y = nf4gemv.matmul(layer, x)
    assert y.shape == (1, shape[0])
    check_matmul(y, x, layer)


def _misaligned_copy(layer):
    """The same NF4 weight with its packed bytes at an address that is 16- but
    not 32-byte aligned (the register-fed kernel's 256-bit loads need 32)."""
    packed = layer.weight.data
    n = packed.numel()
    buf = torch.empty(n + 64, dtype=torch.uint8, device=packed.device)
    off = (16 - buf.data_ptr() % 32) % 32
    view = buf[off:off + n].view(packed.shape)
    view.copy_(packed)
    assert view.data_ptr() % 32 == 16
    other = Linear4bit(layer.in_features, layer.out_features, device=packed.device)
    other.weight = Params4bit(view, layer.weight.quant_state)
    other._keep = buf
    assert nf4gemv.prepare(other)
    return other


@pytest.mark.parametrize("rows", [1, 2])
def test_unaligned_weight_falls_back_to_the_tma_ring_kernel(rows):
    layer = make_linear(6144, 2560, seed=51)
    other = _misaligned_copy(layer)
    x = randn_bf16((rows, 2560), seed=52 + rows, device="cuda")
    fast = nf4gemv.matmul(layer, x)
    ring = nf4gemv.matmul(other, x)
    check_matmul(fast, x, layer)
    check_matmul(ring, x, other)
    # the two kernels sum in different orders: equal within a bf16 ulp or two
    a = orc.bf16_to_f32(to_bits(fast)).astype(np.float64)
    b = orc.bf16_to_f32(to_bits(ring)).astype(np.float64)
    assert np.max(np.abs(a - b)) <= 4 * np.exp2(np.floor(np.log2(np.max(np.abs(a)))) - 7)


def test_repeated_launches_are_bit_identical():
    layer = make_linear(2560, 9728, seed=61)
    x = randn_bf16((1, 9728), seed=62, device="cuda")
    first = nf4gemv.matmul(layer, x)
    for _ in range(4):
        assert torch.equal(nf4gemv.matmul(layer, x), first)
