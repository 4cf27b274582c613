"""The register-fed pair GEMV (B200 only).

Decode calls with 1..8 activation rows, blocksize-64 weights, k_in % 256 == 0
and 32-byte aligned packed weights run `nf4_gemv_reg_kernel`: weights loaded
straight into registers, MMA columns of (activation row, 64-block) in 1, 2 or
4 column tiles (1-2, 3-4, 5-8 rows), x staged chunk-rotated. These cases
complement test_gpu_kernels / test_gpu_gated with the variants that kernel
adds: every row count of each column-tile width (including tiles whose second
row is missing), plain fp32 scales (one 8-byte pair per lane), the gated pair
with plain scales, the fused RMSNorm, the largest x the staging holds, row
counts that do not fill a tile at one activation row, and the fall-back to the
TMA-ring pair kernel when the packed weight is 16- but not 32-byte aligned.
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


@pytest.mark.parametrize("shape", [(6144, 2560), (2560, 4096), (1544, 2560), (2560, 9728)])
@pytest.mark.parametrize("rows", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("epi", [nf4gemv.EPI_NONE, nf4gemv.EPI_RESIDUAL])
def test_every_row_count_of_each_column_tile_width(shape, rows, epi):
    """Rows 1-8: the register-fed kernel with 1, 2 and 4 column tiles (odd
    counts leave a tile's second row empty); k_in = 9728 at 8 rows is the
    largest x its staging holds (155.6 KB)."""
    layer = make_linear(*shape, seed=3 * shape[0] + rows)
    x = randn_bf16((rows, shape[1]), seed=17 + rows, device="cuda")
    y0 = nf4gemv.matmul(layer, x)
    check_matmul(y0, x, layer)
    if epi != nf4gemv.EPI_NONE:
        operand = randn_bf16((rows, shape[0]), seed=19 + rows, device="cuda")
        y = nf4gemv.matmul(layer, x, epi=epi, operand=operand)
        want = orc.epilogue(orc.bf16_to_f32(to_bits(y0)), epi, to_bits(operand))
        assert np.array_equal(to_bits(y), want)


@pytest.mark.parametrize("small,large", [(1, 2), (3, 4), (5, 8), (6, 7)])
def test_rows_do_not_interact(small, large):
    """The first rows of a batch give the same bits as a smaller batch of the
    same column-tile width (same products, same summation order), and within
    rounding of the rows computed alone (one tile: two MMA chains, so another
    summation order)."""
    layer = make_linear(2560, 9728, seed=77)
    x = randn_bf16((large, 9728), seed=78, device="cuda")
    big = nf4gemv.matmul(layer, x)
    few = nf4gemv.matmul(layer, x[:small].contiguous())
    assert torch.equal(few, big[:small])
    for r in range(large):
        alone = nf4gemv.matmul(layer, x[r:r + 1].contiguous())
        d = (alone[0].float() - big[r].float()).abs().max().item()
        assert d <= 2 ** -7 * big[r].float().abs().max().item()


@pytest.mark.parametrize("rows", [3, 8])
def test_fused_norm_on_several_column_tiles(rows):
    from ttspipe_b200 import fusedops

    lin = make_linear(6144, 2560, seed=91 + rows)
    g = torch.Generator().manual_seed(rows)
    nw = (1.0 + 0.1 * torch.randn(2560, generator=g)).to(torch.bfloat16).cuda()
    x = randn_bf16((rows, 2560), seed=92 + rows, device="cuda") * 3
    want = nf4gemv.matmul(lin, fusedops.rms_norm(x, nw, 1e-6))
    got = nf4gemv.matmul(lin, x, norm=(nw, 1e-6))
    assert got is not None and torch.equal(got, want)


@pytest.mark.parametrize("shape", [(9728, 2560), (2560, 4096), (1544, 2560), (2560, 9728)])
@pytest.mark.parametrize("rows", [1, 2, 6])
def test_plain_fp32_scales(shape, rows):
    layer = make_linear(*shape, seed=7 * shape[0] + rows, nested=False)
    x = randn_bf16((rows, shape[1]), seed=31 + rows, device="cuda")
    check_matmul(nf4gemv.matmul(layer, x), x, layer)


def gate_box(x, w1, w3):
    """Per-element [lo, hi] of the gate silu(a) * b when a and b may each
    differ from the plain GEMV's bf16 output by one ulp plus the fp32
    summation-order error of the product (2^-18 of sum |x||w|: near-zero
    products with heavy cancellation move by many of their own ulps), widened
    by one output ulp."""
    xb = to_bits(x).reshape(-1, w1.in_features)
    xa = np.abs(orc.bf16_to_f32(xb)).astype(np.float64)
    bounds = []
    for w in (w1, w3):
        y = orc.bf16_to_f32(to_bits(nf4gemv.matmul(w, x))).reshape(-1, w.out_features).astype(np.float64)
        mag = xa @ np.abs(orc.bf16_to_f32(oracle_dequant(w)).astype(np.float64)).T
        d = np.exp2(np.floor(np.log2(np.maximum(np.abs(y), 2.0 ** -126))) - 7) + mag * 2.0 ** -18
        bounds.append((y - d, y, y + d))
    silu = lambda v: v / (1.0 + np.exp(-v))
    a_lo, _, a_hi = bounds[0]
    b_lo, _, b_hi = bounds[1]
    s_vals = [silu(a_lo), silu(a_hi)]
    s_min = np.minimum(*s_vals)
    s_max = np.maximum(*s_vals)
    stationary = (a_lo < -1.2785) & (a_hi > -1.2785)   # silu's minimum inside [a_lo, a_hi]
    s_min = np.where(stationary, silu(-1.2784645), s_min)
    cands = np.stack([s_min * b_lo, s_min * b_hi, s_max * b_lo, s_max * b_hi])
    lo, hi = cands.min(0), cands.max(0)
    ulp = lambda v: np.exp2(np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -126))) - 7)
    return lo - 2 * ulp(lo), hi + 2 * ulp(hi)


@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("rows", [1, 2, 3, 8])
def test_gated_pair(nested, rows):
    """Against the exact gate (each product rounded once to bf16) in norm, and
    element by element within the gate of the plain GEMV's products (gate_box):
    a gate's error scales with its own magnitude (silu(a) * b of large a and
    b), so a bar relative to the RMS of all outputs does not fit its tail."""
    w1 = make_linear(9728, 2560, seed=41, nested=nested)
    w3 = make_linear(9728, 2560, seed=42, nested=nested)
    x = randn_bf16((rows, 2560), seed=43 + rows, device="cuda") * 3
    got = orc.bf16_to_f32(to_bits(nf4gemv.matmul_gated(w1, w3, x))).reshape(rows, 9728)
    want = exact_gate(x, w1, w3)
    assert np.isfinite(got).all()
    assert orc.norm_relative_error(got, want) < 1e-2
    lo, hi = gate_box(x, w1, w3)
    g = got.reshape(lo.shape).astype(np.float64)
    bad = np.flatnonzero((g < lo) | (g > hi))
    assert bad.size == 0, (bad[:8], g.ravel()[bad[:8]], lo.ravel()[bad[:8]], hi.ravel()[bad[:8]])


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
