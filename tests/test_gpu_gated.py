"""The gated GEMV (nf4b_gemm_gated): the FeedForward gate
y = bf16(bf16(silu(bf16(x W1))) * bf16(x W3)) of a W1/W3 pair in one launch
(B200 only).

Its two products are the GEMV's own (checked against the exact oracle in
test_gpu_kernels), so each is held to one bf16 ulp of the plain GEMV's output
for the same weight, and the gate of those is evaluated by the oracle at the
fork's rounding points. (A bar of max error over output RMS does not suit the
gate: it is a product of two Gaussians, its largest values sit ~12 RMS out,
where one bf16 ulp is already ~5% of the RMS.)
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import make_linear, oracle_dequant, randn_bf16, to_bits
from ttspipe_b200 import _lib, nf4gemv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available() and nf4gemv.install()


def _ulp_neighbours(v):
    """v - 1 ulp, v, v + 1 ulp of bf16 values (as fp32)."""
    v = v.astype(np.float64)
    e = np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -126)))
    ulp = np.exp2(e - 7)
    return [(v - ulp).astype(np.float32), v.astype(np.float32), (v + ulp).astype(np.float32)]


def gated_bounds(x, w1, w3):
    """Per-element [lo, hi] of the gate when each product may differ from the
    plain GEMV's bf16 output by one ulp (the gated launch sums the same units
    in its own split), widened by one ulp for the fp32 exp inside silu."""
    y1 = orc.bf16_to_f32(to_bits(nf4gemv.matmul(w1, x))).reshape(-1, w1.out_features)
    y3 = orc.bf16_to_f32(to_bits(nf4gemv.matmul(w3, x))).reshape(-1, w3.out_features)
    cands = []
    for a in _ulp_neighbours(y1):
        for b in _ulp_neighbours(y3):
            out = orc.epilogue(b, orc.EPI_SILU_GATE, orc.f32_to_bf16(a))
            cands.append(orc.bf16_to_f32(out).astype(np.float64))
    cands = np.stack(cands)
    lo, hi = cands.min(0), cands.max(0)
    mag = np.maximum(np.abs(lo), np.abs(hi))
    ulp = np.exp2(np.floor(np.log2(np.maximum(mag, 2.0 ** -126))) - 7)
    return lo - ulp, hi + ulp


def exact_gate(x, w1, w3):
    """The gate of the exact (fp64) products, each rounded once to bf16."""
    xb = to_bits(x).reshape(-1, w1.in_features)
    y1 = orc.f32_to_bf16(orc.matmul_exact(xb, oracle_dequant(w1)).astype(np.float32))
    y3 = orc.matmul_exact(xb, oracle_dequant(w3)).astype(np.float32)
    return orc.bf16_to_f32(orc.epilogue(y3, orc.EPI_SILU_GATE, y1))


def check_gated(got, x, w1, w3):
    lo, hi = gated_bounds(x, w1, w3)
    g = orc.bf16_to_f32(to_bits(got)).reshape(lo.shape).astype(np.float64)
    assert np.isfinite(g).all()
    bad = np.flatnonzero((g < lo) | (g > hi))
    assert bad.size == 0, (bad[:8], g.ravel()[bad[:8]], lo.ravel()[bad[:8]], hi.ravel()[bad[:8]])
    # each product is within the GEMV's own 5e-3 of its exact value, and the
    # gate's relative error is at most about the sum of its factors'
    assert orc.norm_relative_error(g, exact_gate(x, w1, w3)) < 1e-2


@pytest.mark.parametrize("rows", [1, 2, 3, 4])
def test_s2pro_feed_forward_gate(rows):
    """gate/up 9728x2560 (x staged in shared memory at every row count)."""
    w1 = make_linear(9728, 2560, seed=3)
    w3 = make_linear(9728, 2560, seed=4)
    x = randn_bf16((rows, 2560), seed=10 + rows, device="cuda")
    check_gated(nf4gemv.matmul_gated(w1, w3, x), x, w1, w3)


@pytest.mark.parametrize("rows", [1, 4])
def test_wide_input_reads_x_from_global_when_it_does_not_fit(rows):
    """k_in 9728 at 4 rows is 78 KB of x: too big to stage, read from global."""
    w1 = make_linear(2560, 9728, seed=5)
    w3 = make_linear(2560, 9728, seed=6)
    x = randn_bf16((rows, 9728), seed=20 + rows, device="cuda")
    check_gated(nf4gemv.matmul_gated(w1, w3, x), x, w1, w3)


@pytest.mark.parametrize("shape", [(16, 128), (1544, 2560), (100, 384), (13, 256)])
@pytest.mark.parametrize("nested", [True, False])
def test_small_ragged_and_plain_scales(shape, nested):
    n, k = shape
    w1 = make_linear(n, k, seed=300 + n, nested=nested)
    w3 = make_linear(n, k, seed=400 + n, nested=nested)
    x = randn_bf16((3, k), seed=500 + n, device="cuda")
    check_gated(nf4gemv.matmul_gated(w1, w3, x), x, w1, w3)


def test_replays_from_a_cuda_graph_and_is_deterministic():
    w1 = make_linear(9728, 2560, seed=11)
    w3 = make_linear(9728, 2560, seed=12)
    x = randn_bf16((1, 2560), seed=13, device="cuda")
    eager = nf4gemv.matmul_gated(w1, w3, x)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            out = nf4gemv.matmul_gated(w1, w3, x)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    del g


def test_declines_and_rejects():
    w1 = make_linear(256, 2560, seed=1)
    w3 = make_linear(256, 2560, seed=2)
    odd = make_linear(256, 1024 + 64, seed=3)
    x5 = randn_bf16((9, 2560), seed=4, device="cuda")
    assert nf4gemv.matmul_gated(w1, w3, x5) is None          # more than 8 rows
    assert nf4gemv.matmul_gated(w1, odd, x5[:1]) is None     # shapes differ
    L = _lib.lib()
    y = torch.empty((1, 256), dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    st = L.nf4b_gemm_gated(ctypes.byref(w1._nf4_fast["desc"]), ctypes.byref(odd._nf4_fast["desc"]),
                           x5.data_ptr(), y.data_ptr(), 1, ws.data_ptr(), ws.numel(), None, None)
    assert st == -2 and "differ" in _lib.last_error()
    st = L.nf4b_gemm_gated(ctypes.byref(w1._nf4_fast["desc"]), ctypes.byref(w3._nf4_fast["desc"]),
                           x5.data_ptr(), y.data_ptr(), 9, ws.data_ptr(), ws.numel(), None, None)
    assert st == -2 and "1..8 rows" in _lib.last_error()
    x_odd = randn_bf16((1, 1088), seed=5, device="cuda")
    st = L.nf4b_gemm_gated(ctypes.byref(odd._nf4_fast["desc"]), ctypes.byref(odd._nf4_fast["desc"]),
                           x_odd.data_ptr(), y.data_ptr(), 1, ws.data_ptr(), ws.numel(), None, None)
    assert st == -2
