"""The GEMV chain (nf4b_gemv_chain): dependent decode matmuls in one
persistent launch (B200 only).

At 1-2 rows every step must equal, bit for bit, the separate calls it
replaces - the plain GEMV with its epilogue, nf4b_rms_norm, the gated GEMV -
because each job uses the register-fed kernel's units, runs and summation
order, and the fused norm uses nf4b_rms_norm's arithmetic. At 3-4 rows the
chain runs the TMA-ring pair kernel's arithmetic while a separate call runs
the register-fed kernel's column tiles (another summation order), so the two
agree within a bf16 ulp. Those separate calls are checked against the oracle
in test_gpu_kernels / test_gpu_gated / test_gpu_reg_gemv.
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


def ffn_layer(seed):
    g = torch.Generator().manual_seed(seed)
    norm_w = (1.0 + 0.1 * torch.randn(2560, generator=g)).to(torch.bfloat16).cuda()
    return dict(wo=make_linear(2560, 4096, seed=seed + 1), w1=make_linear(9728, 2560, seed=seed + 2),
                w3=make_linear(9728, 2560, seed=seed + 3), w2=make_linear(2560, 9728, seed=seed + 4),
                norm_w=norm_w)


def separate(layer, attn, x):
    """The decode block's second half as separate launches."""
    h = nf4gemv.matmul(layer["wo"], attn, epi=nf4gemv.EPI_RESIDUAL, operand=x)
    hn = fusedops.rms_norm(h, layer["norm_w"], 1e-6)
    gt = nf4gemv.matmul_gated(layer["w1"], layer["w3"], hn)
    out = nf4gemv.matmul(layer["w2"], gt, epi=nf4gemv.EPI_RESIDUAL, operand=h)
    return h, gt, out


def chained(layer, attn, x):
    return nf4gemv.matmul_chain([
        dict(w=layer["wo"], x=attn, epi=nf4gemv.EPI_RESIDUAL, operand=x),
        dict(w=layer["w1"], w3=layer["w3"], x=0, norm=(layer["norm_w"], 1e-6)),
        dict(w=layer["w2"], x=1, epi=nf4gemv.EPI_RESIDUAL, operand=0),
    ])


@pytest.mark.parametrize("rows", [1, 2])
def test_feed_forward_half_of_a_decode_block_in_one_launch(rows):
    layer = ffn_layer(10 * rows)
    attn = randn_bf16((rows, 4096), seed=1 + rows, device="cuda")
    x = randn_bf16((rows, 2560), seed=2 + rows, device="cuda")
    want = separate(layer, attn, x)
    got = chained(layer, attn, x)
    assert got is not None
    torch.cuda.synchronize()
    for g_, w_ in zip(got, want):
        assert torch.equal(g_, w_)
    assert _lib.lib().nf4b_device_error(1) == 0


def test_two_layers_back_to_back_and_repeated_launches():
    """Eight dependent jobs (two layers); the chain's counters must be left
    zeroed so the next launch sees a clean workspace."""
    layers = [ffn_layer(100), ffn_layer(200)]
    attn = [randn_bf16((1, 4096), seed=7 + i, device="cuda") for i in range(2)]
    x = randn_bf16((1, 2560), seed=9, device="cuda")
    h0, g0, o0 = separate(layers[0], attn[0], x)
    h1, g1, o1 = separate(layers[1], attn[1], o0)
    steps = [
        dict(w=layers[0]["wo"], x=attn[0], epi=nf4gemv.EPI_RESIDUAL, operand=x),
        dict(w=layers[0]["w1"], w3=layers[0]["w3"], x=0, norm=(layers[0]["norm_w"], 1e-6)),
        dict(w=layers[0]["w2"], x=1, epi=nf4gemv.EPI_RESIDUAL, operand=0),
        dict(w=layers[1]["wo"], x=attn[1], epi=nf4gemv.EPI_RESIDUAL, operand=2),
        dict(w=layers[1]["w1"], w3=layers[1]["w3"], x=3, norm=(layers[1]["norm_w"], 1e-6)),
        dict(w=layers[1]["w2"], x=4, epi=nf4gemv.EPI_RESIDUAL, operand=3),
    ]
    for _ in range(3):
        outs = nf4gemv.matmul_chain(steps)
        torch.cuda.synchronize()
        for g_, w_ in zip(outs, [h0, g0, o0, h1, g1, o1]):
            assert torch.equal(g_, w_)


def _same(got, want, rows):
    if rows <= 2:
        assert torch.equal(got, want)
    else:   # another summation order: within one bf16 ulp of the larger magnitude
        a, b = got.float(), want.float()
        ulp = torch.exp2(torch.floor(torch.log2(torch.maximum(a.abs(), b.abs()).clamp_min(2.0 ** -126))) - 7)
        assert bool(((a - b).abs() <= ulp).all())


@pytest.mark.parametrize("shape", [(16, 256), (100, 512), (1544, 2560), (13, 768)])
@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("rows", [1, 3])
def test_small_ragged_and_plain_scale_jobs(shape, nested, rows):
    n, k = shape
    a = make_linear(n, k, seed=n + k, nested=nested)
    x = randn_bf16((rows, k), seed=k, device="cuda")
    r = randn_bf16((rows, n), seed=n, device="cuda")
    outs = nf4gemv.matmul_chain([dict(w=a, x=x), dict(w=a, x=x, epi=nf4gemv.EPI_RESIDUAL, operand=r)])
    assert outs is not None
    _same(outs[0], nf4gemv.matmul(a, x), rows)
    _same(outs[1], nf4gemv.matmul(a, x, epi=nf4gemv.EPI_RESIDUAL, operand=r), rows)


def test_replays_from_a_cuda_graph():
    layer = ffn_layer(300)
    attn = randn_bf16((1, 4096), seed=31, device="cuda")
    x = randn_bf16((1, 2560), seed=32, device="cuda")
    eager = chained(layer, attn, x)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            outs = chained(layer, attn, x)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(outs, eager):
        assert torch.equal(a, b)
    del g


def test_declines_and_rejects():
    a = make_linear(256, 2560, seed=1)
    odd = make_linear(256, 384, seed=2)              # k_in % 256 != 0
    bs128 = make_linear(256, 2560, seed=3, blocksize=128)
    x5 = randn_bf16((5, 2560), seed=4, device="cuda")
    assert nf4gemv.matmul_chain([dict(w=a, x=x5)]) is None           # 5 rows
    assert nf4gemv.matmul_chain([dict(w=odd, x=randn_bf16((1, 384), seed=5, device="cuda"))]) is None
    assert nf4gemv.matmul_chain([dict(w=bs128, x=x5[:1])]) is None
    assert nf4gemv.matmul_chain([dict(w=a, x=x5[:1]), dict(w=a, x=1)]) is None  # forward reference
    arr = (_lib.ChainJob * 1)()
    arr[0].w = ctypes.pointer(a._nf4_fast["desc"])
    big = randn_bf16((4, 9728), seed=6, device="cuda")
    wide = make_linear(256, 9728, seed=7)
    arr[0].w = ctypes.pointer(wide._nf4_fast["desc"])
    y = torch.empty((4, 256), dtype=torch.bfloat16, device="cuda")
    arr[0].x, arr[0].y = big.data_ptr(), y.data_ptr()
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    assert _lib.lib().nf4b_gemv_chain(arr, 1, 4, ws.data_ptr(), ws.numel(), None) == -2   # x too big to stage
    assert "staged" in _lib.last_error()
