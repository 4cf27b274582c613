"""The persistent decode step (nf4b_decode_step): a decode step's dependent
matmuls in one launch (B200 only).

Each job is checked on the inputs it actually read (an earlier job's output
where the chain says so) against the separate call it replaces - nf4b_gemm
with its epilogue and fused RMSNorm, or the gated GEMV - which the other test
files check against the oracle. The step sums each output in its own fixed
order (its CTA and warp split differs from the separate launch's), so a value
may round to the neighbouring bf16; the bars are one ulp for a plain output,
the gated GEMV's own bound for a gate (test_gpu_gated.gated_bounds), and the
oracle's GEMV bar (check_matmul) for outputs without an epilogue.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import make_linear, randn_bf16, to_bits
from tests.test_gpu_gated import gated_bounds
from tests.test_gpu_kernels import check_matmul
from ttspipe_b200 import _lib, fusedops, nf4gemv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available() and nf4gemv.install() and fusedops.install()


def _norm_w(n, seed):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(n, generator=g)).to(torch.bfloat16).cuda()


def block_layer(seed, dim=2560, inter=9728, qkv=6144, attn=4096):
    return dict(wqkv=make_linear(qkv, dim, seed=seed), wo=make_linear(dim, attn, seed=seed + 1),
                w1=make_linear(inter, dim, seed=seed + 2), w3=make_linear(inter, dim, seed=seed + 3),
                w2=make_linear(dim, inter, seed=seed + 4), attn_norm=_norm_w(dim, seed + 5),
                ffn_norm=_norm_w(dim, seed + 6))


def block_steps(layers, h0, attn):
    """A decode step's matmuls per layer, in the order of the reference's
    decode_block (app/engine/fusedlayer.py:212-269) without attention, whose
    output `attn[l]` stands in: wqkv(norm(h)), wo(attn) + h, gate(norm(.)),
    w2(gate) + (wo's output); the next layer reads w2's output."""
    steps = []
    h = h0
    for l, L in enumerate(layers):
        base = len(steps)
        steps.append(dict(w=L["wqkv"], x=h, norm=(L["attn_norm"], 1e-6)))
        steps.append(dict(w=L["wo"], x=attn[l], epi=nf4gemv.EPI_RESIDUAL, operand=h))
        steps.append(dict(w=L["w1"], w3=L["w3"], x=base + 1, norm=(L["ffn_norm"], 1e-6)))
        steps.append(dict(w=L["w2"], x=base + 2, epi=nf4gemv.EPI_RESIDUAL, operand=base + 1))
        h = base + 3
    return steps


def _resolve(v, outs):
    return outs[v] if isinstance(v, int) else v


def _ulp(v):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -126))) - 7)


def check_step(steps, outs):
    """Every job against the separate call on the inputs it read."""
    for i, st in enumerate(steps):
        x = _resolve(st["x"], outs)
        if st.get("norm") is not None:
            x = fusedops.rms_norm(x, st["norm"][0], st["norm"][1])
        got = orc.bf16_to_f32(to_bits(outs[i])).astype(np.float64)
        if st.get("w3") is not None:
            lo, hi = gated_bounds(x, st["w"], st["w3"])
            assert np.all((got.reshape(lo.shape) >= lo) & (got.reshape(hi.shape) <= hi)), f"job {i} (gate)"
            continue
        epi = st.get("epi", nf4gemv.EPI_NONE)
        want = nf4gemv.matmul(st["w"], x, epi=epi, operand=_resolve(st.get("operand"), outs))
        w = orc.bf16_to_f32(to_bits(want)).astype(np.float64).reshape(got.shape)
        rms = float(np.sqrt((w ** 2).mean()))
        assert np.all(np.abs(got - w) <= 2 * _ulp(w) + 1e-3 * rms), f"job {i}"
        if epi == nf4gemv.EPI_NONE:
            check_matmul(outs[i], x, st["w"])


@pytest.mark.parametrize("rows", [1, 2])
def test_two_s2pro_layers_in_one_launch(rows):
    layers = [block_layer(10 * rows + 100 * i) for i in range(2)]
    h0 = randn_bf16((rows, 2560), seed=1 + rows, device="cuda")
    attn = [randn_bf16((rows, 4096), seed=3 + rows + i, device="cuda") for i in range(2)]
    steps = block_steps(layers, h0, attn)
    outs = nf4gemv.decode_step(steps)
    assert outs is not None
    torch.cuda.synchronize()
    check_step(steps, outs)
    assert _lib.lib().nf4b_device_error(1) == 0


def test_repeated_launches_and_graph_replay_are_deterministic():
    """The step keeps a launch counter in its workspace (a new flag space per
    launch): repeated launches, eager and from a CUDA graph, give the same bits."""
    layers = [block_layer(300), block_layer(400)]
    h0 = randn_bf16((1, 2560), seed=31, device="cuda")
    attn = [randn_bf16((1, 4096), seed=32 + i, device="cuda") for i in range(2)]
    steps = block_steps(layers, h0, attn)
    first = [o.clone() for o in nf4gemv.decode_step(steps)]
    for _ in range(3):
        again = nf4gemv.decode_step(steps)
        torch.cuda.synchronize()
        for a, b in zip(again, first):
            assert torch.equal(a, b)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            outs = nf4gemv.decode_step(steps)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(4):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(outs, first):
            assert torch.equal(a, b)
    del g
    assert _lib.lib().nf4b_device_error(1) == 0


@pytest.mark.parametrize("nested", [True, False])
def test_small_jobs_barriers_and_operand_handoff(nested):
    """Jobs too small for every CTA to finish a tile (full-barrier boundaries),
    an x that is not the previous output, an epilogue operand that IS the
    previous output (read from its handoff words), a silu-gate epilogue, and
    plain fp32 scales."""
    a = make_linear(256, 512, seed=1, nested=nested)      # 16 tiles x 2 units: 32 units < 148 CTAs
    b = make_linear(512, 256, seed=2, nested=nested)
    c = make_linear(512, 512, seed=3, nested=nested)
    d = make_linear(2048, 512, seed=4, nested=nested)
    x = randn_bf16((1, 512), seed=5, device="cuda")
    z = randn_bf16((1, 512), seed=6, device="cuda")
    steps = [dict(w=a, x=x),
             dict(w=b, x=0, norm=(_norm_w(256, 7), 1e-6)),
             dict(w=c, x=z, epi=nf4gemv.EPI_RESIDUAL, operand=1),   # operand = previous y
             dict(w=c, x=2, epi=nf4gemv.EPI_SILU_GATE, operand=2),  # x and operand = previous y
             dict(w=d, x=3)]
    outs = nf4gemv.decode_step(steps)
    assert outs is not None
    torch.cuda.synchronize()
    check_step(steps, outs)
    assert _lib.lib().nf4b_device_error(1) == 0


def test_declines_and_rejects():
    a = make_linear(256, 2560, seed=1)
    x = randn_bf16((1, 2560), seed=2, device="cuda")
    assert nf4gemv.decode_step([dict(w=a, x=randn_bf16((3, 2560), seed=3, device="cuda"))]) is None   # 3 rows
    assert nf4gemv.decode_step([dict(w=make_linear(24, 2560, seed=4), x=x)]) is None                 # n_out % 16
    wide = make_linear(256, 12288, seed=5)
    assert nf4gemv.decode_step([dict(w=wide, x=randn_bf16((1, 12288), seed=6, device="cuda"))]) is None  # k_in
    assert nf4gemv.decode_step([dict(w=make_linear(256, 2560, seed=7, blocksize=128), x=x)]) is None
    # a job whose x is the previous y must match its width
    arr = (_lib.ChainJob * 2)()
    y0 = torch.empty((1, 256), dtype=torch.bfloat16, device="cuda")
    y1 = torch.empty((1, 256), dtype=torch.bfloat16, device="cuda")
    for i, (xx, yy) in enumerate(((x, y0), (y0, y1))):
        arr[i].w = ctypes.pointer(a._nf4_fast["desc"])
        arr[i].x, arr[i].y = xx.data_ptr(), yy.data_ptr()
    L = _lib.lib()
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    assert L.nf4b_decode_step(arr, 2, 1, ws.data_ptr(), ws.numel(), None) == _lib.NF4B_ERR_SHAPE
    assert "k_in" in _lib.last_error()
    arr[1].x = x.data_ptr()
    need = int(L.nf4b_decode_step_workspace_size(arr, 2, 1))
    assert need > 0
    assert L.nf4b_decode_step(arr, 2, 1, ws.data_ptr(), need - 8, None) == _lib.NF4B_ERR_WORKSPACE
