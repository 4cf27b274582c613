"""Dual-AR frame bookkeeping kernels (nf4b_embed_rows, nf4b_frame_select,
nf4b_frame_advance) against their torch restatement (B200 only).

The token logic is the reference's decode step (app/engine/graphs.py:105-127):
the semantic draw is replaced by the high-temperature draw when it is a
semantic id already in the recent window; the fast AR's input is the
embedding of each drawn code; the next frame's input is the semantic
embedding plus the codebook embeddings (summed in fp32, codebook order).
Everything here is bit-exact.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from ttspipe_b200 import _lib

pytestmark = pytest.mark.gpu

DIM, VOCAB, CB, NCB, WIN, SEM0 = 2560, 1200, 64, 10, 16, 1000


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _table(rows, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(rows, DIM, generator=g, device="cuda") * 0.02).to(torch.bfloat16)


def test_embed_rows_gathers_and_clamps():
    table = _table(100, 1)
    ids = torch.tensor([7, 150, -5, 99], dtype=torch.long, device="cuda")
    out = torch.empty(4, DIM, dtype=torch.bfloat16, device="cuda")
    _lib.check(_lib.lib().nf4b_embed_rows(table.data_ptr(), 100, ids.data_ptr(), 4, DIM, out.data_ptr(), _stream()))
    want = table[torch.tensor([7, 99, 0, 99], device="cuda")]
    assert torch.equal(out, want)


@pytest.mark.parametrize("main,high,in_window,chosen", [
    (SEM0 + 5, SEM0 + 9, True, SEM0 + 9),    # semantic and repeated: the high-temperature draw
    (SEM0 + 5, SEM0 + 9, False, SEM0 + 5),   # semantic, not repeated
    (17, SEM0 + 9, True, 17),                # repeated but not a semantic id
    (SEM0 + CB, SEM0 + 9, True, SEM0 + CB),  # one past the semantic range
])
def test_frame_select(main, high, in_window, chosen):
    fast_emb = _table(CB, 2)
    recent = torch.full((WIN,), -1, dtype=torch.long, device="cuda")
    if in_window:
        recent[11] = main
    m = torch.tensor([main], dtype=torch.long, device="cuda")
    hi = torch.tensor([high], dtype=torch.long, device="cuda")
    tokens = torch.full((NCB + 1,), -7, dtype=torch.long, device="cuda")
    h = torch.empty(DIM, dtype=torch.bfloat16, device="cuda")
    _lib.check(_lib.lib().nf4b_frame_select(m.data_ptr(), hi.data_ptr(), recent.data_ptr(), WIN, SEM0, CB,
                                            tokens.data_ptr(), fast_emb.data_ptr(), DIM, h.data_ptr(), _stream()))
    a = min(max(chosen - SEM0, 0), CB - 1)
    assert int(tokens[0]) == chosen and int(tokens[1]) == a
    assert int(tokens[2]) == -7
    assert torch.equal(h, fast_emb[a])


def test_frame_advance():
    sem = _table(VOCAB, 3)
    cb = _table(NCB * CB, 4).view(NCB, CB, DIM)
    tokens = torch.tensor([SEM0 + 3] + [(7 * i + 5) % CB for i in range(NCB)], dtype=torch.long, device="cuda")
    recent = torch.arange(WIN, dtype=torch.long, device="cuda") + 100
    before = recent.clone()
    pos = torch.tensor([516], dtype=torch.long, device="cuda")
    step = torch.tensor([9], dtype=torch.long, device="cuda")
    x = torch.empty(DIM, dtype=torch.bfloat16, device="cuda")
    _lib.check(_lib.lib().nf4b_frame_advance(sem.data_ptr(), VOCAB, cb.data_ptr(), CB, NCB, tokens.data_ptr(), DIM,
                                             x.data_ptr(), recent.data_ptr(), WIN, pos.data_ptr(), step.data_ptr(),
                                             _stream()))
    s = torch.zeros(DIM, dtype=torch.float32, device="cuda")
    for i in range(NCB):
        s = s + cb[i, int(tokens[1 + i])].float()
    want = (sem[int(tokens[0])].float() + s).to(torch.bfloat16)
    assert torch.equal(x, want)
    assert int(recent[0]) == SEM0 + 3 and torch.equal(recent[1:], before[:-1])
    assert int(pos) == 517 and int(step) == 10


def test_argument_checks():
    L = _lib.lib()
    t = _table(8, 5)
    ids = torch.zeros(1, dtype=torch.long, device="cuda")
    out = torch.empty(DIM, dtype=torch.bfloat16, device="cuda")
    assert L.nf4b_embed_rows(t.data_ptr(), 8, ids.data_ptr(), 1, 100, out.data_ptr(), _stream()) == \
        _lib.NF4B_ERR_SHAPE  # dim % 8
    assert L.nf4b_embed_rows(None, 8, ids.data_ptr(), 1, DIM, out.data_ptr(), _stream()) == _lib.NF4B_ERR_ARG
    z = torch.zeros(1, dtype=torch.long, device="cuda")
    assert L.nf4b_frame_advance(t.data_ptr(), 8, t.data_ptr(), 8, 33, ids.data_ptr(), DIM, out.data_ptr(),
                                None, 0, z.data_ptr(), z.data_ptr(), _stream()) == _lib.NF4B_ERR_SHAPE
