"""The Dual-AR frame driver (BASELINE config 5 structure) on the device.

A reduced model (2 slow layers) keeps the test short; every frame still runs
the full tail: LM head over 155136 ids, repetition-aware sampling, the fast
AR prime and 9 fast steps with their codebook heads.
"""

from __future__ import annotations

import pytest
import torch

from ttspipe_b200 import nf4gemv
from ttspipe_b200.dualar import DualARConfig, DualARDecoder

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def decoder():
    assert nf4gemv.available()
    dec = DualARDecoder(DualARConfig(), "cuda", seed=3, n_slow=2)
    g = torch.Generator().manual_seed(0)
    dec.prefill(torch.randint(0, dec.cfg.vocab, (64,), generator=g).cuda())
    yield dec
    dec.release()


def snapshot(dec):
    caches = [(b.attention.kv_cache.k_cache.clone(), b.attention.kv_cache.v_cache.clone()) for b in dec.slow + dec.fast]
    return dec.pos.clone(), dec.step.clone(), dec.x.clone(), dec.recent.clone(), caches


def restore(dec, snap):
    pos, step, x, recent, caches = snap
    dec.pos.copy_(pos)
    dec.step.copy_(step)
    dec.x.copy_(x)
    dec.recent.copy_(recent)
    for b, (k, v) in zip(dec.slow + dec.fast, caches):
        b.attention.kv_cache.k_cache.copy_(k)
        b.attention.kv_cache.v_cache.copy_(v)


def test_graph_replay_reproduces_eager_frames(decoder):
    dec = decoder
    snap = snapshot(dec)
    eager = []
    for _ in range(3):
        dec.frame()
        eager.append(dec.tokens.clone())
    torch.cuda.synchronize()
    restore(dec, snap)
    dec.capture()
    replayed = []
    for _ in range(3):
        dec.replay()
        replayed.append(dec.tokens.clone())
    torch.cuda.synchronize()
    for a, b in zip(eager, replayed):
        assert torch.equal(a, b)
    assert int(dec.pos.item()) == 64 + 3 and int(dec.step.item()) == 3


def test_tokens_are_in_range_and_frames_differ(decoder):
    dec = decoder
    if dec.graph is None:
        dec.capture()
    frames = []
    for _ in range(4):
        dec.replay()
        frames.append(dec.tokens.clone())
    torch.cuda.synchronize()
    cfg = dec.cfg
    for t in frames:
        assert 0 <= int(t[0]) < cfg.vocab
        assert bool(((t[1:] >= 0) & (t[1:] < cfg.codebook_size)).all())
    assert len({tuple(t.tolist()) for t in frames}) > 1
