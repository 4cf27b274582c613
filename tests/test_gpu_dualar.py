"""The Dual-AR frame driver (BASELINE config 5 structure) on the device.

A reduced model (2 slow layers) keeps the test short; every frame still runs
the full tail: LM head over 155136 ids, repetition-aware sampling, the fast
AR prime and 9 fast steps with their codebook heads.
"""

from __future__ import annotations

import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import to_bits
from ttspipe_b200 import model, nf4gemv
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


def test_slow_stack_matches_the_reference_blocks_at_the_frame_position(decoder):
    """The frame's fused slow stack at device position p equals the model's own
    block forward (separate norm / wqkv / rotary / KV write / attention / wo /
    norm / w1, w3 / w2 launches) fed freqs_cis[p], the reference's convention:
    q and k are rotated for p, not for position 0."""
    dec = decoder
    snap = snapshot(dec)
    torch.cuda.synchronize()
    p = int(dec.pos.item())
    assert p > 0
    fused = dec.slow_stack(dec.x.clone())
    torch.cuda.synchronize()
    restore(dec, snap)
    forward = getattr(model.TransformerBlock, "_fused_original_forward", model.TransformerBlock.forward)
    x = dec.x.clone()
    ip = torch.tensor([p], dtype=torch.long, device="cuda")
    mask = torch.zeros_like(dec.mask)
    mask[..., :p + 1] = True  # causal row of position p, as the reference's model builds it
    for blk in dec.slow:
        x = forward(blk, x, dec.freqs[p:p + 1], mask, ip)
    torch.cuda.synchronize()
    restore(dec, snap)
    got, want = orc.bf16_to_f32(to_bits(fused)), orc.bf16_to_f32(to_bits(x))
    # Norm-relative, as the reference's own CPU tests compare (tests/test_nf4cpu.py:56-57):
    # the fused gate's silu differs from torch's by an ulp on a few of its 9728
    # elements (a different exp), and the second random-init block's attention
    # amplifies that - at some frame states the max error reaches ~3% of the
    # output RMS while the difference's norm stays below 1% of the output's.
    err = orc.norm_relative_error(got, want)
    assert err < 2e-2
    # and the position matters: position 0's rotation lands measurably further away
    x0 = dec.x.clone()
    for blk in dec.slow:
        x0 = forward(blk, x0, dec.freqs[0:1], mask, ip)
    torch.cuda.synchronize()
    restore(dec, snap)
    err0 = orc.norm_relative_error(orc.bf16_to_f32(to_bits(x0)), want)
    assert err0 > max(5 * err, 1e-4), (err, err0)


def test_state_dict_round_trip_reproduces_the_model():
    """A decoder built from another's state dict (NF4 blocks in bitsandbytes'
    serialisation) computes exactly what the original computes; a decoder
    with other random weights does not."""
    cfg = DualARConfig()
    a = DualARDecoder(cfg, "cuda", seed=5, n_slow=2)
    sd = a.state_dict()
    b = DualARDecoder(cfg, "cuda", seed=6, n_slow=2, state_dict=sd)
    c = DualARDecoder(cfg, "cuda", seed=6, n_slow=2)
    prompt = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(1)).cuda()
    outs = []
    for d in (a, b, c):
        d.prefill(prompt)
        h = d.slow_stack(d.x.clone())
        outs.append((h, torch.matmul(h.view(1, -1).float(), d.lm_head.float().t())))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert not torch.equal(outs[0][0], outs[2][0])
    for d in (a, b, c):
        d.release()
