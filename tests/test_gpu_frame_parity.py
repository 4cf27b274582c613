"""One whole Dual-AR frame on the device against the oracle (B200 only).

The reference's frame is `sample_frame` after the slow forward
(app/engine/graphs.py:92-132): the slow stack at the frame's position, the
final norm and LM head, a main and a hotter draw with the repetition-aware
choice (:105-116), the fast AR's prime at fast position 0 (`_fast_prime`,
:76-89) and the remaining codebook steps, then the next frame's input. Here a
reduced model (hidden 1024, two slow and two fast layers, a 6144-id vocabulary
whose last 1024 ids are codebook-0 tokens, four codebooks) runs one frame
through `DualARDecoder.frame`, and the same frame is recomposed on the CPU from
the oracle's `decode_block`, `rms_norm`, `dense_gemv_exact` and `sample_token`
from the very same state (the KV caches the prompt left behind, the position,
the draw counter, the repetition window) and seeds.

What must agree:
  * every logit row the frame samples from (the LM head's and each codebook
    head's, which the frame keeps in place), within LOGIT_TOL of the oracle's
    (the rows come after up to five chained blocks - two slow, the prime, two
    fast - each of which matches the oracle within the block test's 1e-2);
  * every drawn token, exactly, given the device's own logit row: the device
    sampler and the oracle's `sample_token` apply the same rule to the same
    row. On the oracle's row the oracle draws the same token too, unless the
    draw's uniform lies closer to a CDF boundary than the logit difference can
    move it (|dF| <= 2 max|dL| / T): the device's matmuls accumulate in a
    different order than the oracle's exact sums, and a token whose
    probabilities nearly tie may then flip. The frame continues with the
    device's token either way, so everything after it is compared like for
    like;
  * the KV-cache rows the frame writes (every slow layer at the position,
    every fast layer at fast positions 0..3), within the block tolerance;
  * the next frame's input, bit for bit (a sum of embedding rows in a fixed
    order), the repetition window, the position and the draw counter.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import oracle_dequant, to_bits
from ttspipe_b200 import model, nf4gemv
from ttspipe_b200.dualar import DualARConfig, DualARDecoder

pytestmark = pytest.mark.gpu

CACHE_TOL = 3.2e-2   # a KV row after up to 4 blocks of GEMV rounding: four blocks' bars of 8e-3 added
                     # (seed 6's fast layer-0 v row, after two slow blocks and two norms, exceeded 2e-2)
LOGIT_TOL = 4e-2     # max|dL| / max|L| of a logit row after up to five chained blocks (each within 1e-2)


def _cfg():
    slow = model.ModelArgs(dim=1024, n_head=8, n_local_heads=2, head_dim=128, intermediate_size=2816,
                           max_seq_len=128, n_layer=2)
    return DualARConfig(slow=slow, n_fast_layer=2, vocab=6144, num_codebooks=4, codebook_size=1024,
                        semantic_begin_id=5120)


def _block_weights(blk):
    a, ff = blk.attention, blk.feed_forward
    w = {k: oracle_dequant(l) for k, l in
         (("wqkv", a.wqkv), ("wo", a.wo), ("w1", ff.w1), ("w3", ff.w3), ("w2", ff.w2))}
    w["attn_norm"] = to_bits(blk.attention_norm.weight)
    w["ffn_norm"] = to_bits(blk.ffn_norm.weight)
    w["q_norm"] = w["k_norm"] = None
    return w


def _draw_margin(logit_bits, temp, top_p, top_k, seed, step):
    """Distance of the draw's uniform from the nearest boundary of the kept
    set's CDF (the draw is stable against logit errors much smaller than it)."""
    _, _, q = orc.sample_token(logit_bits, temp, top_p, top_k, seed, step)
    u = orc.sample_uniform(seed, step)
    edges = np.concatenate([[0.0], np.cumsum(q)])
    return float(np.min(np.abs(edges - u)))


class OracleFrame:
    """The frame recomposed from oracle functions, on bf16 bit patterns."""

    def __init__(self, dec: DualARDecoder):
        c = dec.cfg
        self.c, self.seed = c, dec.seed
        self.slow_w = [_block_weights(b) for b in dec.slow]
        self.fast_w = [_block_weights(b) for b in dec.fast]
        self.norm_w, self.fast_norm_w = to_bits(dec.norm_w), to_bits(dec.fast_norm_w)
        self.lm_head = to_bits(dec.lm_head)
        self.cb_heads = [to_bits(h) for h in dec.cb_heads]
        self.sem_emb, self.cb_emb, self.fast_emb = to_bits(dec.sem_emb), to_bits(dec.cb_emb), to_bits(dec.fast_emb)
        self.freqs = orc.bf16_to_f32(to_bits(dec.freqs))
        self.fast_freqs = orc.bf16_to_f32(to_bits(dec.fast_freqs))
        s = c.slow
        self.dims = (s.n_head, s.n_local_heads, s.head_dim, s.norm_eps)

    def _block(self, x, w, kc, vc, pos, freqs_row):
        nh, nkv, hd, eps = self.dims
        return orc.decode_block(x, w, kc, vc, pos, freqs_row, nh, nkv, hd, eps, eps)

    def _draw(self, logits, dev_logits, temp, top_p, seed, step, device_tok, mismatches, what):
        """The oracle's draw on its own row `logits`, checked against the
        device's token and the device's row `dev_logits` (bf16 bits)."""
        lo, lg = orc.bf16_to_f32(logits).astype(np.float64), orc.bf16_to_f32(dev_logits).astype(np.float64)
        assert orc.relative_error(lg, lo) < LOGIT_TOL, what
        # the same rule on the same row: the same token, exactly
        assert orc.sample_token(dev_logits, temp, top_p, self.c.top_k, seed, step)[0] == device_tok, what
        tok = orc.sample_token(logits, temp, top_p, self.c.top_k, seed, step)[0]
        if tok != device_tok:
            margin = _draw_margin(logits, temp, top_p, self.c.top_k, seed, step)
            bound = 2.0 * float(np.max(np.abs(lg - lo))) / max(temp, 1e-5)
            assert margin < bound, f"{what}: device drew {device_tok}, oracle {tok}, margin {margin:.2e} > {bound:.2e}"
            mismatches.append((what, margin, bound))
        return device_tok   # teacher-forced: the frame continues with the device's choice

    def run(self, st, dev_tokens, dev_main, dev_high, dev_logits, dev_cb_logits):
        """One frame from state `st` (dict of bit arrays, modified in place);
        returns (tokens, draw mismatches within the margin)."""
        c = self.c
        nh, nkv, hd, eps = self.dims
        mism = []
        pos, step = st["pos"], st["step"]
        x = st["x"]
        for i, w in enumerate(self.slow_w):
            x = self._block(x, w, st["slow_k"][i], st["slow_v"][i], pos, self.freqs[pos])
        hidden = orc.rms_norm(x.reshape(1, -1), self.norm_w, eps)
        logits = orc.f32_to_bf16(orc.dense_gemv_exact(hidden, self.lm_head).astype(np.float32))
        main = self._draw(logits, dev_logits, c.temperature, c.top_p, self.seed * 7919 + 1, step, dev_main, mism,
                          "main")
        high = self._draw(logits, dev_logits, c.high_temperature, c.high_top_p, self.seed * 7919 + 2, step, dev_high,
                          mism, "high")
        semantic = c.semantic_begin_id <= main < c.semantic_begin_id + c.codebook_size
        chosen = high if (semantic and main in list(st["recent"])) else main
        a = min(max(chosen - c.semantic_begin_id, 0), c.codebook_size - 1)
        tokens = [chosen, a]
        # fast prime at fast position 0: all fast blocks but the last, then the
        # last block's q/k/v projection, rotary and KV write only
        y = hidden
        for i, w in enumerate(self.fast_w[:-1]):
            y = self._block(y, w, st["fast_k"][i], st["fast_v"][i], 0, self.fast_freqs[0])
        w = self.fast_w[-1]
        xn = orc.rms_norm(y.reshape(1, -1), w["attn_norm"], eps)
        qkv = orc.bf16_to_f32(orc.matmul_dequant(xn, w["wqkv"]))[0]
        qs, kvs = nh * hd, nkv * hd
        k = orc.f32_to_bf16(qkv[qs:qs + kvs]).reshape(1, 1, nkv, hd)
        f = self.fast_freqs[0].reshape(1, hd // 2, 2)
        st["fast_k"][-1][:, 0] = orc.rope(k, f).reshape(nkv, hd)
        st["fast_v"][-1][:, 0] = orc.f32_to_bf16(qkv[qs + kvs:]).reshape(nkv, hd)
        h = self.fast_emb[a]
        for i in range(1, c.num_codebooks):
            y = h
            for li, w in enumerate(self.fast_w):
                y = self._block(y, w, st["fast_k"][li], st["fast_v"][li], i, self.fast_freqs[i])
            yn = orc.rms_norm(y.reshape(1, -1), self.fast_norm_w, eps)
            lg = orc.f32_to_bf16(orc.dense_gemv_exact(yn, self.cb_heads[i]).astype(np.float32))
            tok = self._draw(lg, dev_cb_logits[i], c.temperature, c.top_p, self.seed * 7919 + 10 + i, step,
                             dev_tokens[i + 1], mism, f"codebook {i}")
            tokens.append(tok)
            h = self.fast_emb[tok]
        # next input: bf16(float(semantic row) + fp32 sum of the codebook rows in order)
        s = np.zeros(self.sem_emb.shape[1], np.float32)
        for i in range(c.num_codebooks):
            s = (s + orc.bf16_to_f32(self.cb_emb[i, tokens[1 + i]])).astype(np.float32)
        st["x"] = orc.f32_to_bf16(orc.bf16_to_f32(self.sem_emb[tokens[0]]) + s)
        st["recent"] = np.concatenate([[tokens[0]], st["recent"][:-1]])
        st["pos"], st["step"] = pos + 1, step + 1
        return tokens, mism


def _state(dec):
    return {
        "x": to_bits(dec.x).reshape(-1), "pos": int(dec.pos.item()), "step": int(dec.step.item()),
        "recent": dec.recent.cpu().numpy().copy(),
        "slow_k": [to_bits(b.attention.kv_cache.k_cache)[0] for b in dec.slow],
        "slow_v": [to_bits(b.attention.kv_cache.v_cache)[0] for b in dec.slow],
        "fast_k": [to_bits(b.attention.kv_cache.k_cache)[0] for b in dec.fast],
        "fast_v": [to_bits(b.attention.kv_cache.v_cache)[0] for b in dec.fast],
    }


def _close(got, want, tol):
    return orc.relative_error(orc.bf16_to_f32(got), orc.bf16_to_f32(want)) < tol


@pytest.mark.parametrize("seed,repeat", [(5, False), (6, True)])
def test_frame_matches_the_oracle_frame(seed, repeat):
    """`repeat`: the main draw is planted in the repetition window first, so
    the frame must take the hotter draw instead (app/engine/graphs.py:111-116)."""
    assert nf4gemv.available()
    dec = DualARDecoder(_cfg(), "cuda", seed=seed)
    c = dec.cfg
    with torch.no_grad():
        # favour codebook-0 ids so the main draw is a semantic token, as in real
        # decoding, and give the heads a trained model's peaked rows instead of
        # random-init's nearly uniform ones (with 64 near-equal probabilities
        # almost every draw sits near a CDF boundary)
        dec.lm_head[c.semantic_begin_id:] *= 4
        for h in dec.cb_heads:
            h *= 4
    g = torch.Generator().manual_seed(seed)
    dec.prefill(torch.randint(0, c.vocab, (16,), generator=g).cuda())
    orf = OracleFrame(dec)
    for frame in range(2):
        if repeat and frame == 1:
            # plant the main draw the device will make (the frame is deterministic)
            saved = [(t.clone()) for t in (dec.pos, dec.step, dec.x, dec.recent)]
            caches = [(b.attention.kv_cache.k_cache.clone(), b.attention.kv_cache.v_cache.clone())
                      for b in dec.slow + dec.fast]
            dec.frame()
            main_probe = int(dec.main_tok.item())
            for t, s in zip((dec.pos, dec.step, dec.x, dec.recent), saved):
                t.copy_(s)
            for b, (k, v) in zip(dec.slow + dec.fast, caches):
                b.attention.kv_cache.k_cache.copy_(k)
                b.attention.kv_cache.v_cache.copy_(v)
            dec.recent[3] = main_probe
        st = _state(dec)
        dec.frame()
        torch.cuda.synchronize()
        dev_tokens = [int(t) for t in dec.tokens.cpu()]
        dev_main, dev_high = int(dec.main_tok.item()), int(dec.high_tok.item())
        pos = st["pos"]
        tokens, mism = orf.run(st, dev_tokens, dev_main, dev_high, to_bits(dec.logits), to_bits(dec.cb_logits))
        # the rows this frame wrote: every slow layer at pos, every fast layer
        # at fast positions 0 (the prime) .. 3
        for i, b in enumerate(dec.slow):
            gk, gv = to_bits(b.attention.kv_cache.k_cache)[0], to_bits(b.attention.kv_cache.v_cache)[0]
            assert _close(gk[:, pos], st["slow_k"][i][:, pos], CACHE_TOL), (frame, "slow k", i)
            assert _close(gv[:, pos], st["slow_v"][i][:, pos], CACHE_TOL), (frame, "slow v", i)
        for i, b in enumerate(dec.fast):
            gk, gv = to_bits(b.attention.kv_cache.k_cache)[0], to_bits(b.attention.kv_cache.v_cache)[0]
            for r in range(c.num_codebooks):
                assert _close(gk[:, r], st["fast_k"][i][:, r], CACHE_TOL), (frame, "fast k", i, r)
                assert _close(gv[:, r], st["fast_v"][i][:, r], CACHE_TOL), (frame, "fast v", i, r)
        assert tokens == dev_tokens, (frame, tokens, dev_tokens)
        # draws that flipped on the oracle's own rows were each within their
        # bound (checked in _draw); the device's draws equal the oracle's rule
        # on the device's rows exactly
        if repeat and frame == 1:
            assert c.semantic_begin_id <= dev_main < c.semantic_begin_id + c.codebook_size
            assert dev_tokens[0] == dev_high
        # the next frame's input and counters, exactly
        assert np.array_equal(to_bits(dec.x).reshape(-1), st["x"])
        assert list(dec.recent.cpu().numpy()) == list(st["recent"])
        assert int(dec.pos.item()) == st["pos"] and int(dec.step.item()) == st["step"]
    dec.release()
