"""Dense bf16 output heads and the fused sampler (B200 only), against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import randn_bf16, to_bits
from ttspipe_b200 import heads, nf4gemv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def available():
    assert nf4gemv.available()


@pytest.mark.parametrize("n,k", [(155136, 2560), (4096, 2560), (1000, 1024), (333, 2048), (64, 4096)])
def test_dense_head_matches_the_exact_product(n, k):
    w = randn_bf16((n, k), seed=n + k, device="cuda", std=0.02)
    x = randn_bf16((k,), seed=k, device="cuda")
    got = orc.bf16_to_f32(to_bits(heads.dense_linear(w, x))).astype(np.float64)
    want = orc.dense_gemv_exact(to_bits(x), to_bits(w))
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 1e-30))) - 7)
    # fp32 accumulation then one bf16 rounding: within one ulp of the exact value
    assert np.all(np.abs(got - want) <= ulp + 1e-6 * np.sqrt((want ** 2).mean()))


@pytest.mark.parametrize("n,k", [(4096, 2560), (155136, 2560), (100, 1024)])
def test_dense_head_with_fused_norm_equals_norm_then_head(n, k):
    from ttspipe_b200 import fusedops

    w = randn_bf16((n, k), seed=n + 3 * k, device="cuda", std=0.02)
    x = randn_bf16((k,), seed=k + 1, device="cuda") * 4
    g = torch.Generator().manual_seed(k)
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).cuda()
    want = heads.dense_linear(w, fusedops.rms_norm(x.view(1, k), nw, 1e-6))
    got = heads.dense_linear(w, x, norm=(nw, 1e-6))
    assert torch.equal(got, want)


@pytest.mark.parametrize("vocab,scale", [(155136, 3.0), (4096, 2.0), (100, 1.0), (2049, 5.0)])
def test_sampler_draws_the_oracles_token(vocab, scale):
    logits = randn_bf16((vocab,), seed=vocab, device="cuda", std=scale)
    bits = to_bits(logits)
    step = torch.zeros(1, dtype=torch.int64, device="cuda")
    for s in range(12):
        step.fill_(s)
        for temp, top_p, top_k in ((0.7, 0.8, 64), (1.0, 0.95, 30), (0.3, 0.5, 64)):
            got = int(heads.sample(logits, temperature=temp, top_p=top_p, top_k=top_k, seed=1234, step=step).item())
            want, kept, _ = orc.sample_token(bits, temp, top_p, top_k, 1234, s)
            assert got == want, (s, temp, top_p, top_k, got, want, kept[:8])


def test_sampler_limits_are_greedy():
    logits = randn_bf16((155136,), seed=5, device="cuda", std=2.0)
    best = int(np.argmax(orc.bf16_to_f32(to_bits(logits))))
    for kw in (dict(temperature=0.7, top_p=0.0), dict(temperature=1e-9, top_p=0.9), dict(temperature=1.0, top_p=1.0, top_k=1)):
        assert int(heads.sample(logits, seed=9, **kw).item()) == best


def test_sampler_frequencies_follow_the_kept_distribution():
    """2000 draws over a 40-entry vocabulary: every token within 5 sigma of its
    probability, nothing outside the kept set."""
    logits = randn_bf16((40,), seed=3, device="cuda", std=1.5)
    _, kept, q = orc.sample_token(to_bits(logits), 0.9, 0.9, 64, 77, 0)
    step = torch.zeros(1, dtype=torch.int64, device="cuda")
    counts = {}
    for s in range(2000):
        step.fill_(s)
        t = int(heads.sample(logits, temperature=0.9, top_p=0.9, top_k=64, seed=77, step=step).item())
        counts[t] = counts.get(t, 0) + 1
    assert set(counts) <= set(int(i) for i in kept)
    for tok, prob in zip(kept, q):
        n = counts.get(int(tok), 0)
        assert abs(n - 2000 * prob) <= 5 * np.sqrt(2000 * prob * (1 - prob)) + 2


def test_sampler_replays_from_a_cuda_graph():
    logits = randn_bf16((155136,), seed=11, device="cuda", std=3.0)
    step = torch.zeros(1, dtype=torch.int64, device="cuda")
    out = torch.empty(1, dtype=torch.int64, device="cuda")
    heads.sample(logits, temperature=0.7, top_p=0.8, seed=5, step=step, out=out)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            heads.sample(logits, temperature=0.7, top_p=0.8, seed=5, step=step, out=out)
    torch.cuda.current_stream().wait_stream(s)
    bits = to_bits(logits)
    for i in range(5):
        step.fill_(i)
        g.replay()
        torch.cuda.synchronize()
        assert int(out.item()) == orc.sample_token(bits, 0.7, 0.8, 64, 5, i)[0]
    del g


_SAMPLER_GOLDEN = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "sampler.npz")


@pytest.mark.parametrize("case", [str(c) for c in _SAMPLER_GOLDEN["cases"]])
def test_sampler_on_the_reference_sampler_rows(case):
    """The rows whose kept sets and probabilities tests/golden/make_golden.py
    took from the reference's own torch sampler (app/engine/graphs.py:55-73):
    at every step the device draws the oracle's token, and the oracle's kept
    set on these rows is the reference's (tests/test_oracle_golden.py), so
    every token drawn lies in the reference's kept set."""
    from tests.helpers import from_bits

    bits = _SAMPLER_GOLDEN[f"{case}_logits"]
    temp, top_p, top_k = _SAMPLER_GOLDEN[f"{case}_params"]
    ref_kept = set(int(i) for i in _SAMPLER_GOLDEN[f"{case}_kept"])
    logits = from_bits(bits, device="cuda")
    step = torch.zeros(1, dtype=torch.int64, device="cuda")
    for s in range(16):
        step.fill_(s)
        got = int(heads.sample(logits, temperature=float(temp), top_p=float(top_p), top_k=int(top_k), seed=99,
                               step=step).item())
        want = orc.sample_token(bits, float(temp), float(top_p), int(top_k), 99, s)[0]
        assert got == want and got in ref_kept, (s, got, want)
