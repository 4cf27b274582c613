"""Pin the oracle against fixtures computed by the reference itself.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py from
the reference's own C++ CPU kernels (app/engine/nf4cpu.py), its torch
attention (app/engine/fastpath.py:133-174) and its torch sampler
(app/engine/graphs.py:55-73). The bars are the reference's own:
tests/test_nf4cpu.py (norm-relative < 5e-3 for the GEMV, < 2e-2 for a block)
and tests/test_nf4gemv.py (max-relative < 5e-3 for attention).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import nf4_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def gemv():
    return np.load(GOLDEN / "gemv.npz")


def test_nf4_code_table_is_the_references():
    ref = np.load(GOLDEN / "nf4_code.npz")["nf4_code"]
    assert np.array_equal(ref, orc.NF4_CODE)
    from ttspipe_b200.quant import NF4_CODE

    assert np.array_equal(np.asarray(NF4_CODE, dtype=np.float32), ref)


@pytest.mark.parametrize("name", ["g0", "g1", "g2", "g3"])
def test_factorised_gemv_is_bit_exact_to_the_reference_cpu_kernel(gemv, name):
    """Per-block code.x dot times the bf16 absmax (app/engine/nf4cpu.py:104-131):
    the oracle's restatement reproduces the AVX-512 kernel's bits at M=1."""
    got = orc.nf4cpu_gemv(gemv[f"{name}_x"], gemv[f"{name}_packed"], gemv[f"{name}_absmax"],
                          gemv["code16"])
    want = gemv[f"{name}_y"]
    if gemv[f"{name}_x"].shape[0] == 1:
        assert np.array_equal(got, want)
    else:
        assert orc.norm_relative_error(orc.bf16_to_f32(got), orc.bf16_to_f32(want)) < 1e-4


@pytest.mark.parametrize("name", ["g0", "g1", "g2", "g3", "a0", "a1", "a2"])
def test_dequant_matmul_matches_the_reference_cpu_kernels(gemv, name):
    """The oracle's dequantise-then-matmul against nf4_gemv / nf4_amx
    (tests/test_nf4cpu.py:43-57, :125-135: norm-relative < 5e-3)."""
    w = orc.dequantize_bf16(gemv[f"{name}_packed"], orc.bf16_to_f32(gemv[f"{name}_absmax"]))
    got = orc.matmul_dequant(gemv[f"{name}_x"], w)
    want = gemv[f"{name}_y"]
    assert orc.norm_relative_error(orc.bf16_to_f32(got), orc.bf16_to_f32(want)) < 5e-3


@pytest.fixture(scope="module")
def block():
    return np.load(GOLDEN / "decode_block.npz")


def _weights(block, qk: bool):
    w = {}
    for nm in ["wqkv", "wo", "w1", "w3", "w2"]:
        w[nm] = orc.dequantize_bf16(block[f"w_{nm}_packed"], orc.bf16_to_f32(block[f"w_{nm}_absmax"]))
    w["attn_norm"], w["ffn_norm"] = block["n_attn_norm"], block["n_ffn_norm"]
    w["q_norm"] = block["n_q_norm"] if qk else None
    w["k_norm"] = block["n_k_norm"] if qk else None
    return w


@pytest.mark.parametrize("case", ["d0", "d1", "d2"])
def test_decode_block_matches_the_reference_cpu_block(block, case):
    dim, nh, nkv, hd, inter, max_len = (int(v) for v in block["dims"])
    eps, qk_eps = (float(v) for v in block["eps"])
    pos, qk, _ = (int(v) for v in block[f"{case}_meta"])
    kc, vc = block["k_cache0"].copy(), block["v_cache0"].copy()
    y = orc.decode_block(block[f"{case}_x"].reshape(-1), _weights(block, bool(qk)), kc, vc, pos,
                         orc.bf16_to_f32(block["freqs"][pos]), nh, nkv, hd, eps, qk_eps)
    want = orc.bf16_to_f32(block[f"{case}_y"]).ravel()
    assert orc.norm_relative_error(orc.bf16_to_f32(y).ravel(), want) < 2e-2
    for got_rows, key in ((kc, "k_rows"), (vc, "v_rows")):
        ref = orc.bf16_to_f32(block[f"{case}_{key}"][:, 0])
        assert orc.norm_relative_error(orc.bf16_to_f32(got_rows[:, pos]), ref) < 2e-2
    # every other cache row is untouched
    others = [p for p in range(max_len) if p != pos]
    assert np.array_equal(kc[:, others], block["k_cache0"][:, others])


@pytest.fixture(scope="module")
def att():
    return np.load(GOLDEN / "attention.npz")


@pytest.mark.parametrize("case", ["s1", "s17", "s100", "p8"])
def test_attention_matches_the_references_torch_attention(att, case):
    nh, nkv, _ = (int(v) for v in att["dims"])
    q, k, v = att[f"{case}_q"][0], att[f"{case}_k"][0], att[f"{case}_v"][0]
    y = orc.attention_masked(q, k, v, att[f"{case}_mask"][0, 0], nh, nkv)
    want = att[f"{case}_y"][0]
    # same rounding points as the fork: equal to the bit
    assert np.array_equal(y, want)
    if q.shape[1] == 1:
        y1 = orc.attention(q[:, 0], k, v, k.shape[1], nh, nkv)
        assert np.array_equal(y1, want[:, 0])


def test_sampler_oracle_follows_the_reference_rule():
    """Hand-checkable case of the fork's rule: cumulative probability cut,
    first position always kept, temperature after the cut."""
    logits = np.array([2.0, 1.0, 0.0, -1.0, 3.0], dtype=np.float32)
    bits = orc.f32_to_bf16(logits)
    p = np.exp(np.sort(logits.astype(np.float64))[::-1] - 3.0)
    p /= p.sum()                     # 0.6364, 0.2341, 0.0861, 0.0317, 0.0117
    tok, kept, q = orc.sample_token(bits, 1.0, 0.9, 64, 0, 0)
    assert list(kept) == [4, 0]      # cumsum 0.870 <= 0.9, then 0.956 > 0.9 cuts the rest
    assert tok in (4, 0)
    tok, kept, _ = orc.sample_token(bits, 1.0, 0.8, 64, 0, 0)
    assert list(kept) == [4]         # 0.870 > 0.8 already at position 1
    tok, kept, _ = orc.sample_token(bits, 1.0, 0.5, 64, 0, 0)
    assert list(kept) == [4]         # position 0 is always kept
    tok, kept, _ = orc.sample_token(bits, 1.0, 1.0, 3, 0, 0)
    assert list(kept) == [4, 0, 1]   # top_k
    assert 0.0 <= orc.sample_uniform(7, 3) < 1.0


SAMPLER = np.load(GOLDEN / "sampler.npz")


@pytest.mark.parametrize("case", [str(c) for c in SAMPLER["cases"]])
def test_sampler_oracle_matches_the_reference_sampler(case):
    """The kept set and the final probabilities of the reference's own torch
    sampler (sort, softmax of the unscaled row, the top-p / top-k cut that
    always keeps position 0, temperature, softmax; app/engine/graphs.py:64-72),
    run on seeded rows by tests/golden/make_golden.py. The reference works in
    fp32 and the oracle in fp64: the kept set must be the same and the
    probabilities agree to fp32 rounding. (The final draw cannot be compared
    token for token: the reference races one torch.rand per vocabulary entry,
    the device draws one counter-based uniform - both sample this distribution.)"""
    logits = SAMPLER[f"{case}_logits"]
    temp, top_p, top_k = SAMPLER[f"{case}_params"]
    _, kept, q = orc.sample_token(logits, float(temp), float(top_p), int(top_k), seed=1, step=0)
    assert list(kept) == list(SAMPLER[f"{case}_kept"])
    np.testing.assert_allclose(q, SAMPLER[f"{case}_probs"], rtol=2e-6, atol=1e-7)


def test_sampler_uniform_is_uniform():
    """The draw's uniform over consecutive steps (one seed): a Kolmogorov-
    Smirnov test against U(0, 1), so an inverse-CDF draw samples the kept
    distribution, as the reference's exponential race does."""
    from scipy import stats

    u = np.array([orc.sample_uniform(12345, s) for s in range(20000)])
    assert stats.kstest(u, "uniform").pvalue > 1e-3
    assert abs(u.mean() - 0.5) < 0.01
