"""The drop-in Python entry points on a machine without a GPU: every call
declines (None / False) exactly where the reference's would, and nothing
silently computes on the CPU instead of the kernels."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import make_linear, randn_bf16, to_bits
from ttspipe_b200 import fastpath, fusedlayer, fusedops, model, nf4gemv


def test_reference_api_surface():
    for name in ("available", "prepare", "matmul", "install", "stats", "EPI_NONE", "EPI_RESIDUAL",
                 "EPI_SILU_GATE", "MAX_N", "NF4_CODE"):
        assert hasattr(nf4gemv, name)
    assert (nf4gemv.EPI_NONE, nf4gemv.EPI_RESIDUAL, nf4gemv.EPI_SILU_GATE) == (0, 1, 2)
    assert set(nf4gemv.stats()) == {"fast", "fallback", "layers"}
    for name in ("rms_norm", "rope", "install", "stats", "note_rope_fallback"):
        assert hasattr(fusedops, name)
    assert set(fusedops.stats()) == {"norm", "norm_fallback", "rope", "rope_fallback"}
    for name in ("decode_block", "install", "stats"):
        assert hasattr(fusedlayer, name)
    assert hasattr(fastpath, "decode_attention") and fastpath.GROUPED_MAX_QUERY == 64


@pytest.mark.skipif(torch.cuda.is_available(), reason="CPU-only behaviour")
def test_without_a_gpu_everything_declines():
    assert nf4gemv.available() is False
    assert nf4gemv.install() is False
    layer = make_linear(64, 128, seed=1, device="cpu")
    assert nf4gemv.prepare(layer) is False          # weight is not on a CUDA device
    assert nf4gemv.matmul(layer, randn_bf16((1, 128), seed=1)) is None
    w = torch.ones(128, dtype=torch.bfloat16)
    assert fusedops.rms_norm(randn_bf16((1, 128), seed=2), w, 1e-6) is None
    assert fusedops.rope(randn_bf16((1, 1, 2, 8), seed=3), torch.zeros(1, 4, 2)) is None
    assert fusedlayer.install() is False


@pytest.mark.skipif(torch.cuda.is_available(), reason="CPU-only behaviour")
def test_a_linear_without_the_kernels_raises_instead_of_computing():
    layer = make_linear(64, 128, seed=1, device="cpu")
    with pytest.raises(RuntimeError):
        layer(randn_bf16((1, 128), seed=1))


def test_decode_block_declines_a_cpu_block():
    cfg = model.ModelArgs(dim=256, n_head=2, n_local_heads=1, intermediate_size=256, max_seq_len=8)
    blk = model.random_block(cfg, device="cpu", seed=0)
    x = randn_bf16((1, 1, 256), seed=1)
    assert fusedlayer.decode_block(blk, x, torch.zeros(1, 64, 2), torch.ones(1, 1, 1, 4, dtype=torch.bool),
                                   torch.tensor([3])) is None


def test_prefill_attention_formulation_matches_the_oracle_on_cpu():
    """The grouped torch formulation used for spans > 1 (the reference's own,
    app/engine/fastpath.py:158-174), against the oracle."""
    nh, nkv, seqlen, prefix = 8, 2, 5, 11
    L = prefix + seqlen
    q = randn_bf16((1, nh, seqlen, 128), seed=1)
    k = randn_bf16((1, nkv, L, 128), seed=2)
    v = randn_bf16((1, nkv, L, 128), seed=3)
    mask = torch.ones(L, L, dtype=torch.bool).tril()[prefix:][None, None]
    y = fastpath.decode_attention(q, k, v, mask, nh, nkv, 128)
    want = orc.attention_masked(to_bits(q)[0], to_bits(k)[0], to_bits(v)[0], mask[0, 0].numpy(), nh, nkv)
    assert np.array_equal(to_bits(y)[0], want)


def test_model_reference_rotary_matches_the_oracle():
    x = randn_bf16((1, 3, 4, 128), seed=4)
    f = model.precompute_freqs_cis(3, 128)
    assert np.array_equal(to_bits(model.apply_rotary_emb(x, f)),
                          orc.rope(to_bits(x), orc.bf16_to_f32(to_bits(f))))
    assert np.array_equal(to_bits(f), orc.precompute_freqs_cis(3, 128, 1e6))
