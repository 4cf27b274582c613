"""The fused decode block against the oracle's restatement of the fork's
block (app/engine/fusedlayer.py:212-269 vs app/engine/nf4cpu.py:479-617), its
KV-cache side effect, CUDA-graph capture, and the zero-fallback envelope at
the BASELINE shapes (B200 only)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import oracle_dequant, randn_bf16, to_bits
from ttspipe_b200 import fusedlayer, fusedops, model, nf4gemv

pytestmark = pytest.mark.gpu

BLOCK_TOL = 1e-2   # max|err| / max|ref| in bf16 (~2.5 ulp at the largest element)
CACHE_TOL = 8e-3


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.install() and fusedops.install() and fusedlayer.install()


def _oracle_weights(blk):
    a, ff = blk.attention, blk.feed_forward
    w = {k: oracle_dequant(l) for k, l in
         (("wqkv", a.wqkv), ("wo", a.wo), ("w1", ff.w1), ("w3", ff.w3), ("w2", ff.w2))}
    w["attn_norm"] = to_bits(blk.attention_norm.weight)
    w["ffn_norm"] = to_bits(blk.ffn_norm.weight)
    w["q_norm"] = to_bits(a.q_norm.weight) if a.attention_qk_norm else None
    w["k_norm"] = to_bits(a.k_norm.weight) if a.attention_qk_norm else None
    return w


def _run(cfg, pos, window, qk, seed=0):
    blk = model.random_block(cfg, device="cuda", seed=seed)
    cache = blk.attention.kv_cache
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    cache.k_cache.copy_(torch.randn(cache.k_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    cache.v_cache.copy_(torch.randn(cache.v_cache.shape, generator=g, device="cuda").to(torch.bfloat16))
    freqs = model.precompute_freqs_cis(cfg.max_seq_len, cfg.head_dim, cfg.rope_base, device="cuda")
    x = randn_bf16((1, 1, cfg.dim), seed=seed + 2, device="cuda")
    ip = torch.tensor([pos], dtype=torch.long, device="cuda")
    mask = torch.ones(cfg.max_seq_len, cfg.max_seq_len, dtype=torch.bool, device="cuda").tril()[None, None, ip, :window]
    kc0, vc0 = to_bits(cache.k_cache)[0], to_bits(cache.v_cache)[0]
    before = fusedlayer.stats()["fused"]
    with torch.inference_mode():
        y = blk(x, freqs[ip], mask, ip)
    assert fusedlayer.stats()["fused"] == before + 1
    kc, vc = kc0.copy(), vc0.copy()
    want = orc.decode_block(to_bits(x).reshape(-1), _oracle_weights(blk), kc, vc, pos,
                            orc.bf16_to_f32(to_bits(freqs[pos])), cfg.n_head, cfg.n_local_heads,
                            cfg.head_dim, cfg.norm_eps, cfg.norm_eps)
    got = orc.bf16_to_f32(to_bits(y)).ravel()
    assert orc.relative_error(got, orc.bf16_to_f32(want).ravel()) < BLOCK_TOL
    gk, gv = to_bits(cache.k_cache)[0], to_bits(cache.v_cache)[0]
    assert orc.relative_error(orc.bf16_to_f32(gk[:, pos]), orc.bf16_to_f32(kc[:, pos])) < CACHE_TOL
    assert orc.relative_error(orc.bf16_to_f32(gv[:, pos]), orc.bf16_to_f32(vc[:, pos])) < CACHE_TOL
    others = [p for p in range(cfg.max_seq_len) if p != pos]
    assert np.array_equal(gk[:, others], kc0[:, others]) and np.array_equal(gv[:, others], vc0[:, others])
    return blk


@pytest.mark.parametrize("qk_norm", [True, False])
@pytest.mark.parametrize("pos,window", [(0, 1), (37, 64), (200, 256)])
def test_small_block_matches_the_oracle(qk_norm, pos, window):
    cfg = model.ModelArgs(dim=512, n_head=4, n_local_heads=2, head_dim=128, intermediate_size=1024,
                          attention_qk_norm=qk_norm, max_seq_len=256, norm_eps=1e-6)
    _run(cfg, pos, window, qk_norm)


@pytest.mark.parametrize("pos", [0, 1000, 2047])
def test_s2pro_block_matches_the_oracle(pos):
    """BASELINE config 4 dimensions: hidden 2560, 32/8 heads x 128, KV 2048."""
    cfg = model.ModelArgs(max_seq_len=2048)
    _run(cfg, pos, 2048, False, seed=pos)


def test_decode_block_replays_from_a_cuda_graph():
    """Position and window travel through device memory, so a captured block
    serves every position (app/engine/graphs.py:140-217 relies on this)."""
    cfg = model.ModelArgs(dim=512, n_head=4, n_local_heads=2, head_dim=128, intermediate_size=1024,
                          max_seq_len=256)
    blk = model.random_block(cfg, device="cuda", seed=3)
    freqs = model.precompute_freqs_cis(256, 128, 1e6, device="cuda")
    causal = torch.ones(256, 256, dtype=torch.bool, device="cuda").tril()
    x = randn_bf16((1, 1, 512), seed=4, device="cuda")
    ip = torch.zeros(1, dtype=torch.long, device="cuda")
    f = torch.empty(1, 64, 2, dtype=torch.bfloat16, device="cuda")
    mask = causal[None, None, 0:1, :128].clone()
    with torch.inference_mode():
        for p in range(3):                       # warm-up (also sizes workspaces)
            ip.fill_(p); f.copy_(freqs[p:p + 1])
            blk(x, f, mask, ip)
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph):
                out = blk(x, f, mask, ip)
        torch.cuda.current_stream().wait_stream(s)
        for p in (5, 17, 99):
            ip.fill_(p); f.copy_(freqs[p:p + 1])
            graph.replay()
            torch.cuda.synchronize()
            replayed = out.clone()
            eager = blk(x, f, mask, ip)
            assert torch.equal(replayed, eager)
    del graph


def test_no_fallback_at_baseline_shapes():
    cfg = model.ModelArgs(n_layer=1)
    blk = model.random_block(cfg, device="cuda", seed=9)
    freqs = model.precompute_freqs_cis(cfg.max_seq_len, 128, 1e6, device="cuda")
    before_nf4, before_blk = nf4gemv.stats()["fallback"], fusedlayer.stats()["fallback"]
    x = randn_bf16((1, 1, cfg.dim), seed=1, device="cuda")
    ip = torch.tensor([5], device="cuda")
    mask = torch.ones(1, 1, 1, 2048, dtype=torch.bool, device="cuda")
    with torch.inference_mode():
        blk(x, freqs[ip], mask, ip)
        # a prefill of 64 positions goes through the tcgen05 GEMM and the fused norms
        xs = randn_bf16((1, 64, cfg.dim), seed=2, device="cuda")
        ips = torch.arange(64, device="cuda")
        m = torch.ones(2048, 2048, dtype=torch.bool, device="cuda").tril()[None, None, ips, :2048]
        blk(xs, freqs[ips], m, ips)
    assert nf4gemv.stats()["fallback"] == before_nf4
    assert fusedlayer.stats()["fallback"] == before_blk
    assert fusedops.stats()["norm_fallback"] == 0
