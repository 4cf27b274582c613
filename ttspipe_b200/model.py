"""The S2-Pro transformer block structure the hot path plugs into.

The reference patches the fish-speech fork's ``TransformerBlock``,
``Attention``, ``FeedForward``, ``RMSNorm`` and ``KVCache`` at class level
(app/engine/worker.py:534-586). The fork is not vendored by the reference, so
this module restates those classes with the attributes the reference's
patches read (``attention.wqkv/wo/n_head/n_local_heads/head_dim/kv_cache/
attention_qk_norm/q_norm/k_norm``, ``feed_forward.w1/w2/w3``,
``attention_norm``, ``ffn_norm``; app/engine/fusedlayer.py:192-269,
app/engine/fastpath.py:207-271) and the fork's arithmetic as the reference's
CPU twin documents it (app/engine/nf4cpu.py:474-617).

Their own ``forward`` methods are the unfused formulation (torch ops around
the NF4 linears); on the GPU, ``fusedlayer.install()`` routes one-position
calls through ``fusedlayer.decode_block`` and ``fusedops.install()`` the norms
through the fused kernel, exactly as the reference's patches do.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from ttspipe_b200.quant import Linear4bit


@dataclass
class ModelArgs:
    """S2-Pro slow-AR dimensions by default (BASELINE config 2/5)."""

    dim: int = 2560
    n_head: int = 32
    n_local_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 9728
    norm_eps: float = 1e-6
    rope_base: float = 1e6
    attention_qk_norm: bool = False
    max_seq_len: int = 2048
    n_layer: int = 36


class RMSNorm(nn.Module):
    """The fork's RMSNorm: ``_norm(x.float()).type_as(x) * weight``
    (formula quoted at app/engine/fusedops.py:9-13)."""

    def __init__(self, dim: int, eps: float = 1e-6, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, device=device, dtype=dtype), requires_grad=False)

    def _norm(self, x):
        return x * torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + self.eps)

    def forward(self, x):
        return self._norm(x.float()).type_as(x) * self.weight


class HeadRMSNorm(nn.Module):
    """Per-head q/k norm: one rounding of x * rsqrt(mean(x^2) + eps) * w, as
    both reference kernels compute it (app/engine/fusedlayer.py:74-84,
    app/engine/nf4cpu.py:501-510)."""

    def __init__(self, dim: int, eps: float = 1e-6, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, device=device, dtype=dtype), requires_grad=False)

    def forward(self, x):
        xf = x.float()
        r = torch.rsqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + self.eps)
        return (xf * r * self.weight.float()).to(x.dtype)


class KVCache(nn.Module):
    """(1, n_local_heads, max_seq_len, head_dim) bf16 caches, as the fork's."""

    def __init__(self, max_seq_len: int, n_heads: int, head_dim: int, device=None,
                 dtype=torch.bfloat16):
        super().__init__()
        shape = (1, n_heads, max_seq_len, head_dim)
        self.register_buffer("k_cache", torch.zeros(shape, dtype=dtype, device=device))
        self.register_buffer("v_cache", torch.zeros(shape, dtype=dtype, device=device))

    def update(self, input_pos, k, v):
        self.k_cache[:, :, input_pos] = k
        self.v_cache[:, :, input_pos] = v
        return self.k_cache, self.v_cache


def apply_rotary_emb(x, freqs_cis):
    """The fork's interleaved-pair rotary in fp32 ops, cast back (unfused)."""
    xs = x.float().reshape(*x.shape[:-1], -1, 2)
    f = freqs_cis.float().view(1, xs.size(1), 1, xs.size(3), 2)
    out = torch.stack([xs[..., 0] * f[..., 0] - xs[..., 1] * f[..., 1],
                       xs[..., 1] * f[..., 0] + xs[..., 0] * f[..., 1]], -1)
    return out.flatten(3).type_as(x)


def precompute_freqs_cis(seq_len: int, n_elem: int, base: float = 1e6, device=None) -> torch.Tensor:
    """(seq_len, n_elem/2, 2) = (cos, sin) in bf16, the fork's layout."""
    i = torch.arange(0, n_elem, 2, device=device)[: n_elem // 2].float()
    inv = 1.0 / (base ** (i / n_elem))
    t = torch.arange(seq_len, device=device, dtype=torch.float32)
    ang = torch.outer(t, inv)
    cache = torch.stack([torch.cos(ang.double()), torch.sin(ang.double())], -1).float()
    return cache.to(torch.bfloat16)


class Attention(nn.Module):
    def __init__(self, cfg: ModelArgs, device=None):
        super().__init__()
        total = (cfg.n_head + 2 * cfg.n_local_heads) * cfg.head_dim
        self.wqkv = Linear4bit(cfg.dim, total, device=device)
        self.wo = Linear4bit(cfg.n_head * cfg.head_dim, cfg.dim, device=device)
        self.n_head, self.n_local_heads, self.head_dim = cfg.n_head, cfg.n_local_heads, cfg.head_dim
        self.dim = cfg.dim
        self.attention_qk_norm = cfg.attention_qk_norm
        if cfg.attention_qk_norm:
            self.q_norm = HeadRMSNorm(cfg.head_dim, cfg.norm_eps, device=device)
            self.k_norm = HeadRMSNorm(cfg.head_dim, cfg.norm_eps, device=device)
        self.kv_cache: KVCache | None = None

    def forward(self, x, freqs_cis, mask, input_pos=None):
        from ttspipe_b200 import fastpath, fusedops

        bsz, seqlen, _ = x.shape
        qs, kvs = self.n_head * self.head_dim, self.n_local_heads * self.head_dim
        q, k, v = self.wqkv(x).split([qs, kvs, kvs], dim=-1)
        q = q.reshape(bsz, seqlen, self.n_head, self.head_dim)
        k = k.reshape(bsz, seqlen, self.n_local_heads, self.head_dim)
        v = v.reshape(bsz, seqlen, self.n_local_heads, self.head_dim)
        if self.attention_qk_norm:
            q, k = self.q_norm(q), self.k_norm(k)
        fq = fusedops.rope(q.contiguous(), freqs_cis)
        fk = fusedops.rope(k.contiguous(), freqs_cis) if fq is not None else None
        if fk is not None:
            q, k = fq, fk
        else:
            fusedops.note_rope_fallback()
            q, k = apply_rotary_emb(q, freqs_cis), apply_rotary_emb(k, freqs_cis)
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
        if self.kv_cache is not None:
            k, v = self.kv_cache.update(input_pos, k, v)
        if mask is not None and mask.shape[-1] < k.shape[2]:
            k, v = k[:, :, : mask.shape[-1]], v[:, :, : mask.shape[-1]]
        y = fastpath.decode_attention(q, k, v, mask, self.n_head, self.n_local_heads, self.head_dim)
        y = y.transpose(1, 2).contiguous().view(bsz, seqlen, qs)
        return self.wo(y)


class FeedForward(nn.Module):
    def __init__(self, cfg: ModelArgs, device=None):
        super().__init__()
        self.w1 = Linear4bit(cfg.dim, cfg.intermediate_size, device=device)
        self.w3 = Linear4bit(cfg.dim, cfg.intermediate_size, device=device)
        self.w2 = Linear4bit(cfg.intermediate_size, cfg.dim, device=device)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class TransformerBlock(nn.Module):
    def __init__(self, cfg: ModelArgs, device=None):
        super().__init__()
        self.attention = Attention(cfg, device)
        self.feed_forward = FeedForward(cfg, device)
        self.ffn_norm = RMSNorm(cfg.dim, cfg.norm_eps, device=device)
        self.attention_norm = RMSNorm(cfg.dim, cfg.norm_eps, device=device)

    def forward(self, x, freqs_cis, mask, input_pos=None):
        h = x + self.attention(self.attention_norm(x), freqs_cis, mask, input_pos)
        return h + self.feed_forward(self.ffn_norm(h))


@torch.no_grad()
def random_block(cfg: ModelArgs, *, device, seed: int, double_quant: bool = True,
                 weight_std: float = 0.02) -> TransformerBlock:
    """A random-init NF4 block: weights ~ N(0, weight_std) quantised
    bitsandbytes-style, norm weights ~ N(1, 0.1), bf16 KV cache of zeros."""
    g = torch.Generator(device=device).manual_seed(seed)
    blk = TransformerBlock(cfg, device)
    for lin in (blk.attention.wqkv, blk.attention.wo, blk.feed_forward.w1,
                blk.feed_forward.w3, blk.feed_forward.w2):
        w = torch.randn(lin.out_features, lin.in_features, generator=g, device=device) * weight_std
        new = Linear4bit.from_float(w, double_quant=double_quant)
        lin.weight = new.weight
    norms = [blk.attention_norm, blk.ffn_norm]
    if cfg.attention_qk_norm:
        norms += [blk.attention.q_norm, blk.attention.k_norm]
    for n in norms:
        n.weight.copy_((1.0 + 0.1 * torch.randn(n.weight.shape, generator=g, device=device)).to(n.weight.dtype))
    blk.attention.kv_cache = KVCache(cfg.max_seq_len, cfg.n_local_heads, cfg.head_dim, device=device)
    return blk


def head_dim_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
