"""Grouped-query attention for a decode step (sm_100a kernel) or a short prefill.

``decode_attention`` keeps the reference's signature and semantics
(app/engine/fastpath.py:133-174): q (B, n_head, S, D), k/v (B, n_local_heads,
L, D) - possibly views of a longer cache - and a boolean mask (B, 1, S, L),
True = visible; query head i reads KV head i // groups. One query position of
batch 1 (every decode step) runs the split-KV kernel of ``libnf4b200.so``
with the mask applied row by row (masked rows are never read), in bf16 or in
the reference's fp16. A multi-position prefill uses the reference's own
grouped torch formulation (scores of the activation type, fp32 softmax,
probabilities of the activation type), as the reference does for spans up
to ``GROUPED_MAX_QUERY``.
"""

from __future__ import annotations

import ctypes

from ttspipe_b200 import _lib

GROUPED_MAX_QUERY = 64
_stats = {"kernel": 0, "grouped": 0}
_workspaces: dict = {}


def stats() -> dict:
    return dict(_stats)


def attention_workspace(device, n_head: int, head_dim: int, window: int):
    """Zeroed per-device workspace for the decode-attention kernel (grown
    outside graph capture only)."""
    import torch

    need = int(_lib.lib().nf4b_decode_attention_workspace_size(n_head, head_dim, window))
    idx = torch.device(device).index
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("attention workspace must be sized before graph capture")
        ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[idx] = ws
    return ws


def kernel_attention(q, k_cache, v_cache, out, *, n_head: int, n_kv: int, pos=None, mask=None,
                     window: int, max_len: int):
    """Launch the decode-attention kernel on raw tensors (one query position).

    q [n_head, 128] bf16 or fp16; caches [n_kv, max_len, 128] of q's dtype
    (head stride max_len rows); pos: int64 device tensor (rows [0, pos]) or
    None; mask: uint8/bool device tensor of `window` entries or None.
    """
    import torch

    dt = _lib.act_type(q.dtype)
    if dt is None or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype or out.dtype != q.dtype:
        raise ValueError(f"attention dtypes {q.dtype}/{k_cache.dtype}/{v_cache.dtype}/{out.dtype} are not served")
    ws = attention_workspace(q.device, n_head, 128, window)
    st = torch.cuda.current_stream(q.device)
    _lib.check(_lib.lib().nf4b_decode_attention_ex(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        None if pos is None else pos.data_ptr(), None if mask is None else mask.data_ptr(),
        out.data_ptr(), n_head, n_kv, 128, max_len, window, ws.data_ptr(), ws.numel(), dt,
        ctypes.c_void_p(st.cuda_stream)))


def qkv_attention(qkv, k_cache, v_cache, out, *, n_head: int, n_kv: int, pos, window: int, max_len: int,
                  freqs, freqs_dtype: int, q_norm_w=None, k_norm_w=None, eps: float = 1e-6, q_scratch=None):
    """q/k norm + rotary + KV write + decode attention in one launch
    (nf4b_qkv_attention) from the wqkv output `qkv` [n_head + 2 n_kv, 128];
    `freqs` is the position's rotary row, `pos` the int64 device position.
    Activations, weights and caches are all bf16 or all fp16."""
    import torch

    dt = _lib.act_type(qkv.dtype)
    if dt is None or k_cache.dtype != qkv.dtype or v_cache.dtype != qkv.dtype or out.dtype != qkv.dtype:
        raise ValueError(f"attention dtypes {qkv.dtype}/{k_cache.dtype}/{out.dtype} are not served")
    ws = attention_workspace(qkv.device, n_head, 128, window)
    if q_scratch is None:
        q_scratch = torch.empty(n_head * 128, dtype=qkv.dtype, device=qkv.device)
    st = torch.cuda.current_stream(qkv.device)
    _lib.check(_lib.lib().nf4b_qkv_attention_ex(
        qkv.data_ptr(), None if q_norm_w is None else q_norm_w.data_ptr(),
        None if k_norm_w is None else k_norm_w.data_ptr(), float(eps), freqs.data_ptr(), int(freqs_dtype),
        pos.data_ptr(), q_scratch.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
        n_head, n_kv, 128, max_len, window, ws.data_ptr(), ws.numel(), dt, ctypes.c_void_p(st.cuda_stream)))


def _grouped_torch(q, k, v, mask, n_head, n_local_heads, head_dim):
    """The reference's grouped formulation (app/engine/fastpath.py:158-174)."""
    import torch

    bsz, _, seqlen, _ = q.shape
    groups = n_head // n_local_heads
    qg = q.reshape(bsz, n_local_heads, groups * seqlen, head_dim)
    scores = torch.matmul(qg, k.transpose(-2, -1)).float() * (head_dim ** -0.5)
    scores = scores.view(bsz, n_local_heads, groups, seqlen, -1)
    scores = torch.where(mask.unsqueeze(2), scores, float("-inf"))
    probs = torch.softmax(scores, dim=-1).to(v.dtype).view(bsz, n_local_heads, groups * seqlen, -1)
    return torch.matmul(probs, v).view(bsz, n_head, seqlen, head_dim)


def decode_attention(q, k, v, mask, n_head, n_local_heads, head_dim):
    """Grouped-query attention; returns (B, n_head, S, head_dim)."""
    import torch

    bsz, _, seqlen, _ = q.shape
    L = k.shape[2]
    served = (
        q.is_cuda and bsz == 1 and seqlen == 1 and head_dim == 128 and _lib.act_type(q.dtype) is not None
        and k.dtype == q.dtype and v.dtype == q.dtype
        and n_head % n_local_heads == 0 and (n_head // n_local_heads) in (1, 2, 4, 8)
        and k.stride(-1) == 1 and k.stride(-2) == head_dim and v.stride() == k.stride()
        and k.stride(1) % head_dim == 0 and mask is not None and mask.shape[-1] == L
    )
    if served:
        qc = q.reshape(n_head, head_dim).contiguous()
        m = mask.reshape(-1, L)[-1].to(torch.uint8).contiguous()
        if qc.data_ptr() % 16 == 0 and k.data_ptr() % 16 == 0 and v.data_ptr() % 16 == 0:
            out = torch.empty((n_head, head_dim), dtype=q.dtype, device=q.device)
            kernel_attention(qc, k, v, out, n_head=n_head, n_kv=n_local_heads, pos=None, mask=m,
                             window=L, max_len=k.stride(1) // head_dim)
            _stats["kernel"] += 1
            return out.view(1, n_head, 1, head_dim)
    _stats["grouped"] += 1
    return _grouped_torch(q, k, v, mask, n_head, n_local_heads, head_dim)
