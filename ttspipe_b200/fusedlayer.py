"""One decode position through a transformer block, on the sm_100a kernels.

Drop-in for the reference's ``app/engine/fusedlayer.py`` (``decode_block``,
``install``, ``stats``): same launch order and rounding points
(app/engine/fusedlayer.py:212-269):

    rms_norm -> wqkv -> qk_rope_kv -> decode_attention -> wo(+x)
             -> rms_norm -> [w1, w3: silu(w1) * w3] -> w2(+h)

The reference's two attention launches (attn_partial + attn_combine) are one
here (the last CTA of each KV head merges the partials), and so are its w1 and
w3 launches (``nf4gemv.matmul_gated``, same rounding points). The position is read
on the device from ``input_pos`` and the attended window is the mask's width,
so one captured CUDA graph per window serves every position in it. A block
runs in bf16 or in the reference's fp16 (activations, norm weights and KV
cache of one type). Anything that is not a single position of an eligible
block returns None and runs the block's own forward.
"""

from __future__ import annotations


from ttspipe_b200 import _lib

HEAD_DIM = 128
#: One launch for q/k norm + rotary + KV write + attention (nf4b_qkv_attention)
#: instead of nf4b_qk_rope_kv then nf4b_decode_attention. On: with the current
#: attention kernel the Dual-AR frame takes 3.88 ms against 4.00 ms with the two
#: launches (it was 3% slower against an earlier, slower attention kernel).
FUSED_QKV_ATTENTION = True
#: Without q/k norm, run the rotary and the KV-cache write in the wqkv GEMV's
#: store (nf4b_gemm_qkv_rope, one launch less per block); "one_chunk": only
#: where the attention that follows is a plain launch (a window of <= 64 rows).
#: Off: per Dual-AR frame, True measured 4.63 ms and "one_chunk" 4.42-4.43
#: against 4.41-4.43 ms with nf4b_qk_rope_kv as its own launch - that launch is
#: hidden behind the GEMV's tail by programmatic dependent launch, while the
#: 8-CTA attention clusters that follow a whole-GPU GEMV start later.
ROPE_IN_WQKV = False
#: Pass L2 prefetch hints (the next weight of the block) to each matmul: off,
#: measured 1.5% slower per Dual-AR frame with them.
PREFETCH = False
_stats = {"fused": 0, "fallback": 0}
_installed = False
_FTYPE = {"torch.float32": _lib.NF4B_F32, "torch.float16": _lib.NF4B_F16,
          "torch.bfloat16": _lib.NF4B_BF16}


def stats() -> dict:
    from ttspipe_b200 import nf4gemv

    return {**_stats, "ready": nf4gemv.available() and _installed}


def _eligible(block, x, mask, input_pos) -> bool:
    import torch

    from ttspipe_b200 import nf4gemv

    a, ff = block.attention, block.feed_forward
    if x.dim() != 3 or x.shape[0] != 1 or x.shape[1] != 1 or _lib.act_type(x.dtype) is None or not x.is_cuda:
        return False
    if mask is None or input_pos is None or input_pos.numel() != 1 or a.kv_cache is None:
        return False
    if input_pos.dtype != torch.long or not input_pos.is_cuda:
        return False
    if a.head_dim != HEAD_DIM or a.n_head % a.n_local_heads:
        return False
    if (a.n_head // a.n_local_heads) not in (1, 2, 4, 8):
        return False
    kc = a.kv_cache.k_cache
    if kc.dtype != x.dtype or a.kv_cache.v_cache.dtype != x.dtype or not kc.is_contiguous() \
            or not a.kv_cache.v_cache.is_contiguous():
        return False
    if mask.shape[-1] > kc.shape[2]:
        return False
    for linear in (a.wqkv, a.wo, ff.w1, ff.w2, ff.w3):
        if getattr(linear, "bias", None) is not None or not nf4gemv.prepare(linear):
            return False
    return True


def _attention(a, qkv, freqs_cis, input_pos, mask, y, nh: int, nkv: int, max_len: int) -> None:
    """From the wqkv output: q/k norm, rotary and the KV write, then the
    attention into `y` - nf4b_qk_rope_kv and the attention kernel, or both in
    one launch (FUSED_QKV_ATTENTION)."""
    import torch

    from ttspipe_b200 import fastpath

    qn = getattr(a, "q_norm", None) if a.attention_qk_norm else None
    kn = getattr(a, "k_norm", None) if a.attention_qk_norm else None
    eps = float(qn.eps if qn is not None and qn.eps is not None else 1e-6)
    if not FUSED_QKV_ATTENTION:
        q = torch.empty(nh * HEAD_DIM, dtype=qkv.dtype, device=qkv.device)
        _lib.check(_lib.lib().nf4b_qk_rope_kv_ex(
            qkv.data_ptr(), None if qn is None else qn.weight.data_ptr(),
            None if kn is None else kn.weight.data_ptr(), eps, freqs_cis.data_ptr(),
            _FTYPE[str(freqs_cis.dtype)], input_pos.data_ptr(), q.data_ptr(),
            a.kv_cache.k_cache.data_ptr(), a.kv_cache.v_cache.data_ptr(), nh, nkv, HEAD_DIM, max_len,
            _lib.act_type(qkv.dtype), torch.cuda.current_stream(qkv.device).cuda_stream))
        fastpath.kernel_attention(q, a.kv_cache.k_cache, a.kv_cache.v_cache, y, n_head=nh, n_kv=nkv,
                                  pos=input_pos, mask=None, window=int(mask.shape[-1]), max_len=max_len)
        return
    # q/k norm, rotary, the KV write and the attention itself: one launch
    fastpath.qkv_attention(qkv, a.kv_cache.k_cache, a.kv_cache.v_cache, y, n_head=nh, n_kv=nkv, pos=input_pos,
                           window=int(mask.shape[-1]), max_len=max_len, freqs=freqs_cis,
                           freqs_dtype=_FTYPE[str(freqs_cis.dtype)],
                           q_norm_w=None if qn is None else qn.weight,
                           k_norm_w=None if kn is None else kn.weight, eps=eps)


def decode_block(block, x, freqs_cis, mask, input_pos, next_block=None):
    """`TransformerBlock.forward` for one position, or None if it cannot.

    `next_block` (optional, not in the reference's signature): the block that
    runs next, whose first weight is streamed into L2 during this block's
    last matmul."""
    import torch

    from ttspipe_b200 import fastpath, fusedops, nf4gemv

    if not nf4gemv.available() or not _eligible(block, x, mask, input_pos):
        return None
    if str(freqs_cis.dtype) not in _FTYPE or not freqs_cis.is_contiguous() or not freqs_cis.is_cuda:
        return None
    a, ff = block.attention, block.feed_forward
    pf = (lambda m: m) if PREFETCH else (lambda m: None)
    an, fn = block.attention_norm, block.ffn_norm
    nh, nkv = a.n_head, a.n_local_heads
    max_len = a.kv_cache.k_cache.shape[2]
    y = torch.empty((1, 1, nh * HEAD_DIM), dtype=x.dtype, device=x.device)
    q = None
    rope_here = ROPE_IN_WQKV is True or (ROPE_IN_WQKV == "one_chunk" and int(mask.shape[-1]) <= 64)
    if rope_here and not FUSED_QKV_ATTENTION and not a.attention_qk_norm and x.dtype == torch.bfloat16:
        # attention_norm, wqkv, the rotary and the KV write in one launch
        q = torch.empty(nh * HEAD_DIM, dtype=torch.bfloat16, device=x.device)
        if nf4gemv.matmul_qkv_rope(a.wqkv, x, freqs=freqs_cis, pos=input_pos, q_out=q, k_cache=a.kv_cache.k_cache,
                                   v_cache=a.kv_cache.v_cache, n_head=nh, n_kv=nkv,
                                   norm=(an.weight, an.eps)) is None:
            q = None
    if q is not None:
        fastpath.kernel_attention(q, a.kv_cache.k_cache, a.kv_cache.v_cache, y, n_head=nh, n_kv=nkv,
                                  pos=input_pos, mask=None, window=int(mask.shape[-1]), max_len=max_len)
    else:
        # attention_norm fused into the wqkv launch (x staged, normalised in shared memory)
        qkv = nf4gemv.matmul(a.wqkv, x, prefetch=pf(a.wo), norm=(an.weight, an.eps))
        if qkv is None:
            xn = fusedops.rms_norm(x, an.weight, an.eps)
            if xn is None:
                return None
            qkv = nf4gemv.matmul(a.wqkv, xn, prefetch=pf(a.wo))
            if qkv is None:
                return None
        _attention(a, qkv, freqs_cis, input_pos, mask, y, nh, nkv, max_len)
    h = nf4gemv.matmul(a.wo, y, epi=nf4gemv.EPI_RESIDUAL, operand=x, prefetch=pf(ff.w1))
    # w1 and w3 read the same input: one launch normalises h (ffn_norm) and
    # computes the gate silu(hn W1^T) * (hn W3^T) without writing hn or hn W1^T out.
    g = nf4gemv.matmul_gated(ff.w1, ff.w3, h, prefetch=pf(ff.w2), norm=(fn.weight, fn.eps))
    if g is None:
        hn = fusedops.rms_norm(h, fn.weight, fn.eps)
        g = nf4gemv.matmul_gated(ff.w1, ff.w3, hn, prefetch=pf(ff.w2))
        if g is None:
            g1 = nf4gemv.matmul(ff.w1, hn, prefetch=pf(ff.w3))
            g = nf4gemv.matmul(ff.w3, hn, epi=nf4gemv.EPI_SILU_GATE, operand=g1, prefetch=pf(ff.w2))
    nxt = next_block.attention.wqkv if next_block is not None else None
    out = nf4gemv.matmul(ff.w2, g, epi=nf4gemv.EPI_RESIDUAL, operand=h, prefetch=pf(nxt))
    _stats["fused"] += 1
    return out


def install() -> bool:
    """Route single-position ``TransformerBlock.forward`` calls through ``decode_block``."""
    global _installed
    from ttspipe_b200 import model, nf4gemv

    if not nf4gemv.available():
        return False
    classes = [model.TransformerBlock]
    try:
        from fish_speech.models.text2semantic.llama import TransformerBlock as ForkBlock

        classes.append(ForkBlock)
    except Exception:  # noqa: BLE001 - the fork is optional
        pass
    for cls in classes:
        if getattr(cls, "_fused_patched", False):
            continue
        original = cls.forward

        def forward(self, x, freqs_cis, mask, input_pos=None, _orig=original):
            out = decode_block(self, x, freqs_cis, mask, input_pos)
            if out is not None:
                return out
            if x.shape[1] == 1:
                _stats["fallback"] += 1
            return _orig(self, x, freqs_cis, mask, input_pos)

        cls.forward = forward
        cls._fused_patched = True
        cls._fused_original_forward = original
    _installed = True
    return True
