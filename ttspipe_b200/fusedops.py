"""Fused RMSNorm and rotary embedding, one sm_100a kernel each.

Drop-in for the reference's ``app/engine/fusedops.py`` (``rms_norm``,
``rope``, ``install``, ``stats``, ``note_rope_fallback``) in bf16 and in the
reference's fp16. Same formulas and rounding points (:61-132): the norm rounds
to the activation type after the normalisation and again after the weight
multiply; rotary is bit-exact to the unfused fp32 formula. The norm's sum of squares is exact (fp64 on the device),
so unlike the reference's fp32 tree sum it does not depend on reduction order.
Shapes these kernels do not serve return None (the caller uses its own code).
"""

from __future__ import annotations

import ctypes

from ttspipe_b200 import _lib

enabled = True
_stats = {"norm": 0, "norm_fallback": 0, "rope": 0, "rope_fallback": 0}
_FTYPE = {"torch.float32": _lib.NF4B_F32, "torch.float16": _lib.NF4B_F16,
          "torch.bfloat16": _lib.NF4B_BF16}


def stats() -> dict:
    return dict(_stats)


def _stream(t):
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def rms_norm(x, weight, eps: float):
    """``x * rsqrt(mean(x*x) + eps) * weight`` over the last axis, or None."""
    import torch

    if not enabled:
        return None
    dt = _lib.act_type(x.dtype)
    if dt is None or weight.dtype != x.dtype:
        return None
    if x.device.type != "cuda" or not x.is_contiguous() or not weight.is_contiguous():
        return None
    width = x.shape[-1]
    if width != weight.numel() or width == 0 or x.numel() == 0:
        return None
    out = torch.empty_like(x)
    _lib.check(_lib.lib().nf4b_rms_norm_ex(x.data_ptr(), weight.data_ptr(), out.data_ptr(),
                                           x.numel() // width, width, float(eps), dt, _stream(x)))
    _stats["norm"] += 1
    return out


def rope(x, freqs_cis):
    """Rotary embedding of `x` (B, S, H, D) against `freqs_cis` (S, D/2, 2), or None."""
    import torch

    if not enabled:
        return None
    dt = _lib.act_type(x.dtype)
    if dt is None or x.device.type != "cuda" or not x.is_contiguous():
        return None
    if not freqs_cis.is_contiguous() or x.dim() != 4 or freqs_cis.device != x.device:
        return None
    ftype = _FTYPE.get(str(freqs_cis.dtype))
    if ftype is None:
        return None
    bsz, seq, heads, head_dim = x.shape
    if head_dim % 2 or freqs_cis.numel() != seq * (head_dim // 2) * 2 or x.numel() == 0:
        return None
    out = torch.empty_like(x)
    _lib.check(_lib.lib().nf4b_rope_ex(x.data_ptr(), freqs_cis.data_ptr(), ftype, out.data_ptr(),
                                       bsz, seq, heads, head_dim, dt, _stream(x)))
    _stats["rope"] += 1
    return out


def note_rope_fallback() -> None:
    """Called by `fastpath` when it had to use the unfused rotary."""
    _stats["rope_fallback"] += 1


def install() -> bool:
    """Route ``RMSNorm.forward`` of ``ttspipe_b200.model`` (and of the fish-speech
    fork when importable) through the fused kernel. Idempotent."""
    from ttspipe_b200 import nf4gemv

    if not nf4gemv.available():
        return False
    classes = []
    from ttspipe_b200 import model

    classes.append(model.RMSNorm)
    try:
        from fish_speech.models.text2semantic.llama import RMSNorm as ForkRMSNorm

        classes.append(ForkRMSNorm)
    except Exception:  # noqa: BLE001 - the fork is optional
        pass
    for cls in classes:
        if getattr(cls, "_fused_patched", False):
            continue
        original_forward = cls.forward

        def forward(self, x, _orig=original_forward):
            out = rms_norm(x, self.weight, self.eps)
            if out is not None:
                return out
            _stats["norm_fallback"] += 1
            return _orig(self, x)

        cls.forward = forward
        cls._fused_patched = True
        cls._fused_original_forward = original_forward
    return True
