"""ctypes binding of ``libnf4b200.so`` (the C ABI in ``include/nf4b200.h``).

The library is the only compute path: if it is missing or fails to load, every
entry point here raises instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import os

#: The library; NF4B_LIBRARY overrides the in-tree path (as the reference's
#: TTS_NVRTC_PATH does for NVRTC, app/engine/nvrtc.py:49-51).
LIB_PATH = Path(os.environ.get("NF4B_LIBRARY") or Path(__file__).resolve().parent / "libnf4b200.so")

NF4B_OK = 0
NF4B_ERR_ARG, NF4B_ERR_SHAPE, NF4B_ERR_ALIGN, NF4B_ERR_DTYPE = -1, -2, -3, -4
NF4B_ERR_WORKSPACE, NF4B_ERR_LAUNCH, NF4B_ERR_DEVICE = -5, -6, -7
NF4B_EPI_NONE, NF4B_EPI_RESIDUAL, NF4B_EPI_SILU_GATE = 0, 1, 2
NF4B_F32, NF4B_F16, NF4B_BF16 = 0, 1, 2


def act_type(dtype):
    """The library's activation-type code of a torch dtype: NF4B_BF16 for
    bfloat16, NF4B_F16 for float16, None for anything else."""
    import torch

    return {torch.bfloat16: NF4B_BF16, torch.float16: NF4B_F16}.get(dtype)

#: Every symbol the header declares; the CPU tests check the library exports all of them.
EXPORTS = (
    "nf4b_version",
    "nf4b_last_error",
    "nf4b_device_error",
    "nf4b_gemm",
    "nf4b_gemm_ex",
    "nf4b_gemm_workspace_size",
    "nf4b_gemm_noalloc",
    "nf4b_gemm_gated",
    "nf4b_gemm_qkv_rope",
    "nf4b_gemv_chain",
    "nf4b_dense_gemv",
    "nf4b_sample",
    "nf4b_sample_workspace_size",
    "nf4b_embed_rows",
    "nf4b_frame_select",
    "nf4b_frame_advance",
    "nf4b_gemv_chain_workspace_size",
    "nf4b_dequantize",
    "nf4b_rms_norm",
    "nf4b_rope",
    "nf4b_qk_rope_kv",
    "nf4b_decode_attention",
    "nf4b_decode_attention_workspace_size",
    "nf4b_qkv_attention",
    "nf4b_decode_step",
    "nf4b_decode_step_workspace_size",
    "nf4b_debug_decode_step",
    "nf4b_debug_gemm_hook",
    "nf4b_rms_norm_ex",
    "nf4b_rope_ex",
    "nf4b_qk_rope_kv_ex",
    "nf4b_decode_attention_ex",
    "nf4b_qkv_attention_ex",
)


class Nf4Weight(ctypes.Structure):
    """`nf4b_weight`: one bitsandbytes NF4 weight, by pointer."""

    _fields_ = [
        ("packed", ctypes.c_void_p),
        ("absmax_code", ctypes.c_void_p),
        ("absmax", ctypes.c_void_p),
        ("code2", ctypes.c_void_p),
        ("offset", ctypes.c_float),
        ("n_out", ctypes.c_int32),
        ("k_in", ctypes.c_int32),
        ("blocksize", ctypes.c_int32),
        ("blocksize2", ctypes.c_int32),
        ("nested", ctypes.c_int32),
    ]


class ChainJob(ctypes.Structure):
    """`nf4b_chain_job`."""

    _fields_ = [
        ("w", ctypes.POINTER(Nf4Weight)),
        ("w3", ctypes.POINTER(Nf4Weight)),
        ("x", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("operand", ctypes.c_void_p),
        ("epi", ctypes.c_int32),
        ("norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
    ]


class GemmOpts(ctypes.Structure):
    """`nf4b_gemm_opts`."""

    _fields_ = [("prefetch_next", ctypes.POINTER(Nf4Weight)), ("prefetch_next2", ctypes.POINTER(Nf4Weight)),
                ("norm_weight", ctypes.c_void_p), ("norm_eps", ctypes.c_float), ("dtype", ctypes.c_int)]


class RopeKv(ctypes.Structure):
    """`nf4b_rope_kv`: the rotary + KV-cache store fused into a wqkv GEMV."""

    _fields_ = [("freqs", ctypes.c_void_p), ("freqs_dtype", ctypes.c_int), ("pos", ctypes.c_void_p),
                ("q_out", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
                ("n_head", ctypes.c_int), ("n_kv", ctypes.c_int), ("max_len", ctypes.c_int)]


class Nf4bError(RuntimeError):
    """A non-zero status from the library, with its message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"nf4b status {status}: {message}")
        self.status = status


_lock = threading.Lock()
_lib = None


def _declare(lib) -> None:
    vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    wp = ctypes.POINTER(Nf4Weight)
    sig = {
        "nf4b_version": (i32, []),
        "nf4b_last_error": (ctypes.c_char_p, []),
        "nf4b_device_error": (i32, [i32]),
        "nf4b_gemm": (i32, [wp, vp, vp, i32, i32, vp, vp, sz, vp]),
        "nf4b_gemm_ex": (i32, [wp, vp, vp, i32, i32, vp, vp, sz, ctypes.POINTER(GemmOpts), vp]),
        "nf4b_gemm_gated": (i32, [wp, wp, vp, vp, i32, vp, sz, ctypes.POINTER(GemmOpts), vp]),
        "nf4b_gemm_qkv_rope": (i32, [wp, vp, vp, ctypes.POINTER(RopeKv), vp, sz, ctypes.POINTER(GemmOpts), vp]),
        "nf4b_gemv_chain": (i32, [ctypes.POINTER(ChainJob), i32, i32, vp, sz, vp]),
        "nf4b_dense_gemv": (i32, [vp, vp, vp, i32, i32, vp, f32, vp]),
        "nf4b_sample": (i32, [vp, i32, ctypes.c_float, ctypes.c_float, i32, ctypes.c_uint64, vp, vp, vp, sz, vp]),
        "nf4b_sample_workspace_size": (sz, [i32]),
        "nf4b_embed_rows": (i32, [vp, ctypes.c_longlong, vp, i32, i32, vp, vp]),
        "nf4b_frame_select": (i32, [vp, vp, vp, i32, ctypes.c_longlong, ctypes.c_longlong, vp, vp, i32, vp, vp]),
        "nf4b_frame_advance": (i32, [vp, ctypes.c_longlong, vp, ctypes.c_longlong, i32, vp, i32, vp, vp, i32, vp, vp,
                                     vp]),
        "nf4b_gemv_chain_workspace_size": (sz, [ctypes.POINTER(ChainJob), i32, i32]),
        "nf4b_decode_step": (i32, [ctypes.POINTER(ChainJob), i32, i32, vp, sz, vp]),
        "nf4b_decode_step_workspace_size": (sz, [ctypes.POINTER(ChainJob), i32, i32]),
        "nf4b_debug_decode_step": (i32, [ctypes.POINTER(ChainJob), i32, i32, vp, sz, i32, ctypes.c_ulonglong, vp]),
        "nf4b_debug_gemm_hook": (i32, [i32, ctypes.c_ulonglong]),
        "nf4b_gemm_workspace_size": (sz, [wp, i32]),
        "nf4b_gemm_noalloc": (i32, [wp, vp, vp, i32, i32, vp, vp]),
        "nf4b_dequantize": (i32, [wp, vp, vp]),
        "nf4b_rms_norm": (i32, [vp, vp, vp, i32, i32, f32, vp]),
        "nf4b_rope": (i32, [vp, vp, i32, vp, i32, i32, i32, i32, vp]),
        "nf4b_qk_rope_kv": (i32, [vp, vp, vp, f32, vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
        "nf4b_decode_attention": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, sz, vp]),
        "nf4b_decode_attention_workspace_size": (sz, [i32, i32, i32]),
        "nf4b_qkv_attention": (i32, [vp, vp, vp, f32, vp, i32, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, sz,
                                     vp]),
        "nf4b_rms_norm_ex": (i32, [vp, vp, vp, i32, i32, f32, i32, vp]),
        "nf4b_rope_ex": (i32, [vp, vp, i32, vp, i32, i32, i32, i32, i32, vp]),
        "nf4b_qk_rope_kv_ex": (i32, [vp, vp, vp, f32, vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
        "nf4b_decode_attention_ex": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, sz, i32, vp]),
        "nf4b_qkv_attention_ex": (i32, [vp, vp, vp, f32, vp, i32, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp,
                                        sz, i32, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    """The loaded library. Raises if it has not been built or cannot load."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m ttspipe_b200.build` "
                    "(the NF4 kernels have no other implementation)")
            handle = ctypes.CDLL(str(LIB_PATH))
            _declare(handle)
            _lib = handle
    return _lib


def check(status: int) -> None:
    """Raise Nf4bError for a non-zero status."""
    if status != NF4B_OK:
        raise Nf4bError(status, lib().nf4b_last_error().decode(errors="replace"))


def last_error() -> str:
    return lib().nf4b_last_error().decode(errors="replace")
