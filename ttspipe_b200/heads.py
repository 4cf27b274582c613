"""The frame's tail on the device: dense bf16 output heads and the fused
sampler (the reference's ``app/engine/graphs.py:55-132`` sample path and
``app/engine/fusedsample.py``), graph-capturable, behind the C ABI."""

from __future__ import annotations

import ctypes

from ttspipe_b200 import _lib

_workspaces: dict = {}


def dense_linear(weight, x, out=None, norm=None):
    """``x @ weight.T`` for a bf16 weight [N, K] (K in 1024, 2048, 2560, 4096)
    and one bf16 row x [K]; returns bf16 [N] (or writes `out`). `norm` =
    (weight, eps): ``rms_norm(x) @ weight.T`` in the same launch, bit-exact to
    ``fusedops.rms_norm`` first."""
    import torch

    n, k = weight.shape
    xf = x.reshape(-1)
    if out is None:
        out = torch.empty(n, dtype=torch.bfloat16, device=x.device)
    nw, eps = (norm[0].data_ptr(), float(norm[1])) if norm is not None else (None, 0.0)
    st = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(_lib.lib().nf4b_dense_gemv(weight.data_ptr(), xf.data_ptr(), out.data_ptr(), n, k, nw, eps, st))
    return out


def _workspace(device, vocab: int):
    import torch

    need = int(_lib.lib().nf4b_sample_workspace_size(vocab))
    idx = torch.device(device).index
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("sampler workspace must be sized before graph capture")
        ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[idx] = ws
    return ws


def sample(logits, *, temperature: float, top_p: float, top_k: int = 64, seed: int = 0, step=None, out=None):
    """One token id (int64 tensor [1] on the device) drawn from a bf16 logit
    row with the fork's top-k / top-p / temperature rule; `step` is an int64
    device tensor [1] (the draw's counter, e.g. the frame index) or None."""
    import torch

    v = logits.reshape(-1)
    if out is None:
        out = torch.empty(1, dtype=torch.int64, device=v.device)
    ws = _workspace(v.device, v.numel())
    st = ctypes.c_void_p(torch.cuda.current_stream(v.device).cuda_stream)
    _lib.check(_lib.lib().nf4b_sample(v.data_ptr(), v.numel(), float(temperature), float(top_p), int(top_k),
                                      ctypes.c_uint64(seed & ((1 << 64) - 1)),
                                      None if step is None else step.data_ptr(), out.data_ptr(),
                                      ws.data_ptr(), ws.numel(), st))
    return out
