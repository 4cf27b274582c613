"""The NF4 matmul for decode and prefill, on sm_100a, reading bitsandbytes' weights in place.

Drop-in for the reference's ``app/engine/nf4gemv.py``: same entry points
(``available``, ``prepare``, ``matmul``, ``install``, ``stats``, ``EPI_*``,
``MAX_N``, ``NF4_CODE``), same argument meaning and the same "None means
declined" convention (app/engine/nf4gemv.py:315-376, :427-479). The kernels
are nvcc-built sm_100a code in ``libnf4b200.so`` behind a C ABI
(``include/nf4b200.h``) instead of NVRTC + ctypes driver launches:

* 1..8 activation rows: the streaming GEMV (mma.sync fragments fed from a
  shared-memory NF4 pair table, persistent SM-balanced grid; the register-fed
  kernel decodes each weight once for all rows);
* more rows: the tcgen05 GEMM (TMA, bit-exact dequantisation into shared
  memory, TMEM accumulators) - one launch for the whole prompt, where the
  reference slices it into 32-row launches (app/engine/nf4gemv.py:460-478).

Activations are bf16 or fp16. fp16 is the reference's only GPU dtype
(app/engine/nf4gemv.py:439, its TTS_HALF default): ``matmul`` serves it with
the same rounding points as its kernel (fp32 accumulation, the output and each
epilogue op rounded to fp16) - on the register-fed decode GEMV for 1..8 rows
and on the tcgen05 GEMM for every other row count. bf16 follows the bf16
rounding points of app/engine/nf4cpu.py; ``matmul_qkv_rope``, the chain and the
decode step are bf16 only. Other dtypes are declined (None), as the reference
declines non-fp16 ones. There is no CPU or bitsandbytes fallback inside: a
missing library raises.
"""

from __future__ import annotations

import ctypes
import logging
import threading

from ttspipe_b200 import _lib
from ttspipe_b200.quant import NF4_CODE  # noqa: F401 - part of the reference's API

logger = logging.getLogger(__name__)

#: The reference's rows per launch (app/engine/nf4gemv.py:71, :460). Here any
#: row count is one launch (1..8 rows the GEMV, more the tensor-core GEMM);
#: MAX_N bounds the decode-sized calls, which share the workspace `prepare`
#: sizes and captured decode graphs point at.
MAX_N = 32

#: Epilogues `matmul` can fold into the kernel's store (app/engine/nf4gemv.py:424).
EPI_NONE, EPI_RESIDUAL, EPI_SILU_GATE = 0, 1, 2

_lock = threading.Lock()
_stats = {"fast": 0, "fallback": 0, "layers": 0}
_unavailable: str | None = None
_checked = False
_workspaces: dict = {}   # device index -> zeroed uint8 tensor


def stats() -> dict:
    """Calls served by the kernel, calls handed back, layers covered."""
    return dict(_stats)


def available() -> bool:
    """Whether the library loads and the current device is a B200 (sm_100)."""
    global _checked, _unavailable
    if _checked:
        return _unavailable is None
    with _lock:
        if not _checked:
            try:
                import torch

                _lib.lib()
                if not torch.cuda.is_available():
                    raise RuntimeError("no CUDA device")
                cap = torch.cuda.get_device_capability()
                if cap != (10, 0):
                    raise RuntimeError(f"device capability {cap} is not sm_100")
            except Exception as exc:  # noqa: BLE001 - reported, never swallowed silently
                _unavailable = str(exc)
                logger.warning("nf4 kernels unavailable: %s", exc)
            _checked = True
    return _unavailable is None


def decode_workspace_bytes(desc) -> int:
    """Workspace bytes that cover every decode-sized call (1..MAX_N rows) of
    the weight `desc` describes: the GEMV's partial sums (1..8 rows) can
    outgrow the GEMM's split-K sums at MAX_N rows."""
    size = _lib.lib().nf4b_gemm_workspace_size
    return max(int(size(ctypes.byref(desc), rows)) for rows in range(1, MAX_N + 1))


def _workspace(device, nbytes: int, kind: str = "gemv"):
    """The zeroed, 256-byte aligned GEMV workspace of this device (kind
    "gemm": the tensor-core GEMM's split-K workspace, kept apart so that
    growing it for a large prefill never moves the buffer a captured decode
    graph points at).

    One per device, like the reference's single worker stream
    (app/engine/worker.py:1-12): GEMVs issued concurrently on two streams of
    one device must not overlap. Grown only outside CUDA-graph capture;
    `prepare` sizes it for the largest GEMV a layer can issue so captured
    calls never need to grow it.
    """
    import torch

    idx = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    key = idx if kind == "gemv" else (kind, idx)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("nf4 workspace must be sized before graph capture (call prepare())")
        size = max(nbytes, 32 << 20, 0 if ws is None else 2 * ws.numel())
        ws = torch.zeros(size, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def _to_desc(packed, qs) -> tuple[_lib.Nf4Weight, tuple]:
    import torch

    out_f, in_f = (int(v) for v in qs.shape)
    desc = _lib.Nf4Weight()
    desc.packed = packed.data_ptr()
    desc.n_out, desc.k_in = out_f, in_f
    desc.blocksize = int(qs.blocksize)
    if getattr(qs, "nested", False):
        st2 = qs.state2
        code2 = st2.code.to(device=packed.device, dtype=torch.float32).contiguous()
        am2 = st2.absmax.contiguous()
        a8 = qs.absmax.contiguous()
        desc.absmax_code = a8.data_ptr()
        desc.absmax = am2.data_ptr()
        desc.code2 = code2.data_ptr()
        off = qs.offset
        desc.offset = float(off.item() if hasattr(off, "item") else off)
        desc.blocksize2 = int(st2.blocksize)
        desc.nested = 1
        held = (packed, a8, am2, code2)
    else:
        am = qs.absmax.contiguous()
        desc.absmax = am.data_ptr()
        desc.absmax_code = None
        desc.code2 = None
        desc.offset = 0.0
        desc.blocksize2 = 0
        desc.nested = 0
        held = (packed, am)
    return desc, held


def prepare(module) -> bool:
    """Attach what the kernels need to one NF4 linear, or say they cannot serve it.

    Idempotent and cached on ``module._nf4_fast`` (None = declined), reading
    only ``weight.quant_state`` fields and the weight's pointer/device, as the
    reference does (app/engine/nf4gemv.py:315-421). Nothing is copied except
    the nested scales' 1 KB code table when it is not fp32 on the device.
    """
    import torch

    cached = getattr(module, "_nf4_fast", -1)
    if cached != -1:
        return cached is not None

    def reject(why: str) -> bool:
        module._nf4_fast = None
        logger.debug("nf4 kernel declines %s: %s", type(module).__name__, why)
        return False

    weight = getattr(module, "weight", None)
    qs = getattr(weight, "quant_state", None)
    if qs is None:
        return reject("weight is not quantised yet")
    if getattr(qs, "quant_type", None) != "nf4":
        return reject(f"quant_type={getattr(qs, 'quant_type', None)}")
    if weight.device.type != "cuda":
        return reject("weight is not on a CUDA device")
    out_f, in_f = (int(v) for v in qs.shape)
    bs = int(qs.blocksize)
    if bs < 64 or bs & (bs - 1):
        return reject(f"blocksize {bs} is not a power of two >= 64")
    if in_f % bs or in_f % 64:
        return reject(f"in_features {in_f} is not a multiple of 64 and {bs}")
    if weight.data_ptr() % 16:
        return reject("packed weight is not 16-byte aligned")
    nblk = out_f * in_f // bs
    if qs.absmax.numel() != nblk:
        return reject("scales do not form a rectangle over the weight rows")
    if getattr(qs, "nested", False):
        st2 = qs.state2
        bs2 = int(st2.blocksize)
        if bs2 <= 0 or bs2 & (bs2 - 1):
            return reject(f"second-level blocksize {bs2} is not a power of two")
        if qs.absmax.dtype != torch.uint8 or st2.absmax.dtype != torch.float32:
            return reject("second-level scales are not the uint8/fp32 pair the kernel reads")
    elif qs.absmax.dtype != torch.float32:
        return reject(f"scales are {qs.absmax.dtype}, not float32")
    packed = weight.data if weight.data.dim() == 2 else weight.data.reshape(out_f, in_f // 2)
    desc, held = _to_desc(packed, qs)
    module._nf4_fast = {"desc": desc, "held": held, "M": out_f, "K": in_f,
                        "nested": bool(getattr(qs, "nested", False))}
    if available():
        _workspace(weight.device, decode_workspace_bytes(desc))
    _stats["layers"] += 1
    return True


#: Largest x (rows * in_features * 2 bytes) the TMA-ring pair GEMV stages in
#: shared memory (1..4 rows), and the register-fed GEMV's limits (1..8 rows of
#: blocksize-64 weights with in_features % 256 == 0): a fused RMSNorm is
#: served within them.
NORM_X_MAX = 40 * 1024
REG_MAX_ROWS = 8
REG_X_MAX = 227 * 1024 - 1024 - 256 * 256


def _norm_ok(norm, rows: int, K: int, device, dtype=None) -> bool:
    """Whether `norm` = (weight, eps) may be fused into a decode GEMV of this
    shape; the library makes the final call (NF4B_ERR_SHAPE = declined)."""
    import torch

    w = norm[0]
    dtype = torch.bfloat16 if dtype is None else dtype
    return (1 <= rows <= REG_MAX_ROWS and K % 128 == 0 and rows * K * 2 <= REG_X_MAX and w.dtype == dtype
            and w.is_contiguous() and w.numel() == K and w.device == device)


def _opts(prefetch=None, norm=None, dtype=None):
    """`nf4b_gemm_opts`: up to two prepared linears to stream into L2, a fused
    RMSNorm (weight, eps) of x and the activation dtype; None when none is
    given (bf16, nothing fused)."""
    import torch

    descs = []
    if prefetch is not None:
        mods = list(prefetch) if isinstance(prefetch, (list, tuple)) else [prefetch]
        descs = [m._nf4_fast["desc"] for m in mods[:2] if getattr(m, "_nf4_fast", None) is not None]
    f16 = dtype == torch.float16
    if not descs and norm is None and not f16:
        return None
    ptrs = [ctypes.pointer(d) for d in descs] + [None] * (2 - len(descs))
    nw, eps = (norm[0].data_ptr(), float(norm[1])) if norm is not None else (None, 0.0)
    return ctypes.byref(_lib.GemmOpts(ptrs[0], ptrs[1], nw, eps, _lib.NF4B_F16 if f16 else 0))


def matmul(module, x, *, epi: int = EPI_NONE, operand=None, prefetch=None, norm=None):
    """``x @ module.weight.T`` for any number of input rows, or None if not applicable.

    x is bf16 or fp16 (the output has x's dtype). `epi` fuses
    ``operand + xW`` (EPI_RESIDUAL) or ``silu(operand) * xW`` (EPI_SILU_GATE);
    `operand` has the output's shape and x's dtype, on x's device.
    `prefetch` (an extension; None in the reference's API) names one or two
    prepared linears that later calls will read: their weights are streamed
    into L2 while this call runs. `norm` (an extension) = (weight, eps):
    ``rms_norm(x) @ W.T`` in the same launch, bit-exact to
    ``fusedops.rms_norm`` then ``matmul``; served where x fits a decode GEMV's
    staging (the register-fed kernel: 1..8 rows within REG_X_MAX bytes; the
    pair kernel, bf16: 1..4 rows within NORM_X_MAX; None otherwise). Launches
    on ``torch.cuda.current_stream()``.
    """
    import torch

    fast = getattr(module, "_nf4_fast", None)
    if fast is None:
        return None
    if _lib.act_type(x.dtype) is None or x.device.type != "cuda":
        return None
    K, N = fast["K"], fast["M"]
    if x.shape[-1] != K:
        return None
    flat = x.reshape(-1, K)
    if not flat.is_contiguous() or flat.data_ptr() % 16:
        flat = flat.contiguous()
        if flat.data_ptr() % 16:
            return None
    rows = flat.shape[0]
    if rows == 0:
        return x.new_empty((*x.shape[:-1], N))
    if norm is not None and not _norm_ok(norm, rows, K, x.device, x.dtype):
        return None
    op_ptr = None
    if epi != EPI_NONE:
        if operand is None or operand.numel() != rows * N or operand.dtype != x.dtype:
            return None
        operand = operand.reshape(rows, N)
        if not operand.is_contiguous():
            return None
        op_ptr = operand.data_ptr()
    if not available():
        raise RuntimeError(f"nf4 kernels unavailable: {_unavailable}")
    out = torch.empty((rows, N), dtype=x.dtype, device=x.device)
    stream = torch.cuda.current_stream(x.device)
    L = _lib.lib()
    desc = fast["desc"]
    ws_ptr, ws_bytes = None, 0
    need = int(L.nf4b_gemm_workspace_size(ctypes.byref(desc), rows))   # GEMV slots or GEMM split-K sums
    if need > 0:
        ws = _workspace(x.device, need, "gemv" if rows <= MAX_N else "gemm")
        ws_ptr, ws_bytes = ws.data_ptr(), ws.numel()
    opts = _opts(prefetch, norm, x.dtype)
    st = L.nf4b_gemm_ex(ctypes.byref(desc), flat.data_ptr(), out.data_ptr(), rows, int(epi),
                        op_ptr, ws_ptr, ws_bytes, opts, ctypes.c_void_p(stream.cuda_stream))
    if st == _lib.NF4B_ERR_SHAPE and norm is not None:
        return None     # outside the fused RMSNorm's staging envelope
    _lib.check(st)
    _stats["fast"] += 1
    return out.view(*x.shape[:-1], N)


def matmul_qkv_rope(module, x, *, freqs, pos, q_out, k_cache, v_cache, n_head: int, n_kv: int, norm=None):
    """The wqkv projection of one token with the rotary + KV-cache write in
    its store (an extension): ``y = x @ W.T`` as ``matmul``, the query heads
    rotated into `q_out`, the key heads rotated into ``k_cache[.., pos]`` and
    the value heads copied into ``v_cache[.., pos]`` - bit-identical to
    ``matmul`` then ``nf4b_qk_rope_kv`` without q/k norm. `freqs` is the
    token's rotary row (128 values, fp32/fp16/bf16), `pos` an int64 device
    tensor [1], the caches (.., n_kv, max_len, 128) bf16. Returns y, or None
    where the fused store does not serve the call (the two launches then).
    """
    import torch

    fast = getattr(module, "_nf4_fast", None)
    if fast is None or x.dtype != torch.bfloat16 or x.device.type != "cuda":
        return None
    K, N = fast["K"], fast["M"]
    flat = x.reshape(-1, K) if x.shape[-1] == K else None
    if flat is None or flat.shape[0] != 1 or not flat.is_contiguous() or flat.data_ptr() % 16:
        return None
    if N != (n_head + 2 * n_kv) * 128 or freqs.numel() != 128 or not freqs.is_contiguous():
        return None
    ftype = {torch.float32: _lib.NF4B_F32, torch.float16: _lib.NF4B_F16, torch.bfloat16: _lib.NF4B_BF16}.get(
        freqs.dtype)
    if ftype is None or norm is not None and not _norm_ok(norm, 1, K, x.device):
        return None
    max_len = k_cache.shape[-2]
    if not (k_cache.is_contiguous() and v_cache.is_contiguous() and q_out.is_contiguous()
            and k_cache.dtype == torch.bfloat16 and v_cache.dtype == torch.bfloat16 and q_out.dtype == torch.bfloat16
            and q_out.numel() == n_head * 128 and k_cache.numel() == n_kv * max_len * 128
            and v_cache.shape == k_cache.shape and k_cache.shape[-1] == 128):
        return None
    if not available():
        raise RuntimeError(f"nf4 kernels unavailable: {_unavailable}")
    out = torch.empty((1, N), dtype=torch.bfloat16, device=x.device)
    L = _lib.lib()
    desc = fast["desc"]
    need = int(L.nf4b_gemm_workspace_size(ctypes.byref(desc), 1))
    ws = _workspace(x.device, need, "gemv") if need > 0 else None
    rk = _lib.RopeKv(freqs.data_ptr(), ftype, pos.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(),
                     v_cache.data_ptr(), int(n_head), int(n_kv), int(max_len))
    st = L.nf4b_gemm_qkv_rope(ctypes.byref(desc), flat.data_ptr(), out.data_ptr(), ctypes.byref(rk),
                              ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                              _opts(None, norm), ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    if st == _lib.NF4B_ERR_SHAPE:   # outside the fused store's envelope (e.g. a 16-byte aligned weight)
        return None
    _lib.check(st)
    _stats["fast"] += 1
    return out.view(*x.shape[:-1], N)


def matmul_gated(w1, w3, x, *, prefetch=None, norm=None):
    """``silu(x @ w1.weight.T) * (x @ w3.weight.T)`` in ONE launch, with the
    fork's rounding points (app/engine/fusedlayer.py:265-266: two ``matmul``
    launches there, the second with EPI_SILU_GATE); x W1^T is never written
    out. An extension of the reference's API. Serves 1..8 rows on the
    register-fed GEMV and (bf16) 1..4 rows with in_features % 128 == 0 on the
    pair kernel; returns None otherwise (the caller then issues the two
    matmuls) or if either linear is not prepared. `norm` as in ``matmul``.
    """
    import torch

    f1, f3 = getattr(w1, "_nf4_fast", None), getattr(w3, "_nf4_fast", None)
    if f1 is None or f3 is None or _lib.act_type(x.dtype) is None or x.device.type != "cuda":
        return None
    K, N = f1["K"], f1["M"]
    if (f3["K"], f3["M"]) != (K, N) or x.shape[-1] != K or K % 128:
        return None
    flat = x.reshape(-1, K)
    if not flat.is_contiguous() or flat.data_ptr() % 16:
        flat = flat.contiguous()
        if flat.data_ptr() % 16:
            return None
    rows = flat.shape[0]
    if rows < 1 or rows > REG_MAX_ROWS:
        return None
    if norm is not None and not _norm_ok(norm, rows, K, x.device, x.dtype):
        return None
    if not available():
        raise RuntimeError(f"nf4 kernels unavailable: {_unavailable}")
    L = _lib.lib()
    need = int(L.nf4b_gemm_workspace_size(ctypes.byref(f1["desc"]), rows))
    ws = _workspace(x.device, need)
    out = torch.empty((rows, N), dtype=x.dtype, device=x.device)
    stream = torch.cuda.current_stream(x.device)
    st = L.nf4b_gemm_gated(ctypes.byref(f1["desc"]), ctypes.byref(f3["desc"]), flat.data_ptr(),
                           out.data_ptr(), rows, ws.data_ptr(), ws.numel(), _opts(prefetch, norm, x.dtype),
                           ctypes.c_void_p(stream.cuda_stream))
    if st == _lib.NF4B_ERR_SHAPE:
        return None     # outside the gated launch's envelope: the caller issues two matmuls
    _lib.check(st)
    _stats["fast"] += 1
    return out.view(*x.shape[:-1], N)


def _chain_jobs(steps, max_jobs: int):
    """The C job array for a chain of steps (see matmul_chain), their output
    tensors and the tensors the array points into; None if a step is outside
    the envelope of the calls below."""
    import torch

    if not steps or len(steps) > max_jobs:
        return None
    arr = (_lib.ChainJob * len(steps))()
    outs, keep = [], []
    rows = dev = None
    for i, st in enumerate(steps):
        w, w3 = st["w"], st.get("w3")
        fasts = [getattr(m, "_nf4_fast", None) for m in ((w, w3) if w3 is not None else (w,))]
        if any(f is None for f in fasts):
            return None
        K, N = fasts[0]["K"], fasts[0]["M"]
        x = st["x"]
        if isinstance(x, int):
            if not 0 <= x < i:
                return None
            x = outs[x]
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.shape[-1] != K:
            return None
        flat = x.reshape(-1, K)
        if not flat.is_contiguous() or flat.data_ptr() % 16:
            return None
        if rows is None:
            rows, dev = flat.shape[0], x.device
        if flat.shape[0] != rows:
            return None
        epi = int(st.get("epi", EPI_NONE))
        operand = st.get("operand")
        if isinstance(operand, int):
            if not 0 <= operand < i:
                return None
            operand = outs[operand]
        if w3 is None and epi != EPI_NONE:
            if operand is None or operand.numel() != rows * N or operand.dtype != torch.bfloat16 \
                    or not operand.is_contiguous():
                return None
        out = torch.empty((rows, N), dtype=torch.bfloat16, device=dev)
        arr[i].w = ctypes.pointer(fasts[0]["desc"])
        arr[i].w3 = ctypes.pointer(fasts[1]["desc"]) if w3 is not None else None
        arr[i].x, arr[i].y = flat.data_ptr(), out.data_ptr()
        arr[i].epi = epi if w3 is None else EPI_NONE
        arr[i].operand = operand.data_ptr() if (w3 is None and epi != EPI_NONE) else None
        norm = st.get("norm")
        if norm is not None:
            nw, eps = norm
            if nw.dtype != torch.bfloat16 or nw.numel() != K or not nw.is_contiguous():
                return None
            arr[i].norm_weight, arr[i].norm_eps = nw.data_ptr(), float(eps)
            keep.append(nw)
        else:
            arr[i].norm_weight, arr[i].norm_eps = None, 0.0
        keep += [flat, operand]
        outs.append(out)
    return arr, outs, keep, rows, dev


def matmul_chain(steps):
    """Dependent decode matmuls in ONE launch (an extension of the reference's
    API, which launches each matmul, norm and gate separately,
    app/engine/fusedlayer.py:212-269).

    `steps`: a list of dicts, run in order, each with
      ``w`` (prepared linear), ``x`` (bf16 tensor [..., in] or the int index of
      an earlier step, whose output is then the input), optional ``w3`` (the
      FeedForward gate silu(x W^T) * (x W3^T)), ``epi`` / ``operand`` (tensor
      or step index) as for ``matmul``, and ``norm`` = (weight, eps) to
      RMS-normalise x first exactly as ``fusedops.rms_norm``.
    Returns the list of step outputs, or None if any step is outside the
    chain's envelope (1..4 rows, blocksize 64, in_features % 256 == 0,
    rows * in_features * 2 <= 40 KB); then nothing was launched. Every output
    equals the separate call's bit for bit.
    """
    import torch

    built = _chain_jobs(steps, 40)
    if built is None:
        return None
    arr, outs, keep, rows, dev = built
    if not available():
        raise RuntimeError(f"nf4 kernels unavailable: {_unavailable}")
    L = _lib.lib()
    need = int(L.nf4b_gemv_chain_workspace_size(arr, len(steps), rows))
    if need == 0:
        return None
    ws = _workspace(dev, need)
    stream = torch.cuda.current_stream(dev)
    _lib.check(L.nf4b_gemv_chain(arr, len(steps), rows, ws.data_ptr(), ws.numel(),
                                 ctypes.c_void_p(stream.cuda_stream)))
    _stats["fast"] += len(steps)
    return outs


_step_workspaces: dict = {}


def step_workspace(device, need: int):
    """The decode step's own workspace on `device` (it keeps a launch counter
    there, so it is never shared with the other kernels' workspaces)."""
    import torch

    idx = torch.device(device).index
    ws = _step_workspaces.get(idx)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the decode step's workspace must be sized before graph capture")
        ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
        _step_workspaces[idx] = ws
    return ws


def decode_step(steps):
    """A whole decode step's dependent matmuls in ONE persistent launch
    (``nf4b_decode_step``): the steps of ``matmul_chain`` (same dict format),
    up to 152 of them, for 1 or 2 activation rows. The weights of step i + 1
    stream while step i's outputs are handed over. Each output equals the
    separate call up to fp32 summation order. Returns the outputs, or None
    outside the envelope (blocksize 64, in_features % 256 == 0 and <= 10240,
    out_features % 16 == 0); then nothing was launched."""
    import torch

    built = _chain_jobs(steps, 152)
    if built is None:
        return None
    arr, outs, keep, rows, dev = built
    if rows > 2 or any(o.shape[1] % 16 for o in outs):
        return None
    if not available():
        raise RuntimeError(f"nf4 kernels unavailable: {_unavailable}")
    L = _lib.lib()
    need = int(L.nf4b_decode_step_workspace_size(arr, len(steps), rows))
    if need == 0:
        return None
    ws = step_workspace(dev, need)
    stream = torch.cuda.current_stream(dev)
    _lib.check(L.nf4b_decode_step(arr, len(steps), rows, ws.data_ptr(), ws.numel(),
                                  ctypes.c_void_p(stream.cuda_stream)))
    _stats["fast"] += len(steps)
    return outs


def dequantize(module):
    """The bf16 dense weight [out, in] the kernels multiply by (bit-exact
    bitsandbytes dequantisation), computed on the device."""
    import torch

    if not prepare(module):
        return None
    fast = module._nf4_fast
    out = torch.empty((fast["M"], fast["K"]), dtype=torch.bfloat16, device=module.weight.device)
    _lib.check(_lib.lib().nf4b_dequantize(ctypes.byref(fast["desc"]), out.data_ptr(),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return out


def _linear_classes():
    classes = []
    from ttspipe_b200 import quant

    classes.append(quant.Linear4bit)
    try:
        import bitsandbytes as bnb  # optional: real bitsandbytes layers are served too

        classes.append(bnb.nn.Linear4bit)
    except Exception:  # noqa: BLE001
        pass
    return classes


def install(model=None) -> bool:
    """Route 4-bit linear forwards through the kernels (class-level patch).

    Patches ``ttspipe_b200.quant.Linear4bit`` and, when importable,
    ``bitsandbytes.nn.Linear4bit`` (app/engine/nf4gemv.py:482-517). A declined
    call counts as a fallback and goes to the class's original forward.
    """
    if not available():
        return False
    for cls in _linear_classes():
        if getattr(cls, "_nf4_patched", False):
            continue
        original_forward = cls.forward

        def forward(self, x, _orig=original_forward):
            if prepare(self):
                out = matmul(self, x)
                if out is not None:
                    if self.bias is not None:
                        out = out + self.bias
                    return out
            _stats["fallback"] += 1
            return _orig(self, x)

        cls.forward = forward
        cls._nf4_patched = True
        cls._nf4_original_forward = original_forward
    if model is not None:
        _prepare_all(model)
    return True


def _prepare_all(model) -> None:
    """Build every layer's descriptor now, so no step pays for it mid-utterance."""
    classes = tuple(_linear_classes())
    served = declined = 0
    for module in model.modules():
        if isinstance(module, classes):
            if prepare(module):
                served += 1
            else:
                declined += 1
    logger.info("nf4 kernels ready for %d of %d 4-bit layers", served, served + declined)
