"""Benchmark: NF4 decode GEMV GB/s on B200 (one replica per GPU).

Workload (`config.workload`): the decode-time NF4 matmuls of the S2-Pro slow AR
at M=1 (blocksize 64, double-quantised scales), per layer in the order and with
the data flow of the reference's decode block (app/engine/fusedlayer.py:212-269)
minus attention: wqkv 6144x2560 on RMSNorm(h) (attention_norm fused), wo
2560x4096 on the attention output (a seeded stand-in per layer) + h, the
FeedForward gate silu(x W1^T) * (x W3^T) with W1, W3 9728x2560 on
RMSNorm(wo's output) (ffn_norm fused), and w2 2560x9728 on the gate + wo's
output; the next layer's h is w2's output. A step is one pass over 36 distinct
layers (1.87 GB of NF4 weights, far larger than the 126 MB L2, so every step
streams from HBM). Weights ~ N(0, 0.02), norm weights ~ N(1, 0.1), the first
h and the attention stand-ins ~ N(0, 1), seeded per layer and rank
(synthetic; no checkpoint).

Schedules (`--mode`, see MODES): `step` runs the whole step as ONE
nf4b_decode_step launch (the persistent decode-step kernel); `decode` issues
the 4 matmuls of each layer as separate C-ABI launches (nf4b_gemm_ex /
nf4b_gemm_gated with the fused norms), captured as one CUDA graph.

value  = algorithmic bytes of all ranks' steps / max-over-ranks device time
e2e    = the same metric through the C ABI with host buffers: every step
         copies its inputs (the first h and the attention stand-ins) from
         pinned host memory, replays the step and reads every output back to
         pinned host memory, inside the timed region.

`--impl reference` times the reference's own CPU NF4 kernel (nf4cpu.nf4_gemv,
built into oracle/_ref) on the host cores over the same workload definition.
`--case <kernel>` runs one profiling case instead (see "profiling cases").
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "nf4_decode_gemv_GBps"
UNIT = "GB/s"
N_LAYERS = 36
# The layer's weights (name, out, in) and its matmul jobs: (name, weights, epilogue)
# with epilogue 0 none, 1 residual, "gated" = silu(x W1^T) * (x W3^T).
PROJ = [("wqkv", 6144, 2560, 0), ("wo", 2560, 4096, 1), ("w1", 9728, 2560, 0),
        ("w3", 9728, 2560, 2), ("w2", 2560, 9728, 1)]
JOBS = [("wqkv", (0,), 0), ("wo", (1,), 1), ("w13", (2, 3), "gated"), ("w2", (4,), 1)]
BS, BS2 = 64, 256


def algorithmic_bytes(n: int, k: int, rows: int = 1, epi: int = 0, nested: bool = True) -> int:
    """Bytes a matmul must move: packed codes + scales + x + y (+ operand)."""
    nb = n * k // BS
    scales = (nb + 4 * math.ceil(nb / BS2) + 1024) if nested else 4 * nb
    return n * k // 2 + scales + 2 * rows * k + 2 * rows * n + (2 * rows * n if epi else 0)


def weight_bytes(n: int, k: int, nested: bool = True) -> int:
    nb = n * k // BS
    return n * k // 2 + ((nb + 4 * math.ceil(nb / BS2) + 1024) if nested else 4 * nb)


# the jobs whose x is RMS-normalised inside the launch (their norm weight is read)
NORMED = {"wqkv", "w13"}


def job_bytes(job, rows: int = 1) -> int:
    """Weights + x + y (+ operand, + the fused norm's weight) of one job; a
    gated pair reads x once and writes only the gated product."""
    name, widx, epi = job
    n, k = PROJ[widx[0]][1], PROJ[widx[0]][2]
    b = sum(weight_bytes(PROJ[i][1], PROJ[i][2]) for i in widx) + 2 * rows * k + 2 * rows * n
    return b + (2 * rows * n if epi == 1 else 0) + (2 * k if name in NORMED else 0)


LAYER_BYTES = sum(job_bytes(j) for j in JOBS)
STEP_BYTES = N_LAYERS * LAYER_BYTES


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# --------------------------------------------------------------------------
# distributed plumbing (one process per GPU; replicas, no data-path collective)
# --------------------------------------------------------------------------


def dist_init(backend: str):
    import torch.distributed as dist

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1 and not dist.is_initialized():
        from datetime import timedelta

        dist.init_process_group(backend=backend, timeout=timedelta(seconds=300))
    return int(os.environ.get("RANK", "0")), ws, int(os.environ.get("LOCAL_RANK", "0"))


def max_over_ranks(v: float, device) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier():
    import torch.distributed as dist

    if dist.is_initialized():
        dist.barrier()


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.idx = set(gpu_indices)
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                f = [c.strip() for c in line.split(",")]
                if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in self.idx:
                    continue
                rows.append(f)
        except Exception:  # noqa: BLE001
            pass
        finally:
            if self.path:
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        load = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows),
                "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


# --------------------------------------------------------------------------
# the GPU arm
# --------------------------------------------------------------------------


def make_layers(device, rank: int):
    """36 layers x 5 NF4 projections (nested scales), generated on the device."""
    import torch

    from ttspipe_b200 import nf4gemv
    from ttspipe_b200.quant import Linear4bit

    layers = []
    for li in range(N_LAYERS):
        mods = []
        for pi, (_, n, k, _) in enumerate(PROJ):
            g = torch.Generator(device=device).manual_seed(1_000_003 * rank + 100 * li + pi)
            w = torch.randn(n, k, generator=g, device=device) * 0.02
            lin = Linear4bit.from_float(w, double_quant=True)
            del w
            assert nf4gemv.prepare(lin)
            mods.append(lin)
        layers.append(mods)
    torch.cuda.synchronize(device)
    return layers


class StepIO:
    """A step's inputs, outputs and norm weights, and the data flow between
    its jobs. Inputs in `dev_in`: the first layer's h, then one attention
    stand-in [4096] per layer. Outputs in `dev_out`, per layer: wqkv's, wo's,
    the gate's and w2's (the next layer's h). Pinned host mirrors serve the
    end-to-end measurement."""

    def __init__(self, device, rank: int):
        import torch

        dim, attn = PROJ[1][1], PROJ[1][2]
        self.h0_off = 0
        self.attn_off = [dim + l * attn for l in range(N_LAYERS)]
        n_in = dim + N_LAYERS * attn
        widths = [PROJ[0][1], PROJ[1][1], PROJ[2][1], PROJ[4][1]]   # wqkv, wo, gate, w2 outputs
        self.out_off = []
        off = 0
        for _ in range(N_LAYERS):
            offs = []
            for w in widths:
                offs.append(off)
                off += w
            self.out_off.append(offs)
        g = torch.Generator(device=device).manual_seed(77 + rank)
        self.dev_in = torch.randn(n_in, generator=g, device=device).to(torch.bfloat16)
        self.dev_out = torch.zeros(off, dtype=torch.bfloat16, device=device)
        self.norms = (1.0 + 0.1 * torch.randn(N_LAYERS, 2, dim, generator=g, device=device)).to(torch.bfloat16)
        self.scratch = torch.zeros(PROJ[2][1], dtype=torch.bfloat16, device=device)  # w1 output (single mode)
        self.host_in = torch.empty(n_in, dtype=torch.bfloat16, pin_memory=True)
        self.host_in.copy_(self.dev_in.cpu())
        self.host_out = torch.empty(off, dtype=torch.bfloat16, pin_memory=True)
        self.h2d_bytes = self.dev_in.numel() * 2
        self.d2h_bytes = self.dev_out.numel() * 2

    def jobs(self, layers):
        """Per layer and job: (name, descriptors, x, y, epilogue, operand, norm weight) as addresses."""
        ib, ob = self.dev_in.data_ptr(), self.dev_out.data_ptr()
        nb = self.norms.data_ptr()
        dim = PROJ[1][1]
        out = []
        h = ib + 2 * self.h0_off
        for l, mods in enumerate(layers):
            qkv, wo, gate, w2 = (ob + 2 * o for o in self.out_off[l])
            attn_norm, ffn_norm = nb + 2 * (2 * l) * dim, nb + 2 * (2 * l + 1) * dim
            d = [m._nf4_fast["desc"] for m in mods]
            out.append(("wqkv", [d[0]], h, qkv, 0, None, attn_norm))
            out.append(("wo", [d[1]], ib + 2 * self.attn_off[l], wo, 1, h, None))
            out.append(("w13", [d[2], d[3]], wo, gate, "gated", None, ffn_norm))
            out.append(("w2", [d[4]], gate, w2, 1, wo, None))
            h = w2
        return out


def step_workspace(layers, io, device):
    import torch

    from ttspipe_b200 import _lib

    L = _lib.lib()
    need = max(int(L.nf4b_gemm_workspace_size(ctypes.byref(m._nf4_fast["desc"]), 1)) for m in layers[0])
    need = max(need, 64 << 20)   # covers every chain of S2-Pro layers at M=1 (each launch checks)
    return torch.zeros(need, dtype=torch.uint8, device=device)


MODES = {
    "step": "the whole step (36 layers x [wqkv with attention_norm fused, wo + residual, the W1/W3 gate with "
            "ffn_norm fused, w2 + residual] = 144 dependent matmuls) as ONE nf4b_decode_step launch: a persistent "
            "kernel, one CTA per SM, that streams the next matmul's weights while the previous one's outputs are "
            "handed over",
    "decode": "the same 144 matmuls as 4 C-ABI launches per layer in stream order (nf4b_gemm_ex / nf4b_gemm_gated "
              "with the fused norms; programmatic dependent launch between them), captured as one CUDA graph; "
              "with --prefetch-distance > 0 each also names the weights of a later launch for L2 prefetch",
    "single": "one launch per projection (w1, then w3 with the silu-gate epilogue on w1's output): "
              "5 launches per layer",
    "chain": "the same 4 matmuls per layer with the same data flow, issued as nf4b_gemv_chain "
             "launches of --chain-layers layers each (job j reads its inputs only after jobs < j are done)",
}


def _chain_array(jobs):
    from ttspipe_b200 import _lib

    arr = (_lib.ChainJob * len(jobs))()
    for i, (name, descs, x, y, epi, op, nw) in enumerate(jobs):
        arr[i].w = ctypes.pointer(descs[0])
        arr[i].w3 = ctypes.pointer(descs[1]) if epi == "gated" else None
        arr[i].x, arr[i].y = x, y
        arr[i].operand = op if epi == 1 else None
        arr[i].epi = 1 if epi == 1 else 0
        arr[i].norm_weight, arr[i].norm_eps = (nw, 1e-6) if nw is not None else (None, 0.0)
    return arr


class StepPlan:
    """The launches of one step through the C ABI, built once (ctypes structs
    kept alive here) and issued on a stream; CUDA-graph capturable.

    Each launch names the weights of the launch `distance` places later as an
    L2 prefetch hint (0: no hints; separate launches only)."""

    def __init__(self, layers, io: StepIO, ws, mode: str = "step", distance: int = 0, chain_layers: int = 9):
        import torch

        from ttspipe_b200 import _lib

        self.L = _lib.lib()
        self.ws_ptr, self.ws_bytes = ws.data_ptr(), ws.numel()
        self.mode = mode
        self.launches = []   # ("gemm", desc, x, y, epi, operand, norm) | ("gated", d1, d3, x, y, norm) | ...
        weights = []         # per launch: descriptors it reads
        jobs = io.jobs(layers)
        if mode == "step":
            arr = _chain_array(jobs)
            need = int(self.L.nf4b_decode_step_workspace_size(arr, len(jobs), 1))
            if need == 0:
                raise RuntimeError(f"decode step rejected: {_lib.last_error()}")
            self.step_ws = torch.zeros(need, dtype=torch.uint8, device=ws.device)
            self.launches.append(("step", arr))
            weights.append([])
        elif mode == "chain":
            per = 4 * chain_layers
            for first in range(0, len(jobs), per):
                self.launches.append(("chain", _chain_array(jobs[first:first + per])))
                weights.append([])
        else:
            for name, descs, x, y, epi, op, nw in jobs:
                if epi == "gated" and mode == "decode":
                    self.launches.append(("gated", descs[0], descs[1], x, y, nw))
                    weights.append(descs)
                elif epi == "gated":
                    scratch = io.scratch.data_ptr()
                    self.launches.append(("gemm", descs[0], x, scratch, 0, None, nw))
                    weights.append([descs[0]])
                    self.launches.append(("gemm", descs[1], x, y, 2, scratch, nw))
                    weights.append([descs[1]])
                else:
                    self.launches.append(("gemm", descs[0], x, y, epi, op, nw))
                    weights.append(descs)
        n = len(self.launches)
        self.opts = []
        for i in range(n):
            launch = self.launches[i]
            hint = weights[(i + distance) % n][:2] if distance > 0 else []
            nw = launch[-1] if launch[0] in ("gemm", "gated") else None
            if hint or nw is not None:
                ptrs = [ctypes.pointer(d) for d in hint] + [None] * (2 - len(hint))
                self.opts.append(_lib.GemmOpts(ptrs[0], ptrs[1], nw, 1e-6 if nw is not None else 0.0))
            else:
                self.opts.append(None)

    def __len__(self):
        return len(self.launches)

    def issue(self, stream_ptr):
        from ttspipe_b200 import _lib

        L = self.L
        for launch, opts in zip(self.launches, self.opts):
            o = ctypes.byref(opts) if opts is not None else None
            if launch[0] == "step":
                arr = launch[1]
                st = L.nf4b_decode_step(arr, len(arr), 1, self.step_ws.data_ptr(), self.step_ws.numel(), stream_ptr)
            elif launch[0] == "chain":
                arr = launch[1]
                st = L.nf4b_gemv_chain(arr, len(arr), 1, self.ws_ptr, self.ws_bytes, stream_ptr)
            elif launch[0] == "gated":
                _, d1, d3, x, y, _ = launch
                st = L.nf4b_gemm_gated(ctypes.byref(d1), ctypes.byref(d3), x, y, 1, self.ws_ptr, self.ws_bytes,
                                       o, stream_ptr)
            else:
                _, desc, x, y, epi, op, _ = launch
                st = L.nf4b_gemm_ex(ctypes.byref(desc), x, y, 1, epi, op, self.ws_ptr, self.ws_bytes, o,
                                    stream_ptr)
            if st != 0:
                raise RuntimeError(f"{launch[0]} launch failed: {_lib.last_error()}")


def roofline_traffic(alg_bytes_per_launch: float):
    """DRAM bytes per launch of the GEMV: the traffic/algorithmic ratio of the
    committed ncu capture (a 9728x2560 launch, small enough to capture) scaled to
    this workload's algorithmic bytes per launch; None without the capture."""
    p = ROOT / "profiles" / "nf4_gemv_decode_traffic.json"
    try:
        d = json.loads(p.read_text())
        return round(float(d["traffic_to_algorithmic"]) * alg_bytes_per_launch)
    except Exception:  # noqa: BLE001
        return None


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:  # noqa: BLE001
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def detail(layers, io, ws, stream, device):
    """Whole-step timings of every issue mode and prefetch distance (graph
    replay), printed to stderr for the profile notes; not part of the JSON line."""
    import torch

    def graph_of(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn()
            torch.cuda.synchronize(device)
            g.capture_begin()
            fn()
            g.capture_end()
        torch.cuda.synchronize(device)
        return g

    def time_graph(g, reps=5):
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            g.replay()
            st.record(stream)
            for _ in range(reps):
                g.replay()
            en.record(stream)
        torch.cuda.synchronize(device)
        return st.elapsed_time(en) / reps * 1e3  # us per replay

    cases = [("step", 0, 0), ("decode", 0, 0), ("decode", 2, 0), ("single", 0, 0)] + [("chain", 0, c) for c in (1, 9)]
    for mode, dist, cl in cases:
        plan = StepPlan(layers, io, ws, mode, dist, cl or 9)
        g = graph_of(lambda: plan.issue(stream.cuda_stream))
        us = time_graph(g)
        log(f"  step mode={mode} prefetch_distance={dist} chain_layers={cl}: {len(plan)} launches, {us:.1f} us, "
            f"{STEP_BYTES / us / 1e3:.0f} GB/s (graph)")
        del g


def run_dualar(args, device, rank: int, world: int):
    """BASELINE config 5 on this rank's GPU: a random-init Dual-AR model, a
    512-token prompt prefilled, then `args.dualar_frames` frames replayed from
    one captured CUDA graph (device-timed, max over ranks)."""
    import torch

    from ttspipe_b200.dualar import DualARConfig, DualARDecoder

    t0 = time.time()
    dec = DualARDecoder(DualARConfig(), device, seed=17 + rank)
    g = torch.Generator().manual_seed(rank)
    dec.prefill(torch.randint(0, dec.cfg.vocab, (512,), generator=g).to(device))
    dec.capture()
    build_s = time.time() - t0
    for _ in range(3):
        dec.replay()
    torch.cuda.synchronize(device)
    n = args.dualar_frames
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(device)
    start.record()
    for _ in range(n):
        dec.replay()
    end.record()
    torch.cuda.synchronize(device)
    barrier()
    secs = max_over_ranks(start.elapsed_time(end) / 1e3, device)
    per_layer = 52_159_552
    kv = 36 * 2 * 8 * 128 * 2 * (512 + 3 + n / 2)                 # mean cache rows read per frame
    wqkv = weight_bytes(6144, 2560)
    # slow stack + LM head + fast prime (3 blocks and the last block's wqkv) +
    # 9 fast steps x 4 blocks + their codebook heads + the slow KV reads
    frame_bytes = (36 * per_layer + 2560 * 155136 * 2 + 3 * per_layer + wqkv + 36 * per_layer
                   + 9 * 2560 * 4096 * 2 + kv)
    peaks, kind = measured_peaks()
    fps = n / secs
    dec.release()
    del dec
    torch.cuda.empty_cache()
    return {
        "workload": f"config 5: random-init NF4 Dual-AR (36 slow layers + bf16 LM head 2560x155136, 4 fast layers x 9 "
                    f"steps + 2560x4096 codebook heads), 512-token prompt, {n} frames timed (positions from 515 on, "
                    f"after 3 untimed), temperature 0.7, top-p 0.8, top-k 64, repetition-aware resample; one CUDA "
                    f"graph per frame",
        "frames": n, "frames_per_s_per_replica": round(fps, 1), "frames_per_s": round(world * fps, 1),
        "codebook_tokens_per_s": round(world * fps * 10, 1), "ms_per_frame": round(1e3 / fps, 3),
        "bytes_per_frame": int(frame_bytes),
        "roofline": {"bound": "hbm", "achieved_GBps": round(frame_bytes * fps / 1e9, 1), "peak": peaks["hbm_gbs"],
                     "frac": round(frame_bytes * fps / 1e9 / float(peaks["hbm_gbs"]), 4), "peak_source": kind},
        "setup_s": round(build_s, 1),
    }


def _replay_us(issue, stream, reps: int = 5) -> float:
    """Microseconds per replay of a CUDA graph of `issue()` (its launches, in
    stream order), after one warm replay; CUDA events on the capturing stream."""
    import torch

    with torch.cuda.stream(stream):
        issue()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        g.capture_begin()
        issue()
        g.capture_end()
        g.replay()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record(stream)
        for _ in range(reps):
            g.replay()
        en.record(stream)
    stream.synchronize()
    us = st.elapsed_time(en) * 1e3 / reps
    del g
    return us


def _frac(achieved: float, peak: float) -> float:
    return round(achieved / peak, 4) if peak else None


def run_config1(device, stream, peaks) -> dict:
    """one 9728x2560 GEMV at M=1 with plain fp32 absmax,
    cold L2 (48 distinct weight copies, 672 MB, launched in turn)."""
    import torch

    from ttspipe_b200 import _lib
    from ttspipe_b200.quant import Linear4bit

    n, k, copies = 9728, 2560, 48
    mods = []
    for i in range(copies):
        g = torch.Generator(device=device).manual_seed(i)
        lin = Linear4bit.from_float(torch.randn(n, k, generator=g, device=device) * 0.02, double_quant=False)
        mods.append(lin)
    from ttspipe_b200 import nf4gemv

    for m in mods:
        assert nf4gemv.prepare(m)
    L = _lib.lib()
    x = torch.randn(1, k, device=device).to(torch.bfloat16)
    y = torch.empty(1, n, device=device, dtype=torch.bfloat16)
    ws = torch.zeros(int(L.nf4b_gemm_workspace_size(ctypes.byref(mods[0]._nf4_fast["desc"]), 1)),
                     dtype=torch.uint8, device=device)

    def issue():
        for m in mods:
            _lib.check(L.nf4b_gemm(ctypes.byref(m._nf4_fast["desc"]), x.data_ptr(), y.data_ptr(), 1, 0, None,
                                   ws.data_ptr(), ws.numel(), stream.cuda_stream))

    us = _replay_us(issue, stream) / copies
    byts = algorithmic_bytes(n, k, 1, 0, nested=False)
    gbs = byts / us / 1e3
    del mods
    return {"workload": "config 1: one 9728x2560 NF4 GEMV, M=1, blocksize 64, plain fp32 absmax; 48 distinct "
                        "weight copies launched in turn (672 MB > L2: cold)",
            "us_per_launch": round(us, 2), "bytes_per_launch": byts, "value": round(gbs, 1), "unit": "GB/s",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": _frac(gbs, float(peaks["hbm_gbs"]))},
            "kernel": "nf4_gemv_reg_kernel (plain scales)"}


def _layer_weights(layers):
    """Per layer: the five NF4 weights (wqkv = q, k, v fused; wo; w1; w3; w2)."""
    return [[m._nf4_fast["desc"] for m in mods] for mods in layers]


def run_config3(layers, device, stream, peaks) -> dict:
    """the layer's projections at batched decode M in
    {1, 8, 32, 64} (GB/s over all 36 layers: cold) and prefill M in
    {256, 512, 1024} (TFLOP/s over 8 layers, 417 MB of weights)."""
    import torch

    from ttspipe_b200 import _lib

    L = _lib.lib()
    descs = _layer_weights(layers)
    shapes = [(PROJ[i][1], PROJ[i][2]) for i in range(5)]
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device=device)
    out = {"workload": "config 3: the S2-Pro layer's projections (q, k, v fused as wqkv 6144x2560; o 2560x4096; "
                       "gate, up 9728x2560; down 2560x9728), NF4 bs64 + double quant, one launch per projection; "
                       "decode rows over all 36 layers (1.87 GB: cold L2), prefill rows over 8 layers",
           "decode": [], "prefill": []}
    for rows, n_layers, kind in ((1, 36, "decode"), (8, 36, "decode"), (32, 36, "decode"), (64, 36, "decode"),
                                 (256, 8, "prefill"), (512, 8, "prefill"), (1024, 8, "prefill")):
        xs = {kk: torch.randn(rows, kk, device=device).to(torch.bfloat16) for _, kk in shapes}
        ys = {nn: torch.empty(rows, nn, device=device, dtype=torch.bfloat16) for nn, _ in shapes}

        def issue():
            for li in range(n_layers):
                for d, (nn, kk) in zip(descs[li], shapes):
                    _lib.check(L.nf4b_gemm(ctypes.byref(d), xs[kk].data_ptr(), ys[nn].data_ptr(), rows, 0, None,
                                           ws.data_ptr(), ws.numel(), stream.cuda_stream))

        us = _replay_us(issue, stream, reps=3)
        byts = n_layers * sum(algorithmic_bytes(nn, kk, rows) for nn, kk in shapes)
        flops = n_layers * sum(2.0 * rows * nn * kk for nn, kk in shapes)
        gbs, tfs = byts / us / 1e3, flops / us / 1e6
        rec = {"rows": rows, "us_per_layer": round(us / n_layers, 2), "GBps": round(gbs, 1),
               "TFLOPps": round(tfs, 2),
               "kernel": "register-fed GEMV (nf4_gemv_reg_kernel)" if rows <= 8 else "tcgen05 GEMM"}
        if kind == "decode":
            rec["roofline"] = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                               "frac": _frac(gbs, float(peaks["hbm_gbs"]))}
        else:
            rec["roofline"] = {"bound": "tensor", "achieved": round(tfs, 1), "peak": peaks.get("bf16_tflops"),
                               "unit": "TFLOP/s", "frac": _frac(tfs, float(peaks.get("bf16_tflops") or 0)),
                               "frac_of_sustained": _frac(tfs, float(peaks.get("bf16_tflops_sustained") or 0))}
        out[kind].append(rec)
        del xs, ys
    return out


def run_config4(device, stream, peaks) -> dict:
    """RMSNorm over 2560, q/k norm-free rotary + KV write of
    one position (32 q / 8 kv heads x 128, theta 1e6), decode attention over a
    2048-row cache; 16 distinct caches (134 MB > L2) launched in turn."""
    import torch

    from ttspipe_b200 import _lib, fastpath, fusedops, model

    nh, nkv, max_len, layers = 32, 8, 2048, 16
    ks = [torch.randn(nkv, max_len, 128, device=device).to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(nkv, max_len, 128, device=device).to(torch.bfloat16) for _ in range(layers)]
    q = torch.randn(nh, 128, device=device).to(torch.bfloat16)
    o = torch.empty(nh, 128, device=device, dtype=torch.bfloat16)
    pos = torch.tensor([max_len - 1], device=device)
    hidden = torch.randn(1, 2560, device=device).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(2560, device=device)).to(torch.bfloat16)
    qkv = torch.randn((nh + 2 * nkv) * 128, device=device).to(torch.bfloat16)
    freqs = model.precompute_freqs_cis(4096, 128, 1e6, device=device)
    L = _lib.lib()

    def attention():
        for i in range(layers):
            fastpath.kernel_attention(q, ks[i], vs[i], o, n_head=nh, n_kv=nkv, pos=pos, window=max_len,
                                      max_len=max_len)

    def norm():
        for _ in range(layers):
            fusedops.rms_norm(hidden, nw, 1e-6)

    def rope_kv():
        for i in range(layers):
            _lib.check(L.nf4b_qk_rope_kv(qkv.data_ptr(), None, None, 1e-6, freqs.data_ptr(), _lib.NF4B_BF16,
                                         pos.data_ptr(), o.data_ptr(), ks[i].data_ptr(), vs[i].data_ptr(), nh, nkv,
                                         128, max_len, stream.cuda_stream))

    att_us = _replay_us(attention, stream) / layers
    norm_us = _replay_us(norm, stream) / layers
    rope_us = _replay_us(rope_kv, stream) / layers
    kv_bytes = 2 * nkv * max_len * 128 * 2
    gbs = kv_bytes / att_us / 1e3
    return {"workload": "config 4: RMSNorm (hidden 2560, eps 1e-6), rotary + KV write of one position "
                        "(32 q / 8 kv heads x 128, theta 1e6, bf16 freqs), GQA decode attention over L = 2048 "
                        "cached rows; 16 distinct caches (134 MB > L2) in turn",
            "attention_us": round(att_us, 2), "attention_GBps_of_kv": round(gbs, 1), "kv_bytes": kv_bytes,
            "rms_norm_us": round(norm_us, 2), "rope_kv_us": round(rope_us, 2),
            "launches_per_layer_step": 3,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": _frac(gbs, float(peaks["hbm_gbs"])),
                         "kernel": "decode attention (8-CTA cluster per KV head, 2-D TMA chunks, mma.sync scores and P.V)"}}


def run_reference_gpu(layers, device, stream, peaks) -> dict:
    """The reference's own GPU kernel, nf4_mma (app/engine/nf4gemv.py:94-231,
    fp16 only), compiled from its source by oracle/build_ref.py into
    oracle/_ref/nf4mma_ref.so and launched as its matmul does, on the same 36
    layers of NF4 weights at M in {1, 8, 32} (one launch per projection, no
    epilogue): GB/s beside this build's GEMV on the same launches (config 3)."""
    import numpy as np
    import torch

    from oracle import build_ref
    from ttspipe_b200 import _lib

    path = build_ref.gpu_so_path()
    if path is None:
        return {"unavailable": "oracle/_ref/nf4mma_ref.so was not built (the reference checkout is needed to build it)"}
    ref = ctypes.CDLL(str(path))
    ref.nf4mma_ref_launch.restype = ctypes.c_int
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    ref.nf4mma_ref_launch.argtypes = [i32, i32, vp, vp, vp, vp, vp, vp, vp, ctypes.c_float, i32, i32, i32, i32,
                                      i32, vp, i32, vp]
    from oracle import nf4_oracle as orc

    lut = torch.tensor(orc.NF4_CODE, dtype=torch.float32, device=device)
    descs = _layer_weights(layers)
    shapes = [(PROJ[i][1], PROJ[i][2]) for i in range(5)]
    out = {"workload": "the reference's nf4_mma (fp16; NVRTC source compiled with nvcc --use_fast_math for "
                       "sm_100a, launched with its own grid/block choice) on the config-2 layer's projections "
                       "at M rows, 36 layers in turn (cold L2)", "rows": []}
    L = _lib.lib()
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device=device)
    for rows in (1, 8, 32):
        xs = {kk: torch.randn(rows, kk, device=device).to(torch.float16) for _, kk in shapes}
        ys = {nn: torch.empty(rows, nn, device=device, dtype=torch.float16) for nn, _ in shapes}

        def call(d, nn, kk):
            st = ref.nf4mma_ref_launch(rows, 1, xs[kk].data_ptr(), d.packed, d.absmax_code, d.absmax, d.code2,
                                       ys[nn].data_ptr(), lut.data_ptr(), d.offset, nn, kk, kk // 64, 6,
                                       int(d.blocksize2).bit_length() - 1, None, 0, stream.cuda_stream)
            if st != 0:
                raise RuntimeError(f"reference nf4_mma launch failed ({st})")

        def issue():
            for li in range(N_LAYERS):
                for d, (nn, kk) in zip(descs[li], shapes):
                    call(d, nn, kk)

        us = _replay_us(issue, stream, reps=3)
        byts = N_LAYERS * sum(algorithmic_bytes(nn, kk, rows) for nn, kk in shapes)
        gbs = byts / us / 1e3
        # the same products through this build: in fp16 on the very same inputs
        # (like for like, and a check of the outputs), and in bf16
        f16 = ctypes.byref(_lib.GemmOpts(None, None, None, 0.0, _lib.NF4B_F16))
        yh = {nn: torch.empty(rows, nn, device=device, dtype=torch.float16) for nn, _ in shapes}
        xb = {kk: v.to(torch.bfloat16) for kk, v in xs.items()}
        yb = {nn: torch.empty(rows, nn, device=device, dtype=torch.bfloat16) for nn, _ in shapes}

        def ours(x, y, opts):
            for li in range(N_LAYERS):
                for d, (nn, kk) in zip(descs[li], shapes):
                    _lib.check(L.nf4b_gemm_ex(ctypes.byref(d), x[kk].data_ptr(), y[nn].data_ptr(), rows, 0, None,
                                              ws.data_ptr(), ws.numel(), opts, stream.cuda_stream))

        ours_us = _replay_us(lambda: ours(xs, yh, f16), stream, reps=3)
        ours_bf_us = _replay_us(lambda: ours(xb, yb, None), stream, reps=3)
        d, (nn, kk) = descs[0][0], shapes[0]
        call(d, nn, kk)
        _lib.check(L.nf4b_gemm_ex(ctypes.byref(d), xs[kk].data_ptr(), yh[nn].data_ptr(), rows, 0, None,
                                  ws.data_ptr(), ws.numel(), f16, stream.cuda_stream))
        stream.synchronize()
        a, b2 = ys[nn].double().cpu().numpy(), yh[nn].double().cpu().numpy()
        rel = float(np.abs(a - b2).max() / (np.sqrt((a ** 2).mean()) + 1e-12))
        out["rows"].append({"rows": rows, "reference_us_per_layer": round(us / N_LAYERS, 2),
                            "reference_GBps": round(gbs, 1),
                            "reference_frac_of_hbm": _frac(gbs, float(peaks["hbm_gbs"])),
                            "ours_f16_us_per_layer": round(ours_us / N_LAYERS, 2),
                            "ours_f16_GBps": round(byts / ours_us / 1e3, 1),
                            "speedup_f16": round(us / ours_us, 2),
                            "ours_bf16_us_per_layer": round(ours_bf_us / N_LAYERS, 2),
                            "ours_bf16_GBps": round(byts / ours_bf_us / 1e3, 1),
                            "speedup_bf16": round(us / ours_bf_us, 2),
                            "f16_max_abs_diff_over_rms": round(rel, 5)})
    return out


def run_gpu(args):
    import torch

    from ttspipe_b200 import _lib, nf4gemv

    rank, world, local = dist_init("nccl")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    assert nf4gemv.available(), "libnf4b200.so must load on a B200"

    t0 = time.time()
    layers = make_layers(device, rank)
    io = StepIO(device, rank)
    ws = step_workspace(layers, io, device)
    plan = StepPlan(layers, io, ws, args.mode, args.prefetch_distance, args.chain_layers)
    log(f"[rank {rank}] built {N_LAYERS} layers in {time.time() - t0:.1f}s; step bytes {STEP_BYTES / 1e9:.3f} GB")

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        plan.issue(stream.cuda_stream)   # eager warm-up of every call
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        graph.capture_begin()
        plan.issue(stream.cuda_stream)
        graph.capture_end()
    stream.synchronize()

    def timed(fn, steps):
        """Seconds for `steps` calls (first to last event), and each step's ms
        (an event after every step; the same bracket)."""
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        barrier()
        torch.cuda.synchronize(device)
        evs[0].record(stream)
        for i in range(steps):
            fn()
            evs[i + 1].record(stream)
        torch.cuda.synchronize(device)
        barrier()
        per_step = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
        return evs[0].elapsed_time(evs[-1]) / 1e3, per_step

    def step_graph():
        with torch.cuda.stream(stream):
            graph.replay()

    def step_e2e():
        with torch.cuda.stream(stream):
            io.dev_in.copy_(io.host_in, non_blocking=True)
            graph.replay()
            io.host_out.copy_(io.dev_out, non_blocking=True)

    for _ in range(args.warmup):
        step_graph()
    torch.cuda.synchronize(device)

    with ClockSampler([local] if world == 1 else list(range(world))) as clocks:
        torch.cuda.profiler.start()   # bounds an `ncu --profile-from-start off` launch list to the timed steps
        secs, step_ms = timed(step_graph, args.steps)
        torch.cuda.profiler.stop()
    clock = clocks.summary()
    for _ in range(max(1, args.warmup)):
        step_e2e()
    e2e_secs, _ = timed(step_e2e, args.steps)

    secs_max = max_over_ranks(secs, device)
    e2e_max = max_over_ranks(e2e_secs, device)
    value = world * STEP_BYTES * args.steps / secs_max / 1e9
    e2e_value = world * STEP_BYTES * args.steps / e2e_max / 1e9
    per_rank = STEP_BYTES * args.steps / secs / 1e9

    # per-projection timing (eager, events around 20 launches of one shape over
    # rotating layers) - printed to stderr for the profile notes only
    if rank == 0 and args.detail:
        detail(layers, io, ws, stream, device)

    peaks, peak_kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    achieved = STEP_BYTES / (secs / args.steps) / 1e9
    traffic = roofline_traffic(STEP_BYTES / len(plan))
    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(secs_max / args.steps * 1e3, 4),
            "step_ms_quantiles": {q: round(statistics.quantiles(step_ms, n=10)[i], 4) if len(step_ms) >= 2
                                  else round(step_ms[0], 4) for q, i in (("p10", 0), ("p50", 4), ("p90", 8))},
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init NF4 weights N(0,0.02), norm weights N(1,0.1), first h and attention "
                    "stand-ins N(0,1), seeded per rank)",
            "config": {"workload": "S2-Pro slow-AR decode matmuls with the decode block's data flow: 36 layers x "
                                   "[wqkv 6144x2560 on rmsnorm(h), wo 2560x4096 on attn + h, "
                                   "silu(x W1)*(x W3) W1,W3 9728x2560 on rmsnorm(wo out), w2 2560x9728 on the "
                                   "gate + wo out -> next h], M=1, NF4 bs64 + double-quant (bs2 256)",
                       "schedule": f"{args.mode}: {MODES[args.mode]}",
                       "prefetch_distance": args.prefetch_distance,
                       "chain_layers": args.chain_layers if args.mode == "chain" else None,
                       "baseline_config": "configs[1] (one slow-AR layer's linears at M=1) x 36 distinct layers",
                       "bytes_per_step": STEP_BYTES, "rows": 1,
                       "l2": "inputs larger than L2 (1.87 GB of weights per step per GPU)",
                       "parallelism": f"replicas x{world} (no collective on the data path)"},
            "gpu_launches": len(plan) * args.steps,
            "launches_per_step": len(plan),
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": io.h2d_bytes,
                    "d2h_bytes_per_step": io.d2h_bytes,
                    "path": ("C ABI nf4b_decode_step call" if args.mode == "step" else "C ABI nf4b_gemm calls")
                            + " (CUDA graph) + pinned H2D inputs + D2H outputs per step"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_source": peak_kind,
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": STEP_BYTES // len(plan),
                         "kernel": ("nf4_decode_step_kernel (persistent decode step: the step's 144 matmuls "
                                    "in one launch)" if args.mode == "step" else
                                    "nf4_gemv_reg_kernel (register-fed pair GEMV), plain and gated")
                                   + "; achieved = step bytes / step time (handoffs and launch gaps included)"},
            "clocks": clock,
            "per_rank_GBps": round(per_rank, 1),
        }
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    del graph
    if not args.no_configs:
        peaks_d = peaks
        configs = {"config1": run_config1(device, stream, peaks_d),
                   "config3": run_config3(layers, device, stream, peaks_d),
                   "config4": run_config4(device, stream, peaks_d),
                   "reference_gpu_kernel": run_reference_gpu(layers, device, stream, peaks_d)}
        if rank == 0:
            result.update(configs)
    if args.dualar_frames > 0:
        dual = run_dualar(args, device, rank, world)
        if rank == 0:
            result["dualar"] = dual
    import torch.distributed as dist

    if dist.is_initialized():
        barrier()
        dist.destroy_process_group()
    return result


# --------------------------------------------------------------------------
# the CPU reference: the reference's own nf4cpu kernels (oracle/_ref)
# --------------------------------------------------------------------------


CPU_SHAPES = [(6144, 2560), (2560, 4096), (19456, 2560), (2560, 9728)]  # wqkv, wo, w13, w2


def cpu_layer_bytes(rows: int = 1) -> int:
    """Bytes one layer pass of the reference's CPU kernel moves: packed codes,
    the bf16 absmax it reads (2 B per 64-block; it takes no double-quantised
    scales), x and y. The w13 output is 2 x 9728 wide on the CPU path (it
    returns both products); the residual adds are not part of its GEMV."""
    return sum(n * k // 2 + 2 * (n * k // BS) + 2 * rows * k + 2 * rows * n for n, k in CPU_SHAPES)


CPU_LAYER_BYTES = cpu_layer_bytes()


def _cpu_layers(count: int):
    """Random packed NF4 bytes and bf16 absmax for `count` layers, generated
    directly as the reference's own CPU test does (tests/test_nf4cpu.py:31-35);
    the kernel's speed does not depend on the values. w1 and w3 are one fused
    w13 matmul, as the reference's CPU path serves them (app/engine/cpu.py:98-126)."""
    import torch

    layers = []
    for li in range(count):
        g = torch.Generator().manual_seed(li)
        mods = []
        for n, k in CPU_SHAPES:
            packed = torch.randint(0, 255, (n, k // 2), dtype=torch.uint8, generator=g)
            absmax = (torch.rand(n, k // 64, generator=g) * 0.1).to(torch.bfloat16)
            mods.append((packed, absmax, n, k))
        layers.append(mods)
    return layers


def _reference_ext():
    from oracle import build_ref

    return build_ref.load()


def cpu_gemv_runner():
    """(callable(x, packed, absmax, n) -> y, kind, note)."""
    import torch

    from oracle import nf4_oracle as orc

    code16 = torch.tensor(orc.NF4_CODE).to(torch.bfloat16)
    try:
        ext = _reference_ext()
        return (lambda x, p, a, n: ext.nf4_gemv(x, p, a, code16, n)), "reference", \
            "reference app/engine/nf4cpu.py nf4_gemv (AVX-512 BF16), built by oracle/build_ref.py"
    except Exception as exc:  # noqa: BLE001
        def port(x, p, a, n):
            y = orc.nf4cpu_gemv(x.view(torch.int16).numpy().view("uint16"), p.numpy(),
                                a.view(torch.int16).numpy().view("uint16"),
                                code16.view(torch.int16).numpy().view("uint16"))
            return torch.from_numpy(y.view("int16")).view(torch.bfloat16)
        return port, "port", f"oracle port (numpy), reference unavailable: {exc}"


def cpu_baseline(seconds: float) -> dict:
    import torch

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    run, kind, note = cpu_gemv_runner()
    layers = _cpu_layers(4)
    xs = {k: torch.randn(1, k).to(torch.bfloat16) for _, k in CPU_SHAPES}
    for mods in layers[:1]:
        for p, a, n, k in mods:
            run(xs[k], p, a, n)
    done_bytes, t0 = 0, time.perf_counter()
    li = 0
    while time.perf_counter() - t0 < seconds:
        for p, a, n, k in layers[li % len(layers)]:
            run(xs[k], p, a, n)
        done_bytes += CPU_LAYER_BYTES
        li += 1
    el = time.perf_counter() - t0
    return {"value": round(done_bytes / el / 1e9, 2), "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{li} layer passes (wqkv, wo, w13, w2 at M=1; 4 distinct layers cycled) in {el:.1f}s, "
                      f"credited with the bytes the CPU kernel reads ({CPU_LAYER_BYTES} B per layer: bf16 absmax); "
                      f"{note}"}


def run_reference(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    run, kind, note = cpu_gemv_runner()
    n_layers = N_LAYERS if kind == "reference" else 2
    layers = _cpu_layers(n_layers)
    xs = {k: torch.randn(1, k).to(torch.bfloat16) for _, k in CPU_SHAPES}

    def step():
        for mods in layers:
            for p, a, n, k in mods:
                run(xs[k], p, a, n)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    step_bytes = n_layers * CPU_LAYER_BYTES
    value = step_bytes * args.steps / el / 1e9
    # n_gpus: the N of the run this line stands beside (the reference's NF4 path is
    # CPU-only: rank 0 times it on the host cores, the GPUs stay idle)
    return {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": args.gpus, "impl": "reference",
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random packed NF4 bytes, bf16 absmax, x N(0,1))",
            "config": {"workload": f"{n_layers} layers x [wqkv 6144x2560, wo 2560x4096, w13 19456x2560, "
                                   "w2 2560x9728], M=1, NF4 bs64 (bf16 absmax, as the reference's CPU path)",
                       "bytes_per_step": step_bytes,
                       "bytes": "what the CPU kernel reads: packed codes, bf16 absmax, x, y"},
            "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": f"{args.steps} steps of {n_layers} layers; {note}"},
            "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}



# --------------------------------------------------------------------------
# profiling cases (`--case <kernel>`): small, self-contained cases of each
# hot-path kernel for ncu captures and graph-replay timings
# --------------------------------------------------------------------------
#
# `python bench.py --case <kernel> [options]` builds a few distinct weight
# copies or caches (enough to exceed the 126 MB L2, a few hundred MB at most on
# the device), warms up, and issues a bounded number of launches - sized so
# that an `ncu --set full -k <kernel> -c 3` capture of it ends in a minute or
# two. With `--time` it instead replays the launches from a CUDA graph and
# prints CUDA-event timings (never under a profiler).
#
# kernels: gemv (M rows <= 8), gated (the W1/W3 gate, M <= 8), gemm (tcgen05,
# M > 8), head (a bf16 output head, `--n` ids x `--k`), attention (decode,
# qk_rope_kv + attention at a given cache length), prefill (the seven S2-Pro
# projections at M rows through the GEMM, TFLOP/s), dualar (the config-5 frame
# graph: `--frames` replays between cudaProfilerStart/Stop, for an
# `ncu --profile-from-start off` launch list; with --time, ms per frame).

S2PRO = [("q", 4096, 2560), ("k", 1024, 2560), ("v", 1024, 2560), ("o", 2560, 4096),
         ("gate", 9728, 2560), ("up", 9728, 2560), ("down", 2560, 9728)]


def _weights(n: int, k: int, copies: int, nested: bool):
    import torch

    from ttspipe_b200 import nf4gemv
    from ttspipe_b200.quant import Linear4bit

    mods = []
    for i in range(copies):
        g = torch.Generator(device="cuda").manual_seed(i)
        w = torch.randn(n, k, generator=g, device="cuda") * 0.02
        lin = Linear4bit.from_float(w, double_quant=nested)
        assert nf4gemv.prepare(lin)
        mods.append(lin)
    return mods


def _graph_time(fn, reps: int = 5) -> float:
    """Microseconds per call of `fn`, replayed from a CUDA graph."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn()
        g.replay()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record(s)
        for _ in range(reps):
            g.replay()
        en.record(s)
    torch.cuda.synchronize()
    return st.elapsed_time(en) * 1e3 / reps


def run_matmul(n: int, k: int, rows: int, copies: int, launches: int, nested: bool, timed: bool) -> None:
    import torch

    from ttspipe_b200 import nf4gemv

    mods = _weights(n, k, copies, nested)
    x = torch.randn(rows, k, device="cuda").to(torch.bfloat16)
    for m in mods:                       # warm-up: one launch per copy
        nf4gemv.matmul(m, x)
    torch.cuda.synchronize()
    if timed:
        us = _graph_time(lambda: [nf4gemv.matmul(mods[i % copies], x) for i in range(launches)]) / launches
        flops = 2.0 * rows * n * k
        print(f"{n}x{k} rows={rows}: {us:.2f} us/launch, {flops / us / 1e6:.1f} TFLOP/s")
        return
    for i in range(launches):
        nf4gemv.matmul(mods[i % copies], x)
    torch.cuda.synchronize()


def run_prefill(rows: int) -> None:
    """The seven S2-Pro projections at `rows` activation rows."""
    import torch

    from ttspipe_b200 import nf4gemv

    total_flops, total_us = 0.0, 0.0
    for name, n, k in S2PRO:
        mods = _weights(n, k, 2, True)
        x = torch.randn(rows, k, device="cuda").to(torch.bfloat16)
        us = _graph_time(lambda: [nf4gemv.matmul(mods[i % 2], x) for i in range(4)]) / 4
        flops = 2.0 * rows * n * k
        total_flops += flops
        total_us += us
        print(f"  {name} {n}x{k} M={rows}: {us:.1f} us, {flops / us / 1e6:.1f} TFLOP/s")
    print(f"layer M={rows}: {total_us:.1f} us, {total_flops / total_us / 1e6:.1f} TFLOP/s")


def run_gated(n: int, k: int, rows: int, copies: int, launches: int, timed: bool) -> None:
    """The FeedForward gate silu(x W1^T) * (x W3^T) in one launch per pair."""
    import torch

    from ttspipe_b200 import nf4gemv

    mods = _weights(n, k, 2 * copies, True)
    x = torch.randn(rows, k, device="cuda").to(torch.bfloat16)
    for i in range(copies):
        nf4gemv.matmul_gated(mods[2 * i], mods[2 * i + 1], x)
    torch.cuda.synchronize()

    def go(i):
        nf4gemv.matmul_gated(mods[2 * (i % copies)], mods[2 * (i % copies) + 1], x)

    if timed:
        us = _graph_time(lambda: [go(i) for i in range(launches)]) / launches
        print(f"gated 2x{n}x{k} rows={rows}: {us:.2f} us/launch, {2 * n * k / 2 / us / 1e3:.0f} GB/s of codes")
        return
    for i in range(launches):
        go(i)
    torch.cuda.synchronize()


def run_attention(length: int, launches: int, timed: bool) -> None:
    import torch

    from ttspipe_b200 import fastpath

    nh, nkv, max_len = 32, 8, 2048
    layers = 16   # 16 distinct caches of 8.4 MB = 134 MB > L2
    ks = [torch.randn(nkv, max_len, 128, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(nkv, max_len, 128, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    q = torch.randn(nh, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty(nh, 128, device="cuda", dtype=torch.bfloat16)
    pos = torch.tensor([length - 1], device="cuda")

    def go(i):
        fastpath.kernel_attention(q, ks[i % layers], vs[i % layers], out, n_head=nh, n_kv=nkv,
                                  pos=pos, window=max_len, max_len=max_len)

    for i in range(layers):
        go(i)
    torch.cuda.synchronize()
    if timed:
        us = _graph_time(lambda: [go(i) for i in range(layers)]) / layers
        kv_bytes = 2 * nkv * length * 128 * 2
        print(f"decode attention L={length}: {us:.2f} us/launch, {kv_bytes / us / 1e3:.0f} GB/s of KV")
        return
    for i in range(launches):
        go(i)
    torch.cuda.synchronize()


def run_case_dualar(frames: int, timed: bool) -> None:
    """The Dual-AR frame graph (random-init model, 512-token prompt, 3 warm replays)."""
    import torch

    from ttspipe_b200.dualar import DualARConfig, DualARDecoder

    dev = torch.device("cuda", torch.cuda.current_device())
    dec = DualARDecoder(DualARConfig(), dev, seed=17)
    g = torch.Generator().manual_seed(0)
    dec.prefill(torch.randint(0, dec.cfg.vocab, (512,), generator=g).to(dev))
    dec.capture()
    for _ in range(3):
        dec.replay()
    torch.cuda.synchronize()
    if timed:
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(frames):
            dec.replay()
        en.record()
        torch.cuda.synchronize()
        print(f"dual-AR frame: {st.elapsed_time(en) / frames:.3f} ms")
    else:
        torch.cuda.profiler.start()
        for _ in range(frames):
            dec.replay()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    dec.release()


def run_head(n: int, k: int, copies: int, launches: int, timed: bool) -> None:
    """A bf16 output head (the LM head 155136 x 2560, or a codebook head 4096 x
    2560) on one activation row: `heads.dense_linear`."""
    import torch

    from ttspipe_b200 import heads

    copies = max(1, min(copies, (1 << 30) // (n * k * 2) + 1))  # >= 1 GB of distinct weights in all
    ws = [(torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(copies)]
    x = torch.randn(k, device="cuda").to(torch.bfloat16)
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)

    def go(i):
        heads.dense_linear(ws[i % copies], x, out=out)

    for i in range(copies):
        go(i)
    torch.cuda.synchronize()
    if timed:
        reps = max(copies, 4)
        us = _graph_time(lambda: [go(i) for i in range(reps)]) / reps
        print(f"dense head {n}x{k}: {us:.2f} us/launch, {n * k * 2 / us / 1e3:.0f} GB/s")
        return
    for i in range(launches):
        go(i)
    torch.cuda.synchronize()




def run_case(a) -> None:
    from ttspipe_b200 import nf4gemv

    assert nf4gemv.available()
    if a.case in ("gemv", "gemm"):
        rows = a.rows if a.case == "gemv" else max(a.rows, 9)
        run_matmul(a.n, a.k, rows, a.copies, a.launches, not a.plain, a.time)
    elif a.case == "prefill":
        run_prefill(a.rows)
    elif a.case == "gated":
        run_gated(a.n, a.k, a.rows, a.copies, a.launches, a.time)
    elif a.case == "dualar":
        run_case_dualar(a.frames, a.time)
    elif a.case == "head":
        run_head(a.n, a.k, a.copies, a.launches, a.time)
    else:
        run_attention(a.length, a.launches, a.time)
    print("ok", file=sys.stderr)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--detail", action="store_true")
    ap.add_argument("--mode", default="decode", choices=sorted(MODES))
    ap.add_argument("--chain-layers", type=int, default=9, help="layers per nf4b_gemv_chain launch (--mode chain)")
    ap.add_argument("--dualar-frames", type=int, default=1024,
                    help="Dual-AR frames timed after the GEMV step (config 5: 1024 slow steps; 0: skip)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the config 1 / 3 / 4 and reference-GPU-kernel objects of the JSON line")
    ap.add_argument("--prefetch-distance", type=int, default=0,
                    help="launches ahead whose weights each launch streams into L2 (0: none; "
                         "measured slower at 1-3 on B200, so off by default)")
    ap.add_argument("--case", default=None,
                    choices=["gemv", "gated", "gemm", "attention", "prefill", "dualar", "head"],
                    help="run one profiling case instead of the benchmark (see 'profiling cases')")
    ap.add_argument("--n", type=int, default=9728)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--copies", type=int, default=12)
    ap.add_argument("--launches", type=int, default=12)
    ap.add_argument("--plain", action="store_true", help="--case: fp32 absmax instead of double quant")
    ap.add_argument("--length", type=int, default=2048)
    ap.add_argument("--time", action="store_true", help="--case: time from a CUDA graph instead")
    ap.add_argument("--frames", type=int, default=2, help="--case dualar: frames replayed")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.case is not None:
        run_case(args)
        return
    if args.impl == "reference":
        res = run_reference(args)
    else:
        res = run_gpu(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
