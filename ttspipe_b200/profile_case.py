"""Small, self-contained cases of each hot-path kernel, for profiling and timing.

`python -m ttspipe_b200.profile_case <kernel> [options]` builds a few distinct
weight copies or caches (enough to exceed the 126 MB L2, a few hundred MB at
most on the device), warms up, and issues a bounded number of launches - sized
so that an `ncu --set full -k <kernel> -c 3` capture of it ends in a minute or
two. With `--time` it instead replays the launches from a CUDA graph and
prints CUDA-event timings (never under a profiler).

kernels: gemv (M rows <= 32), gated (the W1/W3 gate, M <= 4), gemm (tcgen05, M > 32), head (a bf16
output head, `--n` ids x `--k`), attention (decode,
qk_rope_kv + split-KV attention at a given cache length), prefill (the seven
S2-Pro projections at M rows through the GEMM, TFLOP/s), dualar (the config-5
frame graph: `--frames` replays between cudaProfilerStart/Stop, for an
`ncu --profile-from-start off` launch list; with --time, ms per frame).
"""

from __future__ import annotations

import argparse
import sys

import torch

S2PRO = [("q", 4096, 2560), ("k", 1024, 2560), ("v", 1024, 2560), ("o", 2560, 4096),
         ("gate", 9728, 2560), ("up", 9728, 2560), ("down", 2560, 9728)]


def _weights(n: int, k: int, copies: int, nested: bool):
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


def run_dualar(frames: int, timed: bool) -> None:
    """The Dual-AR frame graph (random-init model, 512-token prompt, 3 warm replays)."""
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


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemv", "gated", "gemm", "attention", "prefill", "dualar", "head"])
    ap.add_argument("--n", type=int, default=9728)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--copies", type=int, default=12)
    ap.add_argument("--launches", type=int, default=12)
    ap.add_argument("--plain", action="store_true", help="fp32 absmax instead of double quant")
    ap.add_argument("--length", type=int, default=2048)
    ap.add_argument("--time", action="store_true", help="time from a CUDA graph instead")
    ap.add_argument("--frames", type=int, default=2, help="dualar: frames replayed")
    a = ap.parse_args(argv)
    from ttspipe_b200 import nf4gemv

    assert nf4gemv.available()
    if a.kernel in ("gemv", "gemm"):
        rows = a.rows if a.kernel == "gemv" else max(a.rows, 33)
        run_matmul(a.n, a.k, rows, a.copies, a.launches, not a.plain, a.time)
    elif a.kernel == "prefill":
        run_prefill(a.rows)
    elif a.kernel == "gated":
        run_gated(a.n, a.k, a.rows, a.copies, a.launches, a.time)
    elif a.kernel == "dualar":
        run_dualar(a.frames, a.time)
    elif a.kernel == "head":
        run_head(a.n, a.k, a.copies, a.launches, a.time)
    else:
        run_attention(a.length, a.launches, a.time)
    print("ok", file=sys.stderr)


if __name__ == "__main__":
    main()
