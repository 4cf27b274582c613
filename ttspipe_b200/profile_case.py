"""Small, self-contained cases of each hot-path kernel for profiling.

`python -m ttspipe_b200.profile_case <kernel> [options]` builds a few distinct
weight copies (enough to exceed the 126 MB L2, a few hundred MB at most on the
device), warms up, and issues a bounded number of launches - sized so that an
`ncu --set full -k <kernel> -c 3` capture of it ends in a minute or two.

kernels: gemv (M rows <= 32), gemm (tcgen05, M > 32), attention, block.
"""

from __future__ import annotations

import argparse
import ctypes
import sys

import torch


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


def run_matmul(n: int, k: int, rows: int, copies: int, launches: int, nested: bool) -> None:
    from ttspipe_b200 import nf4gemv

    mods = _weights(n, k, copies, nested)
    x = torch.randn(rows, k, device="cuda").to(torch.bfloat16)
    for m in mods:                       # warm-up: one launch per copy
        nf4gemv.matmul(m, x)
    torch.cuda.synchronize()
    for i in range(launches):
        nf4gemv.matmul(mods[i % copies], x)
    torch.cuda.synchronize()


def run_attention(length: int, launches: int) -> None:
    from ttspipe_b200 import fastpath

    nh, nkv, max_len = 32, 8, 2048
    layers = 16   # 16 distinct caches of 8.4 MB = 134 MB > L2
    ks = [torch.randn(nkv, max_len, 128, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(nkv, max_len, 128, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    q = torch.randn(nh, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty(nh, 128, device="cuda", dtype=torch.bfloat16)
    pos = torch.tensor([length - 1], device="cuda")
    for i in range(layers + launches):
        fastpath.kernel_attention(q, ks[i % layers], vs[i % layers], out, n_head=nh, n_kv=nkv,
                                  pos=pos, window=max_len, max_len=max_len)
    torch.cuda.synchronize()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemv", "gemm", "attention"])
    ap.add_argument("--n", type=int, default=9728)
    ap.add_argument("--k", type=int, default=2560)
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--copies", type=int, default=12)
    ap.add_argument("--launches", type=int, default=12)
    ap.add_argument("--plain", action="store_true", help="fp32 absmax instead of double quant")
    ap.add_argument("--length", type=int, default=2048)
    a = ap.parse_args(argv)
    from ttspipe_b200 import nf4gemv

    assert nf4gemv.available()
    if a.kernel in ("gemv", "gemm"):
        rows = a.rows if a.kernel == "gemv" else max(a.rows, 33)
        run_matmul(a.n, a.k, rows, a.copies, a.launches, not a.plain)
    else:
        run_attention(a.length, a.launches)
    print("ok", file=sys.stderr)


if __name__ == "__main__":
    main()
