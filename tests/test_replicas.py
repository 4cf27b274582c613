"""The multi-GPU story is one independent replica per GPU with no data-path
collective. The only cross-rank steps are the bench's
barriers and the max-over-ranks of the timed seconds; these run here as gloo
ranks on the CPU, including a rank that dies before the reduction."""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import bench
    from datetime import timedelta

    dist.init_process_group("gloo", timeout=timedelta(seconds=10))
    try:
        if mode == "max":
            got = bench.max_over_ranks(1.5 + rank, torch.device("cpu"))
            bench.barrier()
            out[rank] = got
        elif mode == "dies":
            if rank == 1:
                os._exit(0)     # leaves between steps: no collective in flight
            try:
                bench.max_over_ranks(1.0, torch.device("cpu"))
                out[rank] = "no-error"
            except Exception as exc:  # noqa: BLE001
                out[rank] = f"error:{type(exc).__name__}"
    finally:
        if mode != "dies" or rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _spawn(mode, world=2):
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        assert not p.is_alive()
    return dict(out)


def test_seconds_are_reduced_as_the_max_over_ranks():
    out = _spawn("max")
    assert out == {0: 2.5, 1: 2.5}


def test_a_dead_replica_surfaces_as_an_error_not_a_hang():
    out = _spawn("dies")
    assert out[0].startswith("error:")


def test_the_reference_arm_runs_on_rank_0_only():
    """Launched under torchrun, `bench.py --impl reference` works on rank 0
    alone: every other rank exits 0 at once, prints nothing and joins no
    rendezvous (an unreachable master port would fail it)."""
    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1", MASTER_ADDR="127.0.0.1", MASTER_PORT="1")
    r = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=180, cwd=root, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
