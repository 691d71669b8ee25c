"""Helper to run a function in N spawned ranks (one process per rank) and collect results.

Used by the multi-process tests (Gloo on CPU, NCCL + NVLink kernels on GPUs). Rendezvous is on
127.0.0.1 with a free port; every rank gets a bounded process-group timeout so a missing peer ends
the test with an error instead of a hang.
"""
import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, fn, args, q, env):
    os.environ.update(env)
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    try:
        out = fn(rank, world, *args)
        q.put((rank, "ok", out))
    except BaseException as e:  # report, never hang the parent
        q.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def run_ranks(fn, world: int, *args, env: dict | None = None, timeout: float = 240.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q, dict(env or {}))) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, out = q.get(timeout=timeout)
            results[rank] = (status, out)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    errs = {r: o for r, (s, o) in results.items() if s != "ok"}
    if errs:
        raise AssertionError("rank failures:\n" + "\n".join(f"rank {r}: {o}" for r, o in sorted(errs.items())))
    return [results[r][1] for r in range(world)]
