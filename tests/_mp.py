"""Helper to run a function in N spawned ranks (one process per rank) and collect results.

Used by the multi-process tests (Gloo on CPU, NCCL + NVLink kernels on GPUs). Rendezvous is on
127.0.0.1 with a free port; every rank gets a bounded process-group timeout so a missing peer ends
the test with an error instead of a hang.
"""
import faulthandler
import os
import queue
import socket
import sys
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
    # a rank that is still running near the parent's deadline prints every thread's stack to stderr
    faulthandler.dump_traceback_later(float(os.environ.get("BRAIN_TEST_STACK_DUMP_S", "100")), exit=False,
                                      file=sys.stderr)
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
    missing = []
    try:
        wait = timeout
        for _ in range(world):
            try:
                rank, status, out = q.get(timeout=wait)
            except queue.Empty:
                missing = [r for r in range(world) if r not in results]
                break
            results[rank] = (status, out)
            if status != "ok":
                wait = min(wait, 45.0)  # the others are likely stuck in a collective with the failed rank
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    errs = {r: o for r, (s, o) in results.items() if s != "ok"}
    for r in missing:
        errs[r] = f"no result within {timeout:.0f} s (exit code {procs[r].exitcode})"
    if errs:
        raise AssertionError("rank failures:\n" + "\n".join(f"rank {r}: {o}" for r, o in sorted(errs.items())))
    return [results[r][1] for r in range(world)]
