"""Collective sweep: all_reduce / all_gather / reduce_scatter from 4 KB to 1 GB, bf16 and f32, with
the NVLink P2P kernels (``NvlinkComm``) and with NCCL, on every rank of the launch.

Run: ``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m brain_b200.bench.collective_sweep``.
Each (op, dtype, size, backend) is device-timed with CUDA events over ``iters`` back-to-back calls after
warm-up, max over ranks; rank 0 prints one JSON line per point with algorithm and bus bandwidth
(bus = alg * 2(W-1)/W for all-reduce, alg * (W-1)/W for all-gather / reduce-scatter, where alg is the
full buffer size / time). Data: uniform(-1, 1), seeded per rank.
Reference: the collectives of crates/brain-distributed/src/collective/ (allreduce.rs, allgather.rs,
reduce_scatter.rs) run in-process on the CPU.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch
import torch.distributed as dist


def _sizes(lo: int, hi: int):
    s = lo
    while s <= hi:
        yield s
        s *= 4


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-bytes", type=int, default=4096)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--ops", default="all_reduce,all_gather,reduce_scatter")
    ap.add_argument("--dtypes", default="bf16,f32")
    ap.add_argument("--backends", default="nvlink,nccl")
    a = ap.parse_args(argv)

    from ..parallel import dist as bdist
    from ..parallel.symm import NvlinkComm
    ctx = bdist.init(timeout_s=120)
    rank, W = ctx.rank, ctx.world_size
    dev = ctx.device
    comm = NvlinkComm() if W > 1 else None
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    def bench(fn):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for op in a.ops.split(","):
        for dname in a.dtypes.split(","):
            dt = {"bf16": torch.bfloat16, "f32": torch.float32}[dname]
            esz = torch.empty(0, dtype=dt).element_size()
            for nbytes in _sizes(a.min_bytes, a.max_bytes):
                n = nbytes // esz
                n -= n % (W * 8)
                if n == 0:
                    continue
                full = (torch.rand(n, device=dev, generator=g, dtype=torch.float32) * 2 - 1).to(dt)
                shard = full[:n // W].clone()
                out_full = torch.empty_like(full)
                for be in a.backends.split(","):
                    if be == "nvlink" and comm is None:
                        continue
                    if op == "all_reduce":
                        # mean keeps the values bounded over repetitions; the traffic is that of a sum
                        fn = ((lambda: comm.all_reduce(full, "mean")) if be == "nvlink"
                              else (lambda: dist.all_reduce(full, op=dist.ReduceOp.AVG)))
                        factor = 2 * (W - 1) / W
                    elif op == "all_gather":
                        fn = ((lambda: comm.all_gather_flat(shard, out_full)) if be == "nvlink"
                              else (lambda: dist.all_gather_into_tensor(out_full, shard)))
                        factor = (W - 1) / W
                    else:
                        fn = ((lambda: comm.reduce_scatter_flat(full, shard)) if be == "nvlink"
                              else (lambda: dist.reduce_scatter_tensor(shard, full)))
                        factor = (W - 1) / W
                    ms = bench(fn)
                    alg = n * esz / (ms / 1e3) / 1e9
                    if rank == 0:
                        print(json.dumps({"op": op, "dtype": dname, "bytes": n * esz, "backend": be, "world": W,
                                          "ms": ms, "alg_gbs": alg, "bus_gbs": alg * factor}), flush=True)
    if comm is not None:
        comm.close()
    bdist.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
