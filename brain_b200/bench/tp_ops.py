"""Tensor-parallel prefill operations timed on every rank of the launch (one GPU per rank): the
pipelined all-gather -> GEMM (peer row blocks pulled by a copy kernel or by the copy engines), the
GEMM -> reduce-scatter epilogue push, the row all-gather, and the same GEMMs on local data for
comparison. Shapes default to one rank of Llama-3-70B at TP = N with 8192 tokens per rank.

Run: ``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m brain_b200.bench.tp_ops``.
Rank 0 prints one JSON line per operation: milliseconds (CUDA events, max over ranks) and the NVLink
bytes each rank receives.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch
import torch.distributed as dist


def _peaks() -> dict:
    """Roofline denominators: the measured cuBLAS bf16 burst (MEASURED_PEAKS.json next to the package, else
    1,590 TFLOP/s) and 770 GB/s per direction for a peer copy over NVLink."""
    import os
    out = {"bf16_tflops": 1590.0, "nvlink_gbs": 770.0}
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        v = d.get("bf16_tflops") or d.get("cublas_bf16_tflops")
        if isinstance(v, (int, float)) and v > 0:
            out["bf16_tflops"] = float(v)
    except (OSError, ValueError):
        pass
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens-per-rank", type=int, default=8192)
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--qkv-cols", type=int, default=0, help="per-rank QKV width (default: 70B shape at TP = N)")
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args(argv)

    from ..parallel import dist as bdist
    from ..parallel.tensor_parallel import TPContext, all_gather_rows, gemm_allgather_a, gemm_push
    from ..ops.gemm import gemm
    ctx = bdist.init(timeout_s=120)
    W, rank, dev = ctx.world_size, ctx.rank, ctx.device
    tp = TPContext()
    T, d = a.tokens_per_rank, a.hidden
    qkv = a.qkv_cols or (64 + 16) * 128 // W
    attn = 64 * 128 // W
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(T, d, device=dev, generator=g).bfloat16()
    w_qkv = (torch.randn(qkv, d, device=dev, generator=g) * 0.02).bfloat16()
    a_full = torch.randn(T * W, attn, device=dev, generator=g).bfloat16()
    w_o = (torch.randn(d, attn, device=dev, generator=g) * 0.02).bfloat16()

    def timed(fn):
        for _ in range(2):
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

    def report(name, ms, nvlink_bytes, **extra):
        if rank == 0:
            print(json.dumps({"op": name, "world": W, "ms": round(ms, 3), "nvlink_in_bytes_per_rank": nvlink_bytes,
                              "nvlink_in_gbs": round(nvlink_bytes / (ms / 1e3) / 1e9, 1) if nvlink_bytes else None,
                              **extra}), flush=True)

    xf = torch.randn(T * W, d, device=dev, generator=g).bfloat16()
    report("local_gemm_qkv_all_rows", timed(lambda: gemm(xf, w_qkv, trans_b=True)), 0, M=T * W, N=qkv, K=d)
    for mode in ("sm", "ce"):
        tp.ag_copy = mode
        report(f"ag_gemm_qkv_{mode}", timed(lambda: gemm_allgather_a(tp, x, w_qkv)), (W - 1) * T * d * 2,
               M=T * W, N=qkv, K=d)
    tp.ag_copy = "sm"
    report("local_gemm_o_all_rows", timed(lambda: gemm(a_full, w_o, trans_b=True)), 0, M=T * W, N=d, K=attn)
    from .. import _native
    peaks = _peaks()
    flops_o = 2.0 * T * W * d * attn
    for mode in ("pull", "push", "push_rowstore"):
        # pull: GEMM into symmetric memory, barrier, each rank pulls and sums its rows; push: the GEMM
        # epilogue stores each row block into its owner's slot from the shared-memory staging (owner-rotated
        # tile order), barrier, local sum; push_rowstore: the same push with per-row stores
        tp.rs_mode = "pull" if mode == "pull" else "push"
        old = _native.fn("brain_gemm_set_push_stage")(0 if mode == "push_rowstore" else 1)
        ms = timed(lambda: gemm_push(tp, a_full, w_o, 1, T))
        _native.fn("brain_gemm_set_push_stage")(old)
        nbytes = (W - 1) * T * d * 2
        target = max(flops_o / (peaks["bf16_tflops"] * 1e12), nbytes / (peaks["nvlink_gbs"] * 1e9)) * 1e3
        report(f"gemm_rs_{mode}_o", ms, nbytes, M=T * W, N=d, K=attn, roofline_ms=round(target, 3),
               roofline_fraction=round(target / ms, 3))
    tp.rs_mode = "pull"
    report("all_gather_rows", timed(lambda: all_gather_rows(tp, x)), (W - 1) * T * d * 2)
    # block-scaled fp8 row-parallel Linear d x d (K split over ranks), GEMM -> reduce-scatter
    from ..parallel.tensor_parallel import fp8_gemm_rs
    from ..quantization.fp8 import quantize_fp8_weight_blocks
    kr = d // W
    x8 = torch.randn(T * W, kr, device=dev, generator=g).bfloat16()
    w8 = (torch.randn(d, kr, device=dev, generator=g) * 0.02).bfloat16()
    w8q, w8s = quantize_fp8_weight_blocks(w8)
    flops = 2.0 * T * W * d * kr
    ms = timed(lambda: fp8_gemm_rs(tp, x8, w8q, w8s, T))
    report("fp8_linear_gemm_rs", ms, (W - 1) * T * d * 2, M=T * W, N=d, K=kr,
           tflops_per_rank=round(flops / (ms / 1e3) / 1e12, 1))
    from ..quantization.fp8 import quantize_fp8_rowwise
    w8rq, w8rs = quantize_fp8_rowwise(w8)
    ms_rw = timed(lambda: fp8_gemm_rs(tp, x8, w8rq, w8rs, T, scaling="rowwise"))
    report("fp8_rowwise_linear_gemm_rs", ms_rw, (W - 1) * T * d * 2, M=T * W, N=d, K=kr,
           tflops_per_rank=round(flops / (ms_rw / 1e3) / 1e12, 1))
    ms_bf = timed(lambda: gemm_push(tp, x8, w8, 1, T))
    report("bf16_linear_gemm_rs", ms_bf, (W - 1) * T * d * 2, M=T * W, N=d, K=kr,
           tflops_per_rank=round(flops / (ms_bf / 1e3) / 1e12, 1))
    tp.comm.check()
    tp.close()
    tp.comm.close()
    bdist.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
