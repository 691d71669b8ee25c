"""Tensor-parallel linears with fused communication (GEMM -> reduce-scatter: the GEMM writes partial products
into symmetric memory and each rank pulls and sums its rows over NVLink; GEMM -> all-reduce pushed from the
GEMM epilogue; AG -> GEMM pipelined by row block, each peer block copied over NVLink once into local memory
before its GEMM), forward and backward, against the same products computed on full tensors. 2 GPUs."""
import pytest
import torch

from tests._mp import run_ranks


def _tp_worker(rank, world):
    from brain_b200.parallel import dist as bdist
    from brain_b200.parallel.tensor_parallel import (ColumnParallelLinear, RowParallelLinear, TPContext,
                                                     shard_columns, shard_rows)
    bdist.init(timeout_s=60)
    ctx = TPContext()
    g = torch.Generator(device="cuda").manual_seed(0)
    K, N, T = 512, 768, 128
    W_col = torch.randn(N, K, device="cuda", generator=g).bfloat16() * 0.05   # [out, in]
    W_row = torch.randn(K, N, device="cuda", generator=g).bfloat16() * 0.05   # [out, in]
    x_full = torch.randn(T * world, K, device="cuda", generator=g).bfloat16()
    dy_full = torch.randn(T * world, N, device="cuda", generator=g).bfloat16()
    res = {}
    # ---- column parallel with sequence parallelism: AG -> GEMM
    col = ColumnParallelLinear(K, N, ctx, sequence_parallel=True)
    with torch.no_grad():
        col.weight.copy_(shard_columns(W_col, rank, world))
    x_local = x_full[rank * T:(rank + 1) * T].clone().requires_grad_(True)
    y = col(x_local)
    ref = x_full.float() @ shard_columns(W_col, rank, world).float().t()
    res["col_fwd"] = float((y.float() - ref).abs().max())
    dy_local_cols = shard_rows(dy_full, rank, world)  # this rank's output columns
    y.backward(dy_local_cols)
    # reference dx: sum over ranks of dy_cols_r @ W_r == dy_full @ W_col, rows of this rank
    dx_ref = (dy_full.float() @ W_col.float())[rank * T:(rank + 1) * T]
    res["col_dx"] = float((x_local.grad.float() - dx_ref).abs().max())
    dw_ref = dy_local_cols.float().t() @ x_full.float()
    res["col_dw"] = float((col.weight.grad.float() - dw_ref).abs().max())
    # ---- row parallel, all-reduce (decode-style, no SP)
    row = RowParallelLinear(N, K, ctx, sequence_parallel=False)
    with torch.no_grad():
        row.weight.copy_(shard_rows(W_row, rank, world))
    xin = shard_rows(dy_full, rank, world).clone().requires_grad_(True)  # [T*W, N/W]
    y2 = row(xin)
    ref2 = dy_full.float() @ W_row.float().t()
    res["row_ar_fwd"] = float((y2.float() - ref2).abs().max())
    gy = torch.ones_like(y2)
    y2.backward(gy)
    res["row_ar_dx"] = float((xin.grad.float() - (gy.float() @ shard_rows(W_row, rank, world).float())).abs().max())
    # ---- row parallel with SP: GEMM -> reduce-scatter, backward AG -> GEMM
    rsp = RowParallelLinear(N, K, ctx, sequence_parallel=True)
    with torch.no_grad():
        rsp.weight.copy_(shard_rows(W_row, rank, world))
    xin2 = shard_rows(dy_full, rank, world).clone().requires_grad_(True)
    y3 = rsp(xin2)
    res["row_rs_fwd"] = float((y3.float() - ref2[rank * T:(rank + 1) * T]).abs().max())
    gy3 = x_full[rank * T:(rank + 1) * T]
    y3.backward(gy3)
    dx3_ref = x_full.float() @ shard_rows(W_row, rank, world).float()
    res["row_rs_dx"] = float((xin2.grad.float() - dx3_ref).abs().max())
    ctx.comm.check()
    ctx.close()
    ctx.comm.close()
    bdist.shutdown()
    return res


@pytest.mark.gpu
@pytest.mark.multigpu
def test_tensor_parallel_fused_linears():
    outs = run_ranks(_tp_worker, 2, env={"NCCL_NVLS_ENABLE": "0"})
    for r in outs:
        for k, v in r.items():
            tol = 0.25 if "dw" in k else 0.1
            assert v < tol, (k, v, r)


def _fp8_rs_worker(rank, world):
    from brain_b200.parallel import dist as bdist
    from brain_b200.parallel.tensor_parallel import TPContext, fp8_gemm_rs
    from brain_b200.quantization.fp8 import dequantize_fp8_blockwise, quantize_fp8_blockwise, quantize_fp8_weight_blocks
    bdist.init(timeout_s=60)
    ctx = TPContext()
    g = torch.Generator(device="cuda").manual_seed(7)
    T, K, N = 256, 512, 384  # K split over ranks
    x_full = torch.randn(T * world, K, device="cuda", generator=g).bfloat16()
    w_full = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    kr = K // world
    x_local = x_full[:, rank * kr:(rank + 1) * kr].contiguous()
    wq, ws = quantize_fp8_weight_blocks(w_full[:, rank * kr:(rank + 1) * kr].contiguous())
    y = fp8_gemm_rs(ctx, x_local, wq, ws, T)
    # oracle: sum over ranks of the dequantised products, rows of this rank
    ref = torch.zeros(T * world, N, device="cuda")
    for r in range(world):
        xq, sx = quantize_fp8_blockwise(x_full[:, r * kr:(r + 1) * kr].contiguous())
        wq_r, ws_r = quantize_fp8_weight_blocks(w_full[:, r * kr:(r + 1) * kr].contiguous())
        ref += dequantize_fp8_blockwise(xq, sx, 1) @ dequantize_fp8_blockwise(wq_r, ws_r, 128).t()
    err = float((y.float() - ref[rank * T:(rank + 1) * T]).abs().max())
    scale = float(ref.abs().max())
    ctx.comm.check()
    ctx.close()
    ctx.comm.close()
    bdist.shutdown()
    return err, scale


def _fp8_rs_rowwise_worker(rank, world):
    from brain_b200.parallel import dist as bdist
    from brain_b200.parallel.tensor_parallel import TPContext, fp8_gemm_rs
    from brain_b200.quantization.fp8 import quantize_fp8_rowwise
    bdist.init(timeout_s=60)
    ctx = TPContext()
    g = torch.Generator(device="cuda").manual_seed(9)
    T, K, N = 384, 1024, 512  # M = T * world >= 256: the CTA-pair kernel
    x_full = torch.randn(T * world, K, device="cuda", generator=g).bfloat16()
    w_full = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    kr = K // world
    x_local = x_full[:, rank * kr:(rank + 1) * kr].contiguous()
    wq, ws = quantize_fp8_rowwise(w_full[:, rank * kr:(rank + 1) * kr].contiguous())
    y = fp8_gemm_rs(ctx, x_local, wq, ws, T, scaling="rowwise")
    ref = torch.zeros(T * world, N, device="cuda")
    for r in range(world):
        xq, sx = quantize_fp8_rowwise(x_full[:, r * kr:(r + 1) * kr].contiguous())
        wq_r, ws_r = quantize_fp8_rowwise(w_full[:, r * kr:(r + 1) * kr].contiguous())
        ref += (xq.float() * sx[:, None]) @ (wq_r.float() * ws_r[:, None]).t()
    err = float((y.float() - ref[rank * T:(rank + 1) * T]).abs().max())
    scale = float(ref.abs().max())
    ctx.comm.check()
    ctx.close()
    ctx.comm.close()
    bdist.shutdown()
    return err, scale


@pytest.mark.gpu
@pytest.mark.multigpu
def test_fp8_rowwise_row_parallel_gemm_reduce_scatter():
    outs = run_ranks(_fp8_rs_rowwise_worker, 2, env={"NCCL_NVLS_ENABLE": "0"})
    for err, scale in outs:
        assert err < 2e-2 * max(1.0, scale), (err, scale)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_fp8_row_parallel_gemm_reduce_scatter():
    outs = run_ranks(_fp8_rs_worker, 2, env={"NCCL_NVLS_ENABLE": "0"})
    for err, scale in outs:
        assert err < 2e-2 * max(1.0, scale), (err, scale)
