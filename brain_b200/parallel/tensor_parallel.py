"""Tensor parallelism with communication fused into the tcgen05 GEMM (the reference's
``TensorParallelLinear::forward`` returns zeros, crates/brain-distributed/src/tensor_parallel.rs:8-27).

* ``ColumnParallelLinear`` (QKV / gate-up): weight shard [out/W, in]. With sequence parallelism the
  input is this rank's token shard; the forward is AG -> GEMM pipelined by row block: the local block
  is multiplied at once while the copy engines pull the other ranks' blocks over NVLink, and each
  remote block's GEMM starts when its copy lands. Backward: dx = dy W runs as GEMM -> reduce-scatter
  (the epilogue pushes each row block to its owner's receive slot), dW = dy^T x_full.
* ``RowParallelLinear`` (out-proj / down): weight shard [out, in/W]. Forward GEMM -> reduce-scatter
  (sequence parallel) or GEMM -> all-reduce (the epilogue pushes every row to every rank, used by
  decode); the receiver sums its W slots after a peer barrier. Backward: dx = dy_full W via the
  pipelined AG -> GEMM, dW = dy_full^T x.
Receive / staging buffers are symmetric (CUDA IPC) and double-buffered by call parity, so a fast
rank never overwrites a buffer a slower peer is still reading (every call contains a barrier).
With one rank the layers are plain GEMMs.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _native
from ..nn import init as _init
from ..nn.module import Module
from ..ops._common import same_device
from ..ops.gemm import gemm
from ..ops.linear import _wgrad

_native.register({
    "brain_gemm_bf16_tp": ("brain_kernels", "plpliplpiiiilpliiis"),
    "brain_comm_copy_async": ("brain_comm", "llls"),
})


class TPContext:
    """Communicator + symmetric scratch shared by the tensor-parallel layers of one group."""

    def __init__(self, group=None, comm=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.comm = comm
        if self.world > 1 and self.comm is None:
            from .symm import NvlinkComm
            self.comm = NvlinkComm(group)
        self._bufs: dict = {}
        self._local: dict = {}
        self.side = None
        self.calls = 0
        # how AG -> GEMM pulls the peers' row blocks: "sm" = copy kernel of NVLink peer loads on a side
        # stream, "ce" = copy engines (cudaMemcpyAsync per peer)
        self.ag_copy = "sm"
        # GEMM -> reduce-scatter: "push" = the GEMM epilogue stores each row block into its owner's receive
        # slot over NVLink while later tiles compute (rows leave through the shared-memory staging with
        # coalesced 16-byte stores, tiles visited from the next owner on), barrier, local sum of the slots;
        # "pull" = GEMM into symmetric memory, barrier, every rank pulls and sums its own rows from all
        # peers (2 GPUs, 16384 x 8192 x 4096: push 0.859 ms, pull 0.958, GEMM alone 0.753)
        self.rs_mode = "push"

    def symm(self, name: str, nbytes: int, parity: int):
        """Symmetric buffer `name` (double-buffered by parity) of at least nbytes."""
        key = (name, parity)
        buf = self._bufs.get(key)
        if buf is None or buf.nbytes < nbytes:
            from .symm import SymmetricBuffer
            if buf is not None:
                buf.close()
            buf = SymmetricBuffer(max(nbytes, 1 << 16), self.group)
            self._bufs[key] = buf
        return buf

    def local(self, name: str, shape, dtype=torch.bfloat16) -> torch.Tensor:
        """A reusable plain device buffer (not shared with peers)."""
        n = 1
        for x in shape:
            n *= int(x)
        buf = self._local.get(name)
        if buf is None or buf.numel() < n or buf.dtype != dtype:
            buf = torch.empty(n, device=torch.cuda.current_device(), dtype=dtype)
            self._local[name] = buf
        return buf[:n].view(*shape)

    def side_stream(self) -> torch.cuda.Stream:
        if self.side is None:
            self.side = torch.cuda.Stream()
        return self.side

    def next_parity(self) -> int:
        self.calls += 1
        return self.calls & 1

    def close(self):
        for b in self._bufs.values():
            b.close()
        self._bufs.clear()
        self._local.clear()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _i64(vals):
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def gemm_push(ctx: TPContext, a: torch.Tensor, w: torch.Tensor, mode: int, rows_per_rank: int,
              b_mn: int = 0) -> torch.Tensor:
    """C = a @ w.T (w [N, K]; or a @ w for b_mn=1, w [K, N]), reduced over ranks.

    mode 1 (reduce-scatter): returns this rank's rows [rank*rows_per_rank, ...) of the sum; by default
    (``ctx.rs_mode == "pull"``) each rank pulls its rows from the peers' products, otherwise the GEMM
    epilogue pushes them.
    mode 2 (all-reduce): returns the full sum [M, N]; the GEMM epilogue pushes every row to every rank.
    """
    M, K = a.shape
    N = w.shape[1] if b_mn else w.shape[0]
    W = ctx.world
    same_device(a, w)
    out_rows = rows_per_rank if mode == 1 else M
    slot = out_rows * N
    par = ctx.next_parity()
    if mode == 1 and ctx.rs_mode == "pull":
        full = ctx.symm("rs_full", M * N * 2, par)
        gemm(a, w, trans_b=not b_mn, out=full.view(torch.bfloat16, M * N).view(M, N))
        ctx.comm.barrier(40)
        out = torch.empty(out_rows, N, device=a.device, dtype=torch.bfloat16)
        _native.call("brain_comm_reduce_pull", full.peer_array(0), ctx.rank * slot, ctx.rank, W, out.data_ptr(), slot,
                     1, 1.0, _stream())
        return out
    recv = ctx.symm("recv", W * slot * 2, par)
    _native.call("brain_gemm_bf16_tp", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), b_mn, None, N,
                 recv.peer_array(0), mode, ctx.rank, W, rows_per_rank if mode == 1 else M, slot, None, 0, M, N, K,
                 _stream())
    ctx.comm.barrier(20 + mode)
    out = torch.empty(out_rows, N, device=a.device, dtype=torch.bfloat16)
    slots = _i64([recv.local + s * slot * 2 for s in range(W)])
    _native.call("brain_comm_reduce_pull", slots, 0, ctx.rank, W, out.data_ptr(), slot, 1, 1.0, _stream())
    return out


def fp8_gemm_rs(ctx: TPContext, x_local: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                rows_per_rank: int, scaling: str = "block") -> torch.Tensor:
    """Row-parallel block-scaled fp8 Linear with reduce-scatter: x_local [M, K/W] (bf16, this rank's
    input columns) is quantised 1 x 128 on the fly, multiplied by this rank's pre-quantised weight
    shard wq [N, K/W] (128 x 128 scales ws) on the tcgen05 fp8 kernel straight into symmetric memory,
    and after a peer barrier each rank pulls and sums its rows [rank * rows_per_rank, ...) from all
    ranks' products with coalesced NVLink loads. Returns [rows_per_rank, N] bf16.

    ``scaling="rowwise"``: x_local is quantised per token and wq carries one scale per output channel
    (``quantize_fp8_rowwise`` of this rank's weight columns); the product then runs on the CTA-pair
    ``kind::f8f6f4`` kernel with the scales applied in its epilogue."""
    from ..quantization.fp8 import quantize_fp8_blockwise, quantize_fp8_rowwise
    M = x_local.shape[0]
    N = wq.shape[0]
    W = ctx.world
    same_device(x_local, wq, ws)
    par = ctx.next_parity()
    full = ctx.symm("rs_full", M * N * 2, par)
    if scaling == "rowwise":
        if N % 8:
            raise ValueError("row-wise fp8 GEMM -> RS needs N % 8 == 0")
        xq, sx = quantize_fp8_rowwise(x_local)
        wsf = ws.float().contiguous()
        args = (xq.data_ptr(), xq.stride(0), wq.data_ptr(), wq.stride(0), sx.data_ptr(), wsf.data_ptr(),
                full.local, N, None, 0, M, N, xq.shape[1], _stream())
        rc = _native.fn("brain_fp8_gemm_rowwise_pair")(*args)
        if rc == 801:  # cudaErrorNotSupported: M or N below the pair tile, the single-CTA kernel runs
            rc = _native.fn("brain_fp8_gemm_rowwise")(*args)
        if rc:
            raise _native.NativeError(f"row-wise fp8 GEMM failed with status {rc}")
    else:
        xq, sx = quantize_fp8_blockwise(x_local)
        _native.call("brain_fp8_gemm", xq.data_ptr(), xq.stride(0), wq.data_ptr(), wq.stride(0), sx.data_ptr(),
                     ws.data_ptr(), full.local, N, None, 0, M, N, xq.shape[1], _stream())
    ctx.comm.barrier(41)
    slot = rows_per_rank * N
    out = torch.empty(rows_per_rank, N, device=x_local.device, dtype=torch.bfloat16)
    _native.call("brain_comm_reduce_pull", full.peer_array(0), ctx.rank * slot, ctx.rank, W, out.data_ptr(), slot, 1,
                 1.0, _stream())
    return out


def gemm_allgather_a(ctx: TPContext, a_local: torch.Tensor, w: torch.Tensor, b_mn: int = 0) -> torch.Tensor:
    """C = concat_ranks(a_local) @ w.T (or @ w for b_mn=1), pipelined by row block.

    The local block's GEMM starts at once; a side stream pulls every other rank's block from its
    symmetric staging buffer (nearest peers first; a copy kernel of NVLink peer loads, or the copy
    engines with ``ctx.ag_copy = "ce"``), and each remote block's GEMM waits only for its own copy.
    Compute and NVLink transfer overlap and every GEMM reads this GPU's memory.
    """
    T, K = a_local.shape
    N = w.shape[1] if b_mn else w.shape[0]
    W, r = ctx.world, ctx.rank
    par = ctx.next_parity()
    stage = ctx.symm("ag", T * K * 2, par)
    sv = stage.view(torch.bfloat16, T * K).view(T, K)
    sv.copy_(a_local)
    ctx.comm.barrier(30)
    out = torch.empty(T * W, N, device=a_local.device, dtype=torch.bfloat16)
    gather = ctx.local("ag_gather", (W, T, K))
    main, side = torch.cuda.current_stream(), ctx.side_stream()
    side.wait_stream(main)
    order = [(r + i) % W for i in range(1, W)]
    events = []
    fn = "brain_comm_copy_async" if ctx.ag_copy == "ce" else "brain_comm_copy"
    for j in order:
        _native.call(fn, stage.ptrs[j], gather[j].data_ptr(), T * K * 2, side.cuda_stream)
        ev = torch.cuda.Event()
        ev.record(side)
        events.append(ev)
    gemm(a_local, w, trans_b=not b_mn, out=out[r * T:(r + 1) * T])
    for j, ev in zip(order, events):
        main.wait_event(ev)
        gemm(gather[j], w, trans_b=not b_mn, out=out[j * T:(j + 1) * T])
    return out


def all_gather_rows(ctx: TPContext, x: torch.Tensor) -> torch.Tensor:
    """[T, K] per rank -> [W*T, K] (P2P pull), used where the gathered tensor itself is needed."""
    T, K = x.shape
    full = torch.empty(T * ctx.world, K, device=x.device, dtype=x.dtype)
    return ctx.comm.all_gather_flat(x.contiguous().view(-1), full.view(-1)).view(T * ctx.world, K)


class _ColumnSPFn(torch.autograd.Function):
    @staticmethod
    def forward(c, x_local, w, ctx):
        c.save_for_backward(x_local, w)
        c.tp = ctx
        return gemm_allgather_a(ctx, x_local.contiguous(), w)

    @staticmethod
    def backward(c, dy):
        x_local, w = c.saved_tensors
        ctx = c.tp
        T = x_local.shape[0]
        dx = gemm_push(ctx, dy.contiguous(), w, 1, T, b_mn=1)  # (dy @ W) reduce-scattered by rows
        x_full = all_gather_rows(ctx, x_local)
        dw = _wgrad(dy.contiguous(), x_full, w)
        return dx, dw, None


class _RowFn(torch.autograd.Function):
    @staticmethod
    def forward(c, x, w, ctx, sp):
        c.save_for_backward(x, w)
        c.tp, c.sp = ctx, sp
        M = x.shape[0]
        if sp:
            return gemm_push(ctx, x.contiguous(), w, 1, M // ctx.world)
        return gemm_push(ctx, x.contiguous(), w, 2, M)

    @staticmethod
    def backward(c, dy):
        x, w = c.saved_tensors
        ctx = c.tp
        if c.sp:
            dx = gemm_allgather_a(ctx, dy.contiguous(), w, b_mn=1)
            dy_full = all_gather_rows(ctx, dy.contiguous())
        else:
            dx = gemm(dy.contiguous(), w)
            dy_full = dy.contiguous()
        dw = _wgrad(dy_full, x, w)
        return dx, dw, None, None


def _default_device(ctx: TPContext, device):
    """Sharded layers of a multi-rank group live on the rank's GPU unless told otherwise."""
    if device is None and ctx.world > 1:
        return torch.device("cuda", torch.cuda.current_device())
    return device


class ColumnParallelLinear(Module):
    def __init__(self, in_features: int, out_features: int, ctx: TPContext, sequence_parallel: bool = False,
                 device=None, dtype=torch.bfloat16, init_std: float = 0.02, seed: int = 0):
        super().__init__()
        if out_features % ctx.world:
            raise ValueError("out_features must divide by the tensor-parallel size")
        self.ctx, self.sp = ctx, sequence_parallel
        self.in_features, self.out_features = in_features, out_features
        device = _default_device(ctx, device)
        self.weight = torch.nn.Parameter(torch.empty(out_features // ctx.world, in_features, device=device,
                                                     dtype=dtype))
        g = torch.Generator(device=self.weight.device).manual_seed(seed * 1000 + ctx.rank)
        with torch.no_grad():
            self.weight.copy_(torch.randn(self.weight.shape, generator=g, device=self.weight.device) * init_std)

    def forward(self, x):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if self.ctx.world == 1 or not self.sp:
            y = gemm(x2, self.weight, trans_b=True) if x2.is_cuda else x2 @ self.weight.t()
            return y.view(*shp[:-1], -1)
        y = _ColumnSPFn.apply(x2, self.weight, self.ctx)
        return y.view(-1, self.weight.shape[0])


class RowParallelLinear(Module):
    def __init__(self, in_features: int, out_features: int, ctx: TPContext, sequence_parallel: bool = False,
                 device=None, dtype=torch.bfloat16, init_std: float = 0.02, seed: int = 0):
        super().__init__()
        if in_features % ctx.world:
            raise ValueError("in_features must divide by the tensor-parallel size")
        self.ctx, self.sp = ctx, sequence_parallel
        device = _default_device(ctx, device)
        self.weight = torch.nn.Parameter(torch.empty(out_features, in_features // ctx.world, device=device,
                                                     dtype=dtype))
        g = torch.Generator(device=self.weight.device).manual_seed(seed * 1000 + 500 + ctx.rank)
        with torch.no_grad():
            self.weight.copy_(torch.randn(self.weight.shape, generator=g, device=self.weight.device) * init_std)

    def forward(self, x):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if self.ctx.world == 1:
            y = gemm(x2, self.weight, trans_b=True) if x2.is_cuda else x2 @ self.weight.t()
            return y.view(*shp[:-1], -1)
        y = _RowFn.apply(x2, self.weight, self.ctx, self.sp)
        return y if self.sp else y.view(*shp[:-1], -1)


TensorParallelLinear = ColumnParallelLinear


def shard_columns(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    return torch.tensor_split(w, world, dim=0)[rank].contiguous()


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    return torch.tensor_split(w, world, dim=1)[rank].contiguous()
