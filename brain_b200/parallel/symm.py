"""Symmetric memory over CUDA IPC and the in-kernel NVLink communication backend.

``SymmetricBuffer`` allocates the same number of bytes on every rank with ``cudaMalloc``
(``csrc/comm.cu``), exchanges the 64-byte CUDA IPC handles with ``torch.distributed``, opens the
peers' handles and keeps the table of peer device pointers. Kernels read and write peer memory
directly over NVLink / NVSwitch with plain peer loads and stores (no NVLS objects).

``NvlinkComm`` implements the collectives of the data-parallel engine and of the public API with
those kernels (barrier with epochs and a wall-clock budget, one-/two-shot all-reduce,
reduce-scatter, all-gather, broadcast) plus ``fused_rs_adamw``: one kernel per rank that pulls the
gradient shard from every rank, applies AdamW and pushes the new bf16 weights to every rank.
A timed-out wait inside a kernel raises :class:`PeerTimeout` on the host.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _native

_native.register({
    "brain_comm_allreduce_oneshot": ("brain_comm", "pplifppiiils"),
    "brain_comm_allreduce_twoshot": ("brain_comm", "pplifppiiils"),
    "brain_ipc_alloc": ("brain_comm", "lpp"),
    "brain_ipc_handle_size": ("brain_comm", ""),
    "brain_ipc_open": ("brain_comm", "pp"),
    "brain_ipc_close": ("brain_comm", "l"),
    "brain_ipc_free": ("brain_comm", "l"),
    "brain_comm_barrier": ("brain_comm", "piiilis"),
    "brain_comm_reduce_pull": ("brain_comm", "pliiplifs"),
    "brain_comm_gather_pull": ("brain_comm", "piills"),
    "brain_comm_gather_push": ("brain_comm", "piills"),
    "brain_comm_copy": ("brain_comm", "llls"),
    "brain_comm_ddp_step": ("brain_comm", "ppiiillpppffffffffs"),
    "brain_status_comm": ("brain_comm", "pi"),
})


class PeerTimeout(RuntimeError):
    """A peer rank did not reach a collective within the wait budget."""


class _CAI:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def _check_status() -> None:
    code, where = _native.status("comm", clear=True)
    if code:
        raise PeerTimeout(f"NVLink collective wait gave up (status {code}, site {where >> 4}, peer {where & 15})")


class SymmetricBuffer:
    """``nbytes`` of device memory on every rank of ``group`` with the table of peer pointers."""

    def __init__(self, nbytes: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.nbytes = int(-(-nbytes // 256) * 256)
        hsize = _native.fn("brain_ipc_handle_size")()
        handle = ctypes.create_string_buffer(hsize)
        ptr = ctypes.c_int64(0)
        _native.call("brain_ipc_alloc", self.nbytes, ctypes.byref(ptr), handle)
        self.local = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        self.ptrs = []
        self.opened = []
        for j, h in enumerate(handles):
            if j == self.rank:
                self.ptrs.append(self.local)
            else:
                p = ctypes.c_int64(0)
                _native.call("brain_ipc_open", h, ctypes.byref(p))
                self.ptrs.append(p.value)
                self.opened.append(p.value)
        self.ptr_array = (ctypes.c_int64 * self.world)(*self.ptrs)
        self._bytes = torch.as_tensor(_CAI(self.local, self.nbytes), device=torch.device("cuda", torch.cuda.current_device()))

    def view(self, dtype: torch.dtype, numel: int, offset_bytes: int = 0) -> torch.Tensor:
        """Local memory as a torch tensor (no copy)."""
        esz = torch.empty(0, dtype=dtype).element_size()
        if offset_bytes + numel * esz > self.nbytes:
            raise ValueError("view exceeds the symmetric buffer")
        return self._bytes[offset_bytes:offset_bytes + numel * esz].view(dtype)

    def peer_array(self, offset_bytes: int = 0):
        return (ctypes.c_int64 * self.world)(*[p + offset_bytes for p in self.ptrs])

    def close(self) -> None:
        torch.cuda.synchronize()
        for p in self.opened:
            _native.fn("brain_ipc_close")(p)
        self.opened = []
        if self.local:
            self._bytes = None
            _native.fn("brain_ipc_free")(self.local)
            self.local = 0


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class NvlinkComm:
    """Collectives as P2P kernels over symmetric memory (one process per GPU, one node)."""

    name = "nvlink"
    ONE_SHOT_BYTES = 256 * 1024  # staged fallback (unaligned tensors) up to this size
    ONE_LAUNCH_BYTES = 2 << 20  # one-launch all-reduce up to this size (each rank reads every rank's copy)
    # one-launch reduce-scatter + all-gather up to this size: it wins while launches and barriers dominate
    # (4 MB on 2 GPUs: 37 us vs 60 us staged, NCCL 38 us); past it the staged kernels move more bytes in flight
    TWO_PHASE_BYTES = 8 << 20
    PUSH_BYTES = 4 << 20  # all-gather shards from this size are pushed (one more barrier, more bytes in flight)

    def __init__(self, group=None, timeout_s: float = 60.0):
        _native.load("brain_comm")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("NvlinkComm supports up to 8 ranks (one NVSwitch domain per node)")
        self.timeout_ns = int(timeout_s * 1e9)
        self.pads = SymmetricBuffer(4 * 8, group)
        self.epoch = 0
        self.staging: SymmetricBuffer | None = None
        self.registered: dict[int, SymmetricBuffer] = {}
        # one-launch all-reduce: staging halves by call parity and per-CTA flags (int32 [128][8])
        self.os_stage = SymmetricBuffer(2 * self.ONE_LAUNCH_BYTES, group)
        self.os_stage_arr = [self.os_stage.peer_array(0), self.os_stage.peer_array(self.ONE_LAUNCH_BYTES)]
        self.os_flags = SymmetricBuffer(128 * 8 * 4, group)
        self.os_epoch = 0
        self.os_stream: torch.cuda.Stream | None = None  # stream of the last one-launch all-reduce
        # one-launch two-phase all-reduce: its own staging (grown on demand) and flags
        self.ts_stage: SymmetricBuffer | None = None
        self.ts_flags = SymmetricBuffer(128 * 8 * 4, group)
        self.ts_epoch = 0
        dist.barrier(group)

    # ------------------------------------------------------------------ plumbing
    def alloc(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A zero-initialised symmetric tensor; collectives on it need no staging copy."""
        esz = torch.empty(0, dtype=dtype).element_size()
        buf = SymmetricBuffer(numel * esz, self.group)
        t = buf.view(dtype, numel)
        self.registered[t.data_ptr()] = buf
        return t

    def _buf_of(self, t: torch.Tensor):
        base = t.data_ptr()
        for p, buf in self.registered.items():
            if p <= base < p + buf.nbytes:
                return buf, base - p
        return None, 0

    def _staging(self, nbytes: int) -> SymmetricBuffer:
        if self.staging is None or self.staging.nbytes < nbytes:
            if self.staging is not None:
                self.staging.close()
            self.staging = SymmetricBuffer(max(nbytes, 1 << 20), self.group)
        return self.staging

    def barrier(self, where: int = 0) -> None:
        self.epoch += 1
        _native.call("brain_comm_barrier", self.pads.ptr_array, self.rank, self.world, self.epoch, self.timeout_ns,
                     where, _stream())

    def check(self) -> None:
        """Synchronise and raise PeerTimeout if any collective wait gave up."""
        torch.cuda.synchronize()
        _check_status()

    def _ordered_stream(self):
        """The current stream, made to wait for the stream of the previous one-launch all-reduce when it
        differs: the flag protocols of those kernels rely on each rank's calls running in issue order."""
        cur = torch.cuda.current_stream()
        if self.os_stream is not None and cur != self.os_stream:
            cur.wait_stream(self.os_stream)
        self.os_stream = cur
        return cur

    # ------------------------------------------------------------------ collectives
    def all_reduce(self, t: torch.Tensor, op: str = "sum") -> torch.Tensor:
        if op not in ("sum", "mean", "avg"):
            dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}[op], group=self.group)
            return t
        scale = 1.0 / self.world if op in ("mean", "avg") else 1.0
        if t.dtype not in (torch.float32, torch.bfloat16) or not t.is_contiguous():
            dist.all_reduce(t, group=self.group)
            if scale != 1.0:
                t.mul_(scale)
            return t
        n = t.numel()
        vec = 4 if t.dtype == torch.float32 else 8
        esz = t.element_size()
        dcode = 0 if t.dtype == torch.float32 else 1
        if n * esz <= self.ONE_LAUNCH_BYTES and t.data_ptr() % 16 == 0:
            # one launch: copy into this rank's staging half, signal, pull-sum every rank's copy into t.
            # Reusing a staging half two calls later is safe only if this rank's calls run in issue order,
            # so a call on another stream than the previous one first waits for that one.
            cur = self._ordered_stream()
            self.os_epoch += 1
            _native.call("brain_comm_allreduce_oneshot", t.data_ptr(), t.data_ptr(), n, dcode, scale,
                         self.os_stage_arr[self.os_epoch & 1], self.os_flags.ptr_array, self.rank, self.world,
                         self.os_epoch, self.timeout_ns, cur.cuda_stream)
            return t
        if (n * esz <= self.TWO_PHASE_BYTES and n % (self.world * vec) == 0 and t.data_ptr() % 16 == 0):
            # one launch: copy in, reduce this rank's shard and push it to every rank, copy out
            if self.ts_stage is None or self.ts_stage.nbytes < n * esz:
                if self.ts_stage is not None:
                    self.ts_stage.close()
                self.ts_stage = SymmetricBuffer(max(n * esz, 8 << 20), self.group)
            cur = self._ordered_stream()
            _native.call("brain_comm_allreduce_twoshot", t.data_ptr(), t.data_ptr(), n, dcode, scale,
                         self.ts_stage.ptr_array, self.ts_flags.ptr_array, self.rank, self.world, self.ts_epoch + 1,
                         self.timeout_ns, cur.cuda_stream)
            self.ts_epoch += 2
            return t
        if n * esz <= self.ONE_SHOT_BYTES:
            npad = -(-n // vec) * vec
            st = self._staging(npad * esz)
            sv = st.view(t.dtype, npad)
            sv[:n].copy_(t)
            if npad > n:
                sv[n:].zero_()
            self.barrier(1)
            out = torch.empty(npad, device=t.device, dtype=t.dtype)
            # every rank reduces the whole vector: the same summation order (first rank 0) on all of them
            _native.call("brain_comm_reduce_pull", st.ptr_array, 0, 0, self.world, out.data_ptr(), npad, dcode,
                         scale, _stream())
            t.copy_(out[:n].view_as(t))
            return t
        unit = vec * self.world * 16
        npad = -(-n // unit) * unit
        chunk = npad // self.world
        st = self._staging(npad * esz)
        sv = st.view(t.dtype, npad)
        sv[:n].copy_(t.view(-1))
        if npad > n:
            sv[n:].zero_()
        self.barrier(2)
        mine = sv[self.rank * chunk:(self.rank + 1) * chunk]
        _native.call("brain_comm_reduce_pull", st.ptr_array, self.rank * chunk, self.rank, self.world, mine.data_ptr(),
                     chunk, dcode, scale, _stream())
        # once this rank has reduced chunk r no peer reads chunk r anywhere: push it straight into every
        # peer's copy (remote stores), then one barrier publishes all chunks
        _native.call("brain_comm_gather_push", st.ptr_array, self.rank, self.world, chunk * esz, 0, _stream())
        self.barrier(3)
        t.view(-1).copy_(sv[:n])
        return t

    def reduce_scatter_flat(self, full: torch.Tensor, out: torch.Tensor, op: str = "sum") -> torch.Tensor:
        n = out.numel()
        dcode = 0 if full.dtype == torch.float32 else 1
        buf, off = self._buf_of(full)
        if buf is None:
            st = self._staging(full.numel() * full.element_size())
            st.view(full.dtype, full.numel()).copy_(full.view(-1))
            buf, off = st, 0
        self.barrier(4)
        esz = full.element_size()
        _native.call("brain_comm_reduce_pull", buf.peer_array(off), self.rank * n, self.rank, self.world,
                     out.data_ptr(), n, dcode, 1.0, _stream())
        return out

    def reduce_scatter_inplace(self, full: torch.Tensor, shard: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
        """shard = scale * sum over ranks of their ``full`` at this rank's shard position, written in
        place into the local ``full`` (``shard`` is that view): each rank reads only the peers' pieces
        of its own shard, which no peer reads, so the in-place write races with nothing."""
        buf, off = self._buf_of(full)
        esz = full.element_size()
        n = shard.numel()
        if buf is None or shard.data_ptr() != full.data_ptr() + self.rank * n * esz:
            tmp = torch.empty_like(shard)
            self.reduce_scatter_flat(full, tmp)
            return shard.copy_(tmp.mul_(scale))
        self.barrier(10)
        _native.call("brain_comm_reduce_pull", buf.peer_array(off), self.rank * n, self.rank, self.world,
                     shard.data_ptr(), n, 0 if full.dtype == torch.float32 else 1, float(scale), _stream())
        return shard

    def all_gather_flat(self, shard: torch.Tensor, full: torch.Tensor) -> torch.Tensor:
        esz = full.element_size()
        n = shard.numel()
        buf, off = self._buf_of(full)
        if buf is None:
            st = self._staging(full.numel() * esz)
            sv = st.view(full.dtype, full.numel())
            sv[self.rank * n:(self.rank + 1) * n].copy_(shard.view(-1))
            buf, off, target = st, 0, sv
        else:
            target = None
            if shard.data_ptr() != full.data_ptr() + self.rank * n * esz:
                full.view(-1)[self.rank * n:(self.rank + 1) * n].copy_(shard.view(-1))
        self.barrier(5)
        if n * esz >= self.PUSH_BYTES:
            # large shards: remote stores into every peer, then a second barrier publishes them
            _native.call("brain_comm_gather_push", buf.peer_array(0), self.rank, self.world, n * esz, off, _stream())
            self.barrier(11)
        else:
            _native.call("brain_comm_gather_pull", buf.peer_array(0), self.rank, self.world, n * esz, off, _stream())
        if target is not None:
            full.view(-1).copy_(target)
        return full

    def broadcast(self, t: torch.Tensor, src: int = 0) -> torch.Tensor:
        nbytes = t.numel() * t.element_size()
        pad = -(-nbytes // 16) * 16
        st = self._staging(pad)
        if self.rank == src:
            st._bytes[:nbytes].copy_(t.contiguous().view(-1).view(torch.uint8))
        self.barrier(6)
        if self.rank != src:
            tmp = torch.empty(pad, device=t.device, dtype=torch.uint8)
            _native.call("brain_comm_copy", st.ptrs[src], tmp.data_ptr(), pad, _stream())
            t.view(-1).view(torch.uint8).copy_(tmp[:nbytes])
        self.barrier(7)
        return t

    # ------------------------------------------------------------------ fused DDP optimizer step
    def fused_rs_adamw(self, opt, grad_scale: float) -> None:
        """RS of the gradient bucket + AdamW on this rank's shard + bf16 all-gather push, one kernel."""
        flat = opt.flat
        gbuf, goff = self._buf_of(flat.grad_buf)
        pbuf, poff = self._buf_of(flat.param_buf)
        if gbuf is None or pbuf is None or opt.vmax is not None:
            raise RuntimeError("fused_rs_adamw needs symmetric gradient and parameter buffers (no AMSGrad)")
        b1, b2 = opt.betas
        t = opt.step_count
        self.barrier(8)
        _native.call("brain_comm_ddp_step", gbuf.peer_array(goff), pbuf.peer_array(poff),
                     int(flat.grad_buf.dtype == torch.bfloat16), self.rank, self.world, self.rank * flat.shard_size,
                     flat.shard_size, opt.master.data_ptr(), opt.m.data_ptr(), opt.v.data_ptr(), float(opt.lr),
                     float(b1), float(b2), float(opt.eps), float(opt.weight_decay), float(1 - b1 ** t),
                     float(1 - b2 ** t), float(grad_scale), _stream())
        self.barrier(9)

    def close(self) -> None:
        torch.cuda.synchronize()
        for b in list(self.registered.values()):
            b.close()
        self.registered.clear()
        if self.staging is not None:
            self.staging.close()
            self.staging = None
        for b in (self.os_stage, self.os_flags, self.ts_flags, self.ts_stage):
            if b is not None:
                b.close()
        self.ts_stage = None
        self.pads.close()
