"""Host-side distributed building blocks with the reference's names: ``AllReduceAlgorithm`` /
``AllReduceConfig`` / ``execute_allreduce`` (choosing between the NVLink kernels and NCCL / Gloo),
``GradBucket`` (size-capped gradient buckets that flatten and scatter back), ``ClusterNode`` /
``ClusterTopology`` (host and local-rank layout), ``MessageHeader`` + ``StoreCommBackend`` (point-to-point
byte messages over the rendezvous key-value store, CRC-checked), ``DistributedBuilder`` and
``crc32_checksum``.

Reference: crates/brain-distributed/src/collective/allreduce.rs:5-110 (algorithm enum, config with a
chunk size), grad_allreduce.rs:8-26 (GradBucket), cluster.rs / topology.rs (ClusterNode,
ClusterTopology), comm/mod.rs:8-10 (CommBackend::send_bytes / recv_bytes, declared without an
implementation), comm/message.rs (MessageHeader src / dest / tag), utils.rs (crc32_checksum, IEEE),
builder.rs (DistributedBuilder).
"""
from __future__ import annotations

import enum
import struct
import zlib
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


def crc32_checksum(data: bytes) -> int:
    """IEEE CRC-32 (reflected polynomial 0xEDB88320, initial and final inversion)."""
    return zlib.crc32(data) & 0xFFFFFFFF


class AllReduceAlgorithm(enum.Enum):
    AUTO = "auto"          # NVLink kernels when a comm is given and the tensor qualifies, else the process group
    ONE_SHOT = "one_shot"  # every rank reads every peer's copy (NVLink, small messages)
    TWO_SHOT = "two_shot"  # reduce own shard, push it to every peer (NVLink, mid-size messages)
    RING = "ring"          # the process group's collective (NCCL ring / tree, Gloo ring)
    TREE = "tree"
    BUTTERFLY = "butterfly"


@dataclass
class AllReduceConfig:
    algorithm: AllReduceAlgorithm = AllReduceAlgorithm.AUTO
    chunk_size: int = 65536
    op: str = "sum"


def execute_allreduce(t: torch.Tensor, config: AllReduceConfig | None = None, comm=None, group=None) -> torch.Tensor:
    """All-reduce ``t`` in place. With an ``NvlinkComm`` and AUTO / ONE_SHOT / TWO_SHOT the framework's
    NVLink kernels run (the comm picks one-launch, two-phase or staged by size); RING / TREE / BUTTERFLY
    name the process group's own algorithms and go through it, as does every case without a comm."""
    c = config or AllReduceConfig()
    if comm is not None and c.algorithm in (AllReduceAlgorithm.AUTO, AllReduceAlgorithm.ONE_SHOT,
                                            AllReduceAlgorithm.TWO_SHOT):
        return comm.all_reduce(t, c.op)
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return t
    if c.op in ("mean", "avg"):
        dist.all_reduce(t, group=group)
        return t.div_(dist.get_world_size(group))
    dist.all_reduce(t, op={"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}[c.op],
                    group=group)
    return t


def allreduce_tensor(t: torch.Tensor, op: str = "sum", comm=None) -> torch.Tensor:
    return execute_allreduce(t, AllReduceConfig(op=op), comm)


class GradBucket:
    """Gradients collected until ``max_bytes``: ``push`` returns False when the tensor does not fit
    (the caller starts a new bucket), ``flatten`` packs them into one buffer for one collective,
    ``unflatten`` writes the reduced buffer back into the original tensors."""

    def __init__(self, max_bytes: int):
        self.max_bytes, self.tensors, self.nbytes = max_bytes, [], 0

    def push(self, t: torch.Tensor) -> bool:
        b = t.numel() * t.element_size()
        if self.tensors and self.nbytes + b > self.max_bytes:
            return False
        self.tensors.append(t)
        self.nbytes += b
        return True

    def flatten(self) -> torch.Tensor:
        return torch.cat([t.reshape(-1) for t in self.tensors]) if self.tensors else torch.empty(0)

    def unflatten(self, flat: torch.Tensor) -> None:
        off = 0
        for t in self.tensors:
            n = t.numel()
            t.copy_(flat[off:off + n].view_as(t))
            off += n

    def allreduce(self, op: str = "mean", comm=None) -> None:
        flat = self.flatten()
        execute_allreduce(flat, AllReduceConfig(op=op), comm)
        self.unflatten(flat)


def bucket_gradients(tensors, max_bytes: int) -> list[GradBucket]:
    """Greedy packing in the given order (the order backward produces them)."""
    out = [GradBucket(max_bytes)]
    for t in tensors:
        if not out[-1].push(t):
            out.append(GradBucket(max_bytes))
            out[-1].push(t)
    return out


@dataclass
class ClusterNode:
    rank: int
    address: str = "127.0.0.1"
    local_rank: int = 0
    host_index: int = 0


@dataclass
class ClusterTopology:
    """Ranks laid out host by host with ``gpus_per_host`` each; ranks on one host share an NVLink /
    NVSwitch domain."""
    num_hosts: int = 1
    gpus_per_host: int = 8
    addresses: list = field(default_factory=list)

    @property
    def world_size(self) -> int:
        return self.num_hosts * self.gpus_per_host

    def node(self, rank: int) -> ClusterNode:
        h, l = divmod(rank, self.gpus_per_host)
        addr = self.addresses[h] if h < len(self.addresses) else "127.0.0.1"
        return ClusterNode(rank, addr, l, h)

    def same_host(self, a: int, b: int) -> bool:
        return a // self.gpus_per_host == b // self.gpus_per_host

    def host_ranks(self, host: int) -> list[int]:
        return list(range(host * self.gpus_per_host, (host + 1) * self.gpus_per_host))


@dataclass
class MessageHeader:
    src_rank: int
    dest_rank: int
    tag: int
    seq: int = 0
    nbytes: int = 0
    crc: int = 0
    _FMT = "<IIIQQI"

    def pack(self) -> bytes:
        return struct.pack(self._FMT, self.src_rank, self.dest_rank, self.tag, self.seq, self.nbytes, self.crc)

    @classmethod
    def unpack(cls, b: bytes) -> "MessageHeader":
        return cls(*struct.unpack(cls._FMT, b[:struct.calcsize(cls._FMT)]))

    @classmethod
    def size(cls) -> int:
        return struct.calcsize(cls._FMT)


class StoreCommBackend:
    """Point-to-point byte messages over a torch.distributed key-value store (the rendezvous TCPStore):
    each (src, dest, tag) channel is a numbered sequence of keys holding header + payload. ``recv_bytes``
    blocks up to the store's timeout and checks the CRC. For control-plane traffic (configs, small
    tensors), not bulk data, which goes through NCCL or the NVLink kernels."""

    def __init__(self, store, rank: int, world_size: int):
        self.store, self.rank, self.world = store, rank, world_size
        self._send_seq: dict = {}
        self._recv_seq: dict = {}

    @staticmethod
    def _key(src, dst, tag, seq):
        return f"brain_p2p/{src}->{dst}/{tag}/{seq}"

    def send_bytes(self, dest: int, data: bytes, tag: int = 0) -> None:
        if not 0 <= dest < self.world:
            raise ValueError(f"destination rank {dest} outside world of {self.world}")
        ch = (dest, tag)
        seq = self._send_seq.get(ch, 0)
        self._send_seq[ch] = seq + 1
        hdr = MessageHeader(self.rank, dest, tag, seq, len(data), crc32_checksum(data))
        self.store.set(self._key(self.rank, dest, tag, seq), hdr.pack() + bytes(data))

    def recv_bytes(self, src: int, tag: int = 0) -> bytes:
        ch = (src, tag)
        seq = self._recv_seq.get(ch, 0)
        key = self._key(src, self.rank, tag, seq)
        raw = self.store.get(key)
        self._recv_seq[ch] = seq + 1
        self.store.delete_key(key)
        hdr = MessageHeader.unpack(raw)
        payload = raw[MessageHeader.size():]
        if hdr.nbytes != len(payload) or crc32_checksum(payload) != hdr.crc:
            raise IOError(f"corrupt message from rank {src} (tag {tag}, seq {seq})")
        return payload


class DistributedBuilder:
    """Fluent set-up of the process group: ``DistributedBuilder().backend("gloo").timeout(30).build()``."""

    def __init__(self):
        self._backend, self._timeout, self._device = None, 120.0, None

    def backend(self, name: str) -> "DistributedBuilder":
        self._backend = name
        return self

    def timeout(self, seconds: float) -> "DistributedBuilder":
        self._timeout = seconds
        return self

    def device(self, dev: str) -> "DistributedBuilder":
        self._device = dev
        return self

    def build(self):
        from .dist import init
        return init(self._backend, self._timeout, self._device)
