"""Host-side distributed pieces: all-reduce dispatch, gradient buckets, topology, store messaging."""
import pytest
import torch

from tests._mp import run_ranks
from brain_b200.parallel import cluster as CL


def test_local_pieces():
    assert CL.crc32_checksum(b"123456789") == 0xCBF43926  # the standard CRC-32 check value
    ts = [torch.ones(10), torch.ones(20), torch.ones(30), torch.ones(5)]
    bs = CL.bucket_gradients(ts, max_bytes=120)
    assert [len(b.tensors) for b in bs] == [2, 1, 1]  # 40 + 80 bytes, then 120, then 20
    b = CL.GradBucket(1000)
    a1, a2 = torch.arange(3.0), torch.arange(4.0).reshape(2, 2)
    b.push(a1)
    b.push(a2)
    flat = b.flatten() * 2
    b.unflatten(flat)
    assert a1.tolist() == [0, 2, 4] and a2.tolist() == [[0, 2], [4, 6]]
    big = CL.GradBucket(8)
    assert big.push(torch.ones(10)) and not big.push(torch.ones(1))  # a first oversize tensor still fits
    topo = CL.ClusterTopology(num_hosts=2, gpus_per_host=8, addresses=["10.0.0.1", "10.0.0.2"])
    n = topo.node(11)
    assert topo.world_size == 16 and (n.host_index, n.local_rank, n.address) == (1, 3, "10.0.0.2")
    assert topo.same_host(8, 15) and not topo.same_host(7, 8) and topo.host_ranks(1)[0] == 8
    h = CL.MessageHeader(1, 2, 7, 3, 10, 99)
    assert CL.MessageHeader.unpack(h.pack()) == h
    x = torch.ones(3)
    assert CL.execute_allreduce(x) is x  # no process group: nothing to reduce


def _ranks(rank, world):
    import torch.distributed as dist
    from brain_b200.parallel import cluster as CL
    ctx = CL.DistributedBuilder().backend("gloo").device("cpu").timeout(60).build()
    t = torch.full((4,), float(rank + 1))
    CL.execute_allreduce(t, CL.AllReduceConfig(CL.AllReduceAlgorithm.RING))
    m = torch.full((2,), float(rank))
    CL.allreduce_tensor(m, "mean")
    mx = torch.tensor([float(rank)])
    CL.execute_allreduce(mx, CL.AllReduceConfig(op="max"))
    g1, g2 = torch.full((3,), float(rank)), torch.full((2, 2), float(rank * 10))
    b = CL.GradBucket(1 << 20)
    b.push(g1)
    b.push(g2)
    b.allreduce("mean")
    store = dist.distributed_c10d._get_default_store()
    be = CL.StoreCommBackend(store, rank, world)
    peer = 1 - rank
    be.send_bytes(peer, f"hello from {rank}".encode(), tag=5)
    be.send_bytes(peer, b"second", tag=5)
    got = [be.recv_bytes(peer, tag=5), be.recv_bytes(peer, tag=5)]
    dist.barrier()
    from brain_b200.parallel import dist as bdist
    bdist.shutdown()
    return t.tolist(), m.tolist(), mx.tolist(), g1.tolist(), g2.tolist(), [x.decode() for x in got], ctx.world_size


def test_gloo_cluster_pieces():
    out = run_ranks(_ranks, 2)
    for rank, (t, m, mx, g1, g2, got, ws) in enumerate(out):
        assert t == [3.0] * 4 and m == [0.5, 0.5] and mx == [1.0] and ws == 2
        assert g1 == [0.5] * 3 and g2 == [[5.0, 5.0], [5.0, 5.0]]
        assert got == [f"hello from {1 - rank}", "second"]
