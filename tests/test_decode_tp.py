"""Decode-step kernels (swap-AB skinny tcgen05 GEMM with fused epilogues, fused all-reduce + residual +
RMSNorm, greedy pick + embedding) on one rank, against float32 PyTorch restatements."""
import pytest
import torch

from brain_b200.ops import check_status
from brain_b200.ops.decode import (EPI_ARGMAX, EPI_PUSH, EPI_QKV, EPI_SWIGLU, ar_norm, decode_ext, init_ar_slots,
                                   interleave_gate_up, pick_embed, skinny_gemm)
from brain_b200.ops.rope import rope_ref, rope_table

pytestmark = pytest.mark.gpu


def _rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).bfloat16()


@pytest.mark.parametrize("M,N,K", [(32, 1280, 8192), (1, 8192, 1024), (7, 1000, 520), (50, 384, 3584),
                                   (16, 16032, 2048), (32, 8192, 3584)])
@pytest.mark.parametrize("splits", [None, 1])
def test_skinny_store(M, N, K, splits):
    x, w = _rand(M, K, seed=1), _rand(N, K, scale=0.02, seed=2)
    r = _rand(M, N, seed=3)
    y = skinny_gemm(x, w, residual=r, splits=splits)
    ref = x.float() @ w.float().t() + r.float()
    assert not check_status()
    err = (y.float() - ref).abs().max().item()
    assert err < 3e-2 * max(1.0, ref.abs().max().item()), err


def test_skinny_deterministic():
    x, w = _rand(32, 8192, seed=4), _rand(7168, 8192, scale=0.02, seed=5)
    a = skinny_gemm(x, w)
    b = skinny_gemm(x, w)
    assert torch.equal(a, b)


def test_skinny_swiglu():
    M, F, K = 32, 512, 1024
    x = _rand(M, K, seed=6)
    wg, wu = _rand(F, K, scale=0.03, seed=7), _rand(F, K, scale=0.03, seed=8)
    y = skinny_gemm(x, interleave_gate_up(wg, wu), epi=EPI_SWIGLU)
    g, u = x.float() @ wg.float().t(), x.float() @ wu.float().t()
    ref = torch.nn.functional.silu(g) * u
    assert not check_status()
    assert (y.float() - ref).abs().max().item() < 2e-2


def test_skinny_qkv_rope_paged():
    M, Hq, Hkv, D, K, bs = 5, 4, 2, 128, 512, 16
    x = _rand(M, K, seed=9)
    w = _rand((Hq + 2 * Hkv) * D, K, scale=0.03, seed=10)
    pos = torch.tensor([0, 3, 17, 31, 9], dtype=torch.int32, device="cuda")
    max_blocks = 4
    table = torch.arange(M * max_blocks, dtype=torch.int32, device="cuda").view(M, max_blocks).flip(1).contiguous()
    nblocks = M * max_blocks
    kp = torch.zeros(nblocks, bs, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    cs = rope_table(D, 64, 500000.0, device="cuda")
    ext = decode_ext(hq=Hq, hkv=Hkv, pos=pos, rope_cs=cs, k_pool=kp, v_pool=vp, block_table=table)
    q = skinny_gemm(x, w, epi=EPI_QKV, ext=ext, out_cols=Hq * D)
    assert not check_status()
    full = (x.float() @ w.float().t()).view(M, 1, Hq + 2 * Hkv, D)
    rot = rope_ref(full[:, :, :Hq + Hkv], cs, pos.long()[:, None])
    assert (q.float() - rot[:, 0, :Hq].reshape(M, -1)).abs().max().item() < 3e-2
    for t in range(M):
        p = int(pos[t])
        blk = int(table[t, p // bs])
        assert (kp[blk, p % bs].float() - rot[t, 0, Hq:]).abs().max().item() < 3e-2
        assert (vp[blk, p % bs].float() - full[t, 0, Hq + Hkv:]).abs().max().item() < 3e-2


def test_push_ar_norm_single_rank():
    M, N, K = 32, 2048, 1024
    x, w = _rand(M, K, seed=11), _rand(N, K, scale=0.02, seed=12)
    resid = _rand(M, N, seed=13)
    gamma = (1.0 + 0.1 * _rand(N, seed=14).float()).bfloat16()
    resid0 = resid.clone()
    slot_elems = M * N
    slots = init_ar_slots(torch.empty(2 * slot_elems, device="cuda", dtype=torch.bfloat16))
    ctrl = torch.zeros(4, device="cuda", dtype=torch.int32)
    ext = decode_ext(world=1, rank=0, slot_elems=slot_elems, ctrl=ctrl, peer_slots=[slots.data_ptr()])
    normed = torch.empty_like(resid)
    for step in range(3):  # both slot parities, each reused
        skinny_gemm(x, w, epi=EPI_PUSH, ext=ext)
        ar_norm(slots.data_ptr(), ctrl, 1, slot_elems, resid, gamma, 1e-5, normed)
        h = resid0.float() + (step + 1) * (x.float() @ w.float().t())
        assert not check_status()
        assert (resid.float() - h).abs().max().item() < 0.1 * (step + 1)
        hn = resid.float()
        ref = hn * torch.rsqrt(hn.pow(2).mean(-1, keepdim=True) + 1e-5) * gamma.float()
        assert (normed.float() - ref).abs().max().item() < 5e-2
    # epochs 1..3 produced and consumed; every slot is back to the sentinel
    assert int(ctrl[0]) == 3 and int(ctrl[1]) == 3
    assert bool((slots.view(torch.int16) == -32768).all())


def test_argmax_pick_embed_single_rank():
    M, V, K, N = 8, 3000, 512, 512
    x, w = _rand(M, K, seed=15), _rand(V, K, scale=0.05, seed=16)
    emb = _rand(V, N, seed=17)
    gamma = torch.ones(N, device="cuda", dtype=torch.bfloat16)
    keys = torch.zeros(M, device="cuda", dtype=torch.int64)
    key_slots = torch.zeros(2 * M, device="cuda", dtype=torch.int64)
    ctrl = torch.zeros(4, device="cuda", dtype=torch.int32)
    ext = decode_ext(world=1, rank=0, slot_elems=M, ctrl=ctrl, keys=keys, peer_slots=[key_slots.data_ptr()])
    hist = torch.zeros(M, 16, device="cuda", dtype=torch.int32)
    pos = torch.full((M,), 4, device="cuda", dtype=torch.int32)
    seq_lens = pos + 1
    resid = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    normed = torch.empty_like(resid)
    skinny_gemm(x, w, epi=EPI_ARGMAX, ext=ext)
    pick_embed(key_slots.data_ptr(), ctrl, 1, M, emb, resid, gamma, 1e-5, normed, hist, pos, seq_lens)
    assert not check_status()
    logits = x.float() @ w.float().t()
    tok = hist[:, 5].long()
    # the pick is the max of the kernel's own f32 logits: equal to the reference max up to rounding
    picked = logits.gather(1, tok[:, None])[:, 0]
    assert (picked - logits.max(1).values).abs().max().item() < 2e-2
    assert torch.equal(pos.cpu(), torch.full((M,), 5, dtype=torch.int32))
    assert torch.equal(seq_lens.cpu(), torch.full((M,), 6, dtype=torch.int32))
    assert torch.equal(resid, emb[tok])
    assert int(keys.abs().sum()) == 0 and int(key_slots.abs().sum()) == 0
