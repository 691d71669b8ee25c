"""Paged decode attention and the fused RoPE + KV append against float32 PyTorch restatements."""
import math

import pytest
import torch

from brain_b200.ops import check_status
from brain_b200.ops.decode import _decode_ref, kv_append_rope, paged_decode_attention
from brain_b200.ops.rope import rope_table


def _paged(B, Hkv, D, lens, block_size, device, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    max_blocks = max(-(-L // block_size) for L in lens) + 1
    nblocks = B * max_blocks + 3
    kp = (torch.randn(nblocks, block_size, Hkv, D, generator=g) * 0.5).bfloat16()
    vp = torch.randn(nblocks, block_size, Hkv, D, generator=g).bfloat16()
    perm = torch.randperm(nblocks, generator=g)[:B * max_blocks].view(B, max_blocks).int()
    return kp.to(device), vp.to(device), perm.to(device), torch.tensor(lens, dtype=torch.int32, device=device)


def test_decode_ref_matches_dense_cpu():
    B, Hq, Hkv, D, bs = 2, 4, 2, 16, 8
    lens = [13, 5]
    kp, vp, table, sl = _paged(B, Hkv, D, lens, bs, "cpu")
    q = torch.randn(B, Hq, D).bfloat16()
    out = paged_decode_attention(q, kp, vp, table, sl)
    for b in range(B):
        L = lens[b]
        k = torch.cat([kp[table[b, i]] for i in range(-(-L // bs))])[:L].float()  # [L, Hkv, D]
        v = torch.cat([vp[table[b, i]] for i in range(-(-L // bs))])[:L].float()
        for h in range(Hq):
            hk = h // (Hq // Hkv)
            p = torch.softmax(q[b, h].float() @ k[:, hk].t() / math.sqrt(D), -1)
            ref = p @ v[:, hk]
            assert torch.allclose(out[b, h].float(), ref, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("D,Hq,Hkv,bs,lens", [
    (128, 8, 1, 64, [1, 64, 65, 700]),
    (128, 64, 8, 128, [300, 2048, 17, 1000]),
    (64, 16, 4, 64, [129, 5]),
    (64, 6, 2, 16, [33, 200, 1]),      # 3 query heads per kv head, 16-token blocks
    (128, 5, 5, 32, [100, 31]),        # one query head per kv head, 32-token blocks
])
def test_paged_decode_attention_gpu(D, Hq, Hkv, bs, lens):
    B = len(lens)
    kp, vp, table, sl = _paged(B, Hkv, D, lens, bs, "cuda")
    # rows past each sequence's end hold NaN: they must not leak into the output
    for b, L in enumerate(lens):
        if L % bs:
            blk = int(table[b, L // bs])
            kp[blk, L % bs:] = float("nan")
            vp[blk, L % bs:] = float("nan")
    # q as a strided view of a fused qkv row, as the model produces it
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    q = qkv[:, :Hq * D].view(B, Hq, D)
    out = paged_decode_attention(q, kp, vp, table, sl)
    ref = _decode_ref(q.cpu(), kp.cpu(), vp.cpu(), table.cpu(), sl.cpu(), 1.0 / math.sqrt(D))
    assert not check_status()
    err = (out.cpu().float() - ref.float()).abs().max().item()
    assert err < 2e-2, err
    # every cluster size (split count) gives the same result, including splits that own no keys and
    # the non-portable sizes above 8
    for sp in (1, 2, 5, 8, 11, 16):
        out1 = paged_decode_attention(q, kp, vp, table, sl, splits=sp)
        assert not check_status()
        assert (out1.float() - out.float()).abs().max().item() < 2e-2, sp


@pytest.mark.gpu
def test_kv_append_rope_gpu():
    B, Hq, Hkv, D, bs = 3, 8, 2, 128, 64
    lens = [10, 64, 200]
    kp, vp, table, _ = _paged(B, Hkv, D, [L + 1 for L in lens], bs, "cuda")
    pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
    cs = rope_table(D, 4096, 500000.0, device="cuda")
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    qkv_c, kp_c, vp_c = qkv.cpu(), kp.cpu(), vp.cpu()
    kv_append_rope(qkv, Hq, Hkv, pos, cs, kp, vp, table)
    kv_append_rope(qkv_c, Hq, Hkv, pos.cpu(), cs.cpu(), kp_c, vp_c, table.cpu())
    assert not check_status()
    assert (qkv[:, :Hq * D].cpu().float() - qkv_c[:, :Hq * D].float()).abs().max().item() < 2e-2
    assert (kp.cpu().float() - kp_c.float()).abs().max().item() < 2e-2
    assert torch.equal(vp.cpu(), vp_c)
