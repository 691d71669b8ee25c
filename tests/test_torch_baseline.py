"""The plain-PyTorch comparison arm of the benchmark: it starts from exactly the framework model's
weights, and its float32-master AdamW matches torch.optim.AdamW on float32 weights."""
import pytest
import torch

from brain_b200.bench.torch_baseline import MasterAdamW, build
from brain_b200.models import LlamaLite, LlamaLiteConfig


def _cfg():
    return LlamaLiteConfig(vocab_size=256, hidden_dim=64, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=16,
                           intermediate_dim=96, max_seq_len=32)


def test_same_initial_weights_as_the_framework_model():
    cfg = _cfg()
    ours = dict(LlamaLite(cfg, device="cpu", dtype=torch.bfloat16, seed=3).named_parameters())
    theirs = list(build(cfg, "cpu", seed=3).parameters())
    names = ["embed"] + [f"layers.{i}.{n}" for i in range(cfg.num_layers)
                         for n in ("attn_norm", "wqkv", "wo", "ffn_norm", "w_gate_up", "w_down")] + ["final_norm", "lm_head"]
    assert len(theirs) == len(names)
    for n, t in zip(names, theirs):
        assert torch.equal(ours[n].detach(), t.detach()), n


def test_master_adamw_matches_float32_adamw():
    torch.manual_seed(0)
    p16 = [torch.nn.Parameter(torch.randn(40, 8).bfloat16()), torch.nn.Parameter(torch.randn(8).bfloat16())]
    p32 = [torch.nn.Parameter(p.detach().float().clone()) for p in p16]
    opt = MasterAdamW(p16, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, chunk_bytes=64)
    ref = torch.optim.AdamW(p32, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    assert len(opt.chunks) == 2  # chunked float32 gradients
    for _ in range(3):
        g = [torch.randn_like(p, dtype=torch.float32) for p in p16]
        for p, gi in zip(p16, g):
            p.grad = gi.bfloat16()
        for p, gi in zip(p32, g):
            p.grad = gi.bfloat16().float()
        opt.step()
        ref.step()
    for a, b in zip(p16, p32):
        torch.testing.assert_close(a.float(), b.detach().bfloat16().float())
        torch.testing.assert_close(opt.master[id(a)].detach(), b.detach(), rtol=1e-5, atol=1e-6)


def test_torch_vit_arm_matches_framework_architecture():
    """The ViT comparison arm has the framework ViT's parameter count and trains on CPU."""
    import torch
    from brain_b200.bench.torch_baseline import TorchViT
    from brain_b200.models.config import ViTConfig
    from brain_b200.models.families import ViT
    cfg = ViTConfig(image_size=32, patch_size=16, hidden_dim=64, num_layers=2, num_heads=4, mlp_dim=128,
                    num_classes=10)
    tv = TorchViT(cfg, "cpu", dtype=torch.float32)
    fv = ViT(cfg, device="cpu", dtype=torch.float32)
    assert sum(p.numel() for p in tv.parameters()) == sum(p.numel() for p in fv.parameters())
    x = torch.randn(4, 3, 32, 32)
    y = torch.randint(0, 10, (4,))
    opt = torch.optim.AdamW(tv.parameters(), lr=1e-3)
    l0 = tv(x, y)
    for _ in range(5):
        opt.zero_grad()
        loss = tv(x, y)
        loss.backward()
        opt.step()
    assert torch.isfinite(loss) and loss.item() < l0.item()


def test_torch_decode_arm_cached_steps_match_full_recompute():
    """The PyTorch decode arm's static-shape cached step (masked cache read, device position) produces
    the same greedy tokens as re-running the whole prefix, in float32 on the CPU."""
    from brain_b200.bench.torch_decode import TorchTPDecoder
    cfg = _cfg()
    B, S, NEW = 3, 7, 6
    dec = TorchTPDecoder(cfg, B, S + NEW, "cpu", seed=1, dtype=torch.float32)
    prompts = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(2))
    out = dec.generate(prompts, NEW, graph=False)
    assert out.shape == (B, S + NEW) and torch.equal(out[:, :S], prompts)
    for i in range(NEW):
        ref = dec.prefill(out[:, :S + i], chunk=2)  # full recompute of the prefix
        assert torch.equal(ref, out[:, S + i]), i


def test_torch_decode_arm_shard_shapes():
    from brain_b200.bench.torch_decode import TorchTPDecoder
    cfg = _cfg()
    dec = TorchTPDecoder(cfg, 2, 16, "cpu", shard_of=2, dtype=torch.float32)
    assert (dec.hq, dec.hkv, dec.ffn, dec.vloc) == (2, 1, 48, 128)
    assert dec.layers[0]["wqkv"].shape == ((2 + 2) * 16, 64) and dec.layers[0]["wd"].shape == (64, 48)
    tok = dec.generate(torch.zeros(2, 4, dtype=torch.long), 3, graph=False)
    assert int(tok.max()) < dec.vloc  # a lone shard picks within its own vocabulary slice


def test_bench_link_roofline_fields():
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location("bench_main", os.path.join(os.path.dirname(__file__), "..", "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench._ddp_link_roofline(8_000_000_000, 1, 430.0) is None
    r = bench._ddp_link_roofline(8_000_000_000, 8, 440.0)
    assert r["bytes_in_per_rank_per_step"] == 2 * 7 / 8 * 8e9 * 2
    assert r["transfer_ms_at_link_rate"] == pytest.approx(r["bytes_in_per_rank_per_step"] / 770e9 * 1e3)
    assert 0 < r["share_of_step"] < 1
