"""Race detection by repetition: the kernels that reduce across threads or CTAs (attention backward,
embedding backward, norm weight gradients, the fused training step) must give bit-identical results
when run twice on the same inputs. A data race or an order-dependent atomic shows up as a mismatch.
(``compute-sanitizer`` is not available on the GPU pool, so repetition is the race check.)"""
import pytest
import torch

gpu = pytest.mark.gpu


def _rnd(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).bfloat16()


@gpu
def test_attention_backward_is_bitwise_repeatable():
    from brain_b200.ops import attention as attn
    B, S, Hq, Hkv, D = 2, 512, 8, 2, 128
    q, k, v = _rnd(B, S, Hq, D, seed=1), _rnd(B, S, Hkv, D, seed=2), _rnd(B, S, Hkv, D, seed=3)
    do = _rnd(B, S, Hq, D, seed=4)
    o, lse = attn._fwd(q, k, v, True, D ** -0.5)
    outs = []
    for _ in range(2):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        attn._bwd(q, k, v, o, lse, do, dq, dk, dv, True, D ** -0.5)
        outs.append((dq, dk, dv))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@gpu
def test_embedding_and_norm_backward_are_bitwise_repeatable():
    from brain_b200 import ops
    w = _rnd(1000, 256, seed=5).requires_grad_(True)
    ids = torch.randint(0, 50, (4, 512), device="cuda")  # many repeated ids -> contended rows
    x = _rnd(2048, 256, seed=6).requires_grad_(True)
    nw = (_rnd(256, seed=7, scale=0.1) + 1).requires_grad_(True)
    grads = []
    for _ in range(2):
        w.grad = x.grad = nw.grad = None
        ops.embedding(ids, w).float().pow(2).sum().backward()
        ops.rms_norm(x, nw, 1e-6).float().pow(2).sum().backward()
        grads.append((w.grad.clone(), x.grad.clone(), nw.grad.clone()))
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@gpu
def test_training_step_is_bitwise_repeatable():
    from brain_b200.models import LlamaLite, LlamaLiteConfig
    from brain_b200.parallel import DataParallel
    cfg = LlamaLiteConfig(vocab_size=512, hidden_dim=256, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                          intermediate_dim=512, max_seq_len=256, rope_theta=500000.0)
    tok = torch.randint(0, 512, (2, 257), device="cuda", generator=torch.Generator(device="cuda").manual_seed(0))
    results = []
    for _ in range(2):
        model = LlamaLite(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
        dp = DataParallel(model, lr=1e-3, grad_dtype=torch.float32)
        losses = [float(dp.train_step(tok[:, :-1], tok[:, 1:])) for _ in range(3)]
        results.append((losses, dp.flat.param_buf.clone()))
    assert results[0][0] == results[1][0]
    assert torch.equal(results[0][1], results[1][1])
