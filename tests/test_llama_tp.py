"""Tensor-parallel Llama serving (prefill + CUDA-graph decode with the fused decode kernels) against the
training model's own forward: every greedily generated token must be an argmax (up to bf16 rounding)
of ``LlamaLite`` logits over the generated sequence. 1 GPU, and TP=2 on 2 GPUs."""
import pytest
import torch

from tests._mp import run_ranks


def _cfg():
    from brain_b200.models import LlamaLiteConfig
    return LlamaLiteConfig(vocab_size=1000, hidden_dim=512, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=128,
                           intermediate_dim=1024, max_seq_len=256, rope_theta=500000.0)


def _check_greedy(model, seq, S, tol=0.06):
    """Max shortfall of the chosen token's logit below the row max, over the generated positions."""
    with torch.no_grad():
        logits = model(seq.cuda()).float()
    worst = 0.0
    for p in range(S, seq.shape[1]):
        row = logits[:, p - 1]
        chosen = row.gather(1, seq[:, p:p + 1].cuda())[:, 0]
        worst = max(worst, float((row.max(1).values - chosen).max()))
    return worst


def _run(world_rank_setup, S, new):
    from brain_b200.models import LlamaLite
    from brain_b200.models.llama_tp import LlamaTPServe
    cfg = _cfg()
    model = LlamaLite(cfg, device="cuda", seed=3)
    B = 4
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, cfg.vocab_size, (B, S), generator=g)
    srv = LlamaTPServe(cfg, max_batch=B, max_len=S + new + 8, block_size=16, init=False).load_from(model)
    out_graph = srv.generate(prompt, new, use_graph=True)
    srv.check()
    out_eager = srv.generate(prompt, new, use_graph=False)
    srv.check()
    worst = _check_greedy(model, out_graph, S)
    srv.close()
    return out_graph.numpy(), out_eager.numpy(), worst


@pytest.mark.gpu
@pytest.mark.parametrize("S", [32, 40])
def test_llama_tp_single_gpu(S):
    g, e, worst = _run(None, S, 12)
    assert (g == e).all()
    assert (g[:, :S] >= 0).all()
    assert worst < 0.06, worst


def _tp_worker(rank, world, S):
    from brain_b200.parallel import dist as bdist
    bdist.init(timeout_s=60)
    try:
        return _run(None, S, 10)
    finally:
        bdist.shutdown()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("S", [64, 24])  # 64: sequence-parallel prefill (T / W = 128); 24: replicated prefill
def test_llama_tp_two_gpus(S):
    outs = run_ranks(_tp_worker, 2, S, env={"NCCL_NVLS_ENABLE": "0"})
    for g, e, worst in outs:
        assert (g == e).all()
        assert worst < 0.06, worst
    assert (outs[0][0] == outs[1][0]).all()


def _cfg_wide():
    from brain_b200.models import LlamaLiteConfig
    # 16 q / 8 kv heads and 2048 FFN columns: every rank of an 8-way group gets whole heads and 64-row groups
    return LlamaLiteConfig(vocab_size=1024, hidden_dim=1024, num_layers=2, num_heads=16, num_kv_heads=8, head_dim=128,
                           intermediate_dim=2048, max_seq_len=256, rope_theta=500000.0)


def _tp_worker_n(rank, world, S, new):
    """Greedy decode at TP=world against the 1-GPU model forward, then the same generation again with
    random per-rank delays before every decode step (host sleeps and GPU spin kernels of different
    lengths on each rank), which must reproduce the tokens: the all-reduce slots (sentinel-marked,
    no flags) may not be reused before every rank consumed them, however the ranks drift."""
    import random
    import time
    from brain_b200.models import LlamaLite
    from brain_b200.models.llama_tp import LlamaTPServe
    from brain_b200.parallel import dist as bdist
    bdist.init(timeout_s=120)
    try:
        cfg = _cfg_wide()
        model = LlamaLite(cfg, device="cuda", seed=5)
        B = 4
        prompt = torch.randint(0, cfg.vocab_size, (B, S), generator=torch.Generator().manual_seed(13))
        srv = LlamaTPServe(cfg, max_batch=B, max_len=S + new + 8, block_size=16, init=False).load_from(model)
        out = srv.generate(prompt, new, use_graph=True)
        srv.check()
        worst = _check_greedy(model, out, S)
        rng = random.Random(1000 + rank)
        with torch.no_grad():
            srv.prefill(prompt)
            srv.step()
            for _ in range(new - 2):
                time.sleep(rng.random() * 2e-3)
                torch.cuda._sleep(rng.randrange(0, 400_000))
                srv.replay()
            torch.cuda.synchronize()
        stressed = srv.hist[:, :S + new].to("cpu", torch.int64)
        srv.check()
        srv.close()
        return out.numpy(), stressed.numpy(), worst
    finally:
        bdist.shutdown()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("world", [4, 8])
def test_llama_tp_decode_wide_groups_and_drift(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    outs = run_ranks(_tp_worker_n, world, 32, 16, env={"NCCL_NVLS_ENABLE": "0"}, timeout=300)
    for g, stressed, worst in outs:
        assert worst < 0.06, worst
        assert (g == stressed).all()
    for g, _, _ in outs[1:]:
        assert (g == outs[0][0]).all()
