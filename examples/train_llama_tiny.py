"""A tiny Llama (GQA, RoPE, SwiGLU) trained for a few steps through the data-parallel engine: on a GPU
in bf16 through the sm_100a kernels, on the CPU in float32. Launch on N GPUs with
``torchrun --nproc-per-node N examples/train_llama_tiny.py`` (repository on ``PYTHONPATH``)."""
import torch

from brain_b200.models import LlamaLite, LlamaLiteConfig
from brain_b200.parallel import DataParallel, dist


def main(steps: int = 10):
    ctx = dist.init()
    cuda = ctx.device.type == "cuda"
    cfg = LlamaLiteConfig(vocab_size=512, hidden_dim=256, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                          intermediate_dim=512, max_seq_len=128, rope_theta=500000.0)
    model = LlamaLite(cfg, device=ctx.device, dtype=torch.bfloat16 if cuda else torch.float32, seed=0)
    dp = DataParallel(model, lr=3e-3, weight_decay=0.01)
    g = torch.Generator(device=ctx.device).manual_seed(ctx.rank)
    tok = torch.randint(0, cfg.vocab_size, (4, cfg.max_seq_len + 1), device=ctx.device, generator=g)
    losses = [float(dp.train_step(tok[:, :-1], tok[:, 1:])) for _ in range(steps)]
    if ctx.is_master:
        print(f"{dist.rank_prefix()} loss {losses[0]:.3f} -> {losses[-1]:.3f}")
    dist.shutdown()
    return losses


if __name__ == "__main__":
    main()
