"""Token sampling with the reference's pipeline and defaults.

Order (crates/brain-transformer/src/generate.rs:129-158): repetition penalty -> greedy if
temperature <= 1e-6 -> top-k / top-p / min-p filtering -> temperature sampling. Defaults:
temperature 0.7, top_k 50, top_p 0.9, repetition_penalty 1.1 (generate.rs:20-60). Everything runs
batched on the device; the random stream comes from a seeded ``torch.Generator``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class GenerationConfig:
    max_new_tokens: int = 32
    temperature: float = 0.7
    top_k: int = 50
    top_p: float = 0.9
    min_p: float = 0.0
    repetition_penalty: float = 1.1
    eos_token_id: int | None = None
    seed: int = 0

    @staticmethod
    def greedy(max_new_tokens=32):
        return GenerationConfig(max_new_tokens=max_new_tokens, temperature=0.0, top_k=0, top_p=1.0,
                                repetition_penalty=1.0)


def apply_repetition_penalty(logits: torch.Tensor, history: torch.Tensor, penalty: float) -> torch.Tensor:
    """Divide positive / multiply negative logits of already generated tokens (CTRL-style)."""
    if penalty == 1.0 or history is None or history.numel() == 0:
        return logits
    sel = torch.gather(logits, 1, history)
    sel = torch.where(sel > 0, sel / penalty, sel * penalty)
    return logits.scatter(1, history, sel)


def filter_logits(logits: torch.Tensor, top_k: int = 0, top_p: float = 1.0, min_p: float = 0.0) -> torch.Tensor:
    if top_k and top_k < logits.shape[-1]:
        kth = torch.topk(logits, top_k, dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if top_p < 1.0:
        srt, idx = torch.sort(logits, descending=True, dim=-1)
        probs = torch.softmax(srt, dim=-1)
        cum = probs.cumsum(-1)
        drop = cum - probs > top_p
        srt = srt.masked_fill(drop, float("-inf"))
        logits = torch.full_like(logits, float("-inf")).scatter(-1, idx, srt)
    if min_p > 0.0:
        probs = torch.softmax(logits, dim=-1)
        thresh = probs.amax(-1, keepdim=True) * min_p
        logits = logits.masked_fill(probs < thresh, float("-inf"))
    return logits


def sample_next_token(logits: torch.Tensor, cfg: GenerationConfig, history: torch.Tensor | None = None,
                      generator: torch.Generator | None = None) -> torch.Tensor:
    """logits [B, V] -> next ids [B]."""
    logits = logits.float()
    logits = apply_repetition_penalty(logits, history, cfg.repetition_penalty)
    if cfg.temperature <= 1e-6:
        return logits.argmax(-1)
    logits = filter_logits(logits, cfg.top_k, cfg.top_p, cfg.min_p)
    probs = torch.softmax(logits / cfg.temperature, dim=-1)
    return torch.multinomial(probs, 1, generator=generator).squeeze(-1)
