"""Recurrent networks: RNN / GRU / LSTM (optionally peephole) cells, multi-layer and bidirectional
sequence runners, teacher forcing, beam search, and a character-level LSTM language model.

Reference: crates/brain-rnn. Cells (cells/lstm.rs:25-34, cells/gru.rs, cells/rnn.rs,
cells/lstm_peephole.rs), sequence runners (seq/lstm_seq.rs, seq/gru_seq.rs, seq/bidirectional.rs),
teacher forcing (seq/teacher.rs), beam search with a length penalty (seq/beam.rs:19-120).

The gate math of a whole time step is one GEMM over the concatenated gates ([4H] for LSTM, [3H] for
GRU) through ``brain_b200.nn.Linear``, so on a GPU in bf16 each step runs on the framework's tcgen05
GEMM; the input projection of the whole sequence is hoisted out of the time loop as one [T*B, in] GEMM.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from ..nn.layers import Embedding, Linear
from ..nn.module import Module


class RnnCell(Module):
    def __init__(self, input_dim: int, hidden_dim: int, nonlinearity: str = "tanh", device=None, dtype=None):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.ih = Linear(input_dim, hidden_dim, True, device, dtype)
        self.hh = Linear(hidden_dim, hidden_dim, False, device, dtype)
        self.act = torch.tanh if nonlinearity == "tanh" else torch.relu

    def step(self, xp, h):
        return (self.act(xp + self.hh(h)),)

    def forward(self, x, state=None):
        h = state[0] if state is not None else x.new_zeros(x.shape[0], self.hidden_dim)
        return self.step(self.ih(x), h)


class GruCell(Module):
    """r = σ(W_r x + U_r h), z = σ(W_z x + U_z h), n = tanh(W_n x + r ⊙ (U_n h)), h' = (1 − z) n + z h."""

    def __init__(self, input_dim: int, hidden_dim: int, device=None, dtype=None):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.ih = Linear(input_dim, 3 * hidden_dim, True, device, dtype)
        self.hh = Linear(hidden_dim, 3 * hidden_dim, True, device, dtype)

    def step(self, xp, h):
        H = self.hidden_dim
        hp = self.hh(h)
        r = torch.sigmoid(xp[..., :H] + hp[..., :H])
        z = torch.sigmoid(xp[..., H:2 * H] + hp[..., H:2 * H])
        n = torch.tanh(xp[..., 2 * H:] + r * hp[..., 2 * H:])
        return ((1 - z) * n + z * h,)

    def forward(self, x, state=None):
        h = state[0] if state is not None else x.new_zeros(x.shape[0], self.hidden_dim)
        return self.step(self.ih(x), h)


class LstmCell(Module):
    """Gates i, f, g, o from one [4H] projection; ``peephole`` adds diagonal cell connections to i, f
    (previous cell) and o (new cell). The forget-gate bias starts at 1."""

    def __init__(self, input_dim: int, hidden_dim: int, peephole: bool = False, device=None, dtype=None):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.ih = Linear(input_dim, 4 * hidden_dim, True, device, dtype)
        self.hh = Linear(hidden_dim, 4 * hidden_dim, False, device, dtype)
        with torch.no_grad():
            self.ih.bias[hidden_dim:2 * hidden_dim].fill_(1.0)
        self.peep = torch.nn.Parameter(torch.zeros(3, hidden_dim, device=device, dtype=dtype)) if peephole else None

    def step(self, xp, h, c):
        H = self.hidden_dim
        g = xp + self.hh(h)
        i, f, gg, o = g[..., :H], g[..., H:2 * H], g[..., 2 * H:3 * H], g[..., 3 * H:]
        if self.peep is not None:
            i = i + self.peep[0] * c
            f = f + self.peep[1] * c
        c2 = torch.sigmoid(f) * c + torch.sigmoid(i) * torch.tanh(gg)
        if self.peep is not None:
            o = o + self.peep[2] * c2
        return torch.sigmoid(o) * torch.tanh(c2), c2

    def forward(self, x, state=None):
        if state is None:
            z = x.new_zeros(x.shape[0], self.hidden_dim)
            state = (z, z)
        return self.step(self.ih(x), *state)


class PeepholeLstmCell(LstmCell):
    """LSTM with diagonal peephole weights (input and forget gates see c_{t-1}, the output gate sees c_t),
    started at 0.1 as the reference's cell does (crates/brain-rnn/src/cells/lstm_peephole.rs:21-50)."""

    def __init__(self, input_dim: int, hidden_dim: int, device=None, dtype=None):
        super().__init__(input_dim, hidden_dim, peephole=True, device=device, dtype=dtype)
        with torch.no_grad():
            self.peep.fill_(0.1)


VanillaRnnCell = RnnCell  # the reference's name for the Elman cell (cells/rnn.rs)

_CELLS = {"rnn": RnnCell, "gru": GruCell, "lstm": LstmCell}


class Recurrent(Module):
    """Multi-layer (optionally bidirectional) recurrent network over [B, T, in] inputs (batch first).
    Returns (outputs [B, T, H * dirs], final states per layer and direction)."""

    def __init__(self, kind: str, input_dim: int, hidden_dim: int, num_layers: int = 1, bidirectional: bool = False,
                 device=None, dtype=None, **cell_kw):
        super().__init__()
        self.kind, self.hidden_dim, self.num_layers = kind, hidden_dim, num_layers
        self.dirs = 2 if bidirectional else 1
        cells = []
        for layer in range(num_layers):
            d_in = input_dim if layer == 0 else hidden_dim * self.dirs
            for _ in range(self.dirs):
                cells.append(_CELLS[kind](d_in, hidden_dim, device=device, dtype=dtype, **cell_kw))
        self.cells = torch.nn.ModuleList(cells)

    def _run(self, cell, x, reverse: bool, state):
        B, T, _ = x.shape
        xp = cell.ih(x.reshape(B * T, -1)).view(B, T, -1)  # input projection for all steps at once
        if state is None:
            z = x.new_zeros(B, self.hidden_dim)
            state = (z, z) if self.kind == "lstm" else (z,)
        outs = [None] * T
        for t in (range(T - 1, -1, -1) if reverse else range(T)):
            state = cell.step(xp[:, t], *state)
            outs[t] = state[0]
        return torch.stack(outs, 1), state

    def forward(self, x, states=None):
        finals = []
        for layer in range(self.num_layers):
            ys = []
            for d in range(self.dirs):
                idx = layer * self.dirs + d
                y, st = self._run(self.cells[idx], x, d == 1, None if states is None else states[idx])
                ys.append(y)
                finals.append(st)
            x = torch.cat(ys, -1) if self.dirs == 2 else ys[0]
        return x, finals


class LSTM(Recurrent):
    def __init__(self, input_dim, hidden_dim, num_layers=1, bidirectional=False, device=None, dtype=None,
                 peephole=False):
        super().__init__("lstm", input_dim, hidden_dim, num_layers, bidirectional, device, dtype, peephole=peephole)


class GRU(Recurrent):
    def __init__(self, input_dim, hidden_dim, num_layers=1, bidirectional=False, device=None, dtype=None):
        super().__init__("gru", input_dim, hidden_dim, num_layers, bidirectional, device, dtype)


class RNN(Recurrent):
    def __init__(self, input_dim, hidden_dim, num_layers=1, bidirectional=False, device=None, dtype=None):
        super().__init__("rnn", input_dim, hidden_dim, num_layers, bidirectional, device, dtype)


class LstmLanguageModel(Module):
    """Embedding -> LSTM -> vocabulary projection; ``teacher_forcing_loss`` is next-token cross entropy
    with the ground-truth previous token fed at every step (seq/teacher.rs)."""

    def __init__(self, vocab_size: int, embed_dim: int, hidden_dim: int, num_layers: int = 1, device=None,
                 dtype=None):
        super().__init__()
        self.emb = Embedding(vocab_size, embed_dim, device, dtype)
        with torch.no_grad():
            self.emb.weight.mul_(0.1)
        self.rnn = LSTM(embed_dim, hidden_dim, num_layers, device=device, dtype=dtype)
        self.head = Linear(hidden_dim, vocab_size, True, device, dtype)

    def forward(self, ids, states=None):
        h, st = self.rnn(self.emb(ids), states)
        return self.head(h), st

    def teacher_forcing_loss(self, ids):
        logits, _ = self(ids[:, :-1])
        return torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))

    @torch.no_grad()
    def greedy(self, prefix, steps: int):
        logits, st = self(prefix)
        out = [prefix]
        tok = logits[:, -1].argmax(-1, keepdim=True)
        for _ in range(steps):
            out.append(tok)
            logits, st = self(tok, st)
            tok = logits[:, -1].argmax(-1, keepdim=True)
        return torch.cat(out, 1)


@dataclass
class BeamHypothesis:
    tokens: list[int]
    log_prob: float = 0.0
    finished: bool = False

    def score(self, alpha: float) -> float:
        """Length-normalised score log p / ((5 + L) / 6)^alpha (Wu et al. 2016)."""
        return self.log_prob / (((5 + len(self.tokens)) / 6) ** alpha)


@dataclass
class BeamConfig:
    beam_width: int = 4
    max_len: int = 32
    length_penalty: float = 0.6
    eos_token: int | None = None


class BeamSearch:
    def __init__(self, config: BeamConfig, start_token: int):
        self.config = config
        self.beams = [BeamHypothesis([start_token])]

    def step(self, next_token_log_probs) -> None:
        """``next_token_log_probs[i]`` is the log-probability row (over the vocabulary) for beam i."""
        cand = []
        for b, lp in zip(self.beams, next_token_log_probs):
            if b.finished:
                cand.append(b)
                continue
            lp = torch.as_tensor(lp, dtype=torch.float64)
            top = torch.topk(lp, min(self.config.beam_width, lp.numel()))
            for v, i in zip(top.values.tolist(), top.indices.tolist()):
                cand.append(BeamHypothesis(b.tokens + [i], b.log_prob + v, i == self.config.eos_token))
        cand.sort(key=lambda h: -h.score(self.config.length_penalty))
        self.beams = cand[:self.config.beam_width]

    def done(self) -> bool:
        return all(b.finished or len(b.tokens) >= self.config.max_len for b in self.beams)

    def best(self) -> BeamHypothesis:
        return max(self.beams, key=lambda h: h.score(self.config.length_penalty))


def beam_search(step_fn, start_token: int, config: BeamConfig) -> BeamHypothesis:
    """Runs ``BeamSearch`` with ``step_fn(list_of_token_lists) -> [beams, vocab] log-probs``."""
    bs = BeamSearch(config, start_token)
    while not bs.done():
        bs.step(step_fn([b.tokens for b in bs.beams]))
    return bs.best()
