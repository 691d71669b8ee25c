"""Recurrent-network extras: a layer-normalised LSTM cell, variational (per-sequence) dropout, padded and
packed sequences with masks, sequence attention (dot, scaled dot, additive) and an attention-augmented
cell, a bidirectional runner with concat/sum/average merging, teacher-forcing schedules, a stateful
online streamer, orthogonal/uniform initialisers and gradient-norm clipping.

Reference: crates/brain-rnn/src/cells/normalized.rs (NormLstmCell), reg_ops.rs (VariationalDropout),
utils.rs (pad_sequence, create_padding_mask, truncate_steps, concat/split states, clip_grad_norm),
seq/attention.rs (SeqAttention, AttentionKind), cells/attention_cell.rs (AttentionCell),
seq/bidirectional.rs (BidirectionalMerge), seq/teacher.rs (TeacherSchedule, TeacherForcer),
process.rs (OnlineRnnStreamer), init_rnn.rs (init_orthogonal, init_uniform). The reference's
NormLstmCell forwards to a plain LSTM without using its gamma/beta; this one normalises the gate
pre-activations and the cell output (Ba et al. 2016). Everything runs batched ([B, T, D]).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..nn.layers import Linear
from ..nn.module import Module
from .rnn import GruCell, LstmCell, RnnCell


# ------------------------------------------------------------------------------------------ init / utils
def init_orthogonal(rows: int, cols: int, seed: int = 0, dtype=torch.float32) -> torch.Tensor:
    """A [rows, cols] matrix with orthonormal rows or columns (QR of a Gaussian, signs fixed by R's diagonal)."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(max(rows, cols), min(rows, cols), generator=g, dtype=torch.float64)
    q, r = torch.linalg.qr(a)
    q = q * torch.sign(torch.diagonal(r))
    return (q if rows >= cols else q.t()).to(dtype).contiguous()


def init_uniform(rows: int, cols: int, fan_in: int, seed: int = 0, dtype=torch.float32) -> torch.Tensor:
    """U(-1/sqrt(fan_in), 1/sqrt(fan_in))."""
    g = torch.Generator().manual_seed(seed)
    b = 1.0 / math.sqrt(max(fan_in, 1))
    return ((torch.rand(rows, cols, generator=g, dtype=torch.float64) * 2 - 1) * b).to(dtype)


def clip_grad_norm(grads, max_norm: float) -> float:
    """Scale all tensors in place so their joint L2 norm is at most max_norm; returns the norm before."""
    total = math.sqrt(sum(float(g.double().square().sum()) for g in grads))
    if total > max_norm > 0:
        for g in grads:
            g.mul_(max_norm / (total + 1e-6))
    return total


def pad_sequence(sequences, padding_value: float = 0.0) -> torch.Tensor:
    """List of [T_i, D] -> [B, T_max, D] (batch first)."""
    return torch.nn.utils.rnn.pad_sequence(list(sequences), batch_first=True, padding_value=padding_value)


def create_padding_mask(lengths, max_len: int | None = None) -> torch.Tensor:
    """[B, T] bool, True at valid (non-padded) steps."""
    lengths = torch.as_tensor(lengths)
    T = int(max_len if max_len is not None else lengths.max())
    return torch.arange(T, device=lengths.device)[None, :] < lengths[:, None]


def truncate_steps(sequence: torch.Tensor, max_steps: int) -> torch.Tensor:
    """Keep the first max_steps time steps of [B, T, D] (or [T, D])."""
    return sequence[..., :max_steps, :] if sequence.dim() >= 2 else sequence[:max_steps]


def concat_states(a, b):
    return tuple(torch.cat([x, y], -1) for x, y in zip(a, b))


def split_states(combined, hidden: int):
    return tuple(t[..., :hidden] for t in combined), tuple(t[..., hidden:] for t in combined)


@dataclass
class PackedSequence:
    """Variable-length batch as padded data [B, T, D] plus lengths; ``unpack`` returns the list of rows."""
    data: torch.Tensor
    lengths: torch.Tensor

    @classmethod
    def pack(cls, sequences) -> "PackedSequence":
        seqs = list(sequences)
        return cls(pad_sequence(seqs), torch.tensor([s.shape[0] for s in seqs]))

    def mask(self) -> torch.Tensor:
        return create_padding_mask(self.lengths, self.data.shape[1])

    def unpack(self):
        return [self.data[i, :int(n)] for i, n in enumerate(self.lengths)]


# ------------------------------------------------------------------------------------------ cells
class NormLstmCell(Module):
    """LSTM with layer normalisation of the input and recurrent gate projections (separately) and of the
    new cell state before the output tanh; learnable gain/bias per normalisation."""

    def __init__(self, input_dim: int, hidden_dim: int, device=None, dtype=None):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.ih = Linear(input_dim, 4 * hidden_dim, False, device, dtype)
        self.hh = Linear(hidden_dim, 4 * hidden_dim, False, device, dtype)
        self.ln_i = torch.nn.LayerNorm(4 * hidden_dim, device=device, dtype=dtype)
        self.ln_h = torch.nn.LayerNorm(4 * hidden_dim, device=device, dtype=dtype)
        self.ln_c = torch.nn.LayerNorm(hidden_dim, device=device, dtype=dtype)
        with torch.no_grad():
            self.ln_i.bias[hidden_dim:2 * hidden_dim].fill_(1.0)  # forget-gate bias

    def forward(self, x, state=None):
        B = x.shape[0]
        h, c = state if state is not None else (x.new_zeros(B, self.hidden_dim), x.new_zeros(B, self.hidden_dim))
        g = self.ln_i(self.ih(x)) + self.ln_h(self.hh(h))
        i, f, gg, o = g.chunk(4, -1)
        c = torch.sigmoid(f) * c + torch.sigmoid(i) * torch.tanh(gg)
        h = torch.sigmoid(o) * torch.tanh(self.ln_c(c))
        return h, c


class VariationalDropout(Module):
    """One dropout mask per sequence, shared across time steps ([B, T, D] input; mask [B, 1, D])."""

    def __init__(self, p: float):
        super().__init__()
        self.p = p

    def forward(self, x, generator=None):
        if not self.training or self.p <= 0:
            return x
        keep = (torch.rand(x.shape[0], 1, x.shape[-1], generator=generator, device="cpu") >= self.p).to(x.device)
        return x * keep.to(x.dtype) / (1.0 - self.p)


class AttentionKind:
    DOT, SCALED_DOT, ADDITIVE = "dot", "scaled_dot", "additive"


class SeqAttention(Module):
    """Attention of a query [B, Dq] over keys/values [B, T, Dk]/[B, T, Dv]: dot, dot / sqrt(Dk), or additive
    v^T tanh(W_q q + W_k k) (Bahdanau); masked positions get no weight. Returns (context [B, Dv], weights [B, T])."""

    def __init__(self, query_dim: int, key_dim: int, kind: str = AttentionKind.DOT, attn_dim: int = 64,
                 device=None, dtype=None):
        super().__init__()
        self.kind = kind
        if kind == AttentionKind.ADDITIVE:
            self.wq = Linear(query_dim, attn_dim, False, device, dtype)
            self.wk = Linear(key_dim, attn_dim, False, device, dtype)
            self.v = Linear(attn_dim, 1, False, device, dtype)

    def forward(self, query, keys, values, mask=None):
        if self.kind == AttentionKind.ADDITIVE:
            scores = self.v(torch.tanh(self.wq(query)[:, None] + self.wk(keys))).squeeze(-1)
        else:
            d = min(query.shape[-1], keys.shape[-1])
            scores = (keys[..., :d] @ query[..., :d, None]).squeeze(-1)
            if self.kind == AttentionKind.SCALED_DOT:
                scores = scores / math.sqrt(keys.shape[-1])
        if mask is not None:
            scores = scores.masked_fill(~mask, float("-inf"))
        w = torch.softmax(scores, -1)
        return (w[..., None] * values).sum(1), w


class AttentionCell(Module):
    """A recurrent cell whose input is augmented with attention over a memory: each step attends with the
    previous hidden state, then runs the base LSTM/GRU cell on [x, context]."""

    def __init__(self, input_dim: int, hidden_dim: int, memory_dim: int, kind: str = AttentionKind.ADDITIVE,
                 cell: str = "lstm", device=None, dtype=None):
        super().__init__()
        self.attn = SeqAttention(hidden_dim, memory_dim, kind, device=device, dtype=dtype)
        ctor = {"lstm": LstmCell, "gru": GruCell, "rnn": RnnCell}[cell]
        self.cell = ctor(input_dim + memory_dim, hidden_dim, device=device, dtype=dtype)
        self.hidden_dim, self.kind = hidden_dim, cell

    def forward(self, x, memory, state=None, mask=None):
        B = x.shape[0]
        if state is None:
            z = x.new_zeros(B, self.hidden_dim)
            state = (z, z.clone()) if self.kind == "lstm" else (z,)
        ctx, w = self.attn(state[0], memory, memory, mask)
        return self.cell(torch.cat([x, ctx], -1), state), w


# ------------------------------------------------------------------------------------------ runners
class BidirectionalMerge:
    CONCAT, SUM, AVERAGE = "concat", "sum", "average"


def run_cell(cell, x: torch.Tensor, state=None, reverse: bool = False, mask=None):
    """Unroll a cell over [B, T, D]; with a mask, padded steps keep the previous state and emit zeros.
    Returns (outputs [B, T, H], final state)."""
    T = x.shape[1]
    outs = [None] * T
    order = range(T - 1, -1, -1) if reverse else range(T)
    for t in order:
        new = cell(x[:, t], state)
        if mask is not None:
            m = mask[:, t, None].to(x.dtype)
            new = tuple(m * n + (1 - m) * (s if s is not None else torch.zeros_like(n))
                        for n, s in zip(new, state if state is not None else (None,) * len(new)))
            outs[t] = new[0] * m
        else:
            outs[t] = new[0]
        state = new
    return torch.stack(outs, 1), state


class BidirectionalRnn(Module):
    """A forward and a backward cell over the sequence; outputs merged by concat, sum or average."""

    def __init__(self, fwd, bwd, merge: str = BidirectionalMerge.CONCAT):
        super().__init__()
        self.fwd, self.bwd, self.merge = fwd, bwd, merge

    def forward(self, x, mask=None):
        of, sf = run_cell(self.fwd, x, mask=mask)
        ob, sb = run_cell(self.bwd, x, reverse=True, mask=mask)
        if self.merge == BidirectionalMerge.CONCAT:
            out = torch.cat([of, ob], -1)
        elif self.merge == BidirectionalMerge.SUM:
            out = of + ob
        else:
            out = (of + ob) / 2
        return out, (sf, sb)


class TeacherSchedule:
    """constant(r), linear(start, end, steps) (end after ``steps``), exponential(start, decay, min)."""

    def __init__(self, kind: str, **kw):
        self.kind, self.kw = kind, kw

    @classmethod
    def constant(cls, r):
        return cls("constant", r=r)

    @classmethod
    def linear(cls, start, end, steps):
        return cls("linear", start=start, end=end, steps=steps)

    @classmethod
    def exponential(cls, start, decay_rate, min_ratio):
        return cls("exponential", start=start, decay_rate=decay_rate, min_ratio=min_ratio)

    def ratio(self, step: int) -> float:
        k = self.kw
        if self.kind == "constant":
            return k["r"]
        if self.kind == "linear":
            return k["end"] if step >= k["steps"] else k["start"] + (k["end"] - k["start"]) * step / k["steps"]
        return max(k["start"] * k["decay_rate"] ** step, k["min_ratio"])


class TeacherForcer:
    def __init__(self, schedule: TeacherSchedule, generator=None):
        self.schedule, self.step, self.g = schedule, 0, generator

    def current_ratio(self) -> float:
        return self.schedule.ratio(self.step)

    def advance_step(self) -> None:
        self.step += 1

    def choose(self, ground_truth: torch.Tensor, predicted: torch.Tensor) -> torch.Tensor:
        """Per sample: the ground truth with probability current_ratio, else the model's prediction."""
        use = torch.rand(ground_truth.shape[0], generator=self.g) < self.current_ratio()
        use = use.to(ground_truth.device).view(-1, *([1] * (ground_truth.dim() - 1)))
        return torch.where(use, ground_truth, predicted)


class OnlineRnnStreamer:
    """Feeds a stream one step (or chunk) at a time through a cell, carrying the state between calls;
    ``reset`` clears it (optionally for selected batch rows)."""

    def __init__(self, cell):
        self.cell, self.state = cell, None

    @torch.no_grad()
    def push(self, x: torch.Tensor) -> torch.Tensor:
        """x [B, D] (one step) or [B, T, D] (a chunk); returns the outputs for those steps."""
        if x.dim() == 2:
            self.state = self.cell(x, self.state)
            return self.state[0]
        out, self.state = run_cell(self.cell, x, self.state)
        return out

    def reset(self, rows=None) -> None:
        if rows is None or self.state is None:
            self.state = None
            return
        keep = torch.ones(self.state[0].shape[0], dtype=torch.bool, device=self.state[0].device)
        keep[rows] = False
        self.state = tuple(s * keep[:, None].to(s.dtype) for s in self.state)
