"""BrainMind: the reference's tiny byte-level conversational model (crates/brain-core/src/brain_mind.rs).

Architecture as in brain_mind.rs:31-325: bytes (vocab 256) -> embedding d=64 + 0.1 x sinusoidal
positions -> one pre-norm block (RMSNorm, 4-head causal attention, RMSNorm, FFN 128 with swish and
no gate) -> RMSNorm -> LM head over 256 bytes. Trained with Adam on text (``train_text`` /
``teach_file``, brain_mind.rs:724-778, 1737); ``talk`` (brain_mind.rs:939) answers simple
arithmetic and remembered facts with rules first and otherwise generates bytes greedily.
Checkpoints use the ``.bn`` container (brain_mind.rs:1865-2025).
"""
from __future__ import annotations

import re

import torch

from ..checkpoint.formats import BrainModelFile
from ..optim import Adam
from .position import sinusoidal


class BrainMind(torch.nn.Module):
    D, H, F, V, CTX = 64, 4, 128, 256, 128

    def __init__(self, seed: int = 0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        D, F, V = self.D, self.F, self.V

        def xavier(o, i):
            return torch.nn.Parameter(torch.randn(o, i, generator=g) * (2.0 / (o + i)) ** 0.5)
        self.emb = xavier(V, D)
        self.n1 = torch.nn.Parameter(torch.ones(D))
        self.wqkv = xavier(3 * D, D)
        self.wo = xavier(D, D)
        self.n2 = torch.nn.Parameter(torch.ones(D))
        self.w1 = xavier(F, D)
        self.w2 = xavier(D, F)
        self.nf = torch.nn.Parameter(torch.ones(D))
        self.head = xavier(V, D)
        self.register_buffer("pe", sinusoidal(self.CTX, D) * 0.1)
        self.facts: dict[str, str] = {}

    @staticmethod
    def _rms(x, w, eps=1e-6):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        B, S = ids.shape
        x = self.emb[ids] + self.pe[:S]
        h = self._rms(x, self.n1)
        q, k, v = (h @ self.wqkv.t()).view(B, S, 3, self.H, self.D // self.H).unbind(2)
        att = (q.transpose(1, 2) @ k.transpose(1, 2).transpose(-1, -2)) / (self.D // self.H) ** 0.5
        mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
        att = att.masked_fill(mask, -1e9).softmax(-1)
        o = (att @ v.transpose(1, 2)).transpose(1, 2).reshape(B, S, self.D)
        x = x + o @ self.wo.t()
        h = self._rms(x, self.n2) @ self.w1.t()
        x = x + (h * torch.sigmoid(h)) @ self.w2.t()
        return self._rms(x, self.nf) @ self.head.t()

    @staticmethod
    def encode(text: str) -> torch.Tensor:
        return torch.tensor(list(text.encode("utf-8")), dtype=torch.long)

    def train_text(self, text: str, steps: int = 50, lr: float = 3e-3, window: int = 64) -> list[float]:
        data = self.encode(text)
        if len(data) < 2:
            return []
        opt = Adam(self.parameters(), lr=lr)
        opt.compute_norms = False
        losses = []
        for s in range(steps):
            i = (s * 17) % max(1, len(data) - window - 1) if len(data) > window + 1 else 0
            chunk = data[i:i + window + 1][None]
            opt.zero_grad()
            logits = self.forward(chunk[:, :-1])
            loss = torch.nn.functional.cross_entropy(logits.reshape(-1, self.V), chunk[:, 1:].reshape(-1))
            loss.backward()
            opt.step()
            losses.append(float(loss.detach()))
        for m in re.finditer(r"(\w[\w ]*?) is ([^.]+)\.", text):
            self.facts[m.group(1).strip().lower()] = m.group(2).strip()
        return losses

    def teach_file(self, path: str, steps: int = 100) -> list[float]:
        with open(path, encoding="utf-8") as f:
            return self.train_text(f.read(), steps)

    @torch.no_grad()
    def generate(self, prompt: str, max_new: int = 32) -> str:
        ids = self.encode(prompt)[None] if prompt else torch.zeros(1, 1, dtype=torch.long)
        out = []
        for _ in range(max_new):
            logits = self.forward(ids[:, -self.CTX:])[:, -1]
            nxt = int(logits.argmax(-1))
            out.append(nxt)
            ids = torch.cat([ids, torch.tensor([[nxt]])], 1)
        return bytes(out).decode("utf-8", errors="replace")

    def talk(self, message: str, max_new: int = 32) -> str:
        m = re.fullmatch(r"\s*(?:what is\s+)?(-?\d+(?:\.\d+)?)\s*([-+*/])\s*(-?\d+(?:\.\d+)?)\s*\??\s*", message.lower())
        if m:
            a, op, b = float(m.group(1)), m.group(2), float(m.group(3))
            r = {"+": a + b, "-": a - b, "*": a * b, "/": a / b if b else float("nan")}[op]
            return str(int(r)) if r == int(r) else str(r)
        m = re.fullmatch(r"\s*what is ([\w ]+)\??\s*", message.lower())
        if m and m.group(1).strip() in self.facts:
            return self.facts[m.group(1).strip()]
        return self.generate(message, max_new)

    def save(self, path: str) -> None:
        f = BrainModelFile("brain_mind").with_meta("arch", "brain_mind_v1")
        for k, v in self.facts.items():
            f.with_meta(f"fact:{k}", v)
        for n, p in self.named_parameters():
            f.add_tensor(n, p.detach().double())
        f.save_file(path)

    @staticmethod
    def load(path: str) -> "BrainMind":
        f = BrainModelFile.load_file(path)
        bm = BrainMind()
        with torch.no_grad():
            for n, p in bm.named_parameters():
                p.copy_(f.archive.get(n).float())
        bm.facts = {k[5:]: v for k, v in f.metadata.items() if k.startswith("fact:")}
        return bm
