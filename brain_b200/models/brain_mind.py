"""BrainMind: the reference's tiny byte-level conversational model (crates/brain-core/src/brain_mind.rs).

Architecture as in brain_mind.rs:31-325: bytes (vocab 256) -> embedding d=64 + 0.1 x sinusoidal
positions -> one pre-norm block (RMSNorm, 4-head causal attention, RMSNorm, FFN 128 with swish and
no gate) -> RMSNorm -> LM head over 256 bytes, trained with Adam on text (``train_text``,
brain_mind.rs:724-778).

Around it, the reference's symbolic memory (brain_mind.rs:939-1737): ``learn_sentence`` grows a word
vocabulary, Hebbian bigram transitions and "X is Y" facts with associations; ``teach_file`` indexes
structured records (TYPE / NAME / DEFINITION / FORMULA / STATEMENT / KEY: VALUE, END); ``talk`` routes a
message the way the reference does: arithmetic (symbols, number words and remembered variables),
percentage and speed x time word problems, greetings (Levenshtein-tolerant), feelings, name learning
and recall, identity, newborn imitation, knowledge search (definitions, formulas, fuzzy keys), associative
recall, spreading-activation thoughts, and for questions the neural generator or an honest "I don't
know". Numbers print like Rust's f64 ``Display``. ``prune_memory`` drops weak links. Checkpoints use the
``.bn`` container (brain_mind.rs:1865-2025) with the symbolic memory in its metadata.
"""
from __future__ import annotations

import json
import re
from dataclasses import dataclass

import torch

from ..checkpoint.formats import BrainModelFile, _rust_display
from ..optim import Adam
from .position import sinusoidal


def levenshtein(a: str, b: str) -> int:
    prev = list(range(len(b) + 1))
    for i, ca in enumerate(a, 1):
        cur = [i]
        for j, cb in enumerate(b, 1):
            cur.append(min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (ca != cb)))
        prev = cur
    return prev[-1]


def _num(x: float) -> str:
    return _rust_display(float(x))


def _alnum_strip(w: str) -> str:
    i, j = 0, len(w)
    while i < j and not w[i].isalnum():
        i += 1
    while j > i and not w[j - 1].isalnum():
        j -= 1
    return w[i:j]


def _parse_num(s: str):
    try:
        return float(s)
    except ValueError:
        return None


def _strip_to_number(tok: str, allow_minus: bool = False) -> str:
    keep = lambda c: c.isdigit() or c == "." or (allow_minus and c == "-")  # noqa: E731
    i, j = 0, len(tok)
    while i < j and not keep(tok[i]):
        i += 1
    while j > i and not keep(tok[j - 1]):
        j -= 1
    return tok[i:j]


_QUESTION_STARTS = ("what", "who", "why", "how", "where", "when", "which", "can ", "do ", "does ", "is ", "are ")
_GREETINGS = ("hi", "hello", "hey", "ello", "helo", "yo", "hola", "greetings", "howdy", "sup")
_SUBJECT_STOPS = {
    "what", "who", "where", "when", "why", "how", "this", "that", "the", "a", "an", "is", "are", "tell", "explain",
    "about", "define", "definition", "of", "mean", "meaning", "in", "if", "then", "else", "so", "much", "many", "does",
    "do", "did", "will", "would", "can", "could", "should", "was", "were", "have", "has", "had", "car", "drive",
    "drives", "train", "travel", "travels", "walk", "run", "with", "for", "to", "from", "by", "at", "on", "out", "it",
    "its", "they", "them", "there", "here", "let", "given", "assume", "suppose", "me"}
_TRIGGERS = ("what is ", "what are ", "what's ", "whats ", "what does ", "what do ", "define ", "explain ",
             "meaning of ", "tell me about ", "describe ")
_STATEMENT_STOPS = {
    "a", "an", "the", "is", "are", "was", "were", "be", "been", "being", "in", "on", "at", "to", "for", "from", "by",
    "with", "of", "and", "or", "but", "if", "then", "so", "as", "it", "its", "they", "them", "he", "she", "we", "you",
    "i", "my", "your", "his", "her", "our", "their", "do", "does", "did", "have", "has", "had", "can", "could", "will",
    "would", "shall", "should", "what", "which", "who", "whom"}


@dataclass
class TeachSummary:
    lines_processed: int = 0
    facts_indexed: int = 0
    words_learned: int = 0
    synapses_upgraded: int = 0
    neural_loss: float = 0.0


class BrainMind(torch.nn.Module):
    D, H, F, V, CTX = 64, 4, 128, 256, 128

    def __init__(self, seed: int = 0, name: str = "brain", cube_dim: int = 8):
        super().__init__()
        self.name, self.cube_dim = name, max(2, cube_dim)
        self.vocab: dict[str, int] = {}
        self.inv_vocab: list[str] = []
        self.transitions: dict[str, dict[str, float]] = {}
        self.associations: dict[str, list[tuple[str, float]]] = {}
        self.context_history: list[tuple[str, str]] = []
        self.user_nickname: str | None = None
        self.age_steps = 0
        self.synaptic_weights = torch.zeros(self.cube_dim, self.cube_dim, dtype=torch.float64)
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

    def train_text(self, text: str, steps: int = 50, lr: float = 3e-3, window: int = 64,
                   extract_facts: bool = True) -> list[float]:
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
        if extract_facts:
            for m in re.finditer(r"(\w[\w ]*?) is ([^.]+)\.", text):
                self.facts[m.group(1).strip().lower()] = m.group(2).strip()
        return losses

    def teach_file(self, path: str, steps: int = 100) -> TeachSummary:
        """Structured teaching (``teach_text``), then ``steps`` Adam steps of the byte model on the file."""
        with open(path, encoding="utf-8") as f:
            content = f.read()
        summary = self.teach_text(content)
        losses = self.train_text(content, steps, extract_facts=False)
        if losses:
            summary.neural_loss = losses[-1]
        return summary

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

    # ------------------------------------------------------------------ symbolic memory
    def total_neurons(self) -> int:
        return self.cube_dim ** 3

    def total_synapses(self) -> int:
        return sum(len(m) for m in self.transitions.values()) + sum(len(v) for v in self.associations.values())

    def learn_sentence(self, text: str) -> None:
        """Vocabulary, bigram transitions (+1 per occurrence) and "X is Y" / "X are Y" facts."""
        words = [w for w in (_alnum_strip(t) for t in text.lower().split()) if w]
        for w in words:
            if w not in self.vocab:
                self.vocab[w] = len(self.vocab)
                self.inv_vocab.append(w)
        for w1, w2 in zip(words, words[1:]):
            nxt = self.transitions.setdefault(w1, {})
            nxt[w2] = nxt.get(w2, 0.0) + 1.0
        stops = {"what", "who", "where", "when", "why", "how", "this", "that", "it", "there", "here", "a", "an",
                 "the", "of"}
        if len(words) >= 3:
            for i in range(len(words) - 2):
                if words[i + 1] in ("is", "are") and words[i] not in stops:
                    fact = f"{words[i]} is {' '.join(words[i + 2:])}"
                    self.facts[words[i]] = fact
                    self.associations.setdefault(words[i], []).append((fact, 1.0))
        self.synaptic_weights = (self.synaptic_weights * 0.999 + 0.001 * len(words)).clamp(-5.0, 5.0)

    def _record(self, user: str, reply: str) -> str:
        self.context_history.append((user, reply))
        if len(self.context_history) > 20:
            self.context_history.pop(0)
        return reply

    def is_greeting(self, lower: str, tokens: list[str]) -> bool:
        if lower.strip() in _GREETINGS:
            return True
        for t in tokens:
            if t in ("you", "your", "who", "how", "what"):
                continue
            for root in _GREETINGS:
                if (len(root) > 3 and (t == root or levenshtein(t, root) <= 1)) or (len(root) <= 3 and t == root):
                    return True
        return False

    def lookup_number(self, var: str):
        lower = var.lower()
        for k, v in self.facts.items():
            if k == lower or lower in k:
                n = _parse_num(v.strip())
                if n is not None:
                    return n
                for tok in v.split():
                    n = _parse_num(_strip_to_number(tok, allow_minus=True))
                    if n is not None:
                        return n
        return None

    def evaluate_math_expr(self, text: str):
        """"a op b" with symbols or number words ("plus", "divided by", ...), operands numbers or remembered
        variables; a symbolic description when an operand is unknown."""
        clean = text.lower()
        for prefix in ("what is", "calculate", "compute", "eval", "find", "solve"):
            if clean.startswith(prefix):
                clean = clean[len(prefix):]
        clean = f" {clean.replace('?', '').replace('=', '').strip()} "
        for w, sym in ((" plus ", " + "), (" minus ", " - "), (" times ", " * "), (" multiplied by ", " * "),
                       (" multiply ", " * "), (" divided by ", " / "), (" divide ", " / "), (" add ", " + "),
                       (" subtract ", " - ")):
            clean = clean.replace(w, sym)
        toks = "".join(f" {c} " if c in "+-*/" else c for c in clean).split()
        if len(toks) != 3 or toks[1] not in "+-*/" or len(toks[1]) != 1:
            return None
        sa, op, sb = toks
        na, nb = _parse_num(sa), _parse_num(sb)
        a = na if na is not None else self.lookup_number(sa)
        b = nb if nb is not None else self.lookup_number(sb)
        if a is None or b is None:
            desc = {"+": f"{sa} + {sb} represents the algebraic sum of {sa} and {sb}.",
                    "-": f"{sa} - {sb} represents the algebraic difference obtained by subtracting {sb} from {sa}.",
                    "*": f"{sa} * {sb} represents the algebraic product of {sa} and {sb}.",
                    "/": f"{sa} / {sb} represents the algebraic quotient of {sa} divided by {sb}."}
            return desc[op]
        if op == "/" and b == 0.0:
            return "Division by zero is undefined in standard mathematics."
        r = {"+": a + b, "-": a - b, "*": a * b, "/": a / b if b else 0.0}[op]
        if na is not None and nb is not None:
            return f"{_num(a)} {op} {_num(b)} = {_num(r)}"
        return f"{sa} {op} {sb} = {_num(a)} {op} {_num(b)} = {_num(r)}"

    def evaluate_word_problem(self, text: str):
        """Percentages ("20% of 150") and speed x time = distance (km/h or mph with hours, minutes or
        seconds, tolerating misspellings such as "haurs")."""
        lower = text.lower()
        if "%" in lower or "percent" in lower:
            toks = lower.replace("%", " percent ").replace("what is", "").replace("calculate", "").replace("?", "").split()
            for i, t in enumerate(toks):
                if t == "percent" and i > 0:
                    pct = _parse_num(_strip_to_number(toks[i - 1]))
                    if pct is not None:
                        for t2 in toks[i + 1:]:
                            base = _parse_num(_strip_to_number(t2))
                            if base is not None:
                                ans = pct / 100.0 * base
                                s = str(int(ans)) if ans == int(ans) else f"{ans:.2f}"
                                return f"{_num(pct)}% of {_num(base)} = {s}"
        speed_ind = any(k in lower for k in ("km/h", "kmh", "kmph", "mph", "m/s", "km per hour", "miles per hour",
                                             "speed", "drive", "travel"))
        time_ind = any(k in lower for k in ("hour", "haur", "houre", "hr", "minute", "min", "second", "sec"))
        if not (speed_ind and time_ind):
            return None
        speed = time = hours = None
        speed_unit, dist_unit = "km/h", "km"
        toks = lower.replace("?", " ").replace(",", " ").replace("!", " ").split()

        def number_here_or_before(idx):
            v = _parse_num(_strip_to_number(toks[idx]))
            if v is None and idx > 0:
                v = _parse_num(_strip_to_number(toks[idx - 1]))
            return v
        for idx, tok in enumerate(toks):
            if "km/h" in tok or "kmh" in tok or "kmph" in tok:
                v = number_here_or_before(idx)
                if v is not None:
                    speed, speed_unit, dist_unit = v, "km/h", "km"
            elif "mph" in tok:
                v = number_here_or_before(idx)
                if v is not None:
                    speed, speed_unit, dist_unit = v, "mph", "miles"
            if any(k in tok for k in ("hour", "haur", "houre", "min", "sec")) or tok in ("hrs", "hr"):
                v = number_here_or_before(idx)
                if v is not None:
                    time = v
                    hours = v / 60.0 if "min" in tok else v / 3600.0 if "sec" in tok else v
        if speed is None or time is None:
            return None
        dist = speed * hours
        ds = str(int(dist)) if dist == int(dist) else f"{dist:.2f}"
        ts = str(int(time)) if time == int(time) else _num(time)
        return f"At {_num(speed)} {speed_unit}, in {ts} hours, the distance traveled is {ds} {dist_unit}."

    def question_subject(self, lower: str):
        rest = lower.strip()
        for trig in _TRIGGERS:
            if rest.startswith(trig):
                rest = rest[len(trig):]
                break
        else:
            return None
        for tok in rest.split():
            clean = _alnum_strip(tok)
            if len(clean) >= 2 and clean not in _SUBJECT_STOPS:
                return clean
        return None

    def search_knowledge_facts(self, lower: str):
        subject = self.question_subject(lower)
        if subject is None:
            return None
        for key in (f"{subject}_definition", f"{subject}_formula", subject):
            if self.facts.get(key):
                return f"{subject}: {self.facts[key]}"
        best = None
        for key, ans in self.facts.items():
            if len(key) >= 3 and key not in _SUBJECT_STOPS:
                d = levenshtein(subject, key)
                if (d <= 1 or (len(subject) >= 4 and key.startswith(subject))) and (best is None or d < best[2]):
                    best = (key, ans, d)
        if best is not None:
            key, ans, _ = best
            if f"{key}_definition" in self.facts:
                return f"{key}: {self.facts[key + '_definition']}"
            return f"{key}: {ans}"
        return None

    def synthesize_thought(self, tokens: list[str]):
        """Spreading activation over the bigram graph: the strongest successor and its own successor."""
        for t in tokens:
            if t not in _SUBJECT_STOPS and len(t) >= 3 and self.transitions.get(t):
                nxt = max(self.transitions[t].items(), key=lambda kv: kv[1])[0]
                third = self.transitions.get(nxt)
                if third:
                    return f"When I think of {t}, it connects to {nxt} and {max(third.items(), key=lambda kv: kv[1])[0]}."
                return f"I associate {t} with {nxt}."
        return None

    def talk(self, message: str, max_new: int = 24, neural_train: bool = True) -> str:
        """One conversational turn: learn from the message, then answer with the first rule that applies."""
        trimmed = message.strip()
        if not trimmed:
            return "... (listening)"
        self.age_steps += 1
        self.learn_sentence(trimmed)
        if neural_train and len(trimmed.encode("utf-8")) >= 2:
            self.train_text(trimmed, steps=1, lr=0.01, window=min(64, len(trimmed.encode("utf-8")) - 1),
                            extract_facts=False)
        lower = trimmed.lower()
        tokens = [w for w in (_alnum_strip(t) for t in lower.split()) if w]
        is_question = lower.endswith("?") or lower.startswith(_QUESTION_STARTS)
        for rule in (self.evaluate_math_expr, self.evaluate_word_problem):
            r = rule(lower)
            if r is not None:
                return self._record(trimmed, r)
        if self.is_greeting(lower, tokens):
            r = (f"Hello {self.user_nickname}! Great to talk with you. What would you like to explore or teach me today?"
                 if self.user_nickname else "Hello! I am thinking and listening. How are you doing today?")
            return self._record(trimmed, r)
        if any(k in lower for k in ("how are you", "how r u", "whats up", "what's up")):
            c = self.cube_dim
            return self._record(trimmed, f"I am feeling active! My 3D neural cube ({c}x{c}x{c}) has "
                                         f"{self.total_synapses()} active synapses, and my mind has learned "
                                         f"{len(self.vocab)} words. How can I help you?")
        for prefix in ("my name is ", "call me "):
            if lower.startswith(prefix):
                name = trimmed[len(prefix):].strip().strip(".")
                self.user_nickname = name
                self.facts["user_name"] = name
                return self._record(trimmed, f"Nice to meet you, {name}! I will remember your name in my memory.")
        if lower.startswith("i am ") and "learning" not in lower and "thinking" not in lower:
            name = trimmed[5:].strip().strip(".")
            if name and len(name.split()) <= 2:
                self.user_nickname = name
                self.facts["user_name"] = name
                return self._record(trimmed, f"Hello, {name}! I've stored your identity in my neural network.")
        if any(k in lower for k in ("who am i", "what is my name", "do you know me")):
            r = (f"You are {self.user_nickname}! My teacher and companion." if self.user_nickname
                 else "You haven't told me your name yet. What is your name?")
            return self._record(trimmed, r)
        if any(k in lower for k in ("who are you", "what are you", "tell me about yourself")):
            c = self.cube_dim
            return self._record(trimmed, f"I am {self.name}, an associative biological deep-learning brain mind. "
                                         f"I live in a {c}x{c}x{c} 3D cubic space ({self.total_neurons()} neurons), "
                                         f"currently holding {len(self.vocab)} vocabulary words and "
                                         f"{self.total_synapses()} synaptic memories.")
        if not is_question and self.age_steps <= 2 and not self.facts:
            return self._record(trimmed, f"{trimmed}... {trimmed}")
        r = self.search_knowledge_facts(lower)
        if r is not None:
            return self._record(trimmed, r)
        if not is_question:
            for t in tokens:
                if t not in _STATEMENT_STOPS and len(t) >= 3 and self.associations.get(t):
                    return self._record(trimmed, max(self.associations[t], key=lambda kv: kv[1])[0])
            r = self.synthesize_thought(tokens)
            if r is not None:
                return self._record(trimmed, r)
            kw = tokens[0] if tokens else None
            r = (f"I am thinking about '{kw}'. Could you explain more about how it connects with what we're learning?"
                 if kw else f"I registered '{trimmed}' into my 3D neural memory. Teach me more!")
            return self._record(trimmed, r)
        if len(self.vocab) >= 64:
            gen = self.generate(trimmed, max_new).strip().strip(".!?")
            if len(trimmed) < len(gen) < 120:
                return self._record(trimmed, gen)
        tail = {"why", "how", "what", "where", "when", "which", "and", "or", "the", "a", "an", "is", "are", "to", "of",
                "it", "you", "me"}
        kw = next((t for t in reversed(tokens) if t not in tail), tokens[0] if tokens else "that")
        return self._record(trimmed, f"I don't know about '{kw}' yet. Could you explain it to me so I can learn it?")

    def teach_text(self, content: str, neural_every: int = 50) -> TeachSummary:
        """Index structured knowledge (records of TYPE:, NAME:, DEFINITION:, FORMULA: / STATEMENT: and
        unindented KEY: VALUE lines, closed by END) and learn every line as a sentence."""
        summary = TeachSummary()
        vocab0 = len(self.vocab)
        ctype = cname = ""
        for line in content.splitlines():
            t = line.strip()
            if not t or t.startswith("#"):
                continue
            summary.lines_processed += 1
            if t == "END":
                ctype = cname = ""
                continue
            if t.startswith("TYPE: "):
                ctype = t[6:].strip().lower()
                continue
            if t.startswith("NAME: "):
                cname = t[6:].strip().lower()
                self.facts[cname] = f"an entity of type {ctype}"
                summary.facts_indexed += 1
                continue
            if t.startswith("DEFINITION: "):
                if cname:
                    d = t[12:].strip()
                    self.facts[cname] = d
                    self.facts[f"{cname}_definition"] = d
                    summary.facts_indexed += 1
                continue
            if t.startswith("FORMULA: ") or t.startswith("STATEMENT: "):
                if cname:
                    stmt = (t[9:] if t.startswith("FORMULA: ") else t[11:]).strip()
                    self.facts[cname] = stmt
                    self.facts[f"{cname}_formula"] = stmt
                    summary.facts_indexed += 1
                continue
            if ctype and not line.startswith((" ", "\t")) and ":" in t and not t.startswith("http"):
                k, v = (x.strip() for x in t.split(":", 1))
                k = k.lower()
                if k and v:
                    self.facts[f"{ctype}_{k}"] = v
                    if k not in ("id", "type", "examples"):
                        self.facts[k] = v
                    summary.facts_indexed += 1
            self.learn_sentence(t)
            if summary.lines_processed % neural_every == 0 and len(t.encode("utf-8")) >= 2:
                losses = self.train_text(t, steps=1, lr=0.01, window=min(64, len(t.encode("utf-8")) - 1),
                                         extract_facts=False)
                summary.neural_loss = losses[-1] if losses else 0.0
        summary.words_learned = len(self.vocab) - vocab0
        summary.synapses_upgraded = self.total_synapses()
        return summary

    def prune_memory(self, min_strength: float) -> int:
        removed = 0
        for m in self.transitions.values():
            weak = [k for k, v in m.items() if v < min_strength]
            for k in weak:
                del m[k]
            removed += len(weak)
        for key, lst in self.associations.items():
            keep = [x for x in lst if x[1] >= min_strength]
            removed += len(lst) - len(keep)
            self.associations[key] = keep
        return removed

    def save(self, path: str) -> None:
        f = BrainModelFile("brain_mind").with_meta("arch", "brain_mind_v1")
        for k, v in self.facts.items():
            f.with_meta(f"fact:{k}", v)
        f.with_meta("memory", json.dumps({"vocab": self.inv_vocab, "transitions": self.transitions,
                                          "associations": self.associations, "name": self.name,
                                          "cube_dim": self.cube_dim, "user": self.user_nickname,
                                          "age": self.age_steps}, sort_keys=True))
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
        if "memory" in f.metadata:
            m = json.loads(f.metadata["memory"])
            bm.inv_vocab = list(m["vocab"])
            bm.vocab = {w: i for i, w in enumerate(bm.inv_vocab)}
            bm.transitions = {k: dict(v) for k, v in m["transitions"].items()}
            bm.associations = {k: [tuple(x) for x in v] for k, v in m["associations"].items()}
            bm.name, bm.cube_dim, bm.user_nickname, bm.age_steps = m["name"], m["cube_dim"], m["user"], m["age"]
            bm.synaptic_weights = torch.zeros(bm.cube_dim, bm.cube_dim, dtype=torch.float64)
        return bm
