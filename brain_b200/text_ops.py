"""Token-sequence operations and data collators with the reference's names: padding / truncation /
packing, attention-mask, position and token-type ids, MLM masking (80 % [MASK], 10 % random, 10 %
kept), the language-modelling and seq2seq collators, T5 span corruption, EDA text augmentation,
edit distances (Levenshtein, Damerau), Jaccard and cosine similarity with a pairwise matrix, corpus
BLEU, GPT-2 byte-level symbol mapping and BERT character classes.

Reference: crates/brain-text/src/ops.rs:20-200 (pad_sequences returning a 0/1 mask, truncate_sequences,
create_attention_mask, mask_tokens, pack_sequences appending EOS and keeping the last partial chunk,
one_hot_encode), helper.rs:16-260 (DataCollatorForSeq2Seq with label padding, DataCollatorForLanguageModeling
with -100 labels on unmasked and padded positions, SpanCorruptionHelper, TextAugmenter), utils.rs
(levenshtein / damerau / jaccard / cosine, byte_encode / byte_decode, is_whitespace / is_control /
is_punctuation / is_chinese_char), compute.rs (bleu_score, corpus_bleu), similarity.rs.

The collators and ``mask_tokens`` work on a whole padded batch at once as tensors, so on a GPU the
masking draws and selects on the device instead of looping over tokens.
"""
from __future__ import annotations

import math
import random
import unicodedata
from collections import Counter

import torch

IGNORE_INDEX = -100


# ------------------------------------------------------------------ padding, truncation, packing, ids
def pad_sequences(sequences, pad_id: int = 0, max_len: int | None = None, side: str = "right", device=None):
    """(ids [B, L] int64, mask [B, L] uint8). Longer sequences are cut to max_len (from the right)."""
    L = max_len if max_len is not None else max((len(s) for s in sequences), default=0)
    ids = torch.full((len(sequences), L), pad_id, dtype=torch.long)
    mask = torch.zeros((len(sequences), L), dtype=torch.uint8)
    for i, s in enumerate(sequences):
        s = list(s)[:L]
        n = len(s)
        if side == "right":
            ids[i, :n] = torch.as_tensor(s, dtype=torch.long)
            mask[i, :n] = 1
        else:
            ids[i, L - n:] = torch.as_tensor(s, dtype=torch.long)
            mask[i, L - n:] = 1
    return ids.to(device), mask.to(device)


def truncate_sequences(sequences, max_len: int, side: str = "right"):
    return [list(s)[:max_len] if side == "right" else list(s)[max(0, len(s) - max_len):] for s in sequences]


def pack_sequences(sequences, max_length: int, eos_id: int):
    """Concatenate sequences, each followed by EOS, and cut into chunks of max_length (the last may be
    shorter)."""
    flat = [t for s in sequences for t in list(s) + [eos_id]]
    return [flat[i:i + max_length] for i in range(0, len(flat), max_length)]


def create_attention_mask(ids, pad_id: int = 0) -> torch.Tensor:
    ids = torch.as_tensor(ids)
    return (ids != pad_id).to(torch.uint8)


def create_position_ids(batch_size: int, seq_len: int, device=None) -> torch.Tensor:
    return torch.arange(seq_len, device=device).expand(batch_size, seq_len)


def create_token_type_ids(first_len: int, second_len: int, device=None) -> torch.Tensor:
    return torch.cat([torch.zeros(first_len, dtype=torch.long, device=device),
                      torch.ones(second_len, dtype=torch.long, device=device)])


def one_hot_encode(ids, vocab_size: int) -> torch.Tensor:
    """[N, V] float32; ids outside the vocabulary give a zero row."""
    ids = torch.as_tensor(ids, dtype=torch.long)
    ok = (ids >= 0) & (ids < vocab_size)
    out = torch.zeros(ids.numel(), vocab_size)
    out[torch.arange(ids.numel())[ok], ids[ok]] = 1.0
    return out


def tokens_to_ids(tokens, vocab: dict, unk_id: int = 0) -> list[int]:
    return [vocab.get(t, unk_id) for t in tokens]


def ids_to_tokens(ids, inv_vocab, unk: str = "[UNK]") -> list[str]:
    get = inv_vocab.get if isinstance(inv_vocab, dict) else (lambda i, d: inv_vocab[i] if 0 <= i < len(inv_vocab) else d)
    return [get(int(i), unk) for i in ids]


def mask_tokens(ids: torch.Tensor, mask_prob: float, mask_id: int, vocab_size: int, generator=None,
                special_mask: torch.Tensor | None = None):
    """MLM corruption of a batch: each position is selected with probability mask_prob (never where
    ``special_mask`` is true); a selected token becomes mask_id with probability 0.8, a uniform random
    id with 0.1 and stays with 0.1. Returns (masked ids, selected bool mask)."""
    ids = torch.as_tensor(ids)
    dev = ids.device
    u = torch.rand(ids.shape, device=dev, generator=generator)
    sel = u < mask_prob
    if special_mask is not None:
        sel &= ~special_mask.to(dev, torch.bool)
    p = torch.rand(ids.shape, device=dev, generator=generator)
    rnd = torch.randint(0, vocab_size, ids.shape, device=dev, generator=generator)
    out = torch.where(sel & (p < 0.8), torch.full_like(ids, mask_id), ids)
    out = torch.where(sel & (p >= 0.8) & (p < 0.9), rnd, out)
    return out, sel


class DataCollatorForLanguageModeling:
    """Pads a list of sequences; with ``mlm`` masks them and sets labels to the original ids at the
    selected non-pad positions and -100 elsewhere; without ``mlm`` the labels are the inputs (causal
    LM, pads -100). Returns (input_ids, labels, attention_mask)."""

    def __init__(self, pad_token_id: int, mask_token_id: int, vocab_size: int, mlm: bool = True,
                 mlm_probability: float = 0.15, device=None):
        self.pad, self.mask_id, self.V, self.mlm, self.p, self.device = (pad_token_id, mask_token_id, vocab_size,
                                                                          mlm, mlm_probability, device)

    def collate(self, sequences, generator=None):
        ids, am = pad_sequences(sequences, self.pad, device=self.device)
        if not self.mlm:
            return ids, torch.where(am.bool(), ids, torch.full_like(ids, IGNORE_INDEX)), am
        masked, sel = mask_tokens(ids, self.p, self.mask_id, self.V, generator, special_mask=~am.bool())
        labels = torch.where(sel & (ids != self.pad), ids, torch.full_like(ids, IGNORE_INDEX))
        return masked, labels, am

    __call__ = collate


class DataCollatorForSeq2Seq:
    def __init__(self, pad_token_id: int = 0, label_pad_token_id: int = IGNORE_INDEX, max_length: int | None = None,
                 device=None):
        self.pad, self.label_pad, self.max_length, self.device = pad_token_id, label_pad_token_id, max_length, device

    def collate(self, inputs, labels):
        ids, am = pad_sequences(inputs, self.pad, self.max_length, device=self.device)
        L = self.max_length if self.max_length is not None else max((len(x) for x in labels), default=0)
        lab, _ = pad_sequences([list(x)[:L] for x in labels], self.label_pad, L, device=self.device)
        return ids, lab, am

    __call__ = collate


def corrupt_spans(tokens, noise_density: float = 0.15, mean_noise_span_length: float = 3.0,
                  sentinel_start_id: int = 32000, rng: random.Random | None = None, sentinel_step: int = 1):
    """T5 span corruption: round(len * density) noise tokens in round(noise / mean_span) spans placed at
    random; every span becomes one sentinel in the input, and the target lists each sentinel followed by
    the tokens it replaced. Sentinels count from sentinel_start_id by sentinel_step (T5 counts down from
    the top of the vocabulary: step -1)."""
    rng = rng or random.Random(0)
    n = len(tokens)
    n_noise = min(n - 1, max(1, round(n * noise_density))) if n > 1 else 0
    n_spans = max(1, min(n_noise, round(n_noise / max(mean_noise_span_length, 1.0)))) if n_noise else 0
    if not n_spans:
        return list(tokens), []

    def split(total, parts):  # random composition of total into parts positive lengths
        cuts = sorted(rng.sample(range(1, total), parts - 1)) if parts > 1 else []
        return [b - a for a, b in zip([0] + cuts, cuts + [total])]
    noise_lens = split(n_noise, n_spans)
    keep_lens = split(n - n_noise, n_spans) if n - n_noise >= n_spans else [n - n_noise] + [0] * (n_spans - 1)
    inp, tgt, pos = [], [], 0
    for s in range(n_spans):
        inp += tokens[pos:pos + keep_lens[s]]
        pos += keep_lens[s]
        sid = sentinel_start_id + s * sentinel_step
        inp.append(sid)
        tgt.append(sid)
        tgt += tokens[pos:pos + noise_lens[s]]
        pos += noise_lens[s]
    return inp, tgt


class SpanCorruptionHelper:
    corrupt_spans = staticmethod(corrupt_spans)


class TextAugmenter:
    """EDA-style word-level augmentation (Wei & Zou 2019)."""

    @staticmethod
    def random_deletion(words, prob: float, rng: random.Random | None = None):
        rng = rng or random.Random(0)
        kept = [w for w in words if rng.random() >= prob]
        return kept if kept or not words else [words[rng.randrange(len(words))]]

    @staticmethod
    def random_swap(words, prob: float, rng: random.Random | None = None):
        rng = rng or random.Random(0)
        w = list(words)
        for i in range(len(w)):
            if len(w) > 1 and rng.random() < prob:
                j = rng.randrange(len(w))
                w[i], w[j] = w[j], w[i]
        return w

    @staticmethod
    def random_insertion(words, prob: float, rng: random.Random | None = None):
        rng = rng or random.Random(0)
        w = list(words)
        for x in list(words):
            if rng.random() < prob:
                w.insert(rng.randrange(len(w) + 1), x)
        return w

    @staticmethod
    def char_perturbation(text: str, prob: float, rng: random.Random | None = None,
                          alphabet: str = "abcdefghijklmnopqrstuvwxyz") -> str:
        rng = rng or random.Random(0)
        return "".join(rng.choice(alphabet) if c.isalpha() and rng.random() < prob else c for c in text)


random_deletion = TextAugmenter.random_deletion
random_swap = TextAugmenter.random_swap
random_insertion = TextAugmenter.random_insertion
char_perturbation = TextAugmenter.char_perturbation


# ------------------------------------------------------------------ distances and similarity
def levenshtein_distance(a, b) -> int:
    prev = list(range(len(b) + 1))
    for i, ca in enumerate(a, 1):
        cur = [i] + [0] * len(b)
        for j, cb in enumerate(b, 1):
            cur[j] = min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (ca != cb))
        prev = cur
    return prev[-1]


def damerau_levenshtein_distance(a, b) -> int:
    """Optimal-string-alignment distance: insertions, deletions, substitutions and adjacent swaps."""
    n, m = len(a), len(b)
    d = [[0] * (m + 1) for _ in range(n + 1)]
    for i in range(n + 1):
        d[i][0] = i
    for j in range(m + 1):
        d[0][j] = j
    for i in range(1, n + 1):
        for j in range(1, m + 1):
            c = a[i - 1] != b[j - 1]
            d[i][j] = min(d[i - 1][j] + 1, d[i][j - 1] + 1, d[i - 1][j - 1] + c)
            if i > 1 and j > 1 and a[i - 1] == b[j - 2] and a[i - 2] == b[j - 1]:
                d[i][j] = min(d[i][j], d[i - 2][j - 2] + 1)
    return d[n][m]


def jaccard_similarity(a, b) -> float:
    sa, sb = set(a), set(b)
    return 1.0 if not sa and not sb else len(sa & sb) / len(sa | sb)


def cosine_similarity_slice(a, b) -> float:
    a, b = torch.as_tensor(a, dtype=torch.float64), torch.as_tensor(b, dtype=torch.float64)
    na, nb = a.norm(), b.norm()
    return 0.0 if na == 0 or nb == 0 else float(a @ b / (na * nb))


def pairwise_similarity_matrix(x: torch.Tensor, metric: str = "cosine") -> torch.Tensor:
    """[N, N] similarities of the rows of x (one matrix product on x's device): cosine, dot, or
    negative euclidean distance."""
    x = x.float()
    if metric == "cosine":
        xn = x / x.norm(dim=1, keepdim=True).clamp_min(1e-12)
        return xn @ xn.t()
    if metric == "dot":
        return x @ x.t()
    if metric == "euclidean":
        return -torch.cdist(x, x)
    raise ValueError(f"unknown similarity metric {metric!r}")


def _ngrams(tokens, n):
    return Counter(tuple(tokens[i:i + n]) for i in range(len(tokens) - n + 1))


def corpus_bleu(candidates, references_list, max_n: int = 4) -> float:
    """Papineni et al. 2002 over a corpus: clipped n-gram counts and lengths summed over all sentences,
    geometric mean of the n-gram precisions, brevity penalty against the closest reference length."""
    num = [0] * max_n
    den = [0] * max_n
    c_len = r_len = 0
    for cand, refs in zip(candidates, references_list):
        c_len += len(cand)
        r_len += min((abs(len(r) - len(cand)), len(r)) for r in refs)[1]
        for n in range(1, max_n + 1):
            cc = _ngrams(cand, n)
            mx = Counter()
            for r in refs:
                for g, k in _ngrams(r, n).items():
                    mx[g] = max(mx[g], k)
            num[n - 1] += sum(min(k, mx[g]) for g, k in cc.items())
            den[n - 1] += max(0, len(cand) - n + 1)
    if c_len == 0 or min(num) == 0:
        return 0.0
    logp = sum(math.log(num[i] / den[i]) for i in range(max_n)) / max_n
    bp = 1.0 if c_len > r_len else math.exp(1 - r_len / c_len)
    return bp * math.exp(logp)


def bleu_score(candidate, references, max_n: int = 4) -> float:
    return corpus_bleu([candidate], [references], max_n)


# ------------------------------------------------------------------ byte-level symbols, character classes
def _byte_table():
    printable = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + \
        list(range(ord("®"), ord("ÿ") + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in printable:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


_B2U = _byte_table()
_U2B = {v: k for k, v in _B2U.items()}


def byte_encode(text: str) -> str:
    """UTF-8 bytes of text as printable symbols (GPT-2's byte-level alphabet: printable Latin-1 bytes map
    to themselves, the other 68 to U+0100 onward)."""
    return "".join(_B2U[b] for b in text.encode("utf-8"))


def byte_decode(symbols: str) -> str:
    return bytes(_U2B[c] for c in symbols).decode("utf-8", errors="replace")


def is_whitespace(c: str) -> bool:
    return c in " \t\n\r" or unicodedata.category(c) == "Zs"


def is_control(c: str) -> bool:
    return c not in "\t\n\r" and unicodedata.category(c) in ("Cc", "Cf")


def is_punctuation(c: str) -> bool:
    cp = ord(c)
    if 33 <= cp <= 47 or 58 <= cp <= 64 or 91 <= cp <= 96 or 123 <= cp <= 126:
        return True
    return unicodedata.category(c).startswith("P")


def is_chinese_char(c: str) -> bool:
    cp = ord(c)
    return any(lo <= cp <= hi for lo, hi in ((0x4E00, 0x9FFF), (0x3400, 0x4DBF), (0x20000, 0x2A6DF),
                                             (0x2A700, 0x2B73F), (0x2B740, 0x2B81F), (0x2B820, 0x2CEAF),
                                             (0xF900, 0xFAFF), (0x2F800, 0x2FA1F)))


def split_ws(text: str) -> list[str]:
    return text.split()
