"""Text analysis, n-gram operators, transforms, batch preparation, evaluation scores, vocabulary
optimisation and pretrained word-vector tables.

Reference: crates/brain-text/src/analyze.rs (TextStats, syllables, Flesch / Flesch-Kincaid / Gunning
fog / Coleman-Liau / ARI, hapax ratio, Yule's K, entropies), text_ops.rs (n-grams, character n-grams,
shingles, skip-grams, PMI collocations, term frequencies, character entropy), transform.rs (CaseKind,
case_transform, transliterate_ascii, normalize_punctuation, censor_words, TextPipeline), process.rs
(sentence / paragraph splitting, clean_text, pad_and_collate, truncation, length filter, batching),
compute.rs (chrF, character error rate, bits per character, exact match, token F1), optimize.rs
(prune_vocab, VocabTrie, quantize_embeddings_simple), embedding/pretrained.rs (GloVe / word2vec text
loading, most_similar, analogy).

The word-vector table keeps one [V, D] tensor on its device with precomputed inverse norms, so
``most_similar`` and ``analogy`` are one matrix-vector product and a top-k over the vocabulary
instead of a loop over words.
"""
from __future__ import annotations

import math
import re
import unicodedata
from collections import Counter
from dataclasses import dataclass

import torch


# ------------------------------------------------------------------------------------------ analysis
_SENT_END = set(".!?。！？")


def split_into_sentences(text: str) -> list[str]:
    """Cut after every . ! ? (and their full-width forms); pieces are stripped, empty ones dropped."""
    out, cur = [], []
    for c in text:
        cur.append(c)
        if c in _SENT_END:
            s = "".join(cur).strip()
            if s:
                out.append(s)
            cur = []
    s = "".join(cur).strip()
    if s:
        out.append(s)
    return out


def split_into_paragraphs(text: str) -> list[str]:
    return [p.strip() for p in text.split("\n\n") if p.strip()]


@dataclass
class TextStats:
    char_count: int = 0
    letter_count: int = 0
    digit_count: int = 0
    space_count: int = 0
    punctuation_count: int = 0
    word_count: int = 0
    sentence_count: int = 0
    avg_word_length: float = 0.0
    avg_sentence_length: float = 0.0
    type_token_ratio: float = 0.0


def _is_ascii_punct(c: str) -> bool:
    return c.isascii() and not c.isalnum() and not c.isspace() and c.isprintable()


def analyze_text(text: str) -> TextStats:
    """Character classes, whitespace-separated words (lengths and types counted on their alphanumeric
    characters, types case-folded) and sentences (at least 1)."""
    st = TextStats(char_count=len(text))
    for c in text:
        if c.isalpha():
            st.letter_count += 1
        elif c.isascii() and c.isdigit():
            st.digit_count += 1
        elif c.isspace():
            st.space_count += 1
        elif _is_ascii_punct(c):
            st.punctuation_count += 1
    words = text.split()
    st.word_count = len(words)
    types, total = set(), 0
    for w in words:
        cl = "".join(ch for ch in w if ch.isalnum())
        if cl:
            total += len(cl)
            types.add(cl.lower())
    st.sentence_count = max(len(split_into_sentences(text)), 1)
    if st.word_count:
        st.avg_word_length = total / st.word_count
        st.type_token_ratio = len(types) / st.word_count
    st.avg_sentence_length = st.word_count / st.sentence_count
    return st


def count_syllables(word: str) -> int:
    """Vowel groups (a e i o u y) in the letters of the word, minus a final silent e, at least 1 (0 for
    a word without letters)."""
    ch = [c for c in word.lower() if c.isalpha()]
    if not ch:
        return 0
    n, prev = 0, False
    for c in ch:
        v = c in "aeiouy"
        if v and not prev:
            n += 1
        prev = v
    if len(ch) > 2 and ch[-1] == "e" and n > 1:
        n -= 1
    return max(n, 1)


def _wss(text):
    st = analyze_text(text)
    syl = [count_syllables(w) for w in text.split()]
    return st, syl


def flesch_reading_ease(text: str) -> float:
    st, syl = _wss(text)
    if not st.word_count:
        return 100.0
    return 206.835 - 1.015 * st.word_count / st.sentence_count - 84.6 * sum(syl) / st.word_count


def flesch_kincaid_grade(text: str) -> float:
    st, syl = _wss(text)
    if not st.word_count:
        return 0.0
    return max(0.39 * st.word_count / st.sentence_count + 11.8 * sum(syl) / st.word_count - 15.59, 0.0)


def gunning_fog_index(text: str) -> float:
    st, syl = _wss(text)
    if not st.word_count:
        return 0.0
    return 0.4 * (st.word_count / st.sentence_count + 100.0 * sum(s >= 3 for s in syl) / st.word_count)


def coleman_liau_index(text: str) -> float:
    st = analyze_text(text)
    if not st.word_count:
        return 0.0
    return 0.0588 * st.letter_count / st.word_count * 100 - 0.296 * st.sentence_count / st.word_count * 100 - 15.8


def automated_readability_index(text: str) -> float:
    st = analyze_text(text)
    if not st.word_count:
        return 0.0
    return max(4.71 * st.letter_count / st.word_count + 0.5 * st.word_count / st.sentence_count - 21.43, 0.0)


def hapax_legomena_ratio(words) -> float:
    if not words:
        return 0.0
    return sum(1 for c in Counter(words).values() if c == 1) / len(words)


def yules_k_characteristic(words) -> float:
    """10^4 (sum_i i^2 V_i - N) / N^2 with V_i the number of types seen i times."""
    if not words:
        return 0.0
    n = len(words)
    spectrum = Counter(Counter(words).values())
    return 1e4 * (sum(i * i * v for i, v in spectrum.items()) - n) / (n * n)


def _entropy(counts) -> float:
    tot = sum(counts)
    return -sum((c / tot) * math.log2(c / tot) for c in counts if c) if tot else 0.0


def text_entropy(text: str) -> float:
    """Shannon entropy (bits) of the character distribution."""
    return _entropy(Counter(text).values())


shannon_entropy_chars = text_entropy


def shannon_entropy_words(words) -> float:
    return _entropy(Counter(words).values())


# ------------------------------------------------------------------------------------------ n-grams
def ngrams(tokens, n: int) -> list[list]:
    if n == 0 or len(tokens) < n:
        return []
    return [list(tokens[i:i + n]) for i in range(len(tokens) - n + 1)]


def character_ngrams(text: str, n: int) -> list[str]:
    if n == 0 or len(text) < n:
        return []
    return [text[i:i + n] for i in range(len(text) - n + 1)]


def shingles(text: str, k: int) -> set:
    return set(character_ngrams(text, k))


def word_counts(tokens) -> dict:
    return dict(Counter(tokens))


def ngram_freq(tokens, n: int) -> dict:
    return dict(Counter(tuple(g) for g in ngrams(tokens, n)))


def skipgrams(tokens, n: int, k: int) -> list[list]:
    """n = 1: every token; n = 2: pairs (i, j) with 1 <= j - i <= k + 1; larger n: plain n-grams."""
    if n == 0 or not tokens:
        return []
    if n == 1:
        return [[t] for t in tokens]
    if n == 2:
        return [[tokens[i], tokens[j]] for i in range(len(tokens)) for j in range(i + 1, min(i + k + 2, len(tokens)))]
    return ngrams(tokens, n)


def collocations(tokens, min_count: int = 2, min_pmi: float = 0.0) -> list[tuple]:
    """Adjacent pairs by pointwise mutual information ln(p(w1 w2) / (p(w1) p(w2))), with p(w) over
    tokens and p(w1 w2) over the n - 1 bigrams; sorted by PMI, highest first."""
    if len(tokens) < 2:
        return []
    uni = Counter(tokens)
    bi = Counter(zip(tokens[:-1], tokens[1:]))
    nt, nb = len(tokens), len(tokens) - 1
    out = []
    for (a, b), c in bi.items():
        if c >= min_count:
            pmi = math.log((c / nb) / ((uni[a] / nt) * (uni[b] / nt)))
            if pmi >= min_pmi:
                out.append((a, b, pmi))
    return sorted(out, key=lambda t: -t[2])


def term_frequencies(tokens) -> dict:
    """Relative frequency of each token."""
    n = len(tokens)
    return {t: c / n for t, c in Counter(tokens).items()} if n else {}


# ------------------------------------------------------------------------------------------ transforms
class CaseKind:
    LOWER, UPPER, TITLE, CAMEL, SNAKE, KEBAB = "lower", "upper", "title", "camel", "snake", "kebab"


def _words_for_case(text):
    return [w for w in re.split(r"[\s_\-]+", text) if w]


def case_transform(text: str, kind: str) -> str:
    if kind == CaseKind.LOWER:
        return text.lower()
    if kind == CaseKind.UPPER:
        return text.upper()
    if kind == CaseKind.TITLE:
        return " ".join(w[:1].upper() + w[1:].lower() for w in text.split())
    ws = _words_for_case(text)
    if kind == CaseKind.CAMEL:
        return "".join(w.lower() if i == 0 else w[:1].upper() + w[1:].lower() for i, w in enumerate(ws))
    return ("_" if kind == CaseKind.SNAKE else "-").join(w.lower() for w in ws)


_TRANSLIT = {"ß": "ss", "æ": "ae", "Æ": "AE", "œ": "oe", "Œ": "OE", "ø": "o", "Ø": "O", "©": "(c)", "®": "(r)",
             "™": "TM", "«": '"', "»": '"', "“": '"', "”": '"', "‘": "'", "’": "'", "—": "-", "–": "-", "…": "..."}


def transliterate_ascii(text: str) -> str:
    """Ligatures and typographic symbols by table, then accents stripped (NFD, combining marks dropped)."""
    out = []
    for c in text:
        if c in _TRANSLIT:
            out.append(_TRANSLIT[c])
        else:
            out.append("".join(ch for ch in unicodedata.normalize("NFD", c) if not unicodedata.combining(ch)))
    return "".join(out)


def normalize_punctuation(text: str) -> str:
    """Typographic quotes, dashes and ellipses to ASCII; runs of spaces before punctuation removed."""
    t = "".join(_TRANSLIT.get(c, c) if c in "«»“”‘’—–…" else c for c in text)
    return re.sub(r"\s+([.,;:!?])", r"\1", t)


def replace_patterns(text: str, patterns) -> str:
    for pat, rep in patterns:
        text = re.sub(pat, rep, text)
    return text


def censor_words(text: str, banned, replacement: str = "***") -> str:
    """Whitespace words whose letters (case-folded) are banned become the replacement."""
    banned = {b.lower() for b in banned}
    return " ".join(replacement if "".join(c for c in w if c.isalpha()).lower() in banned else w for w in text.split())


class TextPipeline:
    """An ordered list of str -> str steps."""

    def __init__(self):
        self.steps = []

    def add_step(self, fn) -> "TextPipeline":
        self.steps.append(fn)
        return self

    def run(self, text: str) -> str:
        for f in self.steps:
            text = f(text)
        return text


# ------------------------------------------------------------------------------------------ batch preparation
def clean_text(text: str, remove_html: bool = True, normalize_spaces: bool = True, strip_control: bool = True) -> str:
    """Drop <...> spans, control characters other than newline and tab, and collapse whitespace."""
    if remove_html:
        out, inside = [], False
        for c in text:
            if c == "<":
                inside = True
            elif c == ">":
                inside = False
            elif not inside:
                out.append(c)
        text = "".join(out)
    if strip_control:
        text = "".join(c for c in text if c in "\n\t" or unicodedata.category(c) != "Cc")
    if normalize_spaces:
        text = " ".join(text.split())
    return text


def pad_and_collate(sequences, pad_id: int = 0, max_len: int | None = None, device=None):
    """Token-id lists -> (ids [B, T] int64, attention mask [B, T] bool), right-padded (and truncated to max_len)."""
    T = max((len(s) for s in sequences), default=0)
    if max_len is not None:
        T = min(T, max_len)
    ids = torch.full((len(sequences), T), pad_id, dtype=torch.long)
    mask = torch.zeros(len(sequences), T, dtype=torch.bool)
    for i, s in enumerate(sequences):
        s = list(s)[:T]
        ids[i, :len(s)] = torch.tensor(s, dtype=torch.long)
        mask[i, :len(s)] = True
    return ids.to(device), mask.to(device)


def truncate_batch(sequences, max_len: int):
    return [list(s)[:max_len] for s in sequences]


def filter_by_length(texts, min_words: int = 1, max_words: int | None = None):
    return [t for t in texts if len(t.split()) >= min_words and (max_words is None or len(t.split()) <= max_words)]


def batch_iterator(items, batch_size: int):
    for i in range(0, len(items), batch_size):
        yield items[i:i + batch_size]


# ------------------------------------------------------------------------------------------ scores
def _lev(a, b) -> int:
    prev = list(range(len(b) + 1))
    for i, ca in enumerate(a, 1):
        cur = [i]
        for j, cb in enumerate(b, 1):
            cur.append(min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (ca != cb)))
        prev = cur
    return prev[-1]


def chrf_score(reference: str, candidate: str, n: int = 6, beta: float = 2.0) -> float:
    """F-beta of the character n-gram sets (1 when both are empty, 0 when one is)."""
    r, c = shingles(reference, n), shingles(candidate, n)
    if not r and not c:
        return 1.0
    if not r or not c:
        return 0.0
    inter = len(r & c)
    p, rc = inter / len(c), inter / len(r)
    b2 = beta * beta
    return 0.0 if p + rc == 0 else (1 + b2) * p * rc / (b2 * p + rc)


def character_error_rate(reference: str, hypothesis: str) -> float:
    if not reference:
        return 0.0 if not hypothesis else 1.0
    return _lev(reference, hypothesis) / len(reference)


def bits_per_character(cross_entropy_nats: float) -> float:
    return cross_entropy_nats / math.log(2.0)


def exact_match_score(reference: str, candidate: str) -> float:
    return 1.0 if reference.strip() == candidate.strip() else 0.0


def f1_token_score(reference, candidate) -> float:
    """Unigram-overlap F1 (clipped counts)."""
    if not reference or not candidate:
        return 0.0
    common = sum((Counter(reference) & Counter(candidate)).values())
    if common == 0:
        return 0.0
    p, r = common / len(candidate), common / len(reference)
    return 2 * p * r / (p + r)


# ------------------------------------------------------------------------------------------ vocabulary optimisation
def prune_vocab(counts: dict, min_freq: int = 1, max_size: int | None = None, keep=()) -> list[str]:
    """Tokens with count >= min_freq, most frequent first (ties alphabetical), capped at max_size; tokens in
    ``keep`` are always kept, first."""
    ks = [k for k in keep]
    rest = sorted((t for t, c in counts.items() if c >= min_freq and t not in set(ks)), key=lambda t: (-counts[t], t))
    out = ks + rest
    return out[:max_size] if max_size is not None else out


class VocabTrie:
    """Character trie over a vocabulary: membership and longest-prefix match (used by greedy subword
    segmentation)."""

    def __init__(self):
        self.root: dict = {}

    @classmethod
    def from_vocab(cls, words) -> "VocabTrie":
        t = cls()
        for w in words:
            t.insert(w)
        return t

    def insert(self, word: str) -> None:
        node = self.root
        for c in word:
            node = node.setdefault(c, {})
        node["$"] = True

    def contains(self, word: str) -> bool:
        node = self.root
        for c in word:
            if c not in node:
                return False
            node = node[c]
        return "$" in node

    def longest_prefix_match(self, text: str, start: int = 0) -> int:
        """Length of the longest vocabulary word that starts at ``start`` (0 if none)."""
        node, best = self.root, 0
        for i in range(start, len(text)):
            node = node.get(text[i])
            if node is None:
                break
            if "$" in node:
                best = i - start + 1
        return best


def quantize_embeddings_simple(table: torch.Tensor):
    """Symmetric per-row int8: scale = max|row| / 127; returns (int8 [V, D], scales [V])."""
    s = table.abs().amax(1).clamp_min(1e-12) / 127.0
    return torch.round(table / s[:, None]).clamp(-127, 127).to(torch.int8), s


# ------------------------------------------------------------------------------------------ pretrained vectors
class PretrainedEmbedding:
    """A word -> vector table ([V, D] on a device). Unknown words get zeros (``unk='zero'``), a seeded
    random vector (``'random'``) or the mean vector (``'mean'``)."""

    def __init__(self, words, vectors: torch.Tensor, unk: str = "zero", seed: int = 0):
        self.words = list(words)
        self.index = {w: i for i, w in enumerate(self.words)}
        self.vectors = vectors
        self.inv_norm = 1.0 / vectors.float().norm(dim=1).clamp_min(1e-12)
        self.unk, self.seed = unk, seed

    @classmethod
    def load_glove_str(cls, text: str, device=None, **kw) -> "PretrainedEmbedding":
        """Lines "word v1 v2 ..."; blank lines skipped; all rows must have one width."""
        words, rows = [], []
        for line in text.splitlines():
            parts = line.strip().split()
            if len(parts) < 2:
                continue
            words.append(parts[0])
            rows.append([float(v) for v in parts[1:]])
        if len({len(r) for r in rows}) > 1:
            raise ValueError("inconsistent vector widths")
        return cls(words, torch.tensor(rows, dtype=torch.float32, device=device), **kw)

    @classmethod
    def load_word2vec_text_str(cls, text: str, device=None, **kw) -> "PretrainedEmbedding":
        """word2vec text format: a "count dim" header line, then GloVe-style rows."""
        lines = text.splitlines()
        hdr = lines[0].split() if lines else []
        body = "\n".join(lines[1:]) if len(hdr) == 2 and all(h.isdigit() for h in hdr) else text
        return cls.load_glove_str(body, device, **kw)

    @property
    def dim(self) -> int:
        return self.vectors.shape[1]

    def get_vector(self, word: str) -> torch.Tensor:
        i = self.index.get(word)
        if i is not None:
            return self.vectors[i]
        if self.unk == "mean":
            return self.vectors.mean(0)
        if self.unk == "random":
            g = torch.Generator().manual_seed(self.seed + sum(map(ord, word)))
            return (torch.randn(self.dim, generator=g) * 0.1).to(self.vectors)
        return torch.zeros(self.dim, dtype=self.vectors.dtype, device=self.vectors.device)

    def _nearest(self, q: torch.Tensor, k: int, exclude=()) -> list[tuple[str, float]]:
        sims = (self.vectors.float() @ q.float()) * self.inv_norm / q.float().norm().clamp_min(1e-12)
        for w in exclude:
            if w in self.index:
                sims[self.index[w]] = -float("inf")
        top = torch.topk(sims, min(k, len(self.words)))
        return [(self.words[int(i)], float(v)) for v, i in zip(top.values, top.indices) if math.isfinite(float(v))]

    def most_similar(self, word: str, k: int = 10) -> list[tuple[str, float]]:
        """Cosine neighbours over the whole table in one matrix-vector product (the word itself excluded)."""
        return self._nearest(self.get_vector(word), k, exclude=(word,))

    def analogy(self, a: str, b: str, c: str, k: int = 1) -> list[tuple[str, float]]:
        """a : b :: c : ? by the nearest neighbours of b - a + c (the three inputs excluded)."""
        q = self.get_vector(b) - self.get_vector(a) + self.get_vector(c)
        return self._nearest(q, k, exclude=(a, b, c))

    def to_word_embedding(self, vocab) -> torch.Tensor:
        """Rows for an external vocabulary, unknowns filled by the unk rule."""
        return torch.stack([self.get_vector(w) for w in vocab])
