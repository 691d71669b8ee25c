"""Text tokenisation: vocabulary, normaliser, pre-tokeniser, char / word / BPE / WordPiece / unigram
(SentencePiece-style) / byte-level tokenisers, their trainers, and the post-processor that adds
special tokens, truncates and pads into id tensors for the models.

Reference: crates/brain-text/src. ``Tokenizer`` trait (tokenizer/mod.rs:28-60: encode, decode,
tokenize, vocab_size, id/token lookups), ``Vocab`` with special kinds (vocab.rs:19-190), BPE
segmentation by lowest merge rank (tokenizer/bpe.rs:62-135) and its trainer (tokenizer/trainer.rs:52-136,
``</w>`` end-of-word suffix), WordPiece greedy longest match with a ``##`` continuation prefix
(tokenizer/wordpiece.rs:53-100), unigram Viterbi segmentation over ``▁``-marked text
(tokenizer/sentencepiece.rs:62-140) and its trainer (trainer.rs:138-190), the GPT-2 style byte-to-
character map (tokenizer/bytelevel.rs:29-100), and the post-processor (tokenizer/post.rs:18-200).

These are host-side string algorithms (the data path hands the ids to the GPU as one tensor per
batch). The segmentation algorithms are the standard published ones (Sennrich et al. BPE; WordPiece
greedy longest match; Kudo's unigram model with Viterbi decoding). Unlike the reference's hash-map
iteration, every training tie is broken by a fixed order, so a trained vocabulary is deterministic.
"""
from __future__ import annotations

import collections
import enum
import json
import math
import re
import unicodedata
from dataclasses import dataclass, field

import torch


class SpecialKind(enum.Enum):
    PAD = "pad"
    UNK = "unk"
    BOS = "bos"
    EOS = "eos"
    MASK = "mask"
    SEP = "sep"
    CLS = "cls"
    CUSTOM = "custom"


class Vocab:
    """Token <-> id table with special tokens."""

    def __init__(self, tokens=None):
        self._ids: dict[str, int] = {}
        self._toks: list[str] = []
        self._special: dict[int, SpecialKind] = {}
        for t in tokens or []:
            self.insert(t)

    @classmethod
    def from_tokens(cls, tokens) -> "Vocab":
        return cls(tokens)

    def insert(self, token: str) -> int:
        if token not in self._ids:
            self._ids[token] = len(self._toks)
            self._toks.append(token)
        return self._ids[token]

    def add_special(self, token: str, kind: SpecialKind = SpecialKind.CUSTOM) -> int:
        i = self.insert(token)
        self._special[i] = kind
        return i

    def get_id(self, token: str):
        return self._ids.get(token)

    def get_token(self, i: int):
        return self._toks[i] if 0 <= i < len(self._toks) else None

    def __len__(self) -> int:
        return len(self._toks)

    def contains(self, token: str) -> bool:
        return token in self._ids

    __contains__ = contains

    def is_special(self, i: int) -> bool:
        return i in self._special

    def _kind(self, kind: SpecialKind):
        for i, k in self._special.items():
            if k == kind:
                return i
        return None

    def pad_id(self):
        return self._kind(SpecialKind.PAD)

    def unk_id(self):
        return self._kind(SpecialKind.UNK)

    def bos_id(self):
        return self._kind(SpecialKind.BOS)

    def eos_id(self):
        return self._kind(SpecialKind.EOS)

    def mask_id(self):
        return self._kind(SpecialKind.MASK)

    def sep_id(self):
        return self._kind(SpecialKind.SEP)

    def cls_id(self):
        return self._kind(SpecialKind.CLS)

    def export_json(self) -> str:
        return json.dumps({"tokens": self._toks, "special": {str(i): k.value for i, k in self._special.items()}})

    @classmethod
    def import_json(cls, s: str) -> "Vocab":
        d = json.loads(s)
        v = cls(d["tokens"])
        for i, k in d["special"].items():
            v._special[int(i)] = SpecialKind(k)
        return v


def default_vocab_specials(v: Vocab) -> Vocab:
    for tok, kind in (("[PAD]", SpecialKind.PAD), ("[UNK]", SpecialKind.UNK), ("[BOS]", SpecialKind.BOS),
                      ("[EOS]", SpecialKind.EOS), ("[CLS]", SpecialKind.CLS), ("[SEP]", SpecialKind.SEP),
                      ("[MASK]", SpecialKind.MASK)):
        v.add_special(tok, kind)
    return v


@dataclass
class TokenizedOutput:
    ids: list[int]
    tokens: list[str]
    attention_mask: list[int] = field(default_factory=list)
    type_ids: list[int] = field(default_factory=list)

    def __post_init__(self):
        if not self.attention_mask:
            self.attention_mask = [1] * len(self.ids)
        if not self.type_ids:
            self.type_ids = [0] * len(self.ids)


# ------------------------------------------------------------------ normaliser / pre-tokeniser
@dataclass
class NormalizerConfig:
    lowercase: bool = True
    strip_accents: bool = True
    collapse_whitespace: bool = True
    nfkc: bool = False


class Normalizer:
    def __init__(self, config: NormalizerConfig | None = None):
        self.config = config or NormalizerConfig()

    def normalize(self, text: str) -> str:
        c = self.config
        if c.nfkc:
            text = unicodedata.normalize("NFKC", text)
        if c.lowercase:
            text = text.lower()
        if c.strip_accents:
            text = "".join(ch for ch in unicodedata.normalize("NFD", text) if unicodedata.category(ch) != "Mn")
        if c.collapse_whitespace:
            text = " ".join(text.split())
        return text


_PRE = re.compile(r"\w+|[^\w\s]", re.UNICODE)


class PreTokenizer:
    """Splits on whitespace and isolates punctuation; returns (piece, (start, end)) with char offsets."""

    def __init__(self, split_punctuation: bool = True):
        self.split_punctuation = split_punctuation

    def pre_tokenize(self, text: str):
        if self.split_punctuation:
            return [(m.group(), (m.start(), m.end())) for m in _PRE.finditer(text)]
        return [(m.group(), (m.start(), m.end())) for m in re.finditer(r"\S+", text)]


# ------------------------------------------------------------------ tokenisers
class Tokenizer:
    """Common interface: encode / decode / tokenize / vocab lookups."""

    vocab: Vocab

    def tokenize(self, text: str) -> list[str]:
        raise NotImplementedError

    def encode(self, text: str) -> TokenizedOutput:
        toks = self.tokenize(text)
        unk = self.vocab.unk_id()
        ids = []
        for t in toks:
            i = self.vocab.get_id(t)
            if i is None:
                if unk is None:
                    raise KeyError(f"token {t!r} not in vocabulary and no [UNK] token")
                i = unk
            ids.append(i)
        return TokenizedOutput(ids, toks)

    def decode(self, ids) -> str:
        raise NotImplementedError

    def vocab_size(self) -> int:
        return len(self.vocab)

    def get_vocab(self) -> Vocab:
        return self.vocab

    def id_to_token(self, i: int):
        return self.vocab.get_token(i)

    def token_to_id(self, t: str):
        return self.vocab.get_id(t)

    def pad_token_id(self):
        return self.vocab.pad_id()

    def unk_token_id(self):
        return self.vocab.unk_id()

    def _pieces(self, ids):
        return [self.vocab.get_token(int(i)) for i in ids if not self.vocab.is_special(int(i))]


class CharTokenizer(Tokenizer):
    def __init__(self, vocab: Vocab, lowercase: bool = False):
        self.vocab, self.lowercase = vocab, lowercase

    @classmethod
    def from_corpus(cls, corpus, lowercase: bool = False) -> "CharTokenizer":
        v = default_vocab_specials(Vocab())
        for ch in sorted({c for doc in corpus for c in (doc.lower() if lowercase else doc)}):
            v.insert(ch)
        return cls(v, lowercase)

    def tokenize(self, text):
        return list(text.lower() if self.lowercase else text)

    def decode(self, ids):
        return "".join(self._pieces(ids))


class WordTokenizer(Tokenizer):
    def __init__(self, vocab: Vocab, normalizer: Normalizer | None = None):
        self.vocab, self.normalizer, self.pre = vocab, normalizer or Normalizer(), PreTokenizer()

    @classmethod
    def from_corpus(cls, corpus, min_frequency: int = 1) -> "WordTokenizer":
        t = cls(default_vocab_specials(Vocab()))
        cnt = collections.Counter(w for doc in corpus for w, _ in t.pre.pre_tokenize(t.normalizer.normalize(doc)))
        for w in sorted(w for w, c in cnt.items() if c >= min_frequency):
            t.vocab.insert(w)
        return t

    def tokenize(self, text):
        return [w for w, _ in self.pre.pre_tokenize(self.normalizer.normalize(text))]

    def decode(self, ids):
        return " ".join(self._pieces(ids))


class BpeTokenizer(Tokenizer):
    """Words are split into characters (the last carrying ``end_of_word_suffix``); the adjacent pair with
    the lowest merge rank is merged until no ranked pair is left."""

    def __init__(self, vocab: Vocab, merges, end_of_word_suffix: str = "</w>", normalizer=None):
        self.vocab = vocab
        self.ranks = {tuple(p): r for p, r in merges}
        self.suffix = end_of_word_suffix
        self.normalizer = normalizer or Normalizer(NormalizerConfig(lowercase=False, strip_accents=False))
        self.pre = PreTokenizer(split_punctuation=False)
        self._cache: dict[str, list[str]] = {}

    @classmethod
    def from_vocab_and_merges(cls, vocab, merges, end_of_word_suffix="</w>"):
        return cls(vocab, merges, end_of_word_suffix)

    def bpe_segment_word(self, word: str) -> list[str]:
        if not word:
            return []
        hit = self._cache.get(word)
        if hit is not None:
            return list(hit)
        sym = list(word)
        if self.suffix:
            sym[-1] += self.suffix
        while len(sym) > 1:
            best, idx = None, -1
            for i in range(len(sym) - 1):
                r = self.ranks.get((sym[i], sym[i + 1]))
                if r is not None and (best is None or r < best):
                    best, idx = r, i
            if idx < 0:
                break
            sym[idx:idx + 2] = [sym[idx] + sym[idx + 1]]
        self._cache[word] = list(sym)
        return sym

    def tokenize(self, text):
        out = []
        for w, _ in self.pre.pre_tokenize(self.normalizer.normalize(text)):
            out += self.bpe_segment_word(w)
        return out

    def encode(self, text: str) -> TokenizedOutput:
        """With ``use_native()`` and whitespace-collapsing normalisation, the merge loop runs in C++."""
        nat = getattr(self, "_native", None)
        if nat is not None and self.normalizer.config.collapse_whitespace:
            ids = nat.encode(self.normalizer.normalize(text))
            return TokenizedOutput(ids, [self.vocab.get_token(i) for i in ids])
        return super().encode(text)

    def use_native(self) -> "BpeTokenizer":
        self._native = NativeBpe(self.vocab, [((a, b), r) for (a, b), r in self.ranks.items()], self.suffix)
        return self

    def decode(self, ids):
        s = "".join(self._pieces(ids))
        return s.replace(self.suffix, " ").strip() if self.suffix else s


class NativeBpe:
    """The BPE merge loop in C++ (``csrc/bpe.cpp``, in ``libbrain_runtime``): same segmentation as
    ``BpeTokenizer.bpe_segment_word`` on whitespace-separated words, with a per-word cache."""

    def __init__(self, vocab: Vocab, merges, suffix: str = "</w>"):
        import ctypes

        from . import _native

        lib = _native.load("brain_runtime")
        self._lib = lib
        lib.brain_bpe_create.restype = ctypes.c_void_p
        lib.brain_bpe_create.argtypes = [ctypes.c_char_p]
        lib.brain_bpe_add_token.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int]
        lib.brain_bpe_add_merges.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        lib.brain_bpe_encode.restype = ctypes.c_int64
        lib.brain_bpe_encode.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64, ctypes.c_void_p,
                                         ctypes.c_int64]
        lib.brain_bpe_destroy.argtypes = [ctypes.c_void_p]
        self._h = lib.brain_bpe_create(suffix.encode())
        unk = vocab.unk_id()
        for i, t in enumerate(vocab._toks):
            b = t.encode()
            lib.brain_bpe_add_token(self._h, b, len(b), i, int(i == unk))
        trip = []
        for (a, b), _ in sorted(merges, key=lambda m: m[1]):
            ia, ib, im = vocab.get_id(a), vocab.get_id(b), vocab.get_id(a + b)
            if None in (ia, ib, im):
                raise ValueError(f"merge ({a!r}, {b!r}) refers to tokens missing from the vocabulary")
            trip += [ia, ib, im]
        t = torch.tensor(trip, dtype=torch.int32)
        lib.brain_bpe_add_merges(self._h, t.data_ptr(), len(trip) // 3)

    def encode(self, text: str) -> list[int]:
        b = text.encode()
        cap = max(16, len(b) + 1)
        while True:
            out = torch.empty(cap, dtype=torch.int32)
            n = self._lib.brain_bpe_encode(self._h, b, len(b), out.data_ptr(), cap)
            if n < 0:
                raise RuntimeError(f"brain_bpe_encode failed ({n})")
            if n <= cap:
                return out[:n].tolist()
            cap = n

    def __del__(self):
        try:
            if self._h:
                self._lib.brain_bpe_destroy(self._h)
                self._h = None
        except Exception:
            pass


class BpeTrainer:
    @staticmethod
    def train(corpus, vocab_size: int, min_frequency: int = 1, special_tokens=("[PAD]", "[UNK]"),
              end_of_word_suffix: str = "</w>"):
        """Returns (vocab, merges) with merges as [((a, b), rank)]. Ties between equally frequent pairs go
        to the lexicographically smallest pair."""
        words = collections.Counter(w for doc in corpus for w in doc.split())
        vocab = Vocab()
        kinds = {"[PAD]": SpecialKind.PAD, "[UNK]": SpecialKind.UNK, "[BOS]": SpecialKind.BOS,
                 "[EOS]": SpecialKind.EOS}
        for s in special_tokens:
            vocab.add_special(s, kinds.get(s, SpecialKind.CUSTOM))
        splits = {}
        for w in sorted(words):
            sym = list(w)
            sym[-1] += end_of_word_suffix
            splits[w] = sym
        for s in sorted({s for sym in splits.values() for s in sym}):
            vocab.insert(s)
        merges = []
        while len(vocab) < vocab_size:
            pairs = collections.Counter()
            for w, sym in splits.items():
                for i in range(len(sym) - 1):
                    pairs[(sym[i], sym[i + 1])] += words[w]
            cands = [(c, p) for p, c in pairs.items() if c >= min_frequency]
            if not cands:
                break
            best_c = max(c for c, _ in cands)
            a, b = min(p for c, p in cands if c == best_c)
            vocab.insert(a + b)
            merges.append(((a, b), len(merges)))
            for w, sym in splits.items():
                i, new = 0, []
                while i < len(sym):
                    if i + 1 < len(sym) and sym[i] == a and sym[i + 1] == b:
                        new.append(a + b)
                        i += 2
                    else:
                        new.append(sym[i])
                        i += 1
                splits[w] = new
        return vocab, merges


class WordPieceTokenizer(Tokenizer):
    """Greedy longest-prefix match; non-initial pieces carry ``continuation_prefix``; a word with an
    unmatched remainder (or longer than ``max_input_chars_per_word``) becomes ``[UNK]``."""

    def __init__(self, vocab: Vocab, unk_token: str = "[UNK]", continuation_prefix: str = "##",
                 max_input_chars_per_word: int = 100, normalizer=None):
        self.vocab, self.unk, self.prefix, self.max_chars = vocab, unk_token, continuation_prefix, max_input_chars_per_word
        self.normalizer, self.pre = normalizer or Normalizer(), PreTokenizer()

    def segment_word(self, word: str) -> list[str]:
        if len(word) > self.max_chars:
            return [self.unk]
        out, start = [], 0
        while start < len(word):
            end = len(word)
            piece = None
            while start < end:
                cand = word[start:end] if start == 0 else self.prefix + word[start:end]
                if cand in self.vocab:
                    piece = cand
                    break
                end -= 1
            if piece is None:
                return [self.unk]
            out.append(piece)
            start = end
        return out

    def tokenize(self, text):
        out = []
        for w, _ in self.pre.pre_tokenize(self.normalizer.normalize(text)):
            out += self.segment_word(w)
        return out

    def decode(self, ids):
        s = ""
        for p in self._pieces(ids):
            s += p[len(self.prefix):] if p.startswith(self.prefix) else (" " + p if s else p)
        return s


class WordPieceTrainer:
    @staticmethod
    def train(corpus, vocab_size: int, min_frequency: int = 1, continuation_prefix: str = "##") -> Vocab:
        """BPE merges over words (no end-of-word suffix), pieces after the first written with the
        continuation prefix; every character appears in both forms so any word in the corpus segments."""
        norm, pre = Normalizer(), PreTokenizer()
        words = collections.Counter(w for doc in corpus for w, _ in pre.pre_tokenize(norm.normalize(doc)))
        vocab = default_vocab_specials(Vocab())
        splits = {w: [w[0]] + [continuation_prefix + c for c in w[1:]] for w in sorted(words)}
        for s in sorted({s for sym in splits.values() for s in sym}):
            vocab.insert(s)
        strip = lambda t: t[len(continuation_prefix):] if t.startswith(continuation_prefix) else t  # noqa: E731
        while len(vocab) < vocab_size:
            pairs = collections.Counter()
            for w, sym in splits.items():
                for i in range(len(sym) - 1):
                    pairs[(sym[i], sym[i + 1])] += words[w]
            cands = [(c, p) for p, c in pairs.items() if c >= min_frequency]
            if not cands:
                break
            best_c = max(c for c, _ in cands)
            a, b = min(p for c, p in cands if c == best_c)
            merged = a + strip(b)
            vocab.insert(merged)
            for w, sym in splits.items():
                i, new = 0, []
                while i < len(sym):
                    if i + 1 < len(sym) and sym[i] == a and sym[i + 1] == b:
                        new.append(merged)
                        i += 2
                    else:
                        new.append(sym[i])
                        i += 1
                splits[w] = new
        return vocab


SP_SPACE = "▁"


class SentencePieceTokenizer(Tokenizer):
    """Unigram language model: spaces become ``▁`` (and text is prefixed with one), and the
    segmentation maximising the sum of piece log-probabilities is found by Viterbi. Characters that no
    piece covers become ``[UNK]`` with a fixed penalty."""

    UNK_PENALTY = -20.0

    def __init__(self, vocab: Vocab, piece_scores: dict[str, float], add_dummy_prefix: bool = True):
        self.vocab, self.scores, self.add_dummy_prefix = vocab, dict(piece_scores), add_dummy_prefix
        self.max_len = max((len(p) for p in self.scores), default=1)

    @classmethod
    def from_pieces(cls, vocab, piece_scores, add_dummy_prefix=True):
        return cls(vocab, piece_scores, add_dummy_prefix)

    def preprocess(self, text: str) -> str:
        text = " ".join(text.split())
        if self.add_dummy_prefix:
            text = " " + text
        return text.replace(" ", SP_SPACE)

    def viterbi_decode(self, text: str) -> list[str]:
        s = self.preprocess(text)
        n = len(s)
        best = [-math.inf] * (n + 1)
        back = [(-1, None)] * (n + 1)
        best[0] = 0.0
        for end in range(1, n + 1):
            for start in range(max(0, end - self.max_len), end):
                if best[start] == -math.inf:
                    continue
                piece = s[start:end]
                sc = self.scores.get(piece)
                if sc is None:
                    if end - start != 1:
                        continue
                    sc, piece = self.UNK_PENALTY, None
                if best[start] + sc > best[end]:
                    best[end] = best[start] + sc
                    back[end] = (start, piece)
        out, pos = [], n
        while pos > 0:
            start, piece = back[pos]
            out.append(piece if piece is not None else "[UNK]")
            pos = start
        return out[::-1]

    def tokenize(self, text):
        return self.viterbi_decode(text)

    def decode(self, ids):
        return "".join(self._pieces(ids)).replace(SP_SPACE, " ").strip()


class UnigramTrainer:
    @staticmethod
    def train(corpus, vocab_size: int, max_piece_len: int = 8, em_iters: int = 3):
        """Seed with every substring (up to ``max_piece_len``) seen at least twice plus all characters,
        score by log frequency, then repeat: Viterbi-segment the corpus, re-estimate log probabilities
        from the segment counts, and keep the ``vocab_size`` most probable pieces (characters are
        always kept). Returns (vocab, piece_scores)."""
        docs = [" " + " ".join(d.split()) for d in corpus]
        docs = [d.replace(" ", SP_SPACE) for d in docs]
        chars = sorted({c for d in docs for c in d})
        sub = collections.Counter()
        for d in docs:
            for i in range(len(d)):
                for L in range(2, max_piece_len + 1):
                    # a piece never spans a word boundary: "▁" may only lead it
                    if i + L <= len(d) and SP_SPACE not in d[i + 1:i + L]:
                        sub[d[i:i + L]] += 1
        cand = {p: c for p, c in sub.items() if c >= 2}
        seed = dict(cand)
        for c in chars:
            cand[c] = cand.get(c, 0) + 1
        tot = sum(cand.values())
        scores = {p: math.log(c / tot) for p, c in cand.items()}
        specials = default_vocab_specials(Vocab())
        budget = max(len(chars), vocab_size - len(specials))
        for _ in range(em_iters):
            tok = SentencePieceTokenizer(Vocab(), scores)
            counts = collections.Counter()
            for d in docs:
                counts.update(p for p in tok.viterbi_decode(d.replace(SP_SPACE, " ")) if p != "[UNK]")
            for c in chars:
                counts[c] += 1
            # pieces the current segmentation does not use keep a tenth of their seed frequency, so a
            # piece is dropped only when better ones fill the budget
            for p, c in seed.items():
                counts[p] += 0.1 * c
            keep = sorted(counts, key=lambda p: (-counts[p], p))
            keep = list(dict.fromkeys(chars + [p for p in keep if p not in chars][:max(0, budget - len(chars))]))
            tot = sum(counts[p] for p in keep)
            scores = {p: math.log(counts[p] / tot) for p in keep}
        vocab = specials
        for p in sorted(scores, key=lambda p: (-scores[p], p)):
            vocab.insert(p)
        return vocab, scores


def _byte_map() -> dict[int, str]:
    """Printable bytes map to themselves; the rest to code points from 256 up (GPT-2 byte-level map)."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    out, extra = {}, 0
    for b in range(256):
        if b in keep:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + extra)
            extra += 1
    return out


class ByteLevelEncoder:
    def __init__(self):
        self._b2c = _byte_map()
        self._c2b = {c: b for b, c in self._b2c.items()}

    def byte_to_char(self, b: int) -> str:
        return self._b2c[b]

    def char_to_byte(self, c: str):
        return self._c2b.get(c)

    def encode_bytes(self, data: bytes) -> str:
        return "".join(self._b2c[b] for b in data)

    def decode_bytes(self, text: str) -> bytes:
        return bytes(self._c2b[c] for c in text if c in self._c2b)

    def decode_to_string(self, text: str) -> str:
        return self.decode_bytes(text).decode("utf-8", errors="replace")


# ------------------------------------------------------------------ post-processing
class TruncationStrategy(enum.Enum):
    LONGEST_FIRST = "longest_first"
    ONLY_FIRST = "only_first"
    ONLY_SECOND = "only_second"
    DO_NOT_TRUNCATE = "do_not_truncate"


@dataclass
class PostConfig:
    add_bos_eos: bool = False
    add_cls_sep: bool = False
    max_length: int = 0
    pad_to_max_length: bool = False
    truncation: TruncationStrategy = TruncationStrategy.LONGEST_FIRST


class PostProcessor:
    def __init__(self, vocab: Vocab, config: PostConfig | None = None):
        self.vocab, self.config = vocab, config or PostConfig()

    def _wrap(self, ids, toks, first: bool, last: bool):
        c, v = self.config, self.vocab
        if c.add_cls_sep:
            pre = [v.cls_id()] if first else []
            return pre + ids + [v.sep_id()], ([v.get_token(v.cls_id())] if first else []) + toks + [v.get_token(v.sep_id())]
        if c.add_bos_eos:
            pre = [v.bos_id()] if first else []
            post = [v.eos_id()] if last else []
            return (pre + ids + post, ([v.get_token(v.bos_id())] if first else []) + toks +
                    ([v.get_token(v.eos_id())] if last else []))
        return ids, toks

    def _n_special(self, pair: bool) -> int:
        c = self.config
        if c.add_cls_sep:
            return 3 if pair else 2
        if c.add_bos_eos:
            return 2
        return 0

    def _pad(self, out: TokenizedOutput) -> TokenizedOutput:
        c = self.config
        if c.max_length and c.pad_to_max_length and len(out.ids) < c.max_length:
            k = c.max_length - len(out.ids)
            pad = self.vocab.pad_id() or 0
            out.ids += [pad] * k
            out.tokens += [self.vocab.get_token(pad) or ""] * k
            out.attention_mask += [0] * k
            out.type_ids += [out.type_ids[-1] if out.type_ids else 0] * k
        return out

    def process_single(self, out: TokenizedOutput) -> TokenizedOutput:
        c = self.config
        ids, toks = list(out.ids), list(out.tokens)
        if c.max_length and c.truncation != TruncationStrategy.DO_NOT_TRUNCATE:
            keep = max(0, c.max_length - self._n_special(False))
            ids, toks = ids[:keep], toks[:keep]
        ids, toks = self._wrap(ids, toks, True, True)
        return self._pad(TokenizedOutput(ids, toks))

    def process_pair(self, first: TokenizedOutput, second: TokenizedOutput) -> TokenizedOutput:
        c = self.config
        a_ids, a_t, b_ids, b_t = list(first.ids), list(first.tokens), list(second.ids), list(second.tokens)
        if c.max_length and c.truncation != TruncationStrategy.DO_NOT_TRUNCATE:
            budget = max(0, c.max_length - self._n_special(True))
            while len(a_ids) + len(b_ids) > budget:
                cut_a = (c.truncation == TruncationStrategy.ONLY_FIRST or
                         (c.truncation == TruncationStrategy.LONGEST_FIRST and len(a_ids) >= len(b_ids)))
                if cut_a and a_ids:
                    a_ids.pop(), a_t.pop()
                elif b_ids and c.truncation != TruncationStrategy.ONLY_FIRST:
                    b_ids.pop(), b_t.pop()
                else:
                    break
        ai, at = self._wrap(a_ids, a_t, True, False)
        bi, bt = self._wrap(b_ids, b_t, False, True)
        return self._pad(TokenizedOutput(ai + bi, at + bt, type_ids=[0] * len(ai) + [1] * len(bi)))


def batch_encode(tokenizer: Tokenizer, texts, post: PostProcessor, device=None):
    """Encodes and pads a batch to its longest sequence; returns (ids [B, L] int64, mask [B, L])."""
    outs = [post.process_single(tokenizer.encode(t)) for t in texts]
    L = max(len(o.ids) for o in outs)
    pad = tokenizer.vocab.pad_id() or 0
    ids = torch.full((len(outs), L), pad, dtype=torch.int64)
    mask = torch.zeros((len(outs), L), dtype=torch.int64)
    for i, o in enumerate(outs):
        ids[i, :len(o.ids)] = torch.tensor(o.ids)
        mask[i, :len(o.ids)] = torch.tensor(o.attention_mask)
    return ids.to(device), mask.to(device)


# ------------------------------------------------------------------ language-model preprocessing
class LmPreprocessor:
    """Batches for causal / masked language modelling (reference tokenizer-side helpers,
    crates/brain-text/src/lm.rs:52-170)."""

    @staticmethod
    def prepare_causal_lm(ids: torch.Tensor):
        """(inputs, labels) with labels shifted left by one."""
        return ids[..., :-1], ids[..., 1:]

    @staticmethod
    def prepare_masked_lm(ids: torch.Tensor, mask_id: int, vocab_size: int, prob: float = 0.15,
                          special_ids=(), generator=None, ignore_index: int = -100):
        """BERT masking: each non-special position is selected with ``prob``; of those 80 % become
        ``mask_id``, 10 % a random token and 10 % stay. Labels are the originals at selected positions
        and ``ignore_index`` elsewhere."""
        sel = torch.rand(ids.shape, generator=generator) < prob
        for s in special_ids:
            sel &= ids != s
        labels = torch.where(sel, ids, torch.full_like(ids, ignore_index))
        r = torch.rand(ids.shape, generator=generator)
        out = ids.clone()
        out[sel & (r < 0.8)] = mask_id
        rnd = sel & (r >= 0.8) & (r < 0.9)
        out[rnd] = torch.randint(0, vocab_size, (int(rnd.sum()),), generator=generator)
        return out, labels

    @staticmethod
    def create_causal_mask(seq_len: int) -> torch.Tensor:
        """1 where query i may attend key j (j <= i)."""
        return torch.tril(torch.ones(seq_len, seq_len, dtype=torch.uint8))

    @staticmethod
    def create_prefix_lm_mask(prefix_len: int, total_len: int) -> torch.Tensor:
        """Bidirectional inside the prefix, causal after it."""
        m = LmPreprocessor.create_causal_mask(total_len)
        m[:prefix_len, :prefix_len] = 1
        return m

    @staticmethod
    def pack_documents(docs, seq_len: int, eos_id: int) -> torch.Tensor:
        """Concatenates token lists with ``eos_id`` after each and cuts [N, seq_len] rows (the tail that
        does not fill a row is dropped)."""
        flat = [t for d in docs for t in list(d) + [eos_id]]
        n = len(flat) // seq_len
        return torch.tensor(flat[:n * seq_len], dtype=torch.int64).view(n, seq_len)

    @staticmethod
    def sliding_window_chunks(ids, window: int, stride: int):
        ids = list(ids)
        if len(ids) <= window:
            return [ids]
        out = [ids[i:i + window] for i in range(0, len(ids) - window + 1, stride)]
        if (len(ids) - window) % stride:
            out.append(ids[-window:])
        return out


# ------------------------------------------------------------------ text features
class BagOfWords:
    def __init__(self, vocab: Vocab | None = None):
        self.vocab = vocab or Vocab()

    def fit(self, corpus) -> "BagOfWords":
        for doc in corpus:
            for t in doc:
                self.vocab.insert(t)
        return self

    def transform(self, tokens) -> torch.Tensor:
        v = torch.zeros(len(self.vocab))
        for t in tokens:
            i = self.vocab.get_id(t)
            if i is not None:
                v[i] += 1
        return v

    def fit_transform(self, corpus) -> torch.Tensor:
        self.fit(corpus)
        return torch.stack([self.transform(d) for d in corpus])


class TfIdf:
    """tf = count / len(doc); idf = ln((1 + N) / (1 + df)) + 1 (smoothed); rows L2-normalised."""

    def __init__(self, min_df: int = 1, normalize: bool = True):
        self.min_df, self.normalize = min_df, normalize
        self.vocab, self.idf = Vocab(), None

    def fit(self, corpus) -> "TfIdf":
        df = collections.Counter(t for doc in corpus for t in set(doc))
        for t in sorted(t for t, c in df.items() if c >= self.min_df):
            self.vocab.insert(t)
        n = len(corpus)
        self.idf = torch.tensor([math.log((1 + n) / (1 + df[t])) + 1 for t in self.vocab._toks], dtype=torch.float64)
        return self

    def transform(self, tokens) -> torch.Tensor:
        v = torch.zeros(len(self.vocab), dtype=torch.float64)
        for t in tokens:
            i = self.vocab.get_id(t)
            if i is not None:
                v[i] += 1
        if tokens:
            v /= len(tokens)
        v *= self.idf
        if self.normalize and v.norm() > 0:
            v /= v.norm()
        return v

    def fit_transform(self, corpus) -> torch.Tensor:
        self.fit(corpus)
        return torch.stack([self.transform(d) for d in corpus])


class Bm25:
    """Okapi BM25: idf = ln(1 + (N − df + 0.5) / (df + 0.5)), term score
    idf · tf (k1 + 1) / (tf + k1 (1 − b + b · |d| / avgdl))."""

    def __init__(self, k1: float = 1.5, b: float = 0.75):
        self.k1, self.b = k1, b

    def fit(self, docs) -> "Bm25":
        self.docs = [collections.Counter(d) for d in docs]
        self.lens = [len(d) for d in docs]
        self.avgdl = sum(self.lens) / max(1, len(docs))
        df = collections.Counter(t for d in docs for t in set(d))
        n = len(docs)
        self.idf = {t: math.log(1 + (n - c + 0.5) / (c + 0.5)) for t, c in df.items()}
        return self

    def score(self, query, doc_idx: int) -> float:
        d, L = self.docs[doc_idx], self.lens[doc_idx]
        s = 0.0
        for t in query:
            tf = d.get(t, 0)
            if tf:
                s += self.idf[t] * tf * (self.k1 + 1) / (tf + self.k1 * (1 - self.b + self.b * L / self.avgdl))
        return s

    def score_corpus(self, query) -> list[float]:
        return [self.score(query, i) for i in range(len(self.docs))]


class HashingVectorizer:
    """Token counts hashed into ``num_features`` buckets (FNV-1a 64-bit of the UTF-8 token)."""

    def __init__(self, num_features: int = 1 << 16):
        self.n = num_features

    def transform(self, tokens) -> torch.Tensor:
        from .utils import fnv1a_64

        v = torch.zeros(self.n)
        for t in tokens:
            v[fnv1a_64(t.encode()) % self.n] += 1
        return v


# ------------------------------------------------------------------ similarity
class TextSimilarity:
    @staticmethod
    def cosine(a, b) -> float:
        a, b = torch.as_tensor(a, dtype=torch.float64), torch.as_tensor(b, dtype=torch.float64)
        den = float(a.norm() * b.norm())
        return float(a @ b) / den if den > 0 else 0.0

    @staticmethod
    def dot_product(a, b) -> float:
        return float(torch.as_tensor(a, dtype=torch.float64) @ torch.as_tensor(b, dtype=torch.float64))

    @staticmethod
    def euclidean(a, b) -> float:
        return float((torch.as_tensor(a, dtype=torch.float64) - torch.as_tensor(b, dtype=torch.float64)).norm())

    @staticmethod
    def manhattan(a, b) -> float:
        return float((torch.as_tensor(a, dtype=torch.float64) - torch.as_tensor(b, dtype=torch.float64)).abs().sum())

    @staticmethod
    def levenshtein(s1: str, s2: str) -> int:
        prev = list(range(len(s2) + 1))
        for i, c1 in enumerate(s1, 1):
            cur = [i]
            for j, c2 in enumerate(s2, 1):
                cur.append(min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (c1 != c2)))
            prev = cur
        return prev[-1]

    @staticmethod
    def damerau(s1: str, s2: str) -> int:
        """Optimal string alignment distance (adjacent transpositions count 1)."""
        n, m = len(s1), len(s2)
        d = [[0] * (m + 1) for _ in range(n + 1)]
        for i in range(n + 1):
            d[i][0] = i
        for j in range(m + 1):
            d[0][j] = j
        for i in range(1, n + 1):
            for j in range(1, m + 1):
                cost = s1[i - 1] != s2[j - 1]
                d[i][j] = min(d[i - 1][j] + 1, d[i][j - 1] + 1, d[i - 1][j - 1] + cost)
                if i > 1 and j > 1 and s1[i - 1] == s2[j - 2] and s1[i - 2] == s2[j - 1]:
                    d[i][j] = min(d[i][j], d[i - 2][j - 2] + 1)
        return d[n][m]

    @staticmethod
    def levenshtein_similarity(s1: str, s2: str) -> float:
        m = max(len(s1), len(s2))
        return 1.0 - TextSimilarity.levenshtein(s1, s2) / m if m else 1.0

    @staticmethod
    def damerau_similarity(s1: str, s2: str) -> float:
        m = max(len(s1), len(s2))
        return 1.0 - TextSimilarity.damerau(s1, s2) / m if m else 1.0

    @staticmethod
    def jaro(s1: str, s2: str) -> float:
        if s1 == s2:
            return 1.0
        l1, l2 = len(s1), len(s2)
        if not l1 or not l2:
            return 0.0
        win = max(0, max(l1, l2) // 2 - 1)
        m1, m2 = [False] * l1, [False] * l2
        matches = 0
        for i, c in enumerate(s1):
            for j in range(max(0, i - win), min(l2, i + win + 1)):
                if not m2[j] and s2[j] == c:
                    m1[i] = m2[j] = True
                    matches += 1
                    break
        if not matches:
            return 0.0
        a = [c for c, f in zip(s1, m1) if f]
        b = [c for c, f in zip(s2, m2) if f]
        t = sum(x != y for x, y in zip(a, b)) / 2
        return (matches / l1 + matches / l2 + (matches - t) / matches) / 3

    @staticmethod
    def jaro_winkler(s1: str, s2: str, p: float = 0.1) -> float:
        j = TextSimilarity.jaro(s1, s2)
        prefix = 0
        for a, b in zip(s1[:4], s2[:4]):
            if a != b:
                break
            prefix += 1
        return j + prefix * p * (1 - j)

    @staticmethod
    def jaccard(a, b) -> float:
        A, B = set(a), set(b)
        return len(A & B) / len(A | B) if A | B else 1.0

    @staticmethod
    def sorensen_dice(a, b) -> float:
        A, B = set(a), set(b)
        return 2 * len(A & B) / (len(A) + len(B)) if A or B else 1.0

    @staticmethod
    def n_gram_overlap(s1: str, s2: str, n: int = 2) -> float:
        g1 = {s1[i:i + n] for i in range(len(s1) - n + 1)}
        g2 = {s2[i:i + n] for i in range(len(s2) - n + 1)}
        return len(g1 & g2) / len(g1 | g2) if g1 | g2 else 1.0


# --------------------------------------------------------------------------- fastText subword embeddings
@dataclass
class FastTextConfig:
    """crates/brain-text/src/embedding/fasttext.rs:FastTextConfig (same fields and defaults)."""
    min_n: int = 3
    max_n: int = 6
    bucket_size: int = 10000
    dim: int = 100


class FastTextEmbedding:
    """Word vectors composed from character n-grams (Bojanowski et al. 2017), so that out-of-vocabulary
    words get vectors from the subwords they share with known ones. A word's n-grams are taken from
    "<word>" for n in [min_n, max_n] and hashed into ``bucket_size`` rows of an n-gram table with 64-bit
    FNV-1a (the published hash; the same bucket indices as the reference). ``insert_word`` stores the
    word vector and spreads an equal share of it (vector / (n-grams + 1)) over its n-gram rows;
    ``get_word_vector`` averages the stored vector (if any) and the word's n-gram rows. The table is a
    tensor (``device`` selectable) and ``word_vectors`` batches the lookup with one ``embedding_bag``."""

    def __init__(self, config: FastTextConfig | None = None, device=None):
        self.config = c = config or FastTextConfig()
        self.word_vectors_: dict[str, torch.Tensor] = {}
        self.ngram_buckets = torch.zeros(c.bucket_size, c.dim, device=device)

    @staticmethod
    def compute_ngram_hash(ngram: str, bucket_size: int) -> int:
        h = 0xCBF29CE484222325
        for b in ngram.encode("utf-8"):
            h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
        return h % bucket_size

    def extract_subwords(self, word: str) -> list[str]:
        chars = "<" + word + ">"
        return [chars[i:i + n] for n in range(self.config.min_n, self.config.max_n + 1)
                for i in range(len(chars) - n + 1)]

    def _buckets(self, word: str) -> list[int]:
        return [self.compute_ngram_hash(s, self.config.bucket_size) for s in self.extract_subwords(word)]

    def insert_word(self, word: str, vector) -> None:
        v = torch.as_tensor(vector, dtype=torch.float32, device=self.ngram_buckets.device)
        idx = self._buckets(word)
        share = v / (len(idx) + 1)
        self.ngram_buckets.index_add_(0, torch.tensor(idx, dtype=torch.long, device=v.device),
                                      share.expand(len(idx), -1).contiguous())
        self.word_vectors_[word] = v

    def get_word_vector(self, word: str) -> torch.Tensor:
        idx = self._buckets(word)
        total = torch.zeros(self.config.dim, device=self.ngram_buckets.device)
        count = 0
        if word in self.word_vectors_:
            total += self.word_vectors_[word]
            count += 1
        if idx:
            total += self.ngram_buckets[torch.tensor(idx, dtype=torch.long, device=total.device)].sum(0)
            count += len(idx)
        return total / count if count else total

    def word_vectors(self, words: list[str]) -> torch.Tensor:
        """[len(words), dim] in one embedding_bag over the n-gram rows (stored word vectors added)."""
        dev = self.ngram_buckets.device
        flat, offsets, extra, counts = [], [], torch.zeros(len(words), self.config.dim, device=dev), []
        for i, w in enumerate(words):
            offsets.append(len(flat))
            idx = self._buckets(w)
            flat += idx
            n = len(idx)
            if w in self.word_vectors_:
                extra[i] = self.word_vectors_[w]
                n += 1
            counts.append(max(n, 1))
        sums = torch.nn.functional.embedding_bag(torch.tensor(flat, dtype=torch.long, device=dev),
                                                 self.ngram_buckets, torch.tensor(offsets, dtype=torch.long, device=dev),
                                                 mode="sum")
        return (sums + extra) / torch.tensor(counts, dtype=torch.float32, device=dev)[:, None]

    def most_similar(self, word: str, candidates: list[str], top_k: int) -> list[tuple[str, float]]:
        target = self.get_word_vector(word)
        scored = [(c, TextSimilarity.cosine(target.cpu(), self.get_word_vector(c).cpu())) for c in candidates if c != word]
        scored.sort(key=lambda t: -t[1])
        return scored[:top_k]
