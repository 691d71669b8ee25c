"""Sequence ops, collators, span corruption, augmentation, distances, BLEU and byte-level mapping."""
import random

import pytest
import torch

from brain_b200 import text_ops as T


def test_pad_truncate_pack_ids():
    ids, m = T.pad_sequences([[1, 2, 3], [4]], pad_id=0)
    assert ids.tolist() == [[1, 2, 3], [4, 0, 0]] and m.tolist() == [[1, 1, 1], [1, 0, 0]]
    ids, m = T.pad_sequences([[1, 2, 3], [4]], pad_id=9, max_len=2, side="left")
    assert ids.tolist() == [[1, 2], [9, 4]] and m.tolist() == [[1, 1], [0, 1]]
    assert T.truncate_sequences([[1, 2, 3, 4]], 2, "left") == [[3, 4]]
    assert T.pack_sequences([[1, 2], [3, 4, 5]], 3, 0) == [[1, 2, 0], [3, 4, 5], [0]]
    assert T.create_attention_mask([[5, 0, 7]], 0).tolist() == [[1, 0, 1]]
    assert T.create_position_ids(2, 3).tolist() == [[0, 1, 2]] * 2
    assert T.create_token_type_ids(2, 3).tolist() == [0, 0, 1, 1, 1]
    assert T.one_hot_encode([1, 5, 0], 3).tolist() == [[0, 1, 0], [0, 0, 0], [1, 0, 0]]
    assert T.tokens_to_ids(["a", "zz"], {"a": 3}, 0) == [3, 0]
    assert T.ids_to_tokens([1, 7], ["x", "y"]) == ["y", "[UNK]"]


def test_mlm_masking_statistics_and_collators():
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(5, 1000, (64, 512), generator=g)
    out, sel = T.mask_tokens(ids, 0.15, 4, 1000, generator=g)
    frac = sel.float().mean().item()
    assert abs(frac - 0.15) < 0.01
    masked = (out == 4) & sel
    kept = (out == ids) & sel
    assert abs(masked.sum().item() / sel.sum().item() - 0.8) < 0.02
    assert abs(kept.sum().item() / sel.sum().item() - 0.1) < 0.02 + 0.001  # random ids can equal the original
    assert torch.equal(out[~sel], ids[~sel])
    col = T.DataCollatorForLanguageModeling(pad_token_id=0, mask_token_id=4, vocab_size=50, mlm_probability=0.5)
    x, y, am = col([[7, 8, 9, 10], [11, 12]], generator=torch.Generator().manual_seed(1))
    assert am.tolist() == [[1, 1, 1, 1], [1, 1, 0, 0]]
    assert (y[1, 2:] == -100).all() and (x[1, 2:] == 0).all()  # pads never selected
    sel_pos = y != -100
    orig = torch.tensor([[7, 8, 9, 10], [11, 12, 0, 0]])
    assert torch.equal(y[sel_pos], orig[sel_pos])
    clm = T.DataCollatorForLanguageModeling(0, 4, 50, mlm=False)
    x, y, am = clm([[7, 8], [9]])
    assert y.tolist() == [[7, 8], [9, -100]]
    s2s = T.DataCollatorForSeq2Seq(pad_token_id=0)
    x, y, am = s2s([[1, 2], [3]], [[5], [6, 7, 8]])
    assert x.tolist() == [[1, 2], [3, 0]] and y.tolist() == [[5, -100, -100], [6, 7, 8]]


def test_span_corruption_and_augmentation():
    toks = list(range(100, 140))
    inp, tgt = T.corrupt_spans(toks, 0.15, 3.0, sentinel_start_id=999, rng=random.Random(3), sentinel_step=-1)
    sentinels = [t for t in inp if t > 900]
    assert sentinels == [t for t in tgt if t > 900] == [999 - i for i in range(len(sentinels))]
    # rebuilding: replace each sentinel in the input by its span from the target gives the original
    spans, cur = {}, None
    for t in tgt:
        if t > 900:
            cur = t
            spans[cur] = []
        else:
            spans[cur].append(t)
    rebuilt = [x for t in inp for x in (spans[t] if t > 900 else [t])]
    assert rebuilt == toks
    assert len(tgt) - len(sentinels) == round(40 * 0.15)
    w = "the quick brown fox jumps".split()
    r = random.Random(5)
    assert set(T.random_deletion(w, 0.5, r)) <= set(w) and T.random_deletion(w, 1.0, r)
    sw = T.random_swap(w, 0.5, r)
    assert sorted(sw) == sorted(w)
    ins = T.random_insertion(w, 1.0, r)
    assert len(ins) == 2 * len(w) and sorted(set(ins)) == sorted(set(w))
    assert len(T.char_perturbation("hello, world", 0.5, r)) == 12


def test_distances_similarity_bleu_bytes():
    assert T.levenshtein_distance("kitten", "sitting") == 3
    assert T.damerau_levenshtein_distance("ca", "ac") == 1 and T.levenshtein_distance("ca", "ac") == 2
    assert T.jaccard_similarity("abc", "bcd") == 0.5 and T.jaccard_similarity("", "") == 1.0
    assert T.cosine_similarity_slice([1, 0], [1, 1]) == pytest.approx(2 ** -0.5)
    x = torch.tensor([[1.0, 0.0], [0.0, 2.0], [3.0, 3.0]])
    s = T.pairwise_similarity_matrix(x)
    assert torch.allclose(s.diagonal(), torch.ones(3)) and abs(float(s[0, 1])) < 1e-7
    assert torch.allclose(T.pairwise_similarity_matrix(x, "euclidean")[0, 1], torch.tensor(-5 ** 0.5))
    cand = "the cat sat on the mat".split()
    assert T.bleu_score(cand, [cand]) == pytest.approx(1.0)
    assert T.bleu_score("a b".split(), ["c d".split()]) == 0.0
    c2 = "the cat is on the mat".split()
    b = T.corpus_bleu([c2], [[cand]], max_n=2)
    # unigram 5/6, bigram 3/5, no brevity penalty
    assert b == pytest.approx((5 / 6 * 3 / 5) ** 0.5)
    s = "héllo 世界 \x00!"
    enc = T.byte_encode(s)
    assert all(c.isprintable() for c in enc) and T.byte_decode(enc) == s
    assert T.byte_encode(" ") == "Ġ"  # GPT-2's space symbol
    assert T.is_whitespace("　") and T.is_control("\x00") and not T.is_control("\n")
    assert T.is_punctuation("$") and T.is_punctuation("、") and T.is_chinese_char("世") and not T.is_chinese_char("a")
