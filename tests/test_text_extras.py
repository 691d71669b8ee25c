"""Text analysis, n-gram operators, transforms, batch preparation, scores, vocabulary tools and word-vector
tables (crates/brain-text/src/analyze.rs, text_ops.rs, transform.rs, process.rs, compute.rs, optimize.rs,
embedding/pretrained.rs)."""
import math

import pytest
import torch

from brain_b200 import text_extras as TX


def test_analysis_and_readability():
    text = "The cat sat. The dog ran away quickly! Did it?"
    st = TX.analyze_text(text)
    assert st.word_count == 10 and st.sentence_count == 3 and st.punctuation_count == 3
    assert st.type_token_ratio == pytest.approx(9 / 10)
    assert [TX.count_syllables(w) for w in ("the", "quickly", "make", "beautiful", "42")] == [1, 2, 1, 3, 0]
    syl = sum(TX.count_syllables(w) for w in text.split())
    assert TX.flesch_reading_ease(text) == pytest.approx(206.835 - 1.015 * 10 / 3 - 84.6 * syl / 10)
    assert TX.flesch_kincaid_grade(text) == pytest.approx(max(0.39 * 10 / 3 + 11.8 * syl / 10 - 15.59, 0))
    assert TX.coleman_liau_index(text) == pytest.approx(0.0588 * st.letter_count * 10 - 0.296 * 30 - 15.8)
    assert TX.flesch_reading_ease("") == 100.0 and TX.gunning_fog_index("") == 0.0
    words = "a b a c d d d".split()
    assert TX.hapax_legomena_ratio(words) == pytest.approx(2 / 7)
    assert TX.yules_k_characteristic(words) == pytest.approx(1e4 * ((1 * 2 + 4 * 1 + 9 * 1) - 7) / 49)
    assert TX.text_entropy("aabb") == 1.0 and TX.shannon_entropy_words(["x", "y", "x", "y"]) == 1.0
    assert TX.split_into_sentences("Hi. Yes! no") == ["Hi.", "Yes!", "no"]
    assert TX.split_into_paragraphs("a\n\n\n\nb\n\n") == ["a", "b"]


def test_ngrams_skipgrams_collocations():
    toks = "new york is new york city".split()
    assert TX.ngrams(toks, 2)[0] == ["new", "york"] and len(TX.ngrams(toks, 7)) == 0
    assert TX.character_ngrams("abcd", 3) == ["abc", "bcd"] and TX.shingles("aaaa", 2) == {"aa"}
    assert TX.skipgrams(["a", "b", "c", "d"], 2, 1) == [["a", "b"], ["a", "c"], ["b", "c"], ["b", "d"], ["c", "d"]]
    col = TX.collocations(toks, 2, 0.0)
    assert col[0][:2] == ("new", "york")
    assert col[0][2] == pytest.approx(math.log((2 / 5) / ((2 / 6) * (2 / 6))))
    assert TX.ngram_freq(toks, 2)[("new", "york")] == 2 and TX.term_frequencies(["a", "a", "b", "c"])["a"] == 0.5


def test_transforms_and_pipeline():
    assert TX.case_transform("hello big_world-now", "camel") == "helloBigWorldNow"
    assert TX.case_transform("Hello Big World", "snake") == "hello_big_world"
    assert TX.case_transform("Hello Big World", "kebab") == "hello-big-world"
    assert TX.case_transform("hELLO wORLD", "title") == "Hello World"
    assert TX.transliterate_ascii("Straße café Æsop “x” — ©") == 'Strasse cafe AEsop "x" - (c)'
    assert TX.censor_words("You darn fool!", {"darn", "fool"}) == "You *** ***"
    assert TX.normalize_punctuation("Hi , “there” …") == 'Hi, "there"...'
    p = TX.TextPipeline().add_step(str.strip).add_step(str.upper)
    assert p.run("  ab ") == "AB"
    assert TX.clean_text("<b>Hi</b>\x07   there\n") == "Hi there"


def test_batch_prep_and_scores():
    ids, mask = TX.pad_and_collate([[1, 2, 3], [4]], pad_id=0)
    assert ids.tolist() == [[1, 2, 3], [4, 0, 0]] and mask.tolist() == [[True] * 3, [True, False, False]]
    ids2, _ = TX.pad_and_collate([[1, 2, 3], [4]], max_len=2)
    assert ids2.shape == (2, 2)
    assert list(TX.batch_iterator(list(range(5)), 2)) == [[0, 1], [2, 3], [4]]
    assert TX.filter_by_length(["a b", "a", "a b c d"], 2, 3) == ["a b"]
    assert TX.chrf_score("abcd", "abcd", 2) == 1.0 and TX.chrf_score("", "", 2) == 1.0 and TX.chrf_score("ab", "", 2) == 0.0
    assert TX.character_error_rate("kitten", "sitting") == pytest.approx(3 / 6)
    assert TX.bits_per_character(math.log(2)) == pytest.approx(1.0)
    assert TX.f1_token_score("a b c".split(), "a b d".split()) == pytest.approx(2 / 3)
    assert TX.exact_match_score(" x ", "x") == 1.0


def test_vocab_tools_and_pretrained_vectors():
    v = TX.prune_vocab({"a": 5, "b": 5, "c": 1, "d": 3}, min_freq=2, max_size=3, keep=["<pad>"])
    assert v == ["<pad>", "a", "b"]
    t = TX.VocabTrie.from_vocab(["un", "unb", "unbelievable", "be"])
    assert t.contains("unb") and not t.contains("unbe")
    assert t.longest_prefix_match("unbelievably") == 3 and t.longest_prefix_match("xyz") == 0
    table = torch.randn(10, 8)
    q, s = TX.quantize_embeddings_simple(table)
    assert q.dtype == torch.int8 and float((q.float() * s[:, None] - table).abs().max()) <= float(s.max()) / 2 + 1e-6
    glove = "king 1 0 0 1\nqueen 1 0 1 1\nman 0 0 0 1\nwoman 0 0 1 1\napple 0 1 0 0\n"
    emb = TX.PretrainedEmbedding.load_glove_str(glove)
    assert emb.dim == 4 and emb.get_vector("queen").tolist() == [1, 0, 1, 1]
    assert emb.analogy("man", "king", "woman")[0][0] == "queen"
    ms = emb.most_similar("king", 2)
    assert ms[0][0] in ("queen", "man") and all(w != "king" for w, _ in ms)
    assert float(emb.get_vector("zzz").abs().sum()) == 0.0
    w2v = TX.PretrainedEmbedding.load_word2vec_text_str("2 3\na 1 2 3\nb 4 5 6\n")
    assert w2v.words == ["a", "b"] and w2v.to_word_embedding(["b", "x"]).shape == (2, 3)
    with pytest.raises(ValueError):
        TX.PretrainedEmbedding.load_glove_str("a 1 2\nb 1\n")
