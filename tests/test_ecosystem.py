"""Ecosystem components beyond the transformer stack (CPU): federated learning, text tokenisers, the
model zoo (RNN, CNN, GNN, diffusion, GAN, RL, audio, neuroevolution), the graph IR, the benchmark
harness and the CLI commands for BrainMind."""
import math

import pytest
import torch

from tests._mp import run_ranks


# ------------------------------------------------------------------ federated
def test_fedavg_trimmed_median():
    from brain_b200 import federated as F
    d = [F.ModelDelta(0, [torch.tensor([1.0, 10.0])], 1), F.ModelDelta(1, [torch.tensor([3.0, 20.0])], 3),
         F.ModelDelta(2, [torch.tensor([100.0, -5.0])], 0), F.ModelDelta(3, [torch.tensor([2.0, 0.0])], 0)]
    torch.testing.assert_close(F.fed_avg_aggregate(d[:2])[0], torch.tensor([2.5, 17.5]))
    # trimmed mean with f = 0.25 over 4 clients drops one lowest and one highest per coordinate
    torch.testing.assert_close(F.trimmed_mean_aggregate(d, 0.25)[0], torch.tensor([2.5, 5.0]))
    torch.testing.assert_close(F.median_aggregate(d)[0], torch.tensor([2.5, 5.0]))
    torch.testing.assert_close(F.median_aggregate(d[:3])[0], torch.tensor([3.0, 10.0]))


def test_secure_aggregation_masks_cancel_and_dp():
    from brain_b200 import federated as F
    agg = F.SecureAggregator(5)
    masks = [agg.generate_client_pairwise_mask(i, (3, 4), seed=11) for i in range(5)]
    assert masks[0].abs().max() > 0.1
    torch.testing.assert_close(sum(masks), torch.zeros(3, 4, dtype=torch.float64), atol=1e-12, rtol=0)
    x = torch.full((100,), 1.0, dtype=torch.float64)
    assert abs(float(F.clip_by_norm(x, 1.0).norm()) - 1.0) < 1e-12
    g = F.GaussianNoise(F.DpConfig(epsilon=1.0, delta=1e-5))
    assert abs(g.compute_sigma() - math.sqrt(2 * math.log(1.25e5))) < 1e-12
    noisy = F.add_dp_noise(torch.zeros(20000, dtype=torch.float64), 0.5, seed=3)
    assert abs(float(noisy.std()) - 0.5) < 0.02
    q, lo, hi = F.quantize_tensor(torch.linspace(-1, 1, 101, dtype=torch.float64), 8)
    back = F.dequantize_tensor(q, lo, hi, 8)
    assert float((back - torch.linspace(-1, 1, 101, dtype=torch.float64)).abs().max()) <= 2 / 255 / 2 + 1e-12
    s = F.top_k_sparsify(torch.tensor([0.1, -5.0, 2.0, 0.0]), 0.5)
    assert s.tolist() == [0.0, -5.0, 2.0, 0.0]


def test_federated_rounds_reduce_loss_secure_equals_plain():
    from brain_b200 import federated as F
    torch.manual_seed(0)
    w_true = torch.tensor([[2.0, -1.0]])

    def shard(seed, n):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(n, 2, generator=g)
        return [(x, x @ w_true.t())]

    make = lambda: torch.nn.Linear(2, 1, bias=False)  # noqa: E731
    loss = torch.nn.functional.mse_loss
    w0 = [torch.zeros(1, 2)]
    plain = F.FederatedServer(w0)
    secure = F.FederatedServer(w0, secure=True, seed=5)
    clients = [F.FederatedClient(i, make, shard(i, 16 + 8 * i), loss, lr=0.2, local_epochs=3) for i in range(3)]
    for _ in range(5):
        plain.run_round(clients)
        secure.run_round(clients)
    assert plain.history[-1].mean_client_loss < 0.05 * plain.history[0].mean_client_loss
    torch.testing.assert_close(secure.weights[0], plain.weights[0], atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(plain.weights[0], w_true, atol=0.05, rtol=0)


def _fedavg_rank(rank, world):
    import torch.distributed as dist
    from brain_b200 import federated as F
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = [torch.full((2, 2), float(rank + 1)), torch.tensor([float(10 * rank)])]
        out = F.fed_avg_across_ranks(w, num_samples=rank + 1)
        return [t.tolist() for t in out]
    finally:
        dist.destroy_process_group()


def test_fedavg_across_gloo_ranks():
    res = run_ranks(_fedavg_rank, 2, timeout=120)
    # weights 1 (1 sample) and 2 (2 samples) -> 5/3; biases 0 and 10 -> 20/3
    for r in range(2):
        a, b = res[r]
        assert abs(a[0][0] - 5 / 3) < 1e-6 and abs(b[0] - 20 / 3) < 1e-5


# ------------------------------------------------------------------ text
CORPUS = ["low lower lowest", "new newer newest", "wide wider widest", "low new wide low low"]


def test_bpe_train_and_roundtrip():
    from brain_b200.text import BpeTokenizer, BpeTrainer
    vocab, merges = BpeTrainer.train(CORPUS, vocab_size=40)
    assert merges[0][1] == 0 and len(vocab) <= 40
    tok = BpeTokenizer(vocab, merges)
    assert tok.bpe_segment_word("low") == ["low</w>"]
    enc = tok.encode("lowest newer")
    assert tok.decode(enc.ids) == "lowest newer"
    # deterministic training
    assert BpeTrainer.train(CORPUS, vocab_size=40)[1] == merges


def test_wordpiece_and_char_and_bytelevel():
    from brain_b200.text import ByteLevelEncoder, CharTokenizer, WordPieceTokenizer, WordPieceTrainer
    vocab = WordPieceTrainer.train(CORPUS, vocab_size=60)
    wp = WordPieceTokenizer(vocab)
    pieces = wp.tokenize("Lowest wider")
    assert all(p in vocab for p in pieces) and pieces[0].startswith("low")
    assert wp.decode(wp.encode("lowest wider").ids) == "lowest wider"
    assert wp.tokenize("xyz") == ["[UNK]"]
    ct = CharTokenizer.from_corpus(CORPUS)
    assert ct.decode(ct.encode("lower").ids) == "lower"
    be = ByteLevelEncoder()
    s = "héllo wörld ✓"
    assert be.decode_to_string(be.encode_bytes(s.encode())) == s
    assert be.byte_to_char(ord("A")) == "A" and be.byte_to_char(32) != " "


def test_unigram_viterbi_and_postprocess():
    from brain_b200.text import (PostConfig, PostProcessor, SentencePieceTokenizer, UnigramTrainer,
                                 batch_encode)
    vocab, scores = UnigramTrainer.train(CORPUS * 3, vocab_size=50)
    sp = SentencePieceTokenizer(vocab, scores)
    pieces = sp.tokenize("lowest newer")
    assert "".join(pieces).replace("▁", " ").strip() == "lowest newer"
    assert len(pieces) < len("lowest newer")  # multi-character pieces were learned
    assert sp.decode(sp.encode("lowest newer").ids) == "lowest newer"
    post = PostProcessor(vocab, PostConfig(add_cls_sep=True, max_length=6, pad_to_max_length=True))
    o = post.process_single(sp.encode("wide wider widest lowest"))
    assert len(o.ids) == 6 and o.ids[0] == vocab.cls_id() and vocab.sep_id() in o.ids
    p = post.process_pair(sp.encode("low"), sp.encode("new newer"))
    assert p.type_ids[0] == 0 and p.type_ids[-1] == 1 or p.attention_mask[-1] == 0
    ids, mask = batch_encode(sp, ["low", "newest wider"], PostProcessor(vocab))
    assert ids.shape[0] == 2 and mask.sum(1)[0] < mask.sum(1)[1]
