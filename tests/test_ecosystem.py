"""Ecosystem components beyond the transformer stack (CPU): federated learning, text tokenisers, the
model zoo (RNN, CNN, GNN, diffusion, GAN, RL, audio, neuroevolution), the graph IR, the benchmark
harness and the CLI commands for BrainMind."""
import math
import os

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


# ------------------------------------------------------------------ model zoo
def test_lstm_cell_matches_torch_and_lm_learns():
    from brain_b200.zoo import rnn
    torch.manual_seed(0)
    cell = rnn.LstmCell(5, 7)
    ref = torch.nn.LSTMCell(5, 7)
    with torch.no_grad():
        ref.weight_ih.copy_(cell.ih.weight)
        ref.bias_ih.copy_(cell.ih.bias)
        ref.weight_hh.copy_(cell.hh.weight)
        ref.bias_hh.zero_()
    x, h, c = torch.randn(3, 5), torch.randn(3, 7), torch.randn(3, 7)
    h1, c1 = cell(x, (h, c))
    h2, c2 = ref(x, (h, c))
    torch.testing.assert_close(h1, h2)
    torch.testing.assert_close(c1, c2)
    gru = rnn.GRU(4, 6, num_layers=2, bidirectional=True)
    y, st = gru(torch.randn(2, 5, 4))
    assert y.shape == (2, 5, 12) and len(st) == 4
    lm = rnn.LstmLanguageModel(8, 16, 32)
    seq = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7] * 3] * 4)
    opt = torch.optim.Adam(lm.parameters(), lr=0.03)
    first = None
    for _ in range(60):
        loss = lm.teacher_forcing_loss(seq)
        first = first if first is not None else float(loss)
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < 0.2 * first
    assert lm.greedy(seq[:1, :3], 5)[0, 3:].tolist() == [3, 4, 5, 6, 7]


def test_beam_search_prefers_higher_joint_probability():
    from brain_b200.zoo.rnn import BeamConfig, beam_search
    # greedy picks token 1 first (0.6) but the best two-token sequence is 2 -> 3 (0.4 * 1.0)
    table = {(0,): [0.0, 0.6, 0.4, 0.0], (0, 1): [0.0, 0.0, 0.5, 0.5], (0, 2): [0.0, 0.0, 0.0, 1.0]}

    def step(seqs):
        out = []
        for s in seqs:
            p = torch.tensor(table.get(tuple(s), [0.25] * 4))
            out.append(torch.log(p + 1e-12))
        return out
    best = beam_search(step, 0, BeamConfig(beam_width=2, max_len=3, length_penalty=0.0))
    assert best.tokens == [0, 2, 3]


def test_gcn_matches_dense_formula_and_classifier_trains():
    from brain_b200.zoo import gnn
    torch.manual_seed(0)
    edges = [(0, 1), (1, 2), (2, 0), (3, 4), (4, 5), (5, 3), (2, 3)]
    g = gnn.Graph.from_undirected(edges, 6)
    x = torch.randn(6, 4)
    layer = gnn.GcnLayer(4, 3, bias=False)
    A = torch.zeros(6, 6)
    for a, b in edges:
        A[a, b] = A[b, a] = 1
    A += torch.eye(6)
    d = A.sum(1).rsqrt()
    dense = (d[:, None] * A * d[None]) @ (x @ layer.lin.weight.t())
    torch.testing.assert_close(layer(g, x), dense)
    gat = gnn.GatLayer(4, 2, num_heads=3)
    assert gat(g, x).shape == (6, 6)
    pooled = gnn.global_mean_pool(x, torch.tensor([0, 0, 0, 1, 1, 1]), 2)
    torch.testing.assert_close(pooled[1], x[3:].mean(0))
    for kind in ("gcn", "sage", "gin", "gat"):
        model = gnn.GnnNodeClassifier(4, 8, 2, kind)
        y = torch.tensor([0, 0, 0, 1, 1, 1])
        feats = torch.eye(6)[:, :4] + 0.1
        opt = torch.optim.Adam(model.parameters(), lr=0.05)
        for _ in range(80):
            loss = torch.nn.functional.cross_entropy(model(g, feats), y)
            opt.zero_grad()
            loss.backward()
            opt.step()
        assert (model(g, feats).argmax(1) == y).float().mean() >= 5 / 6, kind


def test_diffusion_schedules_samplers_and_training():
    from brain_b200.zoo import diffusion as D
    for s in (D.LinearSchedule(100), D.CosineSchedule(100), D.ScaledLinearSchedule(100)):
        ac = s.alphas_cumprod
        assert bool((ac[1:] < ac[:-1]).all()) and 0 < float(ac[-1]) < float(ac[0]) <= 1
    # with the exact noise predictor for a point mass at x0, deterministic DDIM returns x0
    sched = D.LinearSchedule(200)
    x0 = torch.tensor([[1.5, -0.5]])

    def oracle(x, t, cond=None):
        ac = sched.at("alphas_cumprod", t, x)
        return (x - ac.sqrt() * x0) / (1 - ac).sqrt()
    out = D.DdimSampler(sched, eta=0.0).sample(oracle, (1, 2), num_steps=20, generator=torch.Generator().manual_seed(0))
    torch.testing.assert_close(out, x0, atol=1e-4, rtol=0)
    ddpm = D.DdpmSampler(D.LinearSchedule(50)).sample(lambda x, t, c=None: torch.zeros_like(x), (4, 2),
                                                      generator=torch.Generator().manual_seed(1))
    assert ddpm.shape == (4, 2) and torch.isfinite(ddpm).all()
    torch.manual_seed(0)
    model = D.MlpDenoiser(2, 64, num_classes=2)
    opt = torch.optim.Adam(model.parameters(), lr=3e-3)
    g = torch.Generator().manual_seed(2)
    data = torch.randn(256, 2, generator=g) * 0.1 + torch.tensor([1.0, -1.0])
    losses = []
    for _ in range(150):
        loss = D.diffusion_loss(model, sched, data, generator=g)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert sum(losses[-20:]) / 20 < 0.7 * sum(losses[:20]) / 20
    guided = D.guided_eps(model, data[:3], torch.tensor([5, 5, 5]), torch.tensor([0, 1, 0]), 2.0)
    assert guided.shape == (3, 2)


def test_gan_losses_penalties_and_training():
    from brain_b200.zoo import gan
    lin = torch.nn.Linear(3, 1)
    with torch.no_grad():
        lin.weight.copy_(torch.tensor([[0.6, 0.8, 0.0]]))  # unit-norm gradient everywhere
    real, fake = torch.randn(8, 3), torch.randn(8, 3)
    assert float(gan.gradient_penalty(lambda x: lin(x).squeeze(-1), real, fake)) < 1e-10
    assert abs(float(gan.r1_penalty(lambda x: lin(x).squeeze(-1), real, gamma=2.0)) - 1.0) < 1e-6
    d_r, d_f = torch.tensor([2.0, 0.5]), torch.tensor([-2.0, 0.5])
    assert float(gan.hinge_loss_d(d_r, d_f)) == pytest.approx(0.25 + 0.75)
    assert float(gan.wgan_loss_d(d_r, d_f)) == pytest.approx(-0.75 - 1.25)
    torch.manual_seed(0)
    G, Dn = gan.MlpGenerator(4, 1, 32), gan.MlpDiscriminator(1, 32)
    og, od = torch.optim.Adam(G.parameters(), 2e-3, betas=(0.5, 0.9)), torch.optim.Adam(Dn.parameters(), 2e-3, betas=(0.5, 0.9))
    g = torch.Generator().manual_seed(0)
    for _ in range(300):
        real = torch.randn(64, 1, generator=g) * 0.5 + 3.0
        gan.train_step(G, Dn, og, od, real, loss="bce", generator=g)
    mean = float(G(torch.randn(512, 4)).mean())
    assert abs(mean - 3.0) < 0.75
    img = gan.DcganGenerator(16, 1, 16, 3)(torch.randn(2, 16))
    assert img.shape == (2, 1, 32, 32)
    assert gan.DcganDiscriminator(1, 16, 3)(img).shape == (2,)
    assert gan.DcganDiscriminator(1, 16, 3, patch=True)(img).shape[0] == 2


def test_rl_gae_buffers_and_dqn_solves_gridworld():
    from brain_b200.zoo import rl
    adv, ret = rl.gae([1.0, 0.0, 1.0], [0.5, 0.5, 0.5], [False, False, True], gamma=0.9, lam=1.0)
    mc = rl.discounted_returns([1.0, 0.0, 1.0], [False, False, True], 0.9)
    torch.testing.assert_close(ret.float(), mc.float())
    obj = rl.PpoClippedObjective(0.2)
    assert float(obj.compute_policy_loss(torch.tensor([1.5]), torch.tensor([1.0]))) == pytest.approx(-1.2)
    pb = rl.PrioritizedReplayBuffer(10)
    for i in range(10):
        pb.push(rl.Transition(torch.zeros(2), 0, float(i), torch.zeros(2), False))
    batch, w = pb.sample_batch(4)
    pb.update_priorities([1.0] * 4)
    assert len(batch) == 4 and float(w.max()) == 1.0
    env = rl.GridWorldEnv(3, 3, max_steps=30)
    agent = rl.DqnAgent(9, 4, rl.DqnConfig(epsilon_decay_steps=600, target_update=50, batch_size=32, lr=3e-3), seed=0)
    s = env.reset()
    for _ in range(1500):
        a = agent.act(s)
        s2, r, d, _ = env.step(a)
        agent.step(rl.Transition(s, a, r, s2, d))
        s = env.reset() if d else s2
    assert rl.evaluate(rl.GridWorldEnv(3, 3, max_steps=30), lambda o: agent.act(o, greedy=True), 1) > 0.9
    cliff, lake = rl.CliffWalkingEnv(), rl.FrozenLakeEnv(4)
    assert cliff.reset().shape == (48,) and cliff.step(1)[1] == -100.0
    assert (0, 0) not in lake.holes
    venv = rl.VectorEnv(lambda: rl.GridWorldEnv(2, 2, 5), 3)
    o, r, d = venv.step([1, 1, 1])
    assert o.shape == (3, 4)
    ppo = rl.PpoAgent(4, 4, rl.PpoConfig(rollout=32, epochs=2))
    assert math.isfinite(ppo.update(rl.GridWorldEnv(2, 2, 10)))
    a2c = rl.A2cAgent(4, 4)
    assert math.isfinite(a2c.update(rl.GridWorldEnv(2, 2, 10)))


def test_audio_features_and_wav(tmp_path):
    from brain_b200.zoo import audio as A
    sr = 16000
    t = torch.arange(sr, dtype=torch.float32) / sr
    x = 0.5 * torch.sin(2 * math.pi * 440 * t)
    mag, ph = A.stft(x)
    back = A.istft(mag, ph, length=x.numel())
    torch.testing.assert_close(back, x, atol=1e-4, rtol=0)
    peak_bin = int(mag.mean(-1).argmax())
    assert abs(peak_bin * sr / 512 - 440) < sr / 512
    fb = A.mel_filterbank(40, 512, sr)
    peaks = fb.argmax(1)
    assert bool((peaks[1:] >= peaks[:-1]).all()) and fb.shape == (40, 257)
    m = A.mfcc(x)
    assert m.shape[0] == 13 and torch.isfinite(m).all()
    cm = A.apply_cmvn(m)
    assert float(cm.mean(-1).abs().max()) < 1e-4
    y = A.resample(x, sr, 8000)
    assert y.numel() == 8000
    mag8, _ = A.stft(y)
    assert abs(int(mag8.mean(-1).argmax()) * 8000 / 512 - 440) < 8000 / 512 * 1.5
    sil = torch.cat([torch.zeros(4000), x[:4000]])
    vad = A.energy_vad(sil)
    assert not bool(vad[0]) and bool(vad[-1])
    p = str(tmp_path / "a.wav")
    A.write_wav(p, x[:1000], sr)
    r, sr2 = A.read_wav(p)
    assert sr2 == sr and r.shape == (1, 1000)
    torch.testing.assert_close(r[0], x[:1000], atol=1 / 16384, rtol=0)
    aug = A.spec_augment(mag, 5, 10, generator=torch.Generator().manual_seed(0))
    assert aug.shape == mag.shape


def test_neuroevolution_ga_es_cmaes():
    from brain_b200.zoo import neuroevolution as N
    target = torch.tensor([3.0, -2.0, 1.0, 0.5], dtype=torch.float64)
    f = lambda g: -float(((g - target) ** 2).sum())  # noqa: E731
    res = N.Ga(N.GaConfig(population=48, genome_len=4, generations=80, mutation_sigma=0.2), seed=0).run(f)
    assert res.best_fitness > -0.1
    fb = lambda P: -((P - target) ** 2).sum(1)  # noqa: E731
    res2 = N.Ga(N.GaConfig(population=48, genome_len=4, generations=80, crossover="blend", selection="rank"),
                seed=1).run(fb, batched=True)
    assert res2.best_fitness > -0.5
    x, fx = N.es_one_plus_one(f, torch.zeros(4), iters=600)
    assert fx > -1e-3
    best, bf = N.Cmaes(N.CmaesConfig(dim=4, sigma=1.0, max_iters=150), seed=0).optimize(fb, batched=True)
    assert bf > -1e-6
    net = torch.nn.Linear(2, 1)
    X = torch.randn(32, 2)
    Y = X @ torch.tensor([[1.0], [-1.0]])
    r = N.evolve_network(net, lambda m: -float(((m(X) - Y) ** 2).mean()),
                         N.GaConfig(population=40, generations=60, mutation_sigma=0.2))
    assert r.best_fitness > -0.05


def test_cv_blocks_detection_and_segmentation():
    from brain_b200.zoo import cv
    torch.manual_seed(0)
    net = cv.ResNetLite(3, (8, 16, 32), (1, 1, 1), 5)
    x = torch.randn(2, 3, 32, 32)
    feats = net.features(x)
    assert [f.shape[-1] for f in feats] == [32, 16, 8] and net(x).shape == (2, 5)
    pyr = cv.FPN([8, 16, 32], 16)(feats)
    assert [p.shape[1] for p in pyr] == [16, 16, 16]
    assert cv.DepthwiseSeparableConv(8, 12)(feats[0]).shape == (2, 12, 32, 32)
    assert cv.GhostConv(8, 12)(feats[0]).shape == (2, 12, 32, 32)
    assert cv.WSConv2d(8, 4, 3, padding=1)(feats[0]).shape == (2, 4, 32, 32)
    boxes = torch.tensor([[0, 0, 10, 10], [1, 1, 11, 11], [20, 20, 30, 30.0]])
    scores = torch.tensor([0.9, 0.8, 0.7])
    assert cv.nms(boxes, scores, 0.5).tolist() == [0, 2]
    iou = cv.compute_iou(boxes[:1], boxes[1:2])
    assert float(iou) == pytest.approx(81 / 119, rel=1e-5)
    anchors = cv.AnchorGenerator((16.0, 32.0), (0.5, 1.0, 2.0)).generate_grid_anchors(4, 5, 8)
    assert anchors.shape == (4 * 5 * 6, 4)
    gt = anchors[:10] + torch.tensor([1.0, -2.0, 3.0, 1.0])
    torch.testing.assert_close(cv.decode_boxes(cv.encode_boxes(gt, anchors[:10]), anchors[:10]), gt, atol=1e-4, rtol=1e-4)
    rois = cv.roi_align(torch.arange(64.0).view(1, 8, 8), torch.tensor([[0.0, 0.0, 8.0, 8.0]]), 4)
    assert rois.shape == (1, 1, 4, 4)
    head = cv.FcnHead(8, 3)
    logits = head(feats[0], (32, 32))
    tgt = torch.randint(0, 3, (2, 32, 32))
    perfect = torch.nn.functional.one_hot(tgt, 3).permute(0, 3, 1, 2).float() * 50
    assert float(cv.dice_loss(perfect, tgt)) < 1e-3 < float(cv.dice_loss(logits, tgt))
    img = torch.rand(3, 16, 16)
    assert cv.random_crop(img, (12, 12), padding=2).shape == (3, 12, 12)
    assert cv.color_jitter(img).shape == img.shape
    xm, ym = cv.mixup(torch.rand(4, 3, 8, 8), torch.eye(4))
    xc, yc = cv.cutmix(torch.rand(4, 3, 8, 8), torch.eye(4))
    torch.testing.assert_close(ym.sum(1), torch.ones(4))
    torch.testing.assert_close(yc.sum(1), torch.ones(4))


# ------------------------------------------------------------------ graph IR / compile / ONNX
def _mlp_graph():
    from brain_b200.graph import GraphIr
    torch.manual_seed(0)
    g = GraphIr("mlp")
    x = g.add_input("x", (4, 8))
    w1, b1 = g.constant("w1", torch.randn(16, 8)), g.constant("b1", torch.randn(16))
    w2 = g.constant("w2", torch.randn(8, 16))
    h = g.add_node("linear", [x, w1, b1])
    h = g.add_node("gelu", [h])
    y = g.add_node("linear", [h, w2])
    y = g.add_node("add", [y, x])
    # redundant work the passes remove: a duplicate, a double transpose, dead code, foldable constants
    dup = g.add_node("gelu", [g.add_node("linear", [x, w1, b1])])
    t = g.add_node("transpose", [g.add_node("transpose", [y])])
    c = g.add_node("mul", [g.constant("two", torch.tensor(2.0)), g.constant("three", torch.tensor(3.0))])
    out = g.add_node("mul", [t, c])
    g.add_node("exp", [dup])  # dead
    g.mark_output(out)
    return g


def test_graph_passes_interpreter_and_plans():
    from brain_b200 import graph as G
    g = _mlp_graph()
    assert G.verify(g) == []
    G.infer_shapes(g)
    x = torch.randn(4, 8)
    ref = G.GraphInterpreter().run(g, [x])[0]
    h = g.clone()
    rep = G.optimize(h, 2)
    assert rep.nodes_after < rep.nodes_before and G.verify(h) == []
    ops = [n.op for n in h.nodes]
    assert "transpose" not in ops and "exp" not in ops and ops.count("linear") == 2
    torch.testing.assert_close(G.GraphInterpreter().run(h, [x])[0], ref)
    assert rep.fusion.num_fused() >= 2  # linear+gelu, linear+add
    d = G.diff_graphs(g, h)
    assert d.removed_ops and not d.added_ops
    G.infer_shapes(h)
    assert G.estimate_flops(h) >= 2 * 4 * 16 * 8 + 2 * 4 * 8 * 16
    plan = G.plan_memory(h)
    assert len(plan.buffer_bytes) < len(plan.assignment)  # buffers were reused
    ip = G.plan_inplace_operations(h)
    assert ip.inplace
    back = G.from_json(G.to_json(h))
    torch.testing.assert_close(G.GraphInterpreter().run(back, [x])[0], ref)
    assert G.to_dot(h).startswith('digraph "mlp"')
    cache = G.JitCache()
    cache.get_or_compile(g)
    cache.get_or_compile(g)
    assert cache.hits == 1 and cache.misses == 1


def test_graph_from_fx_and_onnx_roundtrip(tmp_path):
    from brain_b200 import graph as G
    from brain_b200 import onnx as O

    class Net(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.a = torch.nn.Linear(6, 12)
            self.act = torch.nn.ReLU()
            self.b = torch.nn.Linear(12, 3)

        def forward(self, x):
            return torch.tanh(self.b(self.act(self.a(x)))) * 2.0

    torch.manual_seed(1)
    net = Net()
    x = torch.randn(5, 6)
    g = G.from_fx(net, x)
    torch.testing.assert_close(G.GraphInterpreter().run(g, [x])[0], net(x))
    data = O.export_onnx(g, str(tmp_path / "m.onnx"))
    assert O.check_model(data) == []
    g2 = O.import_onnx(open(tmp_path / "m.onnx", "rb").read())
    torch.testing.assert_close(G.GraphInterpreter().run(g2, [x])[0], net(x))
    # extra op coverage through export -> import
    h = G.GraphIr("ops")
    a = h.add_input("a", (2, 3, 4))
    t = h.add_node("transpose", [a], {"dim0": 1, "dim1": 2})
    r = h.add_node("reshape", [t], {"shape": [2, 12]})
    s = h.add_node("softmax", [r], {"dim": -1})
    m = h.add_node("mean", [s], {"dim": 1, "keepdim": True})
    q = h.add_node("rsqrt", [h.add_node("add", [m, h.constant("one", torch.tensor(1.0))])])
    n = h.add_node("rms_norm", [r, h.constant("g", torch.ones(12))], {"eps": 1e-6})
    h.mark_output(q, h.add_node("swiglu", [n]))
    G.infer_shapes(h)
    xa = torch.randn(2, 3, 4)
    want = G.GraphInterpreter().run(h, [xa])
    got = G.GraphInterpreter().run(O.import_onnx(O.export_onnx(h)), [xa])
    for u, v in zip(got, want):
        torch.testing.assert_close(u, v)


# ------------------------------------------------------------------ CLI: repl / script / init / space
def test_cli_repl_script_init_and_space(tmp_path, capsys):
    import io
    import os
    import subprocess
    import sys

    import importlib

    from brain_b200.cli.repl import ReplState, run_repl
    cli = importlib.import_module("brain_b200.cli.main")

    lines = []
    st = ReplState(device="cpu", out=lines.append)
    st.eval_line("a = ones(2, 3)")
    st.eval_line("b = add(mul(a, 2), ones(2, 3))")
    st.eval_line("sum(b)")
    assert lines[-1] == "ans: [] = 18"
    st.eval_line("c = matmul(b, transpose(a))")
    assert lines[-1] == "c = [2, 2]"
    st.eval_line(":vars")
    assert "  c: [2, 2]" in lines
    out = []
    run_repl(io.StringIO("x = zeros(4)\nfoo(x)\n:quit\ny = ones(1)\n"), out=out.append)
    assert any("unknown function 'foo'" in s for s in out) and out[-1] == "Goodbye!"
    script = tmp_path / "s.bn"
    script.write_text("# comment\nx = randn(3, 3)\n\ny = add(x, x)\n")
    assert cli.main(["script", str(script)]) == 0
    script.write_text("x = ones(2)\ny = sub(x)\n")
    assert cli.main(["script", str(script)]) == 1
    assert cli.main(["script", str(tmp_path / "missing.bn")]) == 3
    proj = tmp_path / "proj"
    assert cli.main(["init", str(proj)]) == 0
    assert (proj / "brain.toml").exists() and (proj / "src" / "model.py").exists()
    assert cli.main(["init", str(proj)]) == 3
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "train.py"], cwd=proj, capture_output=True, text=True, timeout=300,
                       env={**os.environ, "PYTHONPATH": root, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr[-2000:]
    teach = tmp_path / "t.txt"
    teach.write_text("the sky is blue. the grass is green.\n" * 4)
    bn = tmp_path / "mind.bn"
    assert cli.main(["new", str(bn), "--teach", str(teach), "--steps", "5"]) == 0 and bn.exists()
    assert cli.main(["chat", str(bn), "--message", "hello"]) == 0
    assert "> hello" in capsys.readouterr().out
    assert cli.main(["space"]) == 2
    assert cli.main(["version"]) == 0


# ------------------------------------------------------------------ benchmark harness
def test_bench_harness_statistics_welch_baseline_reports(tmp_path):
    from brain_b200.bench import harness as H
    s = H.Statistics.compute([1, 2, 3, 4, 100])
    assert s.median == 3 and s.min == 1 and s.max == 100 and s.p50 == 3 and s.iqr == 2
    assert s.ci_95_lower < s.mean < s.ci_95_upper and s.skewness > 0
    assert H.Statistics.trimmed_mean([1, 2, 3, 4, 100], 20) == 3
    # Welch: scipy's ttest_ind(equal_var=False) is the oracle
    from scipy import stats as st
    a, b = [10.0, 11.0, 9.5, 10.2, 10.8], [12.0, 12.5, 11.8, 13.1, 12.2, 12.9]
    t, p = H.welch_t_test(a, b)
    ref = st.ttest_ind(b, a, equal_var=False)
    assert abs(t - ref.statistic) < 1e-9 and abs(p - ref.pvalue) < 1e-9
    cfg = H.BenchConfig("op", 0, 5)
    base, slow = H.BenchResult(cfg, [100.0, 101, 99, 100, 100.5]), H.BenchResult(cfg, [120.0, 121, 119, 120, 122])
    c = H.compare_runs(base, slow)
    assert c.verdict == "regression" and c.percent_change > 15
    store = H.BaselineStore(str(tmp_path / "b.json"))
    store.add(base)
    store.save()
    store2 = H.BaselineStore(str(tmp_path / "b.json"))
    with pytest.raises(RuntimeError, match="regressed"):
        store2.evaluate_regressions([slow], 5.0)
    assert store2.evaluate_regressions([base], 5.0)[0].verdict == "no_change"
    r = H.Runner.run_benchmark(H.BenchConfig("sleep", 1, 4), lambda: sum(range(1000)))
    assert r.stats.count == 4 and r.mean_nanos() > 0
    sw = H.Runner.run_sweep("sum", [10, 1000], lambda n: (lambda: sum(range(n))), warmup_iters=1, measure_iters=3)
    assert len(sw) == 2
    for fmt in (H.format_console, H.format_markdown, H.format_csv, H.format_json, H.format_html):
        assert "sleep" in fmt([r])
    prom = H.PrometheusExporter.export([r])
    assert 'brain_bench_mean_seconds{name="sleep"}' in prom
    assert "brain.bench.mean_ns" in H.OpenTelemetryExporter.export([r])
    h = H.LogHistogram()
    for v in range(1, 10001):
        h.record(v * 1000)
    assert h.count() == 10000 and abs(h.percentile(50) / 5e6 - 1) < 0.2 and abs(h.percentile(99) / 9.9e6 - 1) < 0.2
    assert H.HardwareInfo.probe().cpu_count > 0
    assert H.EnergyEstimator.estimate_joules(2.0, 500.0) == 1000.0
    suite = H.KernelSuite.run(n=128, iters=2, device="cpu")
    assert [x.config.name for x in suite] == ["gemm", "rms_norm", "softmax_cross_entropy"] and suite[0].tflops() > 0


# ------------------------------------------------------------------ export
def test_export_formats_zip_quant_and_bn_conversion(tmp_path):
    import json as _json
    import zipfile

    from brain_b200 import export as E
    from brain_b200 import graph as G
    from brain_b200.checkpoint.formats import BrainModelFile
    from brain_b200.utils.safetensors import load_safetensors

    g = _mlp_graph()
    G.optimize(g, 2)
    G.infer_shapes(g)
    x = torch.randn(4, 8)
    s = E.export_all(g, str(tmp_path / "out"), example_inputs=[x])
    assert set(s.files) == {"onnx", "webnn", "tflite", "coreml"} and not s.skipped
    web = _json.loads(open(s.files["webnn"]).read())
    assert [o["op"] for o in web["operations"]][:2] == ["gemm", "gelu"]
    tfl = _json.loads(open(s.files["tflite"]).read())
    assert {c["builtin_code"] for c in tfl["operator_codes"]} >= {"FULLY_CONNECTED", "GELU"}
    with zipfile.ZipFile(s.files["coreml"]) as z:
        assert set(z.namelist()) == {"model.mil", "weights.bin", "manifest.json"}
        assert "linear(" in z.read("model.mil").decode()
    h = G.GraphIr("norm")
    a = h.add_input("a", (2, 4))
    h.mark_output(h.add_node("rms_norm", [a]))
    rep = E.supported_ops_report(h, E.ExportFormat.TFLITE)
    assert not rep.ok() and rep.unsupported == ["rms_norm"]
    s2 = E.export_all(h, str(tmp_path / "out2"))
    assert "tflite" in s2.skipped and "onnx" in s2.files
    with pytest.raises(E.ExportError):
        E.verify_export(torch.ones(3), torch.zeros(3), 0.5)
    w = {"w": torch.randn(16, 32), "b": torch.randn(16)}
    err = E.export_quantized_safetensors(w, str(tmp_path / "q.safetensors"))
    q, meta = load_safetensors(str(tmp_path / "q.safetensors"))
    assert q["w"].dtype == torch.int8 and q["w.scale"].shape == (16,) and meta["format"] == "brain-int8"
    assert err["w"] <= float(w["w"].abs().max()) / 127 * 0.51
    m = BrainModelFile("net").with_meta("arch", "mlp")
    m.add_tensor("layer.weight", torch.randn(3, 2, dtype=torch.float64))
    m.save_file(str(tmp_path / "m.bn"))
    E.convert_bn_to_safetensors(str(tmp_path / "m.bn"), str(tmp_path / "m.safetensors"))
    r = E.convert_safetensors_to_bn(str(tmp_path / "m.safetensors"), str(tmp_path / "m2.bn"))
    m2 = BrainModelFile.load_file(str(tmp_path / "m2.bn"))
    assert r.num_tensors == 1 and m2.name == "net" and m2.metadata["arch"] == "mlp"
    torch.testing.assert_close(m2.archive.get("layer.weight").double(), m.archive.get("layer.weight").double())


# ------------------------------------------------------------------ data: native loader, streams, datasets
def test_native_token_loader_matches_oracle_and_resumes(tmp_path):
    import numpy as np
    from brain_b200 import data as D
    toks = np.random.default_rng(0).integers(0, 60000, size=50000).astype(np.uint16)
    p = str(tmp_path / "tok.bin")
    D.write_token_file(p, toks)
    L = D.NativeTokenLoader(p, batch=3, seq=16, seed=5, rank=1, world=2, workers=3, depth=2, pin_memory=False)
    seen = []
    for b in range(8):
        x, y = L.next()
        starts = D.splitmix64_window_starts(5, b, 1, 2, 3, 16, len(toks))
        ref = torch.stack([torch.from_numpy(toks[s:s + 17].astype(np.int64)) for s in starts])
        assert torch.equal(x, ref[:, :-1]) and torch.equal(y, ref[:, 1:])
        seen.append(ref)
    ck = L.checkpoint()
    st = L.stats()
    assert st["consumed"] == 8 and st["tokens"] == len(toks) and ck.sample_offset == 8
    L.close()
    R = D.NativeTokenLoader(p, batch=3, seq=16, seed=5, rank=1, world=2, start_batch=ck.sample_offset, pin_memory=False)
    x, _ = R.next()
    ref = torch.stack([torch.from_numpy(toks[s:s + 17].astype(np.int64))
                       for s in D.splitmix64_window_starts(5, 8, 1, 2, 3, 16, len(toks))])
    assert torch.equal(x, ref[:, :-1]) and torch.equal(R.batch_at(0), seen[0])
    R.close()
    other = D.NativeTokenLoader(p, batch=3, seq=16, seed=5, rank=0, world=2, pin_memory=False)
    assert not torch.equal(other.batch_at(0), seen[0])
    other.close()
    with pytest.raises(RuntimeError, match="I/O"):
        D.NativeTokenLoader(str(tmp_path / "missing.bin"), batch=1, seq=4)


def test_streams_cache_metrics_and_codecs():
    from brain_b200 import data as D
    s = D.StreamDataset(lambda: iter(range(10)))
    assert list(s.shard(1, 3)) == [1, 4, 7]
    assert [b.tolist() for b in s.batches(4)] == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    c = D.CachedDataset(D.SyntheticTokens(100, 8, 10), capacity=2)
    a = c[0]
    assert torch.equal(c[0][0], a[0]) and c.cache.hits == 1 and c.cache.misses == 1
    c[1], c[2], c[0]
    assert c.cache.misses == 4  # index 0 was evicted
    m = D.PipelineMetrics()
    n = sum(1 for _ in m.wrap(D.DataLoader(D.SyntheticTokens(100, 8, 10), batch_size=4)))
    assert n == 3 and m.samples == 10 and m.throughput() > 0
    x, lengths = D.pad_collate([torch.ones(2), torch.ones(4), torch.ones(3)], -1.0)
    assert x.shape == (3, 4) and lengths.tolist() == [2, 4, 3] and float(x[0, 3]) == -1.0
    cat = D.ConcatDataset(D.SyntheticTokens(100, 4, 3, seed=1), D.SyntheticTokens(100, 4, 2, seed=2))
    assert len(cat) == 5 and torch.equal(cat[4][0], D.SyntheticTokens(100, 4, 2, seed=2)[1][0])
    assert D.rle_decode(D.rle_encode([1, 1, 2, 2, 2, 3])) == [1, 1, 2, 2, 2, 3]
    assert D.delta_decode(D.delta_encode([5, 7, 7, 10])) == [5, 7, 7, 10]
    ck = D.PipelineCheckpoint.from_dict(D.PipelineCheckpoint(2, 40).to_dict())
    assert (ck.epoch, ck.sample_offset) == (2, 40)


def test_dataset_library(tmp_path):
    import numpy as np
    from brain_b200.data import datasets as DS
    from brain_b200.zoo.audio import write_wav
    csvp = tmp_path / "t.csv"
    csvp.write_text("a,b,label\n1,2,0\n3,4,1\n5,6,1\n")
    ds = DS.TabularDataset(str(csvp), label_column="label")
    assert len(ds) == 3 and ds.feature_names == ["a", "b"] and ds[1][1].item() == 1
    st = DS.dataset_stats(ds)
    assert st.class_counts == {0: 1, 1: 2} and st.imbalance_ratio() == 2.0
    torch.testing.assert_close(st.feature_mean, torch.tensor([3.0, 4.0]))
    txt = tmp_path / "t.txt"
    txt.write_text("pos\tgood movie\nneg\tbad film\n\npos\tgreat\n")
    tl = DS.TextLineDataset(str(txt), label_sep="\t")
    assert len(tl) == 3 and tl.label_names == ["neg", "pos"] and tl[1] == ("bad film", 0)
    for c in ("cat", "dog"):
        os.makedirs(tmp_path / "img" / c)
        np.save(tmp_path / "img" / c / "0.npy", np.full((4, 4, 3), 255 if c == "dog" else 0, np.uint8))
    im = DS.ImageArrayDataset(str(tmp_path / "img"), transform=DS.Compose(DS.Normalize([0.5] * 3, [0.5] * 3)))
    x, k = im[1]
    assert x.shape == (3, 4, 4) and k == 1 and float(x.mean()) == 1.0
    os.makedirs(tmp_path / "aud" / "beep")
    write_wav(str(tmp_path / "aud" / "beep" / "a.wav"), torch.sin(torch.arange(1600.0)), 16000)
    au = DS.AudioDataset(str(tmp_path / "aud"), sample_rate=8000)
    assert au[0][0].numel() == 800
    sp = DS.random_split_indices(10, 0.6, 0.2)
    assert len(sp.train) == 6 and len(sp.val) == 2 and sorted(sp.train + sp.val + sp.test) == list(range(10))
    folds = DS.k_fold_split_indices(10, 3)
    assert sorted(sum((v for _, v in folds), [])) == list(range(10))
    tr, va = DS.stratified_split_indices([0] * 10 + [1] * 10, 0.7)
    assert len(tr) == 14 and len(va) == 6
    bal = DS.balance_indices([0] * 5 + [1] * 2)
    assert len(bal) == 10
    assert DS.WorkerPool(3).map(lambda v: v * v, range(5)) == [0, 1, 4, 9, 16]
    assert "csv" in DS.list_datasets() and len(DS.create_dataset("synthetic_tokens", vocab_size=10, seq_len=4,
                                                                  num_samples=3)) == 3
    with pytest.raises(KeyError):
        DS.create_dataset("nope")


# ------------------------------------------------------------------ device / BLAS / pruning / pipelines / parsers
def test_device_blas_and_quantized_tensor():
    from brain_b200.device import (CpuBackend, Device, DeviceGuard, DeviceList, DeviceType, QuantizedTensor, blas,
                                   backend_for)
    d = Device.parse("cuda:3")
    assert d.type == DeviceType.CUDA and d.index == 3 and d.name() == "cuda:3" and d.is_accelerator()
    assert Device.parse("CPU").is_cpu() and DeviceType.METAL.has_unified_memory() and not DeviceType.CUDA.has_unified_memory()
    with pytest.raises(ValueError):
        Device.parse("quantum:0")
    with pytest.raises(RuntimeError):
        Device.vulkan(0).to_torch()
    assert DeviceList().cpu() == Device.cpu() and Device.cpu().is_available()
    with DeviceGuard("cpu") as dev:
        assert dev.is_cpu()
    assert isinstance(backend_for("cpu"), CpuBackend)
    x, y = torch.tensor([1.0, 2.0, 3.0]), torch.tensor([4.0, 5.0, 6.0])
    assert float(blas.dot(x, y)) == 32.0 and blas.iamax(torch.tensor([1.0, -7.0, 3.0])) == 1
    assert blas.axpy(2.0, x, y.clone()).tolist() == [6.0, 9.0, 12.0]
    assert abs(float(blas.nrm2(x)) - 14 ** 0.5) < 1e-6 and float(blas.asum(-x)) == 6.0
    a, b = torch.randn(3, 4), torch.randn(5, 4)
    c = torch.randn(3, 5)
    torch.testing.assert_close(blas.gemm(a, b, c.clone(), 2.0, 0.5, trans_b=True), 2 * a @ b.t() + 0.5 * c)
    torch.testing.assert_close(blas.gemv(1.0, a, torch.ones(4), 0.0, torch.zeros(3)), a.sum(1))
    torch.testing.assert_close(blas.ger(1.0, torch.ones(2), torch.ones(3), torch.zeros(2, 3)), torch.ones(2, 3))
    p, q = torch.tensor([1.0]), torch.tensor([0.0])
    blas.rot(p, q, 0.0, 1.0)
    assert p.item() == 0.0 and q.item() == -1.0
    t = torch.linspace(-2, 5, 50)
    qt = QuantizedTensor.quantize(t)
    assert qt.data.dtype == torch.int8 and float((qt.dequantize() - t).abs().max()) <= qt.scale * 0.51
    qs = QuantizedTensor.quantize(t, symmetric=True)
    assert qs.zero_point == 0 and float((qs.dequantize() - t).abs().max()) <= qs.scale * 0.51


def test_pruning_masks_and_module_pruning():
    from brain_b200.nn.pruning import PruningMask, prune_module, remove_pruning
    w = torch.tensor([[0.1, -3.0], [0.5, 2.0]])
    m = PruningMask.from_magnitude(w, 0.5)
    assert m.apply(w).tolist() == [[0.0, -3.0], [0.0, 2.0]] and m.sparsity() == 0.5
    rows = PruningMask.structured_rows(torch.tensor([[1.0, 1.0], [5.0, 5.0], [0.1, 0.0]]), 1 / 3)
    assert rows.mask.tolist() == [[True, True], [True, True], [False, False]]
    net = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.ReLU(), torch.nn.Linear(16, 4))
    masks = prune_module(net, 0.75, global_=True)
    zeros = sum(int((p == 0).sum()) for n, p in net.named_parameters() if n in masks)
    total = sum(p.numel() for n, p in net.named_parameters() if n in masks)
    assert abs(zeros / total - 0.75) < 0.02
    opt = torch.optim.SGD(net.parameters(), lr=0.5)
    net(torch.randn(4, 8)).sum().backward()
    opt.step()
    net(torch.randn(1, 8))  # the hook re-applies the masks
    assert sum(int((p == 0).sum()) for n, p in net.named_parameters() if n in masks) >= zeros
    remove_pruning(net)


def test_transformer_builder_and_pipelines():
    from brain_b200.models.config import BertLiteConfig, GptLiteConfig
    from brain_b200.models.generate import GenerationConfig
    from brain_b200.models.pipelines import (SequenceClassificationPipeline, TextGenerationPipeline,
                                             TransformerBuilder)
    cfg = TransformerBuilder().arch("gpt").vocab_size(64).hidden_dim(32).num_layers(1).num_heads(4).max_seq_len(16).build_config()
    assert cfg.learned_positions and not cfg.rope and cfg.norm == "layer"
    with pytest.raises(ValueError, match="divisible"):
        TransformerBuilder().hidden_dim(30).num_heads(4).build_config()
    for arch in ("llama", "gpt", "bert"):
        m = TransformerBuilder().arch(arch).vocab_size(64).hidden_dim(32).num_layers(1).num_heads(4) \
            .intermediate_dim(64).max_seq_len(16).build_model()
        assert type(m).__name__ == {"llama": "LlamaLite", "gpt": "GptLite", "bert": "BertLite"}[arch]
    cls = SequenceClassificationPipeline(BertLiteConfig(vocab_size=50, hidden_dim=32, num_layers=1, num_heads=4,
                                                        intermediate_dim=64, max_seq_len=16, num_labels=3))
    assert cls.predict_class([1, 2, 3]) in (0, 1, 2)
    torch.testing.assert_close(cls.predict_proba([[1, 2, 3]]).sum(), torch.tensor(1.0))
    gen = TextGenerationPipeline(GptLiteConfig(vocab_size=50, hidden_dim=32, num_layers=1, num_heads=4,
                                               intermediate_dim=64, max_seq_len=16))
    out = gen.generate([1, 2], GenerationConfig(max_new_tokens=5, temperature=0.0))
    assert out[:2] == [1, 2] and len(out) == 7


def test_text_format_parsers():
    from brain_b200.utils import parsers as P
    ini = P.parse_ini("top = 1\n[model]\nname = llama\nlayers = 32\nlr = 3e-4\ntied = false\n")
    assert ini == {"": {"top": 1}, "model": {"name": "llama", "layers": 32, "lr": 3e-4, "tied": False}}
    assert P.parse_ini(P.dump_ini(ini)) == ini
    rows = P.parse_csv("a,b\n1,x\n2.5,true\n")
    assert rows == [{"a": 1, "b": "x"}, {"a": 2.5, "b": True}]
    assert P.parse_csv(P.dump_csv(rows)) == rows
    assert P.parse_json(P.dump_json({"k": [1, 2]})) == {"k": [1, 2]}


# ------------------------------------------------------------------ sharded checkpoints
def _sharded_rank(rank, world, directory, phase):
    from brain_b200.checkpoint.sharded import load_sharded, save_sharded
    from brain_b200.models import LlamaLite, LlamaLiteConfig
    from brain_b200.parallel import DataParallel, dist as bdist
    bdist.init(device="cpu", timeout_s=60)
    try:
        cfg = LlamaLiteConfig.tiny(vocab_size=64)
        model = LlamaLite(cfg, dtype=torch.float32, seed=0 if phase == "train" else 9)
        dp = DataParallel(model, lr=1e-2, betas=(0.9, 0.999), weight_decay=0.01)

        def batch(step):
            g = torch.Generator().manual_seed(1000 * step + rank)
            t = torch.randint(0, 64, (2, 17), generator=g)
            return t[:, :-1], t[:, 1:]
        if phase == "train":
            for s in range(2):
                dp.train_step(*batch(s))
            save_sharded(dp, directory, {"note": "two steps"})
        else:
            meta = load_sharded(dp, directory) if phase != "resume" else dp.load_checkpoint(directory)
            assert meta["note"] == "two steps" and dp.optimizer.step_count == 2
            if phase == "load_only":
                f = dp.flat
                return f.rank * f.shard_size, dp.optimizer.master.clone().numpy(), dp.optimizer.v.clone().numpy()
        dp.train_step(*batch(2))
        return model.layers[0].wqkv.detach().clone().numpy(), dp.optimizer.master.clone().numpy()
    finally:
        bdist.shutdown()


def test_sharded_checkpoint_resume_and_reshard(tmp_path):
    import numpy as np
    from brain_b200.checkpoint.sharded import load_full_state
    d = str(tmp_path / "ck")
    ref = run_ranks(_sharded_rank, 2, d, "train", timeout=180)
    full, meta = load_full_state(d)
    assert meta["world_size"] == 2 and meta["step"] == 2
    again = run_ranks(_sharded_rank, 2, d, "resume", timeout=180)
    for r in range(2):  # resuming on the same world size continues bit-exactly
        assert np.array_equal(ref[r][0], again[r][0]) and np.array_equal(ref[r][1], again[r][1])
    three = run_ranks(_sharded_rank, 3, d, "load_only", timeout=180)  # re-sharded onto three ranks
    n = meta["numel"]
    for key, idx in (("master", 1), ("exp_avg_sq", 2)):
        got = np.concatenate([three[r][idx] for r in range(3)])[:n]
        assert np.array_equal(got, full[key][:n].numpy())


def test_checkpoint_policy_masks():
    from brain_b200.autograd import CheckpointPolicy
    assert CheckpointPolicy("sqrt").mask(9) == [True, False, False] * 3
    assert CheckpointPolicy("all").mask(2) == [True, True] and CheckpointPolicy().mask(2) == [False, False]


def _mesh_rank(rank, world):
    import torch.distributed as dist
    from brain_b200.parallel import dist as bdist
    bdist.init(device="cpu", timeout_s=60)
    try:
        m = bdist.init_mesh(tp=2, pp=1)
        t = torch.tensor([float(rank)])
        dist.all_reduce(t, group=m.tp_group.handle)
        u = torch.tensor([float(rank)])
        dist.all_reduce(u, group=m.dp_group.handle)
        return m.tp_rank, m.dp_rank, m.tp_group.ranks, m.dp_group.ranks, float(t), float(u)
    finally:
        bdist.shutdown()


def test_parallel_mesh_subgroups():
    res = run_ranks(_mesh_rank, 4, timeout=120)
    assert res[0][:4] == (0, 0, [0, 1], [0, 2]) and res[3][:4] == (1, 1, [2, 3], [1, 3])
    assert res[1][4] == 1.0 and res[2][4] == 5.0  # TP sums: 0+1, 2+3
    assert res[0][5] == 2.0 and res[1][5] == 4.0  # DP sums: 0+2, 1+3


def test_memory_efficient_attention_matches_dense_with_alibi():
    from brain_b200.models.blocks import memory_efficient_attention, sdpa_with_bias
    from brain_b200.models.position import alibi_bias
    torch.manual_seed(0)
    B, S, H, Hkv, D = 2, 70, 4, 2, 16
    q, k, v = torch.randn(B, S, H, D), torch.randn(B, S, Hkv, D), torch.randn(B, S, Hkv, D)
    bias = alibi_bias(H, S, S, causal=False)
    for causal in (False, True):
        ref = sdpa_with_bias(q, k, v, bias, causal)
        got = memory_efficient_attention(q, k, v, bias, causal, q_chunk=16, k_chunk=24)
        torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)
    q2 = torch.randn(B, 10, H, D)  # decode-style: fewer queries than keys, bottom-right causal
    torch.testing.assert_close(memory_efficient_attention(q2, k, v, None, True, 4, 16),
                               sdpa_with_bias(q2, k, v, None, True), atol=1e-5, rtol=1e-5)


def test_memory_arena_pool_linalg_and_heads():
    from brain_b200 import linalg as LA
    from brain_b200.memory import BinnedMemoryPool, MemoryArena, aligned_empty, is_aligned, strides_row_major
    from brain_b200.models.heads import ClsHead, EmbConfig, HeadConfig, LmHead, TransformerEmbedding
    ar = MemoryArena(1 << 16)
    a = ar.alloc((10, 3), torch.float32)
    b = ar.alloc((7,), torch.bfloat16)
    assert is_aligned(a, 256) and is_aligned(b, 256) and a.data_ptr() != b.data_ptr()
    m = ar.mark()
    ar.alloc((100,))
    ar.release_to(m)
    assert ar.used() == m
    with pytest.raises(MemoryError):
        ar.alloc((1 << 20,))
    ar.reset()
    assert ar.used() == 0 and ar.stats.peak_bytes > 0
    pool = BinnedMemoryPool(min_bytes=256)
    t = pool.get((100,), torch.float32)
    p0 = t.data_ptr()
    pool.put(t)
    t2 = pool.get((90,), torch.float32)
    assert t2.data_ptr() == p0 and pool.hits == 1 and pool.misses == 1
    assert is_aligned(aligned_empty((5, 5)), 256) and strides_row_major((2, 3, 4)) == [12, 4, 1]
    x = torch.randn(5, 5, dtype=torch.float64)
    spd = x @ x.t() + 5 * torch.eye(5, dtype=torch.float64)
    L, U, perm = LA.lu(spd)
    torch.testing.assert_close(L @ U, spd[perm])
    torch.testing.assert_close(LA.cholesky(spd) @ LA.cholesky(spd).t(), spd)
    w, V = LA.eigh(spd)
    torch.testing.assert_close(V @ torch.diag(w) @ V.t(), spd)
    torch.testing.assert_close(LA.ifft_complex(LA.fft_complex(x[0])).real, x[0])
    coo = LA.SparseCOO((2, 3))
    for r, c, v in ((0, 1, 2.0), (1, 0, 1.0), (1, 2, 3.0)):
        coo.insert(r, c, v)
    dense = torch.tensor([[0.0, 2.0, 0.0], [1.0, 0.0, 3.0]], dtype=torch.float64)
    assert coo.nnz == 3
    torch.testing.assert_close(coo.spmm(torch.eye(3, dtype=torch.float64)), dense)
    emb = TransformerEmbedding(EmbConfig(50, 16, max_positions=8, type_vocab_size=2, norm="layer"))
    h = emb(torch.randint(0, 50, (2, 8)))
    assert h.shape == (2, 8, 16)
    lm = LmHead.new_tied(HeadConfig(16, 50), emb.tok.weight)
    assert lm(h).shape == (2, 8, 50)
    assert LmHead(HeadConfig(16, 50))(h).shape == (2, 8, 50) and ClsHead(HeadConfig(16, num_labels=3))(h).shape == (2, 3)


def test_fx_capture_keeps_exact_gelu():
    from brain_b200 import graph as G
    from brain_b200 import onnx as O
    net = torch.nn.Sequential(torch.nn.Linear(4, 8), torch.nn.GELU(), torch.nn.Linear(8, 2))
    x = torch.randn(3, 4)
    g = G.from_fx(net, x)
    torch.testing.assert_close(G.GraphInterpreter().run(g, [x])[0], net(x))
    torch.testing.assert_close(G.GraphInterpreter().run(O.import_onnx(O.export_onnx(g)), [x])[0], net(x))


def _async_rank(rank, world):
    from brain_b200.parallel import collectives as C
    from brain_b200.parallel import dist as bdist
    bdist.init(device="cpu", timeout_s=60)
    try:
        t = torch.full((4,), float(rank + 1))
        w = C.all_reduce_async(t)
        out = w.wait()
        g = C.all_gather_async(torch.tensor([float(rank)])).wait()
        return out.tolist(), w.is_completed(), g.tolist()
    finally:
        bdist.shutdown()


def test_async_collectives_on_gloo():
    res = run_ranks(_async_rank, 2, timeout=120)
    for r in range(2):
        assert res[r][0] == [3.0] * 4 and res[r][1] and res[r][2] == [0.0, 1.0]


def test_text_lm_features_similarity():
    from brain_b200.text import Bm25, HashingVectorizer, LmPreprocessor, TextSimilarity as TS, TfIdf
    ids = torch.arange(10).view(2, 5)
    x, y = LmPreprocessor.prepare_causal_lm(ids)
    assert x.tolist()[0] == [0, 1, 2, 3] and y.tolist()[0] == [1, 2, 3, 4]
    big = torch.randint(5, 100, (64, 64))
    m, lab = LmPreprocessor.prepare_masked_lm(big, mask_id=3, vocab_size=100, generator=torch.Generator().manual_seed(0))
    sel = lab != -100
    assert 0.10 < float(sel.float().mean()) < 0.20 and 0.7 < float((m[sel] == 3).float().mean()) < 0.9
    assert torch.equal(m[~sel], big[~sel])
    pm = LmPreprocessor.create_prefix_lm_mask(2, 4)
    assert pm.tolist() == [[1, 1, 0, 0], [1, 1, 0, 0], [1, 1, 1, 0], [1, 1, 1, 1]]
    assert LmPreprocessor.pack_documents([[1, 2], [3]], 3, 0).tolist() == [[1, 2, 0]]
    assert LmPreprocessor.sliding_window_chunks(range(7), 4, 2) == [[0, 1, 2, 3], [2, 3, 4, 5], [3, 4, 5, 6]]
    docs = [["the", "cat", "sat"], ["the", "dog", "ran"], ["a", "cat", "ran", "fast"]]
    tf = TfIdf().fit_transform(docs)
    assert tf.shape[0] == 3 and abs(float(tf[0].norm()) - 1) < 1e-9
    bm = Bm25().fit(docs)
    s = bm.score_corpus(["cat"])
    assert s[1] == 0.0 and s[0] > s[2] > 0  # shorter document ranks higher for the same tf
    assert float(HashingVectorizer(16).transform(["a", "a", "b"]).sum()) == 3
    assert TS.levenshtein("kitten", "sitting") == 3 and TS.damerau("ca", "ac") == 1
    assert abs(TS.jaro("MARTHA", "MARHTA") - 0.944444) < 1e-5
    assert abs(TS.jaro_winkler("MARTHA", "MARHTA") - 0.961111) < 1e-5
    assert TS.jaccard(["a", "b"], ["b", "c"]) == 1 / 3 and TS.sorensen_dice(["a", "b"], ["b", "c"]) == 0.5
    assert abs(TS.cosine([1, 0], [1, 1]) - 2 ** -0.5) < 1e-12 and TS.manhattan([1, 2], [3, 5]) == 5


def test_audio_alignment_pitch_chroma_and_dueling():
    from brain_b200.zoo import audio as A
    from brain_b200.zoo import rl
    a = torch.tensor([[0.0], [1.0], [2.0], [3.0]])
    b = torch.tensor([[0.0], [0.0], [1.0], [2.0], [3.0]])
    cost, path = A.dtw(a, b)
    assert cost == 0.0 and path[0] == (0, 0) and path[-1] == (3, 4)
    sr = 16000
    t = torch.arange(2048, dtype=torch.float64) / sr
    f0 = A.yin_pitch(torch.sin(2 * math.pi * 220.0 * t), sr)
    assert abs(f0 - 220.0) < 1.0
    assert A.yin_pitch(torch.zeros(2048), sr) == 0.0
    c = A.chroma(torch.sin(2 * math.pi * 440.0 * torch.arange(sr) / sr).float(), sr)
    assert int(c.mean(1).argmax()) == 9  # A
    q = rl.DuelingQNet(4, 3)(torch.randn(5, 4))
    assert q.shape == (5, 3)


def test_native_bpe_matches_python():
    import random as _r
    from brain_b200.text import BpeTokenizer, BpeTrainer
    rng = _r.Random(0)
    words = ["".join(rng.choice("abcdeéfg") for _ in range(rng.randint(1, 8))) for _ in range(300)]
    corpus = [" ".join(rng.choice(words) for _ in range(20)) for _ in range(50)]
    vocab, merges = BpeTrainer.train(corpus, vocab_size=200, special_tokens=("[PAD]", "[UNK]"))
    py = BpeTokenizer(vocab, merges)
    nat = BpeTokenizer(vocab, merges).use_native()
    for text in corpus[:20] + ["  unseen  zzz  words\tand\nlines ", ""]:
        assert nat.encode(text).ids == py.encode(text).ids, text


def test_nvtx_ranges_around_native_calls(monkeypatch):
    from brain_b200 import _native
    seen = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda n: seen.append(("push", n)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: seen.append(("pop",)))
    _native.register({"brain_bpe_destroy": ("brain_runtime", "p")})
    _native.set_nvtx(True)
    try:
        assert _native.call("brain_bpe_destroy", None) == 0
    finally:
        _native.set_nvtx(False)
    assert seen == [("push", "brain_bpe_destroy"), ("pop",)]


def test_graph_transformer_jk_and_euler_ancestral():
    from brain_b200.zoo import diffusion as D
    from brain_b200.zoo import gnn
    g = gnn.Graph.from_undirected([(0, 1), (1, 2)], 3)
    layer = gnn.GraphTransformerLayer(8, 2)
    h1 = layer(g, torch.randn(3, 8))
    h2 = layer(g, h1)
    assert h1.shape == (3, 8) and gnn.jumping_knowledge([h1, h2]).shape == (3, 16)
    assert gnn.jumping_knowledge([h1, h2], "max").shape == (3, 8)
    sched = D.LinearSchedule(200)
    x0 = torch.tensor([[0.7, -1.2]])

    def oracle(x, t, cond=None):
        ac = sched.at("alphas_cumprod", t, x)
        return (x - ac.sqrt() * x0) / (1 - ac).sqrt()
    out = D.EulerAncestralSampler(sched, eta=0.0).sample(oracle, (1, 2), num_steps=30,
                                                         generator=torch.Generator().manual_seed(0))
    torch.testing.assert_close(out, x0, atol=1e-3, rtol=0)
    noisy = D.EulerAncestralSampler(sched, eta=1.0).sample(oracle, (1, 2), num_steps=30,
                                                           generator=torch.Generator().manual_seed(0))
    torch.testing.assert_close(noisy, x0, atol=1e-3, rtol=0)


def test_periodic_checkpointer_keeps_last_and_resumes(tmp_path):
    import os
    from brain_b200.checkpoint.formats import ModelState
    from brain_b200.train import Batch, TrainerBuilder
    from brain_b200.train.callbacks import PeriodicCheckpointer
    torch.manual_seed(0)
    x, y = torch.randn(32, 4), torch.randint(0, 3, (32,))
    model = torch.nn.Sequential(torch.nn.Linear(4, 8), torch.nn.ReLU(), torch.nn.Linear(8, 3))
    tr = TrainerBuilder().model(model).learning_rate(0.1).build()
    ck = PeriodicCheckpointer(str(tmp_path), every=2, keep_last=2)
    tr.callbacks.append(ck)
    tr.fit([Batch(x, y)], epochs=8)
    files = sorted(f for f in os.listdir(tmp_path) if f.startswith("epoch"))
    assert files == ["epoch000006.brain", "epoch000008.brain"] and os.path.exists(tmp_path / "best.brain")
    model2 = torch.nn.Sequential(torch.nn.Linear(4, 8), torch.nn.ReLU(), torch.nn.Linear(8, 3))
    tr2 = TrainerBuilder().model(model2).learning_rate(0.1).build()
    tr2.load_state(ModelState.load_file(ck.latest()))
    for a, b in zip(model.parameters(), model2.parameters()):
        torch.testing.assert_close(a, b)


# ------------------------------------------------------------------ context / pipeline parallel on Gloo
def _cp_rank(rank, world):
    from brain_b200.models.blocks import sdpa_with_bias
    from brain_b200.parallel import dist as bdist
    from brain_b200.parallel.sequence import gather_sequence, ring_attention, scatter_sequence, ulysses_attention
    bdist.init(device="cpu", timeout_s=60)
    try:
        g = torch.Generator().manual_seed(0)
        B, S, H, Hkv, D = 2, 24, 4, 2, 8
        q, k, v = torch.randn(B, S, H, D, generator=g), torch.randn(B, S, Hkv, D, generator=g), \
            torch.randn(B, S, Hkv, D, generator=g)
        ref = sdpa_with_bias(q, k, v, None, True)
        ql, kl, vl = (scatter_sequence(t, rank, world) for t in (q, k, v))
        ring = gather_sequence(ring_attention(ql, kl, vl, rank, world, causal=True), world)
        kf, vf = k.repeat_interleave(H // Hkv, 2), v.repeat_interleave(H // Hkv, 2)
        uly = gather_sequence(ulysses_attention(ql, scatter_sequence(kf, rank, world),
                                                scatter_sequence(vf, rank, world), world, causal=True), world)
        return float((ring - ref).abs().max()), float((uly - ref).abs().max())
    finally:
        bdist.shutdown()


def test_ring_and_ulysses_attention_match_full_attention():
    res = run_ranks(_cp_rank, 2, timeout=120)
    for r in range(2):
        assert res[r][0] < 1e-5 and res[r][1] < 1e-5


def _cp_train_rank(rank, world, causal):
    """Context-parallel training: ring attention forward and backward against full attention."""
    from brain_b200.models.blocks import sdpa_with_bias
    from brain_b200.parallel import dist as bdist
    from brain_b200.parallel.sequence import ring_attention, scatter_sequence
    bdist.init(device="cpu", timeout_s=60)
    try:
        g = torch.Generator().manual_seed(1)
        B, S, H, Hkv, D = 2, 30, 4, 2, 8
        q, k, v = (torch.randn(B, S, h, D, generator=g, dtype=torch.float64).requires_grad_(True)
                   for h in (H, Hkv, Hkv))
        do = torch.randn(B, S, H, D, generator=g, dtype=torch.float64)
        sdpa_with_bias(q, k, v, None, causal).double().backward(do)
        ql, kl, vl = (scatter_sequence(t.detach(), rank, world).requires_grad_(True) for t in (q, k, v))
        o = ring_attention(ql, kl, vl, rank, world, causal=causal)
        o.backward(scatter_sequence(do, rank, world))
        errs = [float((a.grad if hasattr(a, "grad") and a.grad is not None else a) .sub(scatter_sequence(b, rank, world)).abs().max())
                for a, b in ((ql, q.grad), (kl, k.grad), (vl, v.grad))]
        return errs
    finally:
        bdist.shutdown()


@pytest.mark.parametrize("world,causal", [(2, True), (3, True), (3, False)])
def test_ring_attention_gradients_match_full_attention(world, causal):
    res = run_ranks(_cp_train_rank, world, causal, timeout=120)
    for errs in res:
        assert max(errs) < 1e-5, errs


def _pp_rank(rank, world):
    import torch.distributed as dist
    from brain_b200.parallel import dist as bdist
    from brain_b200.parallel.pipeline import PipelineStage
    bdist.init(device="cpu", timeout_s=60)
    try:
        torch.manual_seed(0)
        layers = [torch.nn.Linear(8, 8) for _ in range(4)]
        stage = torch.nn.Sequential(*layers[2 * rank:2 * rank + 2])
        g = torch.Generator().manual_seed(1)
        mbs = [torch.randn(3, 8, generator=g) for _ in range(4)]
        tgts = [torch.randn(3, 8, generator=g) for _ in range(4)]
        ps = PipelineStage(stage, rank, world, 4, (3, 8), dtype=torch.float32,
                           loss_fn=lambda y, t: torch.nn.functional.mse_loss(y, t))
        loss = ps.step_1f1b(mbs if rank == 0 else None, tgts if rank == world - 1 else None)
        grads = [p.grad.clone() for p in stage.parameters()]
        return loss, [gr.tolist() for gr in grads]
    finally:
        bdist.shutdown()


def test_pipeline_1f1b_matches_single_process_gradients():
    res = run_ranks(_pp_rank, 2, timeout=120)
    torch.manual_seed(0)
    layers = [torch.nn.Linear(8, 8) for _ in range(4)]
    full = torch.nn.Sequential(*layers)
    g = torch.Generator().manual_seed(1)
    mbs = [torch.randn(3, 8, generator=g) for _ in range(4)]
    tgts = [torch.randn(3, 8, generator=g) for _ in range(4)]
    total = 0.0
    for x, t in zip(mbs, tgts):
        loss = torch.nn.functional.mse_loss(full(x), t) / 4
        loss.backward()
        total += float(loss) * 4
    assert abs(res[1][0] - total / 4) < 1e-5
    ref = [p.grad for p in full.parameters()]
    got = [torch.tensor(x) for x in res[0][1] + res[1][1]]
    for a, b in zip(got, ref):
        torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-5)


def test_heartbeat_detects_a_rank_that_stops():
    import time
    import torch.distributed as dist
    from brain_b200.parallel.fault import FaultPolicy, Heartbeat, StepFailed, run_step_with_policy
    store = dist.HashStore()
    hb = [Heartbeat(store, r, 3, interval_s=0.05, timeout_s=0.4).start() for r in range(3)]
    time.sleep(0.3)
    assert hb[0].dead_ranks() == []
    hb[2].stop()  # rank 2 goes silent (a crashed or hung process)
    deadline = time.time() + 5
    dead = []
    while time.time() < deadline and dead != [2]:
        dead = hb[0].dead_ranks()
        time.sleep(0.05)
    assert dead == [2]
    with pytest.raises(StepFailed) as e:
        run_step_with_policy(lambda: (_ for _ in ()).throw(TimeoutError("collective timed out")),
                             FaultPolicy.EXCLUDE_RANK, heartbeat=hb[0])
    assert e.value.dead_ranks == [2]
    for h in hb:
        h.stop()


def test_bench_report_scaling_table(tmp_path):
    import json as _json
    from brain_b200.bench.report import load_runs, scaling_table
    p = tmp_path / "runs.log"
    p.write_text("\n".join(["warming up...", _json.dumps({"value": 18000.0, "n_gpus": 1, "ms_per_step": 450.0,
                                                          "unit": "tokens/s"}),
                            _json.dumps({"value": 140000.0, "n_gpus": 8, "ms_per_step": 468.0, "unit": "tokens/s"}),
                            _json.dumps({"impl": "reference", "unavailable": "x"})]))
    t = scaling_table(load_runs([str(p)]))
    assert "| 8 | 140,000 | 468.0 | 17,500 | 0.972 |" in t and t.count("\n") == 3


def test_bert_t5_vit_train_steps_on_cpu():
    from brain_b200.models import BertLite, T5Lite, ViT
    from brain_b200.models.config import BertLiteConfig, T5LiteConfig, ViTConfig
    torch.manual_seed(0)
    bert = BertLite(BertLiteConfig(vocab_size=100, hidden_dim=32, num_layers=2, num_heads=4, intermediate_dim=64,
                                   max_seq_len=16, num_labels=3))
    t5 = T5Lite(T5LiteConfig(vocab_size=100, hidden_dim=32, num_layers=1, num_decoder_layers=1, num_heads=4,
                             intermediate_dim=64, max_seq_len=16))
    vit = ViT(ViTConfig(image_size=32, patch_size=8, hidden_dim=32, num_layers=1, num_heads=4, mlp_dim=64,
                        num_classes=5))
    ids, src, tgt = torch.randint(0, 100, (4, 12)), torch.randint(0, 100, (4, 10)), torch.randint(0, 100, (4, 7))
    imgs, ylab = torch.randn(4, 3, 32, 32), torch.randint(0, 5, (4,))
    losses = {}
    for name, model, fn in (
            ("bert", bert, lambda: torch.nn.functional.cross_entropy(bert(ids), torch.tensor([0, 1, 2, 0]))),
            ("t5", t5, lambda: torch.nn.functional.cross_entropy(t5(src, tgt).reshape(-1, 100), tgt.reshape(-1))),
            ("vit", vit, lambda: vit.loss(imgs, ylab))):
        opt = torch.optim.Adam(model.parameters(), lr=3e-3)
        seq = []
        for _ in range(15):
            loss = fn()
            opt.zero_grad()
            loss.backward()
            opt.step()
            seq.append(float(loss.detach()))
        losses[name] = seq
        assert seq[-1] < seq[0], (name, seq)


def test_kv_caches_contiguous_and_paged():
    from brain_b200.models.kv_cache import KvCache, KvCacheConfig, PagedKvCache
    c = KvCache(KvCacheConfig(2, 2, 2, 4, 8, torch.float32, "cpu"))
    k1, v1 = torch.randn(2, 3, 2, 4), torch.randn(2, 3, 2, 4)
    fk, fv = c.update(0, k1, v1)
    k2 = torch.randn(2, 2, 2, 4)
    fk, fv = c.update(0, k2, k2)
    assert c.current_seq_len(0) == 5 and c.current_seq_len(1) == 0
    torch.testing.assert_close(fk, torch.cat([k1, k2], 1))
    with pytest.raises(ValueError, match="overflow"):
        c.update(0, torch.randn(2, 4, 2, 4), torch.randn(2, 4, 2, 4))
    c.clear()
    assert c.current_seq_len(0) == 0
    p = PagedKvCache(1, 6, 4, 2, 4, torch.float32, "cpu")
    seqs = {0: torch.randn(7, 2, 4), 1: torch.randn(5, 2, 4)}
    for sid in seqs:
        p.add_sequence(sid)
    # prefill token by token for seq 0 and in one go for seq 1, interleaving block allocation
    for t in range(7):
        p.reserve(0, 1)
        p.write(0, p.slot_mapping([0], 1), seqs[0][t:t + 1], seqs[0][t:t + 1] * 2)
        p.advance([0], 1)
    p.reserve(1, 5)
    p.write(0, p.slot_mapping([1], 5), seqs[1], seqs[1] * 2)
    p.advance([1], 5)
    for sid, ref in seqs.items():
        k, v = p.gather(0, sid)
        torch.testing.assert_close(k, ref)
        torch.testing.assert_close(v, ref * 2)
    assert p.lengths_tensor([0, 1]).tolist() == [7, 5] and p.block_table_tensor([0, 1]).shape == (2, 2)
    assert len(p.free) == 2
    p.free_sequence(0)
    assert len(p.free) == 4
    p.add_sequence(2)
    with pytest.raises(RuntimeError, match="out of blocks"):
        p.reserve(2, 17)


def test_sampling_penalty_filters_and_greedy():
    from brain_b200.models.generate import (GenerationConfig, apply_repetition_penalty, filter_logits,
                                            sample_next_token)
    logits = torch.tensor([[2.0, -1.0, 0.5, 3.0, 1.0]])
    hist = torch.tensor([[0, 1]])
    pen = apply_repetition_penalty(logits, hist, 2.0)
    assert torch.allclose(pen, torch.tensor([[1.0, -2.0, 0.5, 3.0, 1.0]]))
    assert apply_repetition_penalty(logits, hist, 1.0) is logits
    # top-k keeps the k largest
    fk = filter_logits(logits, top_k=2)
    assert torch.isfinite(fk).tolist() == [[True, False, False, True, False]]
    # top-p keeps the smallest prefix whose mass reaches p (the token crossing p stays)
    p = torch.softmax(logits, -1)[0]
    order = torch.argsort(p, descending=True)
    cum = p[order].cumsum(0)
    keep_n = int((cum - p[order] <= 0.8).sum())
    fp = filter_logits(logits, top_p=0.8)
    assert int(torch.isfinite(fp).sum()) == keep_n
    assert set(torch.nonzero(torch.isfinite(fp[0])).flatten().tolist()) == set(order[:keep_n].tolist())
    # min-p drops tokens below min_p * max prob
    fm = filter_logits(logits, min_p=0.3)
    kept = (p >= p.max() * 0.3).tolist()
    assert torch.isfinite(fm[0]).tolist() == kept
    # greedy after the penalty: token 0 (2.0) would beat token 4 (1.0) but not token 3
    cfg = GenerationConfig(temperature=0.0, repetition_penalty=10.0)
    assert sample_next_token(torch.tensor([[5.0, 0.0, 0.0, 4.0]]), cfg, torch.tensor([[0]])).item() == 3
    # sampling with top_k=1 is deterministic
    cfg = GenerationConfig(temperature=1.0, top_k=1, top_p=1.0, repetition_penalty=1.0)
    g = torch.Generator().manual_seed(0)
    out = sample_next_token(logits.repeat(8, 1), cfg, None, g)
    assert out.tolist() == [3] * 8
    # empirical distribution follows softmax(logits / T) when nothing is filtered
    cfg = GenerationConfig(temperature=2.0, top_k=0, top_p=1.0, min_p=0.0, repetition_penalty=1.0)
    draws = sample_next_token(logits.repeat(20000, 1), cfg, None, torch.Generator().manual_seed(1))
    freq = torch.bincount(draws, minlength=5).float() / draws.numel()
    assert torch.allclose(freq, torch.softmax(logits[0] / 2.0, -1), atol=0.015)


def test_fused_layer_norm_one_pass_variance():
    from brain_b200.ops import fused_layer_norm, layer_norm
    torch.manual_seed(0)
    x = torch.randn(6, 64, dtype=torch.float64)
    w, b = torch.randn(64, dtype=torch.float64), torch.randn(64, dtype=torch.float64)
    assert torch.allclose(fused_layer_norm(x, w, b), layer_norm(x, w, b), atol=1e-5)
    # a constant row: the one-pass variance may round below zero; the clamp keeps it finite
    c = torch.full((2, 64), 1e4, dtype=torch.float32) + torch.tensor([[0.0], [1e-3]])
    y = fused_layer_norm(c, torch.ones(64), None)
    assert torch.isfinite(y).all()


def test_adamw_group_weight_decay_overrides_default():
    from brain_b200.optim.optimizers import AdamW
    a, b = torch.nn.Parameter(torch.ones(2)), torch.nn.Parameter(torch.ones(2))
    opt = AdamW([{"params": [a]}, {"params": [b], "weight_decay": 0.0}], lr=0.1, weight_decay=0.5)
    a.grad, b.grad = torch.zeros(2), torch.zeros(2)
    opt.step()
    # decoupled decay p -= lr * wd * p before the moments; a zero gradient leaves only the decay
    assert torch.allclose(a.data, torch.full((2,), 0.95)) and torch.equal(b.data, torch.ones(2))


def test_diffusion_model_wrapper_and_helpers():
    import torch
    from brain_b200.zoo import diffusion as D
    torch.manual_seed(0)
    assert D.linspace_timesteps(1000, 5).tolist() == [999, 749, 500, 250, 0]
    vals = torch.arange(10.0)
    assert D.extract_at_t(vals, torch.tensor([2, 7]), torch.zeros(2, 3, 4)).shape == (2, 1, 1)
    assert float(D.eps_loss(torch.ones(3), torch.zeros(3))) == 1.0
    net = D.MlpDenoiser(2, hidden=32, time_dim=16, num_classes=3)
    dm = D.DiffusionModel(net, D.LinearSchedule(50), sampler="ddim", guidance=D.GuidanceConfig(scale=2.0))
    opt = torch.optim.Adam(net.parameters(), 1e-2)
    g = torch.Generator().manual_seed(1)
    x0 = torch.randn(64, 2, generator=g) * 0.1 + torch.tensor([1.0, -1.0])
    cond = torch.randint(0, 3, (64,), generator=g)
    losses = [dm.train_step(opt, x0, cond, generator=g) for _ in range(30)]
    assert sum(losses[-5:]) < sum(losses[:5])
    out = dm.sample((8, 2), cond=cond[:8], generator=g, num_steps=10)
    assert out.shape == (8, 2) and torch.isfinite(out).all()
    assert D.DiffusionRunner is D.DiffusionModel and D.sinusoidal_timestep_embedding is D.timestep_embedding


def test_benchmark_suite_and_timers():
    import torch
    from brain_b200.bench import harness as H
    suite = H.BenchmarkSuite("s")
    suite.add(H.FnBenchmark.from_fn("matmul_64", lambda: torch.randn(64, 64) @ torch.randn(64, 64), flops=2 * 64 ** 3,
                                    iters=3, tags=["kernel"]))
    suite.add(H.FnBenchmark.from_fn("copy", lambda: torch.zeros(1000).clone(), iters=3))
    res = suite.run_all()
    assert set(res) == {"matmul_64", "copy"} and len(res["copy"].raw_nanos) == 3
    assert set(suite.run_filtered(tag="kernel")) == {"matmul_64"} and set(suite.run_filtered("cop")) == {"copy"}
    t = H.BenchTimer.start_new()
    assert t.is_running()
    t.stop()
    assert not t.is_running() and t.elapsed_nanos() >= 0 and t.elapsed_secs() == t.elapsed_nanos() / 1e9
    assert H.calibrate_timer_overhead(50) >= 0
    assert H.format_gflops(2e12, 1.0) == "2.00 TFLOP/s" and H.format_gflops(5e9, 1.0) == "5.00 GFLOP/s"
    assert H.format_throughput(2.5e6, 1.0, "tok") == "2.50 Mtok/s"
    assert H.estimate_memory_bandwidth_gbps(1 << 20, "cpu", 2) > 0 and H.get_peak_rss_kb() > 0
