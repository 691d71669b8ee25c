"""RNN extras (crates/brain-rnn/src/cells/normalized.rs, reg_ops.rs, utils.rs, seq/attention.rs,
cells/attention_cell.rs, seq/bidirectional.rs, seq/teacher.rs, process.rs, init_rnn.rs)."""
import math

import pytest
import torch

from brain_b200.zoo import rnn_extras as RX
from brain_b200.zoo.rnn import GruCell, LstmCell


def test_inits_clip_padding_packing():
    q = RX.init_orthogonal(8, 4, seed=1).double()
    torch.testing.assert_close(q.t() @ q, torch.eye(4, dtype=torch.float64), rtol=1e-5, atol=1e-5)
    q2 = RX.init_orthogonal(3, 6, seed=2).double()
    torch.testing.assert_close(q2 @ q2.t(), torch.eye(3, dtype=torch.float64), rtol=1e-5, atol=1e-5)
    u = RX.init_uniform(50, 50, 25, seed=0)
    assert float(u.abs().max()) <= 0.2
    g = [torch.full((3,), 3.0), torch.full((1,), 4.0)]
    n = RX.clip_grad_norm(g, 1.0)
    assert n == pytest.approx(math.sqrt(27 + 16)) and math.sqrt(sum(float(t.square().sum()) for t in g)) <= 1.0
    seqs = [torch.ones(3, 2), torch.ones(1, 2) * 2]
    p = RX.PackedSequence.pack(seqs)
    assert p.data.shape == (2, 3, 2) and p.mask().tolist() == [[True, True, True], [True, False, False]]
    assert [t.shape[0] for t in p.unpack()] == [3, 1]
    assert RX.truncate_steps(torch.zeros(2, 5, 3), 2).shape == (2, 2, 3)
    a, b = RX.split_states(RX.concat_states((torch.ones(2, 3),), (torch.zeros(2, 4),)), 3)
    assert a[0].shape == (2, 3) and b[0].shape == (2, 4)


def test_norm_lstm_and_variational_dropout():
    torch.manual_seed(0)
    cell = RX.NormLstmCell(5, 8)
    h, c = cell(torch.randn(4, 5))
    assert h.shape == (4, 8) and c.shape == (4, 8)
    h2, _ = cell(torch.randn(4, 5) * 100.0, (h, c))  # layer norm keeps the gates in range
    assert torch.isfinite(h2).all() and float(h2.detach().abs().max()) <= 1.0
    vd = RX.VariationalDropout(0.5)
    x = torch.ones(3, 6, 10)
    y = vd(x, generator=torch.Generator().manual_seed(1))
    assert torch.equal(y[:, 0], y[:, 5])  # same mask at every step
    assert set(y.unique().tolist()) <= {0.0, 2.0}
    vd.eval()
    assert torch.equal(vd(x), x)


def test_seq_attention_kinds_and_attention_cell():
    torch.manual_seed(0)
    q, k, v = torch.randn(2, 4), torch.randn(2, 5, 4), torch.randn(2, 5, 3)
    ctx, w = RX.SeqAttention(4, 4, "dot")(q, k, v)
    ref_w = torch.softmax((k @ q[..., None]).squeeze(-1), -1)
    torch.testing.assert_close(w, ref_w)
    torch.testing.assert_close(ctx, (ref_w[..., None] * v).sum(1))
    _, ws = RX.SeqAttention(4, 4, "scaled_dot")(q, k, v)
    torch.testing.assert_close(ws, torch.softmax((k @ q[..., None]).squeeze(-1) / 2.0, -1))
    mask = torch.tensor([[True] * 5, [True, True, False, False, False]])
    _, wa = RX.SeqAttention(4, 4, "additive", attn_dim=6)(q, k, v, mask)
    assert float(wa[1, 2:].sum()) == 0.0 and torch.allclose(wa.sum(-1), torch.ones(2))
    cell = RX.AttentionCell(3, 8, 4, cell="gru")
    (h,), w = cell(torch.randn(2, 3), k)
    assert h.shape == (2, 8) and w.shape == (2, 5)


def test_bidirectional_merges_and_masked_unroll():
    torch.manual_seed(0)
    f, b = LstmCell(3, 4), LstmCell(3, 4)
    x = torch.randn(2, 6, 3)
    out, _ = RX.BidirectionalRnn(f, b, "concat")(x)
    of, _ = RX.run_cell(f, x)
    ob, _ = RX.run_cell(b, x, reverse=True)
    torch.testing.assert_close(out, torch.cat([of, ob], -1))
    torch.testing.assert_close(RX.BidirectionalRnn(f, b, "sum")(x)[0], of + ob)
    torch.testing.assert_close(RX.BidirectionalRnn(f, b, "average")(x)[0], (of + ob) / 2)
    mask = RX.create_padding_mask(torch.tensor([6, 3]), 6)
    om, (hm, cm) = RX.run_cell(f, x, mask=mask)
    short, (hs, cs) = RX.run_cell(f, x[1:, :3])
    torch.testing.assert_close(hm[1], hs[0])  # the padded row's final state is that of its 3 valid steps
    assert float(om[1, 3:].abs().sum()) == 0.0


def test_teacher_forcing_and_streamer():
    assert RX.TeacherSchedule.constant(0.7).ratio(100) == 0.7
    lin = RX.TeacherSchedule.linear(1.0, 0.0, 10)
    assert lin.ratio(5) == 0.5 and lin.ratio(20) == 0.0
    assert RX.TeacherSchedule.exponential(1.0, 0.5, 0.2).ratio(3) == 0.2
    tf = RX.TeacherForcer(RX.TeacherSchedule.constant(1.0))
    gt, pr = torch.ones(4, 2), torch.zeros(4, 2)
    assert torch.equal(tf.choose(gt, pr), gt)
    tf.advance_step()
    assert tf.step == 1
    torch.manual_seed(0)
    cell = GruCell(3, 5)
    x = torch.randn(2, 7, 3)
    full, _ = RX.run_cell(cell, x)
    st = RX.OnlineRnnStreamer(cell)
    a = st.push(x[:, :4])
    b = st.push(x[:, 4])
    c = st.push(x[:, 5:])
    torch.testing.assert_close(torch.cat([a, b[:, None], c], 1), full)
    st.reset([0])
    assert float(st.state[0][0].abs().sum()) == 0.0 and float(st.state[0][1].abs().sum()) > 0


def test_peephole_lstm_cell_gate_equations():
    from brain_b200.zoo.rnn import PeepholeLstmCell, VanillaRnnCell, RnnCell
    torch.manual_seed(3)
    cell = PeepholeLstmCell(3, 4)
    assert torch.equal(cell.peep.detach(), torch.full((3, 4), 0.1))
    x, h, c = torch.randn(2, 3), torch.randn(2, 4), torch.randn(2, 4)
    h2, c2 = cell(x, (h, c))
    i, f, g, o = (cell.ih(x) + cell.hh(h)).chunk(4, -1)
    cn = torch.sigmoid(f + 0.1 * c) * c + torch.sigmoid(i + 0.1 * c) * torch.tanh(g)
    hn = torch.sigmoid(o + 0.1 * cn) * torch.tanh(cn)
    assert torch.allclose(c2, cn, atol=1e-6) and torch.allclose(h2, hn, atol=1e-6)
    assert VanillaRnnCell is RnnCell
