"""Transformer front-ends and backward-graph utilities against plain fp32 PyTorch references."""
import math

import pytest
import torch

from brain_b200.autograd import (Value, topological_sort, compute_dag_levels, values_close, TapeBuilder,
                                 RecomputeGraph, OpRecord)
from brain_b200.models import (FlashAttentionLite, FlashLiteConfig, XformersAttentionLite, XformersConfig,
                               RelativeAttention, AlibiPositionalBias, LayerKvCache, TransformerDecoderLayer,
                               TransformerDecoder, repeat_kv, quick_gelu, all_close)


def _ref(q, k, v, causal, scale=None, bias=None):
    qh, kh, vh = (t.transpose(1, 2).double() for t in (q, k, v))
    if kh.shape[1] != qh.shape[1]:
        kh = repeat_kv(kh, qh.shape[1] // kh.shape[1])
        vh = repeat_kv(vh, qh.shape[1] // vh.shape[1])
    s = qh @ kh.transpose(-1, -2) * (scale if scale is not None else qh.shape[-1] ** -0.5)
    if bias is not None:
        s = s + bias.double()
    if causal:
        Sq, Sk = s.shape[-2:]
        m = torch.ones(Sq, Sk, dtype=torch.bool).tril(Sk - Sq)
        s = s.masked_fill(~m, float("-inf"))
    return (s.softmax(-1) @ vh).transpose(1, 2).float()


@pytest.mark.parametrize("causal", [False, True])
def test_flash_and_xformers_lite_match_reference(causal):
    torch.manual_seed(0)
    q = torch.randn(2, 37, 4, 16)
    k = torch.randn(2, 53, 2, 16)
    v = torch.randn(2, 53, 2, 16)
    ref = _ref(q, k, v, causal)
    a = FlashAttentionLite(FlashLiteConfig(block_m=8, block_n=16, is_causal=causal))(q, k, v)
    b = XformersAttentionLite(XformersConfig(chunk_size=7, is_causal=causal))(q, k, v)
    assert torch.allclose(a, ref, atol=1e-5) and torch.allclose(b, ref, atol=1e-5)
    c = FlashAttentionLite(FlashLiteConfig(8, 8, scale=0.05, is_causal=causal))(q, k, v)
    assert torch.allclose(c, _ref(q, k, v, causal, scale=0.05), atol=1e-5)


def test_alibi_and_relative_attention():
    torch.manual_seed(1)
    q, k, v = torch.randn(1, 9, 4, 8), torch.randn(1, 9, 4, 8), torch.randn(1, 9, 4, 8)
    ab = AlibiPositionalBias(4)
    dense = ab.bias(9, 9).dense()
    assert dense.shape == (4, 9, 9)
    assert torch.allclose(dense[:, 5, 2], -ab.slopes * 3)
    ra = RelativeAttention(4, num_buckets=8, max_distance=16)
    torch.nn.init.normal_(ra.table)
    out = ra(q, k, v)
    assert torch.allclose(out, _ref(q, k, v, False, bias=ra.bias(9, 9)), atol=1e-5)
    out.sum().backward()
    assert ra.table.grad is not None and ra.table.grad.abs().sum() > 0


def test_layer_kv_cache_and_helpers():
    c = LayerKvCache(2, 2, 4, 6, dtype=torch.float32)
    k1, v1 = c.update(torch.ones(2, 2, 4, 4), torch.zeros(2, 2, 4, 4))
    assert k1.shape == (2, 2, 4, 4) and c.current_seq_len == 4
    k2, _ = c.update(torch.full((2, 2, 2, 4), 2.0), torch.zeros(2, 2, 2, 4))
    assert k2.shape[2] == 6 and float(k2[0, 0, 5, 0]) == 2.0
    with pytest.raises(ValueError):
        c.update(torch.zeros(2, 2, 1, 4), torch.zeros(2, 2, 1, 4))
    c.clear()
    assert c.current_seq_len == 0
    x = torch.arange(12.0).reshape(1, 2, 3, 2)
    r = repeat_kv(x, 3)
    assert r.shape == (1, 6, 3, 2) and torch.equal(r[:, 2], x[:, 0]) and torch.equal(r[:, 3], x[:, 1])
    t = torch.linspace(-3, 3, 11)
    assert torch.allclose(quick_gelu(t), t / (1 + torch.exp(-1.702 * t)))
    assert all_close(t, t + 1e-9) and not all_close(t, t + 1e-3) and not all_close(t, t[:5])


def test_transformer_decoder_cross_attends():
    torch.manual_seed(2)
    dec = TransformerDecoder(2, 32, 4, 64)
    x, mem = torch.randn(2, 5, 32), torch.randn(2, 7, 32)
    y = dec(x, memory=mem)
    assert y.shape == (2, 5, 32)
    mem2 = mem.clone()
    mem2[:, 3] += torch.randn(32)
    assert not torch.allclose(dec(x, memory=mem2), y)
    # causal self-attention: the first position ignores later ones
    x2 = x.clone()
    x2[:, 4] += torch.randn(32)
    y2 = dec(x2, memory=mem)
    assert torch.allclose(y2[:, :4], y[:, :4], atol=1e-5) and not torch.allclose(y2[:, 4], y[:, 4])
    assert isinstance(dec.layers[0], TransformerDecoderLayer)


def test_topological_sort_and_levels():
    a = torch.randn(3, requires_grad=True)
    b = torch.randn(3, requires_grad=True)
    c = a * b
    d = c.exp() + a
    order = topological_sort(Value(d) if not isinstance(d, Value) else d)
    assert order[-1] is d.grad_fn
    pos = {id(n): i for i, n in enumerate(order)}
    for n in order:
        for p, _ in n.next_functions:
            if p is not None:
                assert pos[id(p)] < pos[id(n)]
    levels = compute_dag_levels(order)
    assert {type(n).__name__ for n in levels[0]} == {"AccumulateGrad"}
    assert levels[-1] == [d.grad_fn]
    level_of = {id(n): i for i, lv in enumerate(levels) for n in lv}
    for n in order:
        for p, _ in n.next_functions:
            if p is not None:
                assert level_of[id(p)] < level_of[id(n)]
    # a deep chain does not exhaust the Python stack
    x = torch.ones(1, requires_grad=True)
    y = x
    for _ in range(5000):
        y = y * 1.0
    assert len(topological_sort(y)) == 5001
    assert topological_sort(torch.ones(2)) == []


def test_values_close_tape_builder_recompute():
    assert values_close(Value(torch.ones(3)), Value(torch.ones(3) + 1e-4), 1e-3)
    assert not values_close(Value(torch.ones(3)), Value(torch.ones(3) + 1e-2), 1e-3)
    assert not values_close(Value(torch.ones(3)), Value(torch.ones(4)), 1.0)
    tape = TapeBuilder().add_op(OpRecord("mul", [0, 1], 2, (3,))).add_op(OpRecord("exp", [2], 3, (3,))).build()
    assert tape.ops() == ["mul", "exp"]
    g = RecomputeGraph([torch.tensor(2.0), torch.tensor(3.0)], "mul", lambda a, b: a * b)
    assert g.input_count() == 2 and g.op_name() == "mul" and float(g.recompute()) == 6.0
    with pytest.raises(RuntimeError):
        RecomputeGraph([], "noop").recompute()


def _rope_oracle(x, cos, sin, pos):
    """x [B, H, S, D] float64, pairs (i, i + D/2)."""
    half = x.shape[-1] // 2
    c, s = cos[pos][None, None], sin[pos][None, None]
    a, b = x[..., :half], x[..., half:]
    return torch.cat([a * c - b * s, a * s + b * c], -1)


def test_rotary_embedding_4d_and_2d():
    from brain_b200.models import RopeConfig, RotaryEmbedding
    torch.manual_seed(3)
    re = RotaryEmbedding(RopeConfig(dim=16, max_seq_len=10, theta=500.0, scaling_factor=2.0))
    cos, sin = RotaryEmbedding.compute_frequencies(16, 10, 500.0, 2.0)
    x = torch.randn(2, 3, 6, 16)
    y = re.apply_rope_4d(x.clone(), pos_offset=2)
    ref = _rope_oracle(x.double(), cos, sin, torch.arange(2, 8)).float()
    assert torch.allclose(y, ref, atol=1e-5)
    # positions past the table stay as they are
    z = re.apply_rope_4d(x.clone(), pos_offset=7)
    assert torch.equal(z[:, :, 3:], x[:, :, 3:])
    assert torch.allclose(z[:, :, :3], _rope_oracle(x[:, :, :3].double(), cos, sin, torch.arange(7, 10)).float(),
                          atol=1e-5)
    p = torch.randn(1, 2, 6, 16)
    out = re.apply_rope_2d(p.clone(), 2, 3)
    q = 4
    exp = p.double().clone()
    for n in range(6):
        r, c = divmod(n, 3)
        for base, pos in ((0, r), (2 * q, c)):
            a, b = p.double()[..., n, base:base + q], p.double()[..., n, base + q:base + 2 * q]
            exp[..., n, base:base + q] = a * cos[pos, :q] - b * sin[pos, :q]
            exp[..., n, base + q:base + 2 * q] = a * sin[pos, :q] + b * cos[pos, :q]
    assert torch.allclose(out, exp.float(), atol=1e-5)


def test_encoder_positional_encoding_and_heads():
    from brain_b200.models import (TransformerEncoder, PositionalEncoding, RelativePositionBias, split_heads,
                                   merge_heads, build_encoder, build_decoder)
    from brain_b200.nn import MultiHeadAttention, MultiheadAttention, FeedForwardNetwork, FeedForward
    torch.manual_seed(4)
    enc = build_encoder(2, 32, 4, 64)
    assert isinstance(enc, TransformerEncoder)
    x = torch.randn(2, 6, 32)
    y = enc(x)
    x2 = x.clone()
    x2[:, 5] += torch.randn(32)
    assert not torch.allclose(enc(x2)[:, 0], y[:, 0])  # bidirectional: position 0 sees position 5
    assert build_decoder(1, 32, 4, 64)(x, memory=y).shape == x.shape
    pe = PositionalEncoding(32, max_len=16)
    assert torch.allclose(pe(torch.zeros(1, 4, 32), offset=2)[0, 0, :2], torch.tensor([math.sin(2.0), math.cos(2.0)]))
    assert PositionalEncoding(32, 16, kind="learned").pe.requires_grad
    rb = RelativePositionBias(4, num_buckets=8, max_distance=16)
    assert rb.compute_bias(5, 7).shape == (4, 5, 7)
    t = torch.randn(2, 5, 12)
    h = split_heads(t, 3)
    assert h.shape == (2, 3, 5, 4) and torch.equal(merge_heads(h), t)
    assert MultiHeadAttention is MultiheadAttention and FeedForwardNetwork is FeedForward


@pytest.mark.gpu
def test_front_ends_on_cuda_kernels():
    from brain_b200.models import RopeConfig, RotaryEmbedding
    torch.manual_seed(5)
    dev = "cuda"
    q = torch.randn(2, 256, 8, 64, device=dev).bfloat16()
    k = torch.randn(2, 256, 2, 64, device=dev).bfloat16()
    v = torch.randn(2, 256, 2, 64, device=dev).bfloat16()
    for causal in (False, True):
        out = FlashAttentionLite(FlashLiteConfig(is_causal=causal))(q, k, v)
        ref = _ref(q.float().cpu(), k.float().cpu(), v.float().cpu(), causal)
        assert float((out.float().cpu() - ref).norm() / ref.norm()) < 1e-2
    re = RotaryEmbedding(RopeConfig(dim=64, max_seq_len=300), device=dev)
    cos, sin = RotaryEmbedding.compute_frequencies(64, 300, 10000.0)
    x = torch.randn(2, 4, 256, 64, device=dev)
    ref = _rope_oracle(x.double().cpu(), cos, sin, torch.arange(10, 266)).float()
    y = re.apply_rope_4d(x.clone(), pos_offset=10)  # float32: tensor ops
    assert torch.allclose(y.cpu(), ref, atol=1e-4)
    xb = x.bfloat16()
    refb = _rope_oracle(xb.double().cpu(), cos, sin, torch.arange(10, 266)).float()
    yb = re.apply_rope_4d(xb.clone(), pos_offset=10)  # bf16: the rope kernel, strided [B, S, H, D] view
    assert float((yb.float().cpu() - refb).abs().max()) < 3e-2


def test_vit_entry_points():
    from brain_b200.models import ViT, ViTConfig, VitModel
    from brain_b200.models import vit_extras as VX
    torch.manual_seed(6)
    cfg = ViTConfig(image_size=32, patch_size=8, in_channels=3, hidden_dim=32, num_layers=1, num_heads=2, mlp_dim=64,
                    num_classes=5)
    m = VitModel(cfg)
    img = torch.randn(2, 3, 32, 32)
    feats = m.forward_features(img)
    assert feats.shape == (2, 17, 32) and torch.allclose(m(img), m.head(feats[:, 0]))
    assert VX.num_patches_for(32, 8) == 16
    pe = VX.PatchEmbed(3, 8, 32)
    conv = torch.nn.functional.conv2d(img, pe.proj.weight.view(32, 3, 8, 8), pe.proj.bias, stride=8)
    assert torch.allclose(pe(img), conv.flatten(2).transpose(1, 2), atol=1e-5)
    assert torch.equal(VX.reconstruct_patches(m.patchify(img), 32, 8, 3), img)
    head = VX.VitHead(32, 5, pool="mean")
    assert head(feats).shape == (2, 5)
    assert VX.position_ids(4, 2).tolist() == [[0, 1, 2, 3]] * 2
    logits = torch.randn(3, 5, requires_grad=True)
    VX.label_smooth_ce(logits, torch.tensor([0, 1, 2])).backward()
    assert VX.GradientClipper(1e-3).clip([logits]) > 1e-3 and float(logits.grad.norm()) <= 1e-3 + 1e-9
