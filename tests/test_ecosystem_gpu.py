"""Ecosystem modules on the GPU through the framework's kernels: the graph interpreter's GEMM nodes, the
BLAS gemm with alpha / beta, the LSTM cell's gate projections, and the native token loader feeding a
CUDA tensor. Each result is compared with a float32 PyTorch computation of the same op."""
import numpy as np
import pytest
import torch

gpu = pytest.mark.gpu


def _close(a, b, tol=3e-2):
    torch.testing.assert_close(a.float(), b.float(), rtol=tol, atol=tol)


@gpu
def test_graph_interpreter_gemm_nodes_on_tcgen05():
    from brain_b200 import graph as G
    from brain_b200 import ops
    g = G.GraphIr("mlp")
    x = g.add_input("x", (256, 128), "bfloat16")
    w1 = g.constant("w1", (torch.randn(256, 128) * 0.05).bfloat16())
    b1 = g.constant("b1", (torch.randn(256) * 0.1).bfloat16())
    w2 = g.constant("w2", (torch.randn(256, 64) * 0.05).bfloat16())
    h = g.add_node("gelu", [g.add_node("linear", [x, w1, b1])])
    g.mark_output(g.add_node("matmul", [h, w2]))
    xi = torch.randn(256, 128, device="cuda").bfloat16()
    out = G.GraphInterpreter().run(g, [xi])[0]
    cw = {v.name: v.constant.float().cuda() for v in g.values.values() if v.constant is not None}
    ref = torch.nn.functional.gelu(xi.float() @ cw["w1"].t() + cw["b1"], approximate="tanh") @ cw["w2"]
    _close(out, ref)
    assert not ops.check_status()


@gpu
def test_blas_gemm_alpha_beta_bf16():
    from brain_b200.device import CudaBackend, blas
    a = torch.randn(256, 512, device="cuda").bfloat16()
    b = torch.randn(384, 512, device="cuda").bfloat16()
    c = torch.randn(256, 384, device="cuda", dtype=torch.float32)
    ref = 0.5 * a.float() @ b.float().t() + 2.0 * c
    out = blas.gemm(a, b, c.clone(), alpha=0.5, beta=2.0, trans_b=True)
    _close(out, ref, 0.15)
    _close(CudaBackend().matmul(a, b.t().contiguous()), a.float() @ b.float().t(), 0.3)


@gpu
def test_lstm_cell_bf16_on_gpu_matches_fp32():
    from brain_b200.zoo import rnn
    torch.manual_seed(0)
    cell = rnn.LstmCell(128, 128)
    x, h, c = torch.randn(64, 128), torch.randn(64, 128), torch.randn(64, 128)
    h_ref, c_ref = cell(x, (h, c))
    cg = rnn.LstmCell(128, 128, device="cuda", dtype=torch.bfloat16)
    cg.load_state_dict({k: v.bfloat16() for k, v in cell.state_dict().items()})
    h1, c1 = cg(x.cuda().bfloat16(), (h.cuda().bfloat16(), c.cuda().bfloat16()))
    _close(h1.cpu(), h_ref, 5e-2)
    _close(c1.cpu(), c_ref, 5e-2)


@gpu
def test_native_loader_to_device(tmp_path):
    from brain_b200 import data as D
    toks = np.random.default_rng(1).integers(0, 32000, size=20000).astype(np.uint16)
    p = str(tmp_path / "t.bin")
    D.write_token_file(p, toks)
    L = D.NativeTokenLoader(p, batch=2, seq=64, seed=3, device="cuda")
    x, y = L.next()
    torch.cuda.synchronize()
    ref = L.batch_at(0)
    assert x.is_cuda and torch.equal(x.cpu(), ref[:, :-1]) and torch.equal(y.cpu(), ref[:, 1:])
    L.close()


@gpu
def test_cpu_offloader_gives_same_gradients():
    from brain_b200.autograd import CpuOffloader
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(512, 1024), torch.nn.GELU(), torch.nn.Linear(1024, 512)).cuda()
    x = torch.randn(1024, 512, device="cuda")
    net(x).pow(2).mean().backward()
    ref = [p.grad.clone() for p in net.parameters()]
    net.zero_grad()
    with CpuOffloader(min_bytes=1 << 16) as off:
        y = net(x)
    y.pow(2).mean().backward()
    assert off.offloaded > 0
    for p, r in zip(net.parameters(), ref):
        torch.testing.assert_close(p.grad, r)


@gpu
def test_zoo_models_train_on_gpu_kernels():
    """GNN, diffusion denoiser, GAN and RL networks in bf16 on the GPU: one optimisation step each runs
    forward and backward through the framework's GEMM kernels and stays finite."""
    from brain_b200 import ops
    from brain_b200.zoo import diffusion as D
    from brain_b200.zoo import gan, gnn, rl
    torch.manual_seed(0)
    dev, dt = "cuda", torch.bfloat16
    g = gnn.Graph.from_undirected([(0, 1), (1, 2), (2, 3), (3, 0)], 4, device=dev)
    net = gnn.GnnNodeClassifier(64, 64, 2, "gcn", device=dev, dtype=dt)
    x = torch.randn(4, 64, device=dev, dtype=dt)
    loss = torch.nn.functional.cross_entropy(net(g, x).float(), torch.tensor([0, 1, 0, 1], device=dev))
    loss.backward()
    assert torch.isfinite(loss) and all(torch.isfinite(p.grad).all() for p in net.parameters())
    den = D.MlpDenoiser(64, 128, device=dev, dtype=dt)
    sched = D.LinearSchedule(100)
    l2 = D.diffusion_loss(den, sched, torch.randn(32, 64, device=dev, dtype=dt))
    l2.backward()
    assert torch.isfinite(l2)
    G, Dn = gan.MlpGenerator(16, 64, 64, device=dev, dtype=dt), gan.MlpDiscriminator(64, 64, device=dev, dtype=dt)
    og, od = torch.optim.SGD(G.parameters(), 1e-3), torch.optim.SGD(Dn.parameters(), 1e-3)
    ld, lg = gan.train_step(G, Dn, og, od, torch.randn(32, 64, device=dev, dtype=dt))
    assert ld == ld and lg == lg
    q = rl.MlpNet(64, 4, 64, device=dev, dtype=dt)
    out = q(torch.randn(8, 64, device=dev, dtype=dt))
    assert out.shape == (8, 4) and torch.isfinite(out.float()).all()
    assert not ops.check_status()
