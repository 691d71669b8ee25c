"""The data-parallel training step against a float32 PyTorch oracle.

* One GPU: every parameter's gradient (the flat ``main_grad`` written by the fused backward kernels)
  against the float32 restatement of the model (``models.llama_oracle``), on consecutive steps (a
  gradient left over from the previous step, or a zeroed one, fails); the master weights after
  several steps against ``torch.optim.AdamW`` fed the same gradients (a skipped, zeroed or mis-scaled
  update fails); one layer of the Llama-3-8B shape at sequence 4096 (vocabulary 128256, d 4096, GQA
  32/8) for the production-size GEMM, attention and cross-entropy paths.
* Two ranks: a data-parallel step on batches (a, b) equals a one-rank step on cat(a, b), for the NCCL
  path, the fused NVLink step and both overlapped modes. The test uses AdamW with a large epsilon so
  the update is proportional to the reduced gradient: a missing 1/world, a skipped shard or a stale
  gradient changes it by O(1).
"""
import pytest
import torch

from brain_b200.models import llama_oracle as O

GRAD_TOL = 0.05     # bf16 activations and weights against the float32 oracle (measured: ~0.01)
UPDATE_TOL = 1e-4   # same float32 AdamW arithmetic, different summation order


def _cfg(**kw):
    from brain_b200.models import LlamaLiteConfig
    base = dict(vocab_size=2048, hidden_dim=512, num_layers=2, num_heads=8, num_kv_heads=2, head_dim=64,
                intermediate_dim=1536, max_seq_len=512, rope_theta=500000.0)
    base.update(kw)
    return LlamaLiteConfig(**base)


def _grad_errors(model, ref_grads):
    return {n: O.rel_err(p.main_grad.float(), ref_grads[n]) for n, p in model.named_parameters()}


@pytest.mark.gpu
@pytest.mark.parametrize("grad_dtype", [torch.float32, torch.bfloat16])
def test_single_gpu_step_matches_fp32_oracle(grad_dtype):
    from brain_b200.models import LlamaLite
    from brain_b200.parallel import DataParallel, dist as bdist
    bdist.init(timeout_s=60)
    cfg = _cfg()
    model = LlamaLite(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    lr, betas, eps, wd = 1e-3, (0.9, 0.95), 1e-8, 0.1
    dp = DataParallel(model, lr=lr, betas=betas, eps=eps, weight_decay=wd, grad_dtype=grad_dtype)
    master0 = dp.optimizer.master.clone()
    g = torch.Generator(device="cuda").manual_seed(3)
    grads = []
    for step in range(3):
        tok = torch.randint(0, cfg.vocab_size, (2, 513), device="cuda", generator=g)
        ref_loss, ref = O.loss_and_grads(model, tok[:, :-1], tok[:, 1:])
        loss = dp.train_step(tok[:, :-1], tok[:, 1:])
        assert abs(float(loss) - float(ref_loss)) < 2e-2 * float(ref_loss), (step, float(loss), float(ref_loss))
        errs = _grad_errors(model, ref)
        worst = max(errs, key=errs.get)
        assert errs[worst] < GRAD_TOL, (step, worst, errs)
        grads.append(dp.flat.grad_buf.float().clone())
    ref_master = O.adamw_reference(master0, grads, lr, betas, eps, wd)
    delta, ref_delta = dp.optimizer.master - master0, ref_master - master0
    assert O.rel_err(delta, ref_delta) < UPDATE_TOL
    # the bf16 compute weights are the rounded master weights
    assert torch.equal(dp.flat.param_buf, dp.optimizer.master.to(torch.bfloat16))
    bdist.shutdown()


@pytest.mark.gpu
@pytest.mark.slow
def test_llama8b_shape_layer_gradients_match_fp32_oracle():
    """One block of the 8B shape at seq 4096: the GEMMs at K = 4096 / 14336, N = 6144 / 28672 /
    128256, the tcgen05 attention at S = 4096 and the 128256-class cross-entropy."""
    from brain_b200.models import LlamaLite, LlamaLiteConfig
    from brain_b200.parallel import DataParallel, dist as bdist
    bdist.init(timeout_s=60)
    cfg = LlamaLiteConfig.llama3_8b(max_seq_len=4096).replace(num_layers=1)
    model = LlamaLite(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
    dp = DataParallel(model, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, grad_dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(5)
    for step in range(2):
        tok = torch.randint(0, cfg.vocab_size, (1, 4097), device="cuda", generator=g)
        ref_loss, ref = O.loss_and_grads(model, tok[:, :-1], tok[:, 1:])
        loss = dp.train_step(tok[:, :-1], tok[:, 1:])
        assert abs(float(loss) - float(ref_loss)) < 1e-2 * float(ref_loss), (float(loss), float(ref_loss))
        errs = _grad_errors(model, ref)
        del ref
        worst = max(errs, key=errs.get)
        assert errs[worst] < GRAD_TOL, (step, worst, errs)
    bdist.shutdown()


# --------------------------------------------------------------------------- two ranks vs one
LINEAR_ADAM = dict(lr=1e-2, betas=(0.9, 0.95), eps=1.0, weight_decay=0.0)  # update ~ lr * gradient


def _batches(cfg, n_steps, world):
    g = torch.Generator().manual_seed(11)
    return [torch.randint(0, cfg.vocab_size, (2 * world, 129), generator=g) for _ in range(n_steps)]


def _dp_run(rank, world, kind, device):
    """Two steps of DataParallel on rank ``rank``'s slice of each global batch; returns the f32 master
    delta of this rank's shard (flat layout) and the losses."""
    from brain_b200.models import LlamaLite
    from brain_b200.parallel import DataParallel, dist as bdist
    if device == "cpu":
        bdist.init(backend="gloo", device="cpu", timeout_s=120)
        dtype = torch.float32
    else:
        bdist.init(timeout_s=120)
        dtype = torch.bfloat16
    cfg = _cfg(vocab_size=512, hidden_dim=256, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
               intermediate_dim=512, max_seq_len=128)
    dev = "cpu" if device == "cpu" else "cuda"
    model = LlamaLite(cfg, device=dev, dtype=dtype, seed=0)
    overlap = kind.startswith("nvlink-overlap")
    comm = "nccl" if kind in ("nccl", "gloo") else "nvlink"
    dp = DataParallel(model, **LINEAR_ADAM, grad_dtype=torch.float32, comm=comm, overlap=overlap,
                      bucket_bytes=64 << 10, overlap_mode="sm" if kind.endswith("-sm") else "ce")
    opt = dp.overlapped if dp.overlapped is not None else dp.optimizer
    master0 = opt.master.clone()
    losses = []
    for t in _batches(cfg, 2, 2):
        per = t.shape[0] // world
        t = t[rank * per:(rank + 1) * per].to(dev)
        losses.append(float(dp.train_step(t[:, :-1], t[:, 1:])))
    if hasattr(dp.comm, "check"):
        dp.comm.check()
    delta = (opt.master - master0).cpu().numpy()  # numpy: tensors in the result queue need the sender alive
    pieces = getattr(dp.overlapped, "pieces", None)
    weights = dp.flat.param_buf.float().cpu().numpy()
    if hasattr(dp.comm, "close") and comm == "nvlink":
        if dp.overlapped is not None:
            dp.overlapped.close()
        dp.comm.close()
    bdist.shutdown()
    return delta, losses, pieces, weights


def _full_delta(outs):
    """Concatenate the ranks' shard deltas into the flat layout."""
    pieces = outs[0][2]
    if pieces is None:
        return torch.cat([torch.from_numpy(o[0]) for o in outs])
    total = max(a + n for o in outs for a, n, _ in o[2])
    full = torch.zeros(total)
    for delta, _, ps, _ in outs:
        for a, n, s in ps:
            full[a:a + n] = torch.from_numpy(delta[s:s + n])
    return full


def _check_losses(two, one, tol):
    # each rank's loss is the mean over its half of the global batch; the single rank's over all of it
    for step, single in enumerate(one[0][1]):
        mean2 = sum(o[1][step] for o in two) / len(two)
        assert abs(mean2 - single) < tol * abs(single), (step, mean2, single)


@pytest.mark.parametrize("kind", ["gloo"])
def test_two_rank_step_equals_one_rank_on_concatenated_batch_cpu(kind):
    from _mp import run_ranks
    two = run_ranks(_dp_run, 2, kind, "cpu")
    one = run_ranks(_dp_run, 1, kind, "cpu")
    d2, d1 = _full_delta(two), _full_delta(one)
    n = min(d2.numel(), d1.numel())
    d2, d1 = d2[:n], d1[:n]
    assert O.rel_err(d2, d1) < 1e-4, O.rel_err(d2, d1)
    _check_losses(two, one, 1e-5)
    assert (two[0][3] == two[1][3]).all()
    # a step with no update, or one with twice the gradient, is far outside that
    assert O.rel_err(torch.zeros_like(d1), d1) > 0.5 and O.rel_err(2 * d1, d1) > 0.5


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("kind", ["nccl", "nvlink", "nvlink-overlap", "nvlink-overlap-sm"])
def test_two_rank_step_equals_one_rank_on_concatenated_batch(kind):
    from _mp import run_ranks
    env = {"NCCL_NVLS_ENABLE": "0"}
    two = run_ranks(_dp_run, 2, kind, "cuda", env=env)
    one = run_ranks(_dp_run, 1, "nccl", "cuda", env=env)
    d2, d1 = _full_delta(two), _full_delta(one)
    n = min(d2.numel(), d1.numel())
    err = O.rel_err(d2[:n], d1[:n])
    assert err < GRAD_TOL, (kind, err)
    _check_losses(two, one, 2e-2)
    assert (two[0][3] == two[1][3]).all()  # the replicas hold identical weights after the push


# --------------------------------------------------------------------------- guarded step
def _guard_run(rank, world, kind, device, inject_step=1, max_norm=0.0):
    """Three steps with dynamic loss scaling (and optional clipping); on ``inject_step`` rank 1 (or
    rank 0 alone) writes a NaN into flat gradient element 0 (owned by rank 0's shard or piece) after
    backward. Returns per-step master deltas of this rank's shard, the scaler's scales and the skip count."""
    from brain_b200.autograd.functional import GradScaler
    from brain_b200.models import LlamaLite
    from brain_b200.parallel import DataParallel, dist as bdist
    if device == "cpu":
        bdist.init(backend="gloo", device="cpu", timeout_s=120)
        dtype, dev = torch.float32, "cpu"
    else:
        bdist.init(timeout_s=120)
        dtype, dev = torch.bfloat16, "cuda"
    cfg = _cfg(vocab_size=512, hidden_dim=256, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
               intermediate_dim=512, max_seq_len=128)
    model = LlamaLite(cfg, device=dev, dtype=dtype, seed=0)
    overlap = kind.startswith("nvlink-overlap")
    comm = "nccl" if kind in ("nccl", "gloo") else "nvlink"
    scaler = GradScaler(init_scale=1024.0, growth_interval=1000)
    dp = DataParallel(model, lr=1e-3, grad_dtype=torch.float32, comm=comm, overlap=overlap, bucket_bytes=64 << 10,
                      overlap_mode="sm" if kind.endswith("-sm") else "ce", grad_scaler=scaler, max_grad_norm=max_norm)
    opt = dp.overlapped if dp.overlapped is not None else dp.optimizer
    culprit = 1 if world > 1 else 0
    step_no = [0]

    def inject(d):
        if step_no[0] == inject_step and d.rank == culprit:
            d.flat.grad_buf[0] = float("nan")
    dp.after_backward.append(inject)
    deltas, scales = [], []
    for t in _batches(cfg, 3, 2):
        per = t.shape[0] // world
        t = t[rank * per:(rank + 1) * per].to(dev)
        before = opt.master.clone()
        dp.train_step(t[:, :-1], t[:, 1:])
        deltas.append(float((opt.master - before).abs().max()))
        scales.append(scaler.scale)
        step_no[0] += 1
    if hasattr(dp.comm, "check"):
        dp.comm.check()
    out = (deltas, scales, dp.skipped_steps, dp.optimizer.step_count)
    if comm == "nvlink":
        if dp.overlapped is not None:
            dp.overlapped.close()
        dp.comm.close()
    bdist.shutdown()
    return out


def _check_skip(outs):
    for deltas, scales, skipped, count in outs:
        assert deltas[0] > 0 and deltas[2] > 0, deltas   # normal steps update
        assert deltas[1] == 0.0, deltas                   # the poisoned step is skipped on every rank
        assert scales == [1024.0, 512.0, 512.0], scales  # and the loss scale backs off once
        assert skipped == 1 and count == 2, (skipped, count)


def test_nan_on_one_rank_skips_the_step_on_every_rank_cpu():
    from _mp import run_ranks
    _check_skip(run_ranks(_guard_run, 2, "gloo", "cpu"))


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("kind", ["nccl", "nvlink", "nvlink-overlap", "nvlink-overlap-sm"])
def test_nan_on_one_rank_skips_the_step_on_every_rank(kind):
    from _mp import run_ranks
    _check_skip(run_ranks(_guard_run, 2, kind, "cuda", env={"NCCL_NVLS_ENABLE": "0"}))


@pytest.mark.gpu
def test_nan_skips_the_step_single_gpu():
    from _mp import run_ranks
    _check_skip(run_ranks(_guard_run, 1, "nccl", "cuda"))


def _clip_single(rank, world, device):
    """DataParallel with max_grad_norm against torch: clip_grad_norm_ over the same gradients, then
    torch.optim.AdamW; returns the relative error of the master weights after two steps."""
    from brain_b200.models import LlamaLite
    from brain_b200.parallel import DataParallel, dist as bdist
    if device == "cpu":
        bdist.init(backend="gloo", device="cpu", timeout_s=60)
    else:
        bdist.init(timeout_s=60)
    dtype = torch.float32 if device == "cpu" else torch.bfloat16
    cfg = _cfg(vocab_size=512, hidden_dim=256, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
               intermediate_dim=512, max_seq_len=128)
    model = LlamaLite(cfg, device=device, dtype=dtype, seed=0)
    lr, betas, eps, wd, max_norm = 1e-3, (0.9, 0.95), 1e-8, 0.1, 0.05
    dp = DataParallel(model, lr=lr, betas=betas, eps=eps, weight_decay=wd, grad_dtype=torch.float32,
                      max_grad_norm=max_norm)
    master0 = dp.optimizer.master.clone()
    clipped, norms = [], []
    for t in _batches(cfg, 2, 1):
        t = t.to(device)
        dp.train_step(t[:, :-1], t[:, 1:])
        g = dp.flat.grad_buf.float().clone()
        norm = float(g.norm())
        norms.append((dp.grad_norm(), norm))
        clipped.append(g * min(1.0, max_norm / (norm + 1e-6)))
    ref = O.adamw_reference(master0, clipped, lr, betas, eps, wd)
    err = O.rel_err(dp.optimizer.master - master0, ref - master0)
    bdist.shutdown()
    return err, norms


def test_global_norm_clipping_matches_torch_cpu():
    from _mp import run_ranks
    err, norms = run_ranks(_clip_single, 1, "cpu")[0]
    assert err < 1e-4, err
    for mine, ref in norms:
        assert abs(mine - ref) < 1e-3 * ref and ref > 0.05  # the clip is active


@pytest.mark.gpu
def test_global_norm_clipping_matches_torch_single_gpu():
    from _mp import run_ranks
    err, norms = run_ranks(_clip_single, 1, "cuda")[0]
    assert err < 1e-4, err
    for mine, ref in norms:
        assert abs(mine - ref) < 1e-3 * ref and ref > 0.05
