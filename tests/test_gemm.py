"""tcgen05 GEMM numerics against a float32 PyTorch oracle (all four operand majornesses)."""
import pytest
import torch

from brain_b200.ops.gemm import gemm


def _ref(a, b, ta, tb, alpha=1.0, bias=None, residual=None, out=None, beta=0.0):
    A = a.float().t() if ta else a.float()
    B = b.float().t() if tb else b.float()
    r = alpha * (A @ B)
    if out is not None and beta:
        r = r + beta * out.float()
    if bias is not None:
        r = r + bias.float()
    if residual is not None:
        r = r + residual.float()
    return r


def _mk(shape, device, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(shape, generator=g).to(device=device, dtype=torch.bfloat16)


def test_gemm_cpu_contract():
    a = _mk((33, 40), "cpu", 0)
    b = _mk((40, 17), "cpu", 1)
    c = gemm(a, b, out_dtype=torch.float32)
    torch.testing.assert_close(c, _ref(a, b, False, False), rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("shape", [(128, 256, 64), (256, 512, 192), (300, 200, 136), (1024, 1024, 1024), (64, 96, 40)])
def test_gemm_tc_layouts(ta, tb, shape):
    M, N, K = shape
    a = _mk((K, M) if ta else (M, K), "cuda", 1)
    b = _mk((N, K) if tb else (K, N), "cuda", 2)
    c = gemm(a, b, ta, tb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = _ref(a, b, ta, tb)
    torch.testing.assert_close(c, ref, rtol=2e-3, atol=2e-3 * K ** 0.5)
    from brain_b200 import _native
    assert _native.status("gemm")[0] == 0


@pytest.mark.gpu
def test_gemm_epilogue_bias_residual_accumulate():
    M, N, K = 512, 384, 256
    a = _mk((M, K), "cuda", 3)
    w = _mk((N, K), "cuda", 4)
    bias = _mk((N,), "cuda", 5)
    res = _mk((M, N), "cuda", 6)
    y = gemm(a, w, trans_b=True, bias=bias, residual=res, alpha=0.5)
    ref = _ref(a, w, False, True, alpha=0.5, bias=bias, residual=res)
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=0.1)
    acc = torch.randn(M, N, device="cuda")
    acc0 = acc.clone()
    gemm(a, w, trans_b=True, out=acc, beta=1.0)
    torch.testing.assert_close(acc, acc0 + _ref(a, w, False, True), rtol=2e-3, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("extra_cols", [0, 24, 3])  # 3: row stride not a multiple of 16 B (row-store epilogue)
def test_gemm_bf16_out_view_accumulate(extra_cols):
    """bf16 output into a column slice of a wider buffer, overwrite then accumulate, ragged tiles."""
    M, N, K = 300, 520, 136
    a = _mk((M, K), "cuda", 21)
    w = _mk((N, K), "cuda", 22)
    big = torch.full((M, N + extra_cols), 7.0, device="cuda", dtype=torch.bfloat16)
    out = big[:, :N]
    gemm(a, w, trans_b=True, out=out, beta=0.0)
    ref = _ref(a, w, False, True)
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=5e-2)
    gemm(a, w, trans_b=True, out=out, beta=1.0)
    torch.testing.assert_close(out.float(), 2 * ref, rtol=2e-2, atol=1e-1)
    if extra_cols:
        assert torch.all(big[:, N:] == 7.0)  # columns past N untouched


@pytest.mark.gpu
def test_gemm_simt_fallback_matches():
    M, N, K = 100, 70, 48
    a = _mk((M, K), "cuda", 7)
    b = _mk((K, N), "cuda", 8)
    c = gemm(a, b, out_dtype=torch.float32, force_simt=True)
    torch.testing.assert_close(c, _ref(a, b, False, False), rtol=2e-3, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("shape", [(256, 256, 64), (512, 768, 320), (300, 520, 136), (2048, 1024, 1024)])
def test_gemm_pair_and_single_cta(pair, ta, tb, shape):
    from brain_b200.ops.gemm import set_pair_mode
    M, N, K = shape
    a = _mk((K, M) if ta else (M, K), "cuda", 11)
    b = _mk((N, K) if tb else (K, N), "cuda", 12)
    old = set_pair_mode(pair)
    try:
        c = gemm(a, b, ta, tb, out_dtype=torch.float32)
        acc = torch.ones(M, N, device="cuda")
        gemm(a, b, ta, tb, out=acc, beta=1.0)
        torch.cuda.synchronize()
    finally:
        set_pair_mode(old)
    ref = _ref(a, b, ta, tb)
    torch.testing.assert_close(c, ref, rtol=2e-3, atol=2e-3 * K ** 0.5)
    torch.testing.assert_close(acc, ref + 1, rtol=2e-3, atol=2e-3 * K ** 0.5)
    from brain_b200 import _native
    assert _native.status("gemm")[0] == 0


def _tp_call(A, lda, B, ldb, b_mn, C, ldc, push_peers, mode, rank, world, push_chunk, slot, M, N, K):
    import brain_b200.parallel.tensor_parallel  # noqa: F401  (registers the entry point)
    from brain_b200 import _native
    from brain_b200.ops._common import i64_array, stream
    _native.call("brain_gemm_bf16_tp", A, lda, B.data_ptr(), ldb, b_mn, C, ldc,
                 None if push_peers is None else i64_array(push_peers), mode, rank, world, push_chunk, slot, None, 0,
                 M, N, K, stream(B))


@pytest.mark.gpu
@pytest.mark.parametrize("staged", [1, 0])
@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("M,N,W,rank", [(256, 384, 2, 1), (512, 256, 2, 1), (256, 128, 2, 1), (2048, 768, 4, 2),
                                        (3072, 520, 4, 3)])
def test_gemm_push_local_slots(staged, mode, M, N, W, rank):
    """GEMM -> reduce-scatter (mode 1) / all-reduce (mode 2) pushes into W local receive buffers: through the
    shared-memory staging with owner-rotated tile order (staged 1) or with per-row stores (staged 0)."""
    from brain_b200 import _native
    K = 256
    a, w = _mk((M, K), "cuda", 30), _mk((N, K), "cuda", 31)
    rows = M // W if mode == 1 else M
    slot = rows * N
    recv = [torch.zeros(W * slot, device="cuda", dtype=torch.bfloat16) for _ in range(W)]
    old = _native.fn("brain_gemm_set_push_stage")(staged)
    try:
        _tp_call(a.data_ptr(), K, w, K, 0, 0, N, [r.data_ptr() for r in recv], mode, rank, W,
                 rows if mode == 1 else M, slot, M, N, K)
        torch.cuda.synchronize()
    finally:
        _native.fn("brain_gemm_set_push_stage")(old)
    ref = a.float() @ w.float().t()
    for j in range(W):
        got = recv[j][rank * slot:(rank + 1) * slot].view(rows, N).float()
        exp = ref[j * rows:(j + 1) * rows] if mode == 1 else ref
        torch.testing.assert_close(got, exp, rtol=2e-2, atol=2e-1)
        others = torch.cat([recv[j][:rank * slot], recv[j][(rank + 1) * slot:]])
        assert others.abs().sum().item() == 0  # nothing outside this rank's slot
    assert _native.status("gemm")[0] == 0


@pytest.mark.gpu
def test_gemm_rejects_operand_on_other_device():
    a = _mk((128, 64), "cuda", 40)
    b = _mk((64, 128), "cpu", 41)
    with pytest.raises(ValueError):
        gemm(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("ta,tb", [(True, False), (False, True), (False, False)])
@pytest.mark.parametrize("shape", [(768, 768, 12608), (2304, 768, 8192), (300, 520, 6144)])
def test_gemm_splitk_matches_oracle(ta, tb, shape):
    """Under-filled GEMMs (fewer 256 x 256 tiles than SM pairs, long K) take the split-K path: each
    K slice on its own SM pair into an f32 workspace, then an ordered reduction with the epilogue."""
    from brain_b200.ops.gemm import _splitk_plan
    from brain_b200 import _native
    M, N, K = shape
    assert _splitk_plan(M, N, K) > 1
    a = _mk((K, M) if ta else (M, K), "cuda", 31)
    b = _mk((N, K) if tb else (K, N), "cuda", 32)
    ref = _ref(a, b, ta, tb)
    tol = dict(rtol=2e-3, atol=2e-3 * K ** 0.5)
    c = gemm(a, b, ta, tb, out_dtype=torch.float32)
    torch.testing.assert_close(c, ref, **tol)
    acc = torch.randn(M, N, device="cuda")  # main-grad style accumulation into f32
    acc0 = acc.clone()
    gemm(a, b, ta, tb, out=acc, beta=1.0)
    torch.testing.assert_close(acc, acc0 + ref, **tol)
    bias = _mk((N,), "cuda", 33)
    res = _mk((M, N), "cuda", 34)
    y = gemm(a, b, ta, tb, bias=bias, residual=res, alpha=0.25)
    torch.testing.assert_close(y.float(), _ref(a, b, ta, tb, alpha=0.25, bias=bias, residual=res), rtol=1e-2,
                               atol=0.25 * 2e-3 * K ** 0.5 + 0.1)
    c2 = gemm(a, b, ta, tb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(c, c2)  # the slices are added in a fixed order
    assert _native.status("gemm")[0] == 0


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(300, 520, 136), (8192, 1024, 256), (4096, 768, 768), (256, 2304, 64)])
def test_gemm_residual_by_tma_matches_oracle(shape):
    """bf16 output with bias and residual on the CTA-pair kernel: the residual boxes arrive by TMA one
    64-column unit ahead (across tiles too when a pair runs several); ragged edges are zero-filled."""
    M, N, K = shape
    a = _mk((M, K), "cuda", 41)
    w = _mk((N, K), "cuda", 42)
    bias = _mk((N,), "cuda", 43)
    res = _mk((M, N), "cuda", 44)
    y = gemm(a, w, trans_b=True, bias=bias, residual=res)
    ref = _ref(a, w, False, True, bias=bias, residual=res)
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=2e-3 * K ** 0.5 + 0.05)
    big = torch.randn(M, N + 64, device="cuda").to(torch.bfloat16)  # residual as a strided view
    y2 = gemm(a, w, trans_b=True, residual=big[:, 8:8 + N])
    torch.testing.assert_close(y2.float(), _ref(a, w, False, True, residual=big[:, 8:8 + N]), rtol=1e-2,
                               atol=2e-3 * K ** 0.5 + 0.05)
    from brain_b200 import _native
    assert _native.status("gemm")[0] == 0


@pytest.mark.gpu
@pytest.mark.parametrize("ta,tb,shape", [
    (False, True, (8192, 28672, 4096)),   # gate_up forward: many waves of the persistent scheduler
    (False, True, (8192, 4096, 14336)),   # down forward: K = 14336 through the stage ring
    (False, False, (8192, 14336, 4096)),  # dgrad of down
    (True, False, (4096, 6144, 8192)),    # weight gradient of qkv (A transposed)
    (False, True, (4096, 128256, 4096)),  # LM head: N = 128256 with a ragged last tile column
])
def test_gemm_production_shapes_sampled_rows(ta, tb, shape):
    """Llama-3-8B training shapes on the CTA-pair kernel: full GEMM in bf16, then 96 sampled rows (the
    first and last rows, rows around 256-row tile edges, random rows) against a float32 oracle."""
    from brain_b200 import _native
    M, N, K = shape
    a = (torch.randn((K, M) if ta else (M, K), device="cuda") * 0.5).to(torch.bfloat16)
    b = (torch.randn((N, K) if tb else (K, N), device="cuda") * 0.5).to(torch.bfloat16)
    c = gemm(a, b, ta, tb)
    torch.cuda.synchronize()
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    edges = [0, 1, 255, 256, 257, M // 2 - 1, M // 2, M - 257, M - 256, M - 2, M - 1]
    rows = torch.tensor(sorted(set(edges + torch.randint(0, M, (96 - len(edges),), generator=g).tolist())),
                        device="cuda")
    A = a.float().t()[rows] if ta else a.float()[rows]
    B = b.float().t() if tb else b.float()
    ref = A @ B
    torch.testing.assert_close(c[rows].float(), ref, rtol=1e-2, atol=2e-3 * K ** 0.5 * 0.25 + 0.02)
    assert _native.status("gemm")[0] == 0
