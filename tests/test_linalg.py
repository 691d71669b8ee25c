"""Linear algebra, FFT and sparse routines: the reference's own test vectors
(crates/brain-core/src/tensor/linalg.rs, fft.rs, sparse.rs test modules) on the CPU, float64 oracles for
the factorisations, and the batched Jacobi SVD / CSR SpMM kernels against torch on the GPU."""
import math

import pytest
import torch

from brain_b200 import linalg as LA

T = lambda *rows: torch.tensor(rows, dtype=torch.float64)  # noqa: E731


def test_norms_and_trace_reference_vectors():
    a = T([1.0, -2.0], [3.0, -4.0])
    assert LA.norm_l1(a) == 10.0 and LA.norm_linf(a) == 4.0 and LA.trace(a) == -3.0
    assert abs(LA.norm_l2(a) - math.sqrt(30.0)) < 1e-12 and LA.norm_frobenius(a) == LA.norm_l2(a)
    assert abs(LA.norm_p(a, 3.0) - (1 + 8 + 27 + 64) ** (1 / 3)) < 1e-12
    with pytest.raises(ValueError):
        LA.norm_p(a, 0.5)
    assert abs(LA.norm_nuclear(a) - float(torch.linalg.svdvals(a).sum())) < 1e-10


def test_det_logdet_inv_reference_vectors():
    a = T([4.0, 7.0], [2.0, 6.0])
    assert LA.det(a) == 10.0
    torch.testing.assert_close(a @ LA.inv(a), torch.eye(2, dtype=torch.float64))
    a4 = T([2, 1, 3, 4], [0, 3, 2, 1], [0, 0, 5, 6], [0, 0, 0, 7])
    assert abs(LA.det(a4) - 210.0) < 1e-9 and abs(LA.logdet(a4) - math.log(210.0)) < 1e-9
    a8 = torch.diag(torch.arange(1, 9, dtype=torch.float64))
    assert abs(LA.det(a8) - 40320.0) < 1e-7
    g = torch.Generator().manual_seed(0)
    for n in (3, 5, 9):
        x = torch.randn(n, n, generator=g, dtype=torch.float64)
        assert abs(LA.det(x) - float(torch.linalg.det(x))) < 1e-9 * max(1.0, abs(float(torch.linalg.det(x))))
        sign, ld = LA.slogdet(x)
        s2, l2 = torch.linalg.slogdet(x)
        assert sign == float(s2) and abs(ld - float(l2)) < 1e-9
    assert LA.slogdet(torch.zeros(3, 3, dtype=torch.float64)) == (0.0, -math.inf)


def test_lu_pivoting_and_solve():
    a = T([3.0, 2.0, -1.0], [2.0, -2.0, 4.0], [-1.0, 0.5, -1.0])
    l, u, p = LA.lu(a)
    torch.testing.assert_close(l @ u, a[p])
    x = LA.lu_solve(l, u, p, T(1.0, -2.0, 0.0).view(-1))
    torch.testing.assert_close(a @ x, T(1.0, -2.0, 0.0).view(-1))
    # ties keep the earlier row; the first row of largest magnitude below becomes the pivot
    l2, u2, p2 = LA.lu(T([1.0, 2.0], [-1.0, 3.0]))
    assert p2 == [0, 1]
    _, _, p3 = LA.lu(T([1.0, 2.0], [4.0, 3.0], [-4.0, 1.0]))
    assert p3[0] == 1
    # rectangular shapes
    for shape in ((5, 3), (3, 5)):
        r = torch.randn(*shape, dtype=torch.float64, generator=torch.Generator().manual_seed(1))
        l, u, p = LA.lu(r)
        assert l.shape == (shape[0], min(shape)) and u.shape == (min(shape), shape[1])
        torch.testing.assert_close(l @ u, r[p])
    # a zero pivot column is left un-eliminated and its unknown set to 0, as in the reference
    s = T([0.0, 1.0], [0.0, 2.0])
    l, u, p = LA.lu(s)
    assert torch.isfinite(LA.lu_solve(l, u, p, T(1.0, 2.0).view(-1))).all()


def test_qr_cholesky_solves():
    a = T([12.0, -51.0], [6.0, 167.0])
    q, r = LA.qr(a)
    torch.testing.assert_close(q @ r, a)
    torch.testing.assert_close(q.t() @ q, torch.eye(2, dtype=torch.float64))
    assert float(r[1, 0]) == pytest.approx(0.0, abs=1e-12)
    g = torch.Generator().manual_seed(2)
    m = torch.randn(6, 4, generator=g, dtype=torch.float64)
    q, r = LA.qr(m)
    assert q.shape == (6, 6) and r.shape == (6, 4)
    torch.testing.assert_close(q @ r, m)
    assert torch.allclose(torch.tril(r, -1), torch.zeros_like(r), atol=1e-12)
    assert float(r[0, 0]) < 0 if float(m[0, 0]) >= 0 else float(r[0, 0]) > 0  # reflect onto -sign(r_kk)|x|
    sq = torch.randn(5, 5, generator=g, dtype=torch.float64)
    b = torch.randn(5, generator=g, dtype=torch.float64)
    q, r = LA.qr(sq)
    torch.testing.assert_close(sq @ LA.qr_solve(q, r, b), b)
    l = LA.cholesky(T([4.0, 12.0], [12.0, 45.0]))
    assert (float(l[0, 0]), float(l[1, 0]), float(l[1, 1])) == (2.0, 6.0, 3.0)
    spd = sq @ sq.t() + 5 * torch.eye(5, dtype=torch.float64)
    l = LA.cholesky(spd)
    torch.testing.assert_close(l, torch.linalg.cholesky(spd))
    torch.testing.assert_close(spd @ LA.cholesky_solve(l, b), b)
    with pytest.raises(ValueError):
        LA.cholesky(T([1.0, 2.0], [2.0, 1.0]))
    torch.testing.assert_close(LA.solve(sq, b), torch.linalg.solve(sq, b))


def test_jacobi_svd_cpu_reference_matrix_and_derived():
    m = T([1.0, 2.0, 0.5], [2.0, 3.0, 1.0], [0.5, 1.0, 4.0])
    r = LA.svd_symmetric(m)
    rec = (r.u * r.singular_values) @ r.v.t()
    assert float((rec - m).norm()) < 1e-6
    torch.testing.assert_close(r.singular_values.sort(descending=True).values, torch.linalg.svdvals(m))
    w, v = LA.eigh(m)  # singular values = |eigenvalues|
    torch.testing.assert_close(w.sort().values, torch.linalg.eigvalsh(m).abs().sort().values)
    a = T([2.0, 1.0], [1.0, 2.0])
    torch.testing.assert_close(LA.inv(a), LA.matrix_power(a, -1))
    assert LA.matrix_power(a, 0).tolist() == [[1.0, 0.0], [0.0, 1.0]]
    torch.testing.assert_close(LA.matrix_power(a, 5), torch.linalg.matrix_power(a, 5))
    torch.testing.assert_close(LA.pinv(m), torch.linalg.inv(m))
    assert abs(LA.condition_number(a) - 3.0) < 1e-12
    assert LA.condition_number(T([1.0, 1.0], [1.0, 1.0])) == math.inf
    b = T(1.0, 2.0, 3.0).view(-1)
    torch.testing.assert_close(m @ LA.svd_solve(r.u, r.singular_values, r.v, b), b)
    batch = torch.randn(3, 4, 4, dtype=torch.float64, generator=torch.Generator().manual_seed(3))
    rb = LA.svd_symmetric(batch)
    torch.testing.assert_close((rb.u * rb.singular_values.unsqueeze(-2)) @ rb.v.transpose(-1, -2), batch)


def test_fft_reference_roundtrips_and_windows():
    for size in (4, 8, 16, 64, 128):
        orig = torch.sin(torch.arange(size, dtype=torch.float64) * 0.3)
        re, im = orig.clone(), torch.zeros(size, dtype=torch.float64)
        LA.fft_radix2(re, im, False)
        want = torch.fft.fft(orig)
        torch.testing.assert_close(re, want.real)
        torch.testing.assert_close(im, want.imag)
        LA.fft_radix2(re, im, True)
        assert float((re - orig).abs().max()) < 1e-6 and float(im.abs().max()) < 1e-6
    for size in (3, 5, 7, 13, 17, 25, 50):
        orig = torch.cos(torch.arange(size, dtype=torch.float64) * 0.5)
        re, im = orig.clone(), torch.zeros(size, dtype=torch.float64)
        LA.dft(re, im, False)
        torch.testing.assert_close(re, torch.fft.fft(orig).real)
        LA.dft(re, im, True)
        assert float((re - orig).abs().max()) < 1e-6 and float(im.abs().max()) < 1e-6
    re, im = LA.rfft(T(1.0, 2.0, 3.0, 4.0).view(-1))
    assert re.shape == (3,) and im.shape == (3,) and float(re[0]) == 10.0
    h, hm = LA.hann_window(16), LA.hamming_window(16)
    assert h.shape == (16,) and float(h[0]) == 0.0 and abs(float(hm[0]) - 0.08) < 1e-6
    with pytest.raises(ValueError):
        LA.fft_radix2(torch.zeros(6), torch.zeros(6))
    batch = torch.randn(3, 32, dtype=torch.float64)
    re, im = batch.clone(), torch.zeros_like(batch)
    LA.fft_radix2(re, im)
    torch.testing.assert_close(re, torch.fft.fft(batch).real)


def test_sparse_coo_reference_vectors_and_spmm():
    coo = LA.SparseCOO((2, 2))
    coo.insert(0, 0, 5.0)
    coo.insert(1, 1, 3.0)
    assert coo.to_dense().tolist() == [[5.0, 0.0], [0.0, 3.0]]
    coo = LA.SparseCOO((2, 3))
    coo.insert(0, 1, 5.0)
    coo.insert(1, 2, 10.0)
    coo.insert(1, 2, 1.0)  # duplicates add up
    d = coo.to_dense()
    assert d.shape == (2, 3) and float(d[0, 1]) == 5.0 and float(d[1, 2]) == 11.0
    b = torch.randn(3, 4, dtype=torch.float64)
    torch.testing.assert_close(coo.spmm(b), d @ b)
    indptr, idx, vals = coo.to_csr()
    assert indptr.tolist() == [0, 1, 3] and idx.tolist() == [1, 2, 2]
    with pytest.raises(IndexError):
        coo.insert(2, 0, 1.0)


# ------------------------------------------------------------------------------------ GPU kernels
@pytest.mark.gpu
@pytest.mark.parametrize("n,nb,dtype", [(3, 1, torch.float64), (16, 64, torch.float32), (33, 10, torch.float64),
                                        (64, 300, torch.float32), (96, 4, torch.float64)])
def test_jacobi_svd_kernel_matches_torch(n, nb, dtype):
    """Batched one-sided Jacobi on the GPU: reconstruction, orthogonality and singular values against
    torch.linalg.svdvals in float64, for odd sizes (a bye in every round) and many matrices per launch."""
    from brain_b200 import _native
    g = torch.Generator(device="cpu").manual_seed(n * 7 + nb)
    a = torch.randn(nb, n, n, generator=g, dtype=torch.float64)
    r = LA.svd_symmetric(a.to("cuda", dtype))
    torch.cuda.synchronize()
    u, s, v = r.u.double().cpu(), r.singular_values.double().cpu(), r.v.double().cpu()
    tol = 1e-9 if dtype == torch.float64 else 2e-4
    scale = float(torch.linalg.svdvals(a).max())
    assert float(((u * s.unsqueeze(-2)) @ v.transpose(-1, -2) - a).abs().max()) < tol * scale * n
    eye = torch.eye(n, dtype=torch.float64)
    assert float((v.transpose(-1, -2) @ v - eye).abs().max()) < tol * n
    assert float((u.transpose(-1, -2) @ u - eye).abs().max()) < tol * n * 10
    torch.testing.assert_close(s.sort(dim=-1, descending=True).values, torch.linalg.svdvals(a), rtol=tol * 10,
                               atol=tol * scale)
    assert int(r.sweeps.max()) < 50  # converged, not cut off
    assert _native.status("linalg")[0] == 0


@pytest.mark.gpu
@pytest.mark.parametrize("ncols", [128, 33, 4096])
def test_csr_spmm_kernel_matches_dense(ncols):
    g = torch.Generator(device="cpu").manual_seed(ncols)
    rows, k = 300, 257
    mask = torch.rand(rows, k, generator=g) < 0.05
    dense_a = torch.randn(rows, k, generator=g) * mask
    coo = LA.SparseCOO((rows, k))
    for r, c in mask.nonzero().tolist():
        coo.insert(r, c, float(dense_a[r, c]))
    b = torch.randn(k, ncols, generator=g)
    out = coo.spmm(b.cuda())
    torch.testing.assert_close(out.cpu(), dense_a @ b, rtol=1e-5, atol=1e-4)
    wide = torch.randn(k, ncols + 8, generator=g).cuda()  # strided dense operand
    torch.testing.assert_close(coo.spmm(wide[:, :ncols]).cpu(), dense_a @ wide[:, :ncols].cpu(), rtol=1e-5, atol=1e-4)
