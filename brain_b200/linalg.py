"""Linear algebra, FFT and sparse routines with the reference's semantics.

Reference: crates/brain-core/src/tensor/linalg.rs (norms, trace, det/logdet/slogdet, LU with partial
pivoting, lu_solve, Householder QR, qr_solve, Cholesky, cholesky_solve, one-sided Jacobi SVD
``svd_symmetric``, svd_solve, eigh, inv, pinv, condition_number, matrix_power), tensor/fft.rs
(in-place radix-2 FFT on (real, imag) arrays, ``dft`` for other lengths, ``rfft`` returning the half
spectrum as (real, imag), Hann and Hamming windows) and tensor/sparse.rs (COO matrix with ``insert``,
``to_dense`` and ``spmm``).

The factorisations follow the reference's algorithm steps and thresholds, so outputs agree with it
element for element up to rounding: the LU pivot is the first row of largest magnitude and a pivot
of magnitude <= 1e-15 leaves its column un-eliminated; triangular solves put 0 where a diagonal is
<= 1e-15; QR reflects onto ``-sign(r_kk) * |x|``; SVD singular values stay in column order, and
``eigh`` returns the SVD's singular values with V (so for an indefinite symmetric matrix it gives
the eigenvalues' magnitudes, as the reference does). Each step is a vector operation over a whole
row or column block in torch (float64 on the CPU, or on the GPU for GPU tensors).

B200 kernels (``csrc/linalg.cu``): the SVD of CUDA tensors runs as a batched one-sided Jacobi kernel,
one CTA per matrix with the columns in shared memory and every disjoint column pair of a
round-robin round rotated by its own warp (square matrices up to 96 x 96; any leading batch
dimensions); ``SparseCOO.spmm`` of a CUDA dense operand runs a CSR kernel (warp per sparse row,
float4 lanes over the dense columns). ``norm_nuclear``, ``pinv``, ``condition_number`` and ``eigh``
use that SVD. Complex FFTs of large signals are left to ``torch.fft`` (cuFFT) under
``fft_complex``/``ifft_complex``.
"""
from __future__ import annotations

import math

import torch

from . import _native

_native.register({
    "brain_jacobi_svd": ("brain_kernels", "pppppliiids"),
    "brain_csr_spmm": ("brain_kernels", "pppplpllls"),
    "brain_status_linalg": ("brain_kernels", "pi"),
})

_PIVOT_EPS = 1e-15
SVD_MAX_N = 96


def _as2d(a: torch.Tensor, name: str) -> torch.Tensor:
    if a.dim() != 2:
        raise ValueError(f"{name} requires a 2D matrix, got shape {tuple(a.shape)}")
    return a if a.is_floating_point() else a.double()


def _square(a: torch.Tensor, name: str) -> torch.Tensor:
    a = _as2d(a, name)
    if a.shape[0] != a.shape[1]:
        raise ValueError(f"{name} requires a square matrix, got shape {tuple(a.shape)}")
    return a


# ---------------------------------------------------------------------------------------- norms
def norm_l1(a: torch.Tensor) -> float:
    """Sum of absolute values over all elements."""
    return float(a.abs().sum())


def norm_l2(a: torch.Tensor) -> float:
    """Euclidean norm over all elements (the Frobenius norm of a matrix)."""
    return float(a.double().square().sum().sqrt())


def norm_linf(a: torch.Tensor) -> float:
    """Largest absolute value (-inf for an empty tensor, as the reference's fold starts there)."""
    return float(a.abs().max()) if a.numel() else -math.inf


def norm_frobenius(a: torch.Tensor) -> float:
    return norm_l2(a)


def norm_p(a: torch.Tensor, p: float) -> float:
    if p < 1.0:
        raise ValueError("p-norm requires p >= 1")
    return float(a.double().abs().pow(p).sum().pow(1.0 / p))


def norm_nuclear(a: torch.Tensor) -> float:
    """Sum of the singular values (Jacobi SVD)."""
    return float(svd_symmetric(a).singular_values.sum())


def trace(a: torch.Tensor) -> float:
    """Sum of the diagonal over min(rows, cols)."""
    a = _as2d(a, "trace")
    return float(torch.diagonal(a).sum())


# ---------------------------------------------------------------------------------------- LU
def lu(a: torch.Tensor):
    """LU with partial pivoting: returns (L [m, min(m,n)], U [min(m,n), n], perm) with
    a[perm] = L @ U. The pivot of column k is the first row (from k) of largest magnitude."""
    a = _as2d(a, "lu")
    m, n = a.shape
    kmax = min(m, n)
    u = a.clone()
    l = torch.zeros(m, kmax, dtype=a.dtype, device=a.device)
    perm = list(range(m))
    for k in range(kmax):
        col = u[k:, k].abs()
        piv = k + int(torch.argmax(col))  # the first maximal index: row k stays unless another is larger
        if piv != k:
            u[[k, piv]] = u[[piv, k]]
            perm[k], perm[piv] = perm[piv], perm[k]
            if k:
                l[[k, piv], :k] = l[[piv, k], :k]
        pivot = u[k, k]
        if abs(float(pivot)) > _PIVOT_EPS and k + 1 < m:
            f = u[k + 1:, k] / pivot
            l[k + 1:, k] = f
            u[k + 1:, k + 1:] -= f[:, None] * u[k, k + 1:][None, :]
            u[k + 1:, k] = 0.0
    l[torch.arange(kmax), torch.arange(kmax)] = 1.0
    return l, u[:kmax], perm


def _forward_sub(l: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Lower-triangular solve, one row at a time (b: a vector or columns of right-hand sides)."""
    n = l.shape[0]
    y = torch.zeros_like(b)
    for i in range(n):
        s = b[i] - (l[i, :i] @ y[:i] if i else 0.0)
        y[i] = s / l[i, i]
    return y


def _back_sub(u: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Upper-triangular solve; a diagonal of magnitude <= 1e-15 gives 0 (the reference's rule)."""
    n = u.shape[1]
    x = torch.zeros(n, *y.shape[1:], dtype=y.dtype, device=y.device)
    for i in range(n - 1, -1, -1):
        s = y[i] - (u[i, i + 1:n] @ x[i + 1:] if i + 1 < n else 0.0)
        d = u[i, i]
        x[i] = s / d if abs(float(d)) > _PIVOT_EPS else 0.0
    return x


def lu_solve(l: torch.Tensor, u: torch.Tensor, perm, b: torch.Tensor) -> torch.Tensor:
    """Solve a x = b from lu(a); b is a vector or a matrix of right-hand sides."""
    idx = torch.as_tensor(list(perm), device=b.device)
    y = _forward_sub(l, b.to(l.dtype)[idx])
    return _back_sub(u, y)


def det(a: torch.Tensor) -> float:
    """Determinant: closed forms for n <= 2, else the product of U's diagonal times the sign of the
    pivot permutation (counted by cycles)."""
    a = _square(a, "det")
    n = a.shape[0]
    if n == 0:
        return 1.0
    if n == 1:
        return float(a[0, 0])
    if n == 2:
        return float(a[0, 0] * a[1, 1] - a[0, 1] * a[1, 0])
    _, u, perm = lu(a)
    d = float(torch.diagonal(u).double().prod())
    seen, swaps = [False] * n, 0
    for i in range(n):
        cur, cyc = i, 0
        while not seen[cur]:
            seen[cur] = True
            cur = perm[cur]
            cyc += 1
        swaps += max(cyc - 1, 0)
    return -d if swaps % 2 else d


def logdet(a: torch.Tensor) -> float:
    """ln |det a| (-inf for a singular matrix)."""
    d = abs(det(a))
    return math.log(d) if d > 0 else -math.inf


def slogdet(a: torch.Tensor):
    d = det(a)
    if d == 0.0:
        return 0.0, -math.inf
    return (1.0, math.log(d)) if d > 0 else (-1.0, math.log(-d))


def inv(a: torch.Tensor) -> torch.Tensor:
    """Inverse from one LU factorisation, all unit columns solved at once."""
    a = _square(a, "inv")
    l, u, perm = lu(a)
    eye = torch.eye(a.shape[0], dtype=a.dtype, device=a.device)
    return lu_solve(l, u, perm, eye)


# ---------------------------------------------------------------------------------------- QR
def qr(a: torch.Tensor):
    """Householder QR: (Q [m, m], R [m, n]) with a = Q @ R. Column k is reflected onto
    alpha = -|x| when r_kk >= 0, else +|x|; columns of norm < 1e-15 are skipped."""
    a = _as2d(a, "qr")
    m, n = a.shape
    q = torch.eye(m, dtype=a.dtype, device=a.device)
    r = a.clone()
    for k in range(min(m, n)):
        x = r[k:, k]
        nx = float(x.double().square().sum().sqrt())
        if nx < _PIVOT_EPS:
            continue
        alpha = -nx if float(r[k, k]) >= 0.0 else nx
        v = x.clone()
        v[0] = v[0] - alpha
        nv = float(v.double().square().sum().sqrt())
        if nv < _PIVOT_EPS:
            continue
        v = v / nv
        r[k:, k:] -= 2.0 * v[:, None] * (v @ r[k:, k:])[None, :]
        q[:, k:] -= 2.0 * (q[:, k:] @ v)[:, None] * v[None, :]
    return q, r


def qr_solve(q: torch.Tensor, r: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Least-squares / exact solve from qr(a): back substitution on R x = Q^T b."""
    return _back_sub(r, q.t() @ b.to(q.dtype))


# ---------------------------------------------------------------------------------------- Cholesky
def cholesky(a: torch.Tensor) -> torch.Tensor:
    """Lower-triangular L with a = L L^T, row by row; raises ValueError when a pivot is not positive."""
    a = _square(a, "cholesky")
    n = a.shape[0]
    l = torch.zeros_like(a)
    for i in range(n):
        for j in range(i + 1):
            s = a[i, j] - (l[i, :j] @ l[j, :j] if j else 0.0)
            if i == j:
                if not float(s) > 0.0:
                    raise ValueError("cholesky: matrix is not positive-definite")
                l[i, i] = torch.sqrt(torch.as_tensor(s, dtype=a.dtype))
            else:
                l[i, j] = s / l[j, j]
    return l


def cholesky_solve(l: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Solve (L L^T) x = b: forward substitution with L, back substitution with L^T."""
    y = _forward_sub(l, b.to(l.dtype))
    n = l.shape[0]
    x = torch.zeros_like(y)
    for i in range(n - 1, -1, -1):
        s = y[i] - (l[i + 1:, i] @ x[i + 1:] if i + 1 < n else 0.0)
        x[i] = s / l[i, i]
    return x


# ---------------------------------------------------------------------------------------- SVD
class SvdResult:
    """u [.., n, n], singular_values [.., n] (column order, not sorted), v [.., n, n]: a = u diag(s) v^T."""

    def __init__(self, u, singular_values, v, sweeps=None):
        self.u, self.singular_values, self.v, self.sweeps = u, singular_values, v, sweeps

    def __iter__(self):
        return iter((self.u, self.singular_values, self.v))


def _jacobi_cpu(a: torch.Tensor, max_sweeps: int, tol: float):
    """One-sided Jacobi on one matrix, cyclic-by-row pair order (the reference's order), float64.
    The reference runs a fixed 50 sweeps; once a sweep rotates nothing, further sweeps change nothing,
    so stopping there gives the same result."""
    w = a.double().clone()
    n = w.shape[0]
    v = torch.eye(n, dtype=torch.float64, device=a.device)
    sweeps = 0
    for sweeps in range(1, max_sweeps + 1):
        rotated = False
        for i in range(n):
            for j in range(i + 1, n):
                ci, cj = w[:, i], w[:, j]
                dii, djj, dij = float(ci @ ci), float(cj @ cj), float(ci @ cj)
                if abs(dij) < tol:
                    continue
                rotated = True
                tau = (djj - dii) / (2.0 * dij)
                t = 1.0 / (tau + math.sqrt(1.0 + tau * tau)) if tau >= 0 else -1.0 / (-tau + math.sqrt(1.0 + tau * tau))
                c = 1.0 / math.sqrt(1.0 + t * t)
                s = t * c
                wi, wj = ci.clone(), cj.clone()
                w[:, i], w[:, j] = c * wi - s * wj, s * wi + c * wj
                vi, vj = v[:, i].clone(), v[:, j].clone()
                v[:, i], v[:, j] = c * vi - s * vj, s * vi + c * vj
        if not rotated:
            break
    sv = w.square().sum(0).sqrt()
    u = torch.where(sv > 1e-15, w / torch.where(sv > 1e-15, sv, torch.ones_like(sv)), torch.zeros_like(w))
    return u.to(a.dtype), sv.to(a.dtype), v.to(a.dtype), sweeps


def svd_symmetric(a: torch.Tensor, max_sweeps: int = 50, tol: float | None = None) -> SvdResult:
    """One-sided Jacobi SVD of a square matrix (or a batch [..., n, n]).

    CPU tensors: the reference's cyclic order and its absolute stop rule |a_i . a_j| < 1e-15.
    CUDA tensors: the batched kernel (round-robin order, relative stop rule
    |a_i . a_j| <= tol * |a_i| |a_j|, default 1e-15 for float64 and 1e-7 for float32), n <= 96; one
    CTA per matrix. Both converge to the same factorisation up to the order and signs of the
    singular triplets."""
    if a.dim() < 2 or a.shape[-1] != a.shape[-2]:
        raise ValueError(f"svd_symmetric requires square matrices, got shape {tuple(a.shape)}")
    if not a.is_floating_point():
        a = a.double()
    n = a.shape[-1]
    if a.is_cuda:
        if n > SVD_MAX_N:
            raise ValueError(f"the batched Jacobi kernel takes n <= {SVD_MAX_N}, got {n}")
        _native.require_cuda_lib(a)
        dt = a.dtype if a.dtype in (torch.float32, torch.float64) else torch.float32
        x = a.to(dt).contiguous()
        batch = x.shape[:-2]
        nb = int(torch.tensor(batch).prod()) if batch else 1
        u, v = torch.empty_like(x), torch.empty_like(x)
        s = torch.empty(*batch, n, dtype=dt, device=a.device)
        sweeps = torch.zeros(max(nb, 1), dtype=torch.int32, device=a.device)
        if tol is None:
            tol = 1e-15 if dt == torch.float64 else 1e-7
        _native.call("brain_jacobi_svd", x.data_ptr(), u.data_ptr(), s.data_ptr(), v.data_ptr(), sweeps.data_ptr(),
                     nb, n, 1 if dt == torch.float64 else 0, int(max_sweeps), float(tol),
                     torch.cuda.current_stream().cuda_stream)
        return SvdResult(u, s, v, sweeps[:nb].view(batch) if batch else sweeps[0])
    tol = 1e-15 if tol is None else tol
    if a.dim() == 2:
        return SvdResult(*_jacobi_cpu(a, max_sweeps, tol))
    flat = a.reshape(-1, n, n)
    outs = [_jacobi_cpu(m, max_sweeps, tol) for m in flat]
    u = torch.stack([o[0] for o in outs]).view_as(a)
    s = torch.stack([o[1] for o in outs]).view(*a.shape[:-1])
    v = torch.stack([o[2] for o in outs]).view_as(a)
    return SvdResult(u, s, v, torch.tensor([o[3] for o in outs]).view(a.shape[:-2]))


def svd_solve(u: torch.Tensor, s: torch.Tensor, v: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """x = V diag(1/s) U^T b, dropping singular values <= 1e-12."""
    s = torch.as_tensor(s, dtype=u.dtype, device=u.device)
    inv_s = torch.where(s > 1e-12, 1.0 / torch.where(s > 1e-12, s, torch.ones_like(s)), torch.zeros_like(s))
    utb = u.t() @ b.to(u.dtype)
    return v @ (inv_s.view(-1, *([1] * (utb.dim() - 1))) * utb)


def eigh(a: torch.Tensor):
    """(values, vectors) from the Jacobi SVD: the singular values (column order) and V. For a
    positive semi-definite matrix these are its eigenpairs; for an indefinite one the values are
    the eigenvalues' magnitudes (the reference's definition, kept)."""
    r = svd_symmetric(a)
    return r.singular_values, r.v


def pinv(a: torch.Tensor) -> torch.Tensor:
    """Moore-Penrose pseudo-inverse V diag(1/s) U^T of a square matrix (s <= 1e-12 dropped)."""
    r = svd_symmetric(a)
    s = r.singular_values
    inv_s = torch.where(s > 1e-12, 1.0 / torch.where(s > 1e-12, s, torch.ones_like(s)), torch.zeros_like(s))
    return (r.v * inv_s.unsqueeze(-2)) @ r.u.transpose(-1, -2)


def condition_number(a: torch.Tensor) -> float:
    """Largest over smallest singular value; inf when the smallest is below 1e-15."""
    s = svd_symmetric(a).singular_values
    lo, hi = float(s.min()), float(s.max().clamp_min(0.0))
    return math.inf if lo < 1e-15 else hi / lo


def matrix_power(a: torch.Tensor, n: int) -> torch.Tensor:
    """a^n by binary exponentiation; n < 0 raises the inverse; n = 0 gives the identity."""
    a = _square(a, "matrix_power")
    if n == 0:
        return torch.eye(a.shape[0], dtype=a.dtype, device=a.device)
    if n < 0:
        return matrix_power(inv(a), -n)
    result = torch.eye(a.shape[0], dtype=a.dtype, device=a.device)
    base, e = a, n
    while e:
        if e & 1:
            result = result @ base
        base = base @ base
        e >>= 1
    return result


def solve(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Solve a x = b through lu / lu_solve."""
    return lu_solve(*lu(_square(a, "solve")), b)


# ---------------------------------------------------------------------------------------- FFT
def fft_radix2(real: torch.Tensor, imag: torch.Tensor, inverse: bool = False) -> None:
    """In-place iterative radix-2 FFT over the last dimension of (real, imag) (any leading batch
    dimensions): bit-reversal permutation, then log2(n) butterfly stages, each one vector operation
    over all butterflies of the stage; the inverse divides by n. The length must be a power of two."""
    n = real.shape[-1]
    if imag.shape != real.shape:
        raise ValueError("real and imag must have the same shape")
    if n == 0 or n & (n - 1):
        raise ValueError("FFT size must be a power of two")
    bits = n.bit_length() - 1
    idx = torch.arange(n, device=real.device)
    rev = torch.zeros_like(idx)
    for b in range(bits):
        rev |= ((idx >> b) & 1) << (bits - 1 - b)
    re, im = real[..., rev].double(), imag[..., rev].double()
    sign = 1.0 if inverse else -1.0
    length = 2
    while length <= n:
        half = length // 2
        ang = sign * 2.0 * math.pi * torch.arange(half, device=real.device, dtype=torch.float64) / length
        wr, wi = torch.cos(ang), torch.sin(ang)
        shp = re.shape[:-1] + (n // length, length)
        r2, i2 = re.reshape(shp), im.reshape(shp)
        ur, ui = r2[..., :half], i2[..., :half]
        xr, xi = r2[..., half:], i2[..., half:]
        vr = xr * wr - xi * wi
        vi = xr * wi + xi * wr
        re = torch.cat([ur + vr, ur - vr], dim=-1).reshape(re.shape)
        im = torch.cat([ui + vi, ui - vi], dim=-1).reshape(im.shape)
        length *= 2
    if inverse:
        re, im = re / n, im / n
    real.copy_(re)
    imag.copy_(im)


def dft(real: torch.Tensor, imag: torch.Tensor, inverse: bool = False) -> None:
    """In-place discrete Fourier transform of any length: radix-2 for powers of two, else the direct
    O(n^2) sum as one complex matrix product (the inverse divides by n)."""
    n = real.shape[-1]
    if n == 0:
        return
    if n & (n - 1) == 0:
        fft_radix2(real, imag, inverse)
        return
    sign = 1.0 if inverse else -1.0
    k = torch.arange(n, device=real.device, dtype=torch.float64)
    ang = sign * 2.0 * math.pi * torch.outer(k, k).remainder(n) / n
    c, s = torch.cos(ang), torch.sin(ang)
    xr, xi = real.double(), imag.double()
    out_r = xr @ c.t() - xi @ s.t()
    out_i = xr @ s.t() + xi @ c.t()
    if inverse:
        out_r, out_i = out_r / n, out_i / n
    real.copy_(out_r)
    imag.copy_(out_i)


def rfft(x: torch.Tensor):
    """Half spectrum of a real signal (power-of-two length): (real [n/2 + 1], imag [n/2 + 1])."""
    re = x.double().clone()
    im = torch.zeros_like(re)
    fft_radix2(re, im, False)
    h = x.shape[-1] // 2 + 1
    return re[..., :h].to(x.dtype if x.is_floating_point() else torch.float64), \
        im[..., :h].to(x.dtype if x.is_floating_point() else torch.float64)


def hann_window(n: int, dtype=torch.float64, device=None) -> torch.Tensor:
    """0.5 (1 - cos(2 pi i / (n - 1))): the symmetric window."""
    i = torch.arange(n, dtype=torch.float64, device=device)
    return (0.5 * (1.0 - torch.cos(2.0 * math.pi * i / (n - 1.0)))).to(dtype)


def hamming_window(n: int, dtype=torch.float64, device=None) -> torch.Tensor:
    """0.54 - 0.46 cos(2 pi i / (n - 1)): the symmetric window."""
    i = torch.arange(n, dtype=torch.float64, device=device)
    return (0.54 - 0.46 * torch.cos(2.0 * math.pi * i / (n - 1.0))).to(dtype)


def fft_complex(x: torch.Tensor, n: int | None = None) -> torch.Tensor:
    """Complex FFT of large or batched signals through cuFFT / pocketfft (torch.fft)."""
    return torch.fft.fft(x, n)


def ifft_complex(x: torch.Tensor, n: int | None = None) -> torch.Tensor:
    return torch.fft.ifft(x, n)


# ---------------------------------------------------------------------------------------- sparse
class SparseCOO:
    """Coordinate-format sparse matrix: entries are appended with ``insert`` (duplicates add up).

    ``spmm`` with a CUDA dense operand sorts the entries into CSR rows once (cached until the next
    insert) and runs the native CSR kernel; on the CPU it scatters val * B[col] into the rows."""

    def __init__(self, shape):
        self.shape = (int(shape[0]), int(shape[1]))
        self.row_indices: list[int] = []
        self.col_indices: list[int] = []
        self.values: list[float] = []
        self._csr = None

    def insert(self, row: int, col: int, val: float) -> None:
        if not (0 <= row < self.shape[0] and 0 <= col < self.shape[1]):
            raise IndexError(f"({row}, {col}) outside {self.shape}")
        self.row_indices.append(int(row))
        self.col_indices.append(int(col))
        self.values.append(float(val))
        self._csr = None

    @property
    def nnz(self) -> int:
        return len(self.values)

    def _coo(self, device, dtype):
        r = torch.tensor(self.row_indices, dtype=torch.long, device=device)
        c = torch.tensor(self.col_indices, dtype=torch.long, device=device)
        v = torch.tensor(self.values, dtype=dtype, device=device)
        return r, c, v

    def to_dense(self, dtype=torch.float64, device=None) -> torch.Tensor:
        out = torch.zeros(self.shape, dtype=dtype, device=device)
        if self.nnz:
            r, c, v = self._coo(device, dtype)
            out.index_put_((r, c), v, accumulate=True)
        return out

    def to_csr(self, device=None):
        """(indptr [rows + 1], indices [nnz], values [nnz] float32), rows sorted, entry order kept within a row."""
        dev = torch.device(device) if device is not None else torch.device("cpu")
        if self._csr is not None and self._csr[0].device == dev:
            return self._csr
        r, c, v = self._coo(dev, torch.float32)
        order = torch.argsort(r, stable=True)
        counts = torch.bincount(r, minlength=self.shape[0]) if self.nnz else torch.zeros(self.shape[0], dtype=torch.long,
                                                                                         device=dev)
        indptr = torch.zeros(self.shape[0] + 1, dtype=torch.long, device=dev)
        indptr[1:] = torch.cumsum(counts, 0)
        self._csr = (indptr, c[order].contiguous(), v[order].contiguous())
        return self._csr

    def spmm(self, b: torch.Tensor) -> torch.Tensor:
        """Sparse [rows, K] @ dense b [K, N]."""
        if b.dim() != 2 or b.shape[0] != self.shape[1]:
            raise ValueError(f"spmm: dense operand {tuple(b.shape)} does not match {self.shape}")
        if b.is_cuda:
            _native.require_cuda_lib(b)
            indptr, idx, vals = self.to_csr(b.device)
            dense = b.float()
            if dense.stride(1) != 1:
                dense = dense.contiguous()
            out = torch.empty(self.shape[0], b.shape[1], dtype=torch.float32, device=b.device)
            _native.call("brain_csr_spmm", indptr.data_ptr(), idx.data_ptr(), vals.data_ptr(), dense.data_ptr(),
                         dense.stride(0), out.data_ptr(), out.stride(0), self.shape[0], b.shape[1],
                         torch.cuda.current_stream().cuda_stream)
            return out
        dt = b.dtype if b.is_floating_point() else torch.float64
        out = torch.zeros(self.shape[0], b.shape[1], dtype=dt)
        if self.nnz:
            r, c, v = self._coo(None, dt)
            out.index_add_(0, r, v[:, None] * b.to(dt)[c])
        return out


CsrMatrix = SparseCOO  # the CSR form is SparseCOO.to_csr(); the old name stays importable
