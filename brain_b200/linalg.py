"""Linear algebra, FFT and sparse routines under the reference's names, on torch (cuSOLVER / cuFFT /
cuSPARSE on a GPU). No custom kernels: these are not on a hot path of the benchmarked workloads.

Reference: crates/brain-core/src/tensor/linalg.rs (LU with partial pivoting, QR, Cholesky, symmetric
eigen-decomposition, SVD via the symmetric route, solve, det, inverse), tensor/fft.rs (radix-2 FFT
and its inverse on complex pairs), tensor/sparse.rs (CSR matrix and ``spmm``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def lu(a: torch.Tensor):
    """(P, L, U) with a = P @ L @ U."""
    return torch.linalg.lu(a)


def qr(a: torch.Tensor):
    return torch.linalg.qr(a)


def cholesky(a: torch.Tensor) -> torch.Tensor:
    return torch.linalg.cholesky(a)


def eigh(a: torch.Tensor):
    """Eigenvalues ascending and eigenvectors of a symmetric matrix."""
    return torch.linalg.eigh(a)


def svd(a: torch.Tensor, full_matrices: bool = False):
    return torch.linalg.svd(a, full_matrices=full_matrices)


def solve(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.linalg.solve(a, b)


def det(a: torch.Tensor) -> torch.Tensor:
    return torch.linalg.det(a)


def inverse(a: torch.Tensor) -> torch.Tensor:
    return torch.linalg.inv(a)


def fft(x: torch.Tensor, n: int | None = None) -> torch.Tensor:
    return torch.fft.fft(x, n)


def ifft(x: torch.Tensor, n: int | None = None) -> torch.Tensor:
    return torch.fft.ifft(x, n)


def rfft(x: torch.Tensor, n: int | None = None) -> torch.Tensor:
    return torch.fft.rfft(x, n)


def irfft(x: torch.Tensor, n: int | None = None) -> torch.Tensor:
    return torch.fft.irfft(x, n)


@dataclass
class CsrMatrix:
    """Compressed sparse rows: ``indptr`` [rows + 1], ``indices`` [nnz], ``values`` [nnz]."""
    indptr: torch.Tensor
    indices: torch.Tensor
    values: torch.Tensor
    shape: tuple

    @classmethod
    def from_dense(cls, d: torch.Tensor) -> "CsrMatrix":
        s = d.to_sparse_csr()
        return cls(s.crow_indices(), s.col_indices(), s.values(), tuple(d.shape))

    def to_torch(self) -> torch.Tensor:
        return torch.sparse_csr_tensor(self.indptr, self.indices, self.values, self.shape)

    def to_dense(self) -> torch.Tensor:
        return self.to_torch().to_dense()

    def nnz(self) -> int:
        return int(self.values.numel())


def spmm(a: CsrMatrix, b: torch.Tensor) -> torch.Tensor:
    """Sparse (CSR) x dense."""
    return torch.sparse.mm(a.to_torch(), b)
