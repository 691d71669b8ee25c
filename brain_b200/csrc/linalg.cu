// Dense and sparse linear-algebra kernels, sm_100a.
//
// 1. Batched one-sided Jacobi SVD (Hestenes' method) of many small square matrices, one CTA per matrix.
//    The reference factorises one matrix at a time on the CPU with cyclic-by-row column sweeps
//    (crates/brain-core/src/tensor/linalg.rs:410-475, svd_symmetric). Here a matrix's columns and the
//    accumulated right rotations live in shared memory as float64 (column-major, so a column is
//    contiguous), and each sweep is the round-robin ("circle") ordering: n-1 rounds of n/2 disjoint
//    column pairs, so every pair of a round is rotated at the same time by its own warp (the pairs
//    touch disjoint columns). A warp reduces the three dot products of its pair with shuffles, then
//    rotates both columns of A and of V. The rotation itself is the one the reference applies
//    (tau = (a_jj - a_ii) / (2 a_ij), t = sign(tau) / (|tau| + sqrt(1 + tau^2)), c = 1/sqrt(1 + t^2),
//    s = t c). Sweeps stop when a whole sweep rotates nothing (|a_ij| <= tol * sqrt(a_ii a_jj)) or
//    after max_sweeps. Outputs: S_j = |A V e_j|, U e_j = A V e_j / S_j (zero column when S_j <= 1e-15),
//    V; singular values stay in column order (unsorted), as the reference leaves them.
// 2. CSR sparse x dense product (crates/brain-core/src/tensor/sparse.rs:52-70 spmm over COO entries):
//    one warp per sparse row, lanes over the dense columns in float4 vectors, float32 accumulation.
#include "common.cuh"

using namespace brain;

namespace {

constexpr int kSvdThreads = 256;
constexpr int kSvdMaxN = 96;  // 2 * 96 * 96 doubles = 144 KB of shared memory

template <typename T>
__global__ void __launch_bounds__(kSvdThreads) jacobi_svd_kernel(const T* __restrict__ a, T* __restrict__ u,
                                                                 T* __restrict__ s, T* __restrict__ v, int* sweeps_out,
                                                                 int n, int max_sweeps, double tol) {
  extern __shared__ double smem[];
  double* A = smem;          // column-major n x n: A[j * n + i] = a[i][j]
  double* V = smem + n * n;  // column-major accumulated rotations
  __shared__ int rotated;
  const int b = blockIdx.x;
  const T* ab = a + (int64_t)b * n * n;
  for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
    const int i = e / n, j = e % n;
    A[j * n + i] = (double)ab[e];
    V[j * n + i] = i == j ? 1.0 : 0.0;
  }
  const int m = n + (n & 1);  // even number of players; index n is a bye when n is odd
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  int sweep = 0;
  for (; sweep < max_sweeps; ++sweep) {
    if (threadIdx.x == 0) rotated = 0;
    __syncthreads();
    for (int r = 0; r < m - 1; ++r) {
      for (int pr = warp; pr < m / 2; pr += nwarps) {
        // circle method: player m-1 is fixed, the others rotate by one position per round
        int p, q;
        if (pr == 0) {
          p = r;
          q = m - 1;
        } else {
          p = (r + pr) % (m - 1);
          q = (r - pr + (m - 1)) % (m - 1);
        }
        int i = p < q ? p : q, j = p < q ? q : p;
        if (j >= n) continue;  // bye
        double* ci = A + i * n;
        double* cj = A + j * n;
        double aii = 0.0, ajj = 0.0, aij = 0.0;
        for (int k = lane; k < n; k += 32) {
          const double x = ci[k], y = cj[k];
          aii = fma(x, x, aii);
          ajj = fma(y, y, ajj);
          aij = fma(x, y, aij);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          aii += __shfl_xor_sync(0xffffffffu, aii, o);
          ajj += __shfl_xor_sync(0xffffffffu, ajj, o);
          aij += __shfl_xor_sync(0xffffffffu, aij, o);
        }
        aii = __shfl_sync(0xffffffffu, aii, 0);  // one value per warp, so the branch below stays uniform
        ajj = __shfl_sync(0xffffffffu, ajj, 0);
        aij = __shfl_sync(0xffffffffu, aij, 0);
        if (fabs(aij) <= tol * sqrt(aii * ajj) || aij == 0.0) continue;  // warp-uniform
        const double tau = (ajj - aii) / (2.0 * aij);
        const double t = tau >= 0.0 ? 1.0 / (tau + sqrt(1.0 + tau * tau)) : -1.0 / (-tau + sqrt(1.0 + tau * tau));
        const double c = 1.0 / sqrt(1.0 + t * t), sn = t * c;
        double* vi = V + i * n;
        double* vj = V + j * n;
        for (int k = lane; k < n; k += 32) {
          const double x = ci[k], y = cj[k];
          ci[k] = c * x - sn * y;
          cj[k] = sn * x + c * y;
          const double vx = vi[k], vy = vj[k];
          vi[k] = c * vx - sn * vy;
          vj[k] = sn * vx + c * vy;
        }
        if (lane == 0) rotated = 1;
      }
      __syncthreads();
    }
    const int any = rotated;
    __syncthreads();  // every thread has read the flag before thread 0 clears it
    if (!any) break;
  }
  // column norms -> singular values; U columns normalised
  __shared__ double norms[kSvdMaxN];
  for (int j = warp; j < n; j += nwarps) {
    double acc = 0.0;
    for (int k = lane; k < n; k += 32) acc = fma(A[j * n + k], A[j * n + k], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) norms[j] = sqrt(acc);
  }
  __syncthreads();
  T* ub = u + (int64_t)b * n * n;
  T* vb = v + (int64_t)b * n * n;
  for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
    const int i = e / n, j = e % n;
    const double sj = norms[j];
    ub[e] = (T)(sj > 1e-15 ? A[j * n + i] / sj : 0.0);
    vb[e] = (T)V[j * n + i];
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x) s[(int64_t)b * n + j] = (T)norms[j];
  if (threadIdx.x == 0 && sweeps_out) sweeps_out[b] = sweep;
}

// out[r, :] = sum over the nonzeros (k, val) of row r of val * dense[k, :]   (float32)
__global__ void csr_spmm_kernel(const int64_t* __restrict__ indptr, const int64_t* __restrict__ indices,
                                const float* __restrict__ vals, const float* __restrict__ dense, int64_t ldd,
                                float* __restrict__ out, int64_t ldo, int64_t rows, int64_t ncols, int vec4) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t e0 = indptr[r], e1 = indptr[r + 1];
  if (vec4) {
    for (int64_t c0 = (int64_t)lane * 4; c0 < ncols; c0 += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t e = e0; e < e1; ++e) {
        const float w = vals[e];
        const float4 x = *reinterpret_cast<const float4*>(dense + indices[e] * ldd + c0);
        acc.x = fmaf(w, x.x, acc.x);
        acc.y = fmaf(w, x.y, acc.y);
        acc.z = fmaf(w, x.z, acc.z);
        acc.w = fmaf(w, x.w, acc.w);
      }
      *reinterpret_cast<float4*>(out + r * ldo + c0) = acc;
    }
  } else {
    for (int64_t c = lane; c < ncols; c += 32) {
      float acc = 0.f;
      for (int64_t e = e0; e < e1; ++e) acc = fmaf(vals[e], dense[indices[e] * ldd + c], acc);
      out[r * ldo + c] = acc;
    }
  }
}

}  // namespace

// Batched SVD of nb square n x n matrices (row-major, contiguous). dtype 0 = float32, 1 = float64 (the
// arithmetic is float64 either way). u, v: nb x n x n; s: nb x n; sweeps (optional, int32[nb]) receives
// the number of sweeps each matrix took. tol: relative orthogonality threshold of a column pair.
BRAIN_API int brain_jacobi_svd(const void* a, void* u, void* s, void* v, int* sweeps, int64_t nb, int n, int dtype,
                               int max_sweeps, double tol, cudaStream_t st) {
  if (n < 1 || n > kSvdMaxN || nb < 0 || max_sweeps < 0 || (dtype != 0 && dtype != 1)) return (int)cudaErrorInvalidValue;
  if (nb == 0) return 0;
  const size_t smem = (size_t)2 * n * n * sizeof(double);
  if (dtype == 0) {
    auto k = jacobi_svd_kernel<float>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)nb, kSvdThreads, smem, st>>>(static_cast<const float*>(a), static_cast<float*>(u),
                                               static_cast<float*>(s), static_cast<float*>(v), sweeps, n, max_sweeps, tol);
  } else {
    auto k = jacobi_svd_kernel<double>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)nb, kSvdThreads, smem, st>>>(static_cast<const double*>(a), static_cast<double*>(u),
                                               static_cast<double*>(s), static_cast<double*>(v), sweeps, n, max_sweeps,
                                               tol);
  }
  return (int)cudaGetLastError();
}

// out [rows x ncols] (leading dimension ldo) = CSR [rows x K] @ dense [K x ncols] (leading dimension ldd), float32.
BRAIN_API int brain_csr_spmm(const int64_t* indptr, const int64_t* indices, const float* vals, const float* dense,
                             int64_t ldd, float* out, int64_t ldo, int64_t rows, int64_t ncols, cudaStream_t st) {
  if (rows < 0 || ncols < 0 || ldd < ncols || ldo < ncols) return (int)cudaErrorInvalidValue;
  if (rows == 0 || ncols == 0) return 0;
  const int vec4 = (ncols % 4 == 0) && (ldd % 4 == 0) && (ldo % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(dense) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  const int warps = 8;
  const int64_t grid = (rows + warps - 1) / warps;
  csr_spmm_kernel<<<(unsigned)grid, warps * 32, 0, st>>>(indptr, indices, vals, dense, ldd, out, ldo, rows, ncols, vec4);
  return (int)cudaGetLastError();
}

BRAIN_STATUS_READER(linalg)
