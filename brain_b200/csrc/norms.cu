// Row normalisations (RMSNorm, LayerNorm) forward and backward, bf16 in/out, f32 statistics.
//
// One CTA per row for the forward pass: each thread keeps its slice of the row in registers
// (16-byte vector loads, up to 4 vectors = 32 values per thread), so a row is read from HBM once.
// The optional residual input is added first and the sum is written out (fused add+norm).
// Backward is a persistent grid: each CTA walks rows blockIdx.x, blockIdx.x + gridDim.x, ... and
// accumulates dgamma/dbeta for its fixed columns in registers, then writes one f32 partial row;
// a column-reduction kernel sums the partials (deterministic, no atomics).
//
// Reference semantics (f64 in the reference):
//   RMSNorm  y = x * (mean(x^2) + eps)^-1/2 * w       crates/brain-transformer/src/ops.rs:103-131,
//            fused_add_rmsnorm returns (norm, sum)      crates/brain-core/src/tensor/ops_fused.rs:77-125
//   LayerNorm y = (x - mean) / sqrt(var + eps) * w + b, biased variance
//                                                      crates/brain-transformer/src/ops.rs:57-101
#include <atomic>

#include "common.cuh"
#include "no_alloc.h"

using namespace brain;

namespace {

constexpr int VPT = 4;  // 8-element vectors per thread

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32, nw = (blockDim.x + 31) / 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < nw) ? red[l] : 0.f;
  return warp_sum(t);
}

// ---------------------------------------------------------------- forward
template <bool LAYERNORM>
__global__ void __launch_bounds__(1024) norm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ res, int64_t ldres,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y,
    int64_t ldy, __nv_bfloat16* __restrict__ sum_out, int64_t ldsum, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int D, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = D / 8;
  // the row stays packed (8 bf16 per 16 bytes) in registers and is unpacked where it is used: fewer
  // registers per thread means more resident CTAs, i.e. more rows in flight per SM
  bf16x8 v[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      v[i] = *reinterpret_cast<const bf16x8*>(x + row * ldx + vi * 8);
      if (res) {
        const bf16x8 r = *reinterpret_cast<const bf16x8*>(res + row * ldres + vi * 8);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          // the sum is rounded to bf16 before normalisation, exactly what a separate add would store
          const float2 a = __bfloat1622float2(v[i].h[k]), c = __bfloat1622float2(r.h[k]);
          v[i].h[k] = __floats2bfloat162_rn(a.x + c.x, a.y + c.y);
        }
        *reinterpret_cast<bf16x8*>(sum_out + row * ldsum + vi * 8) = v[i];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = __bfloat1622float2(v[i].h[k]);
        s += LAYERNORM ? a.x + a.y : a.x * a.x + a.y * a.y;
      }
    }
  }
  float mean = 0.f, rstd;
  if (LAYERNORM) {
    mean = block_sum(s, red) / D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = threadIdx.x + i * blockDim.x;
      if (vi < nvec) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 a = __bfloat1622float2(v[i].h[k]);
          q += (a.x - mean) * (a.x - mean) + (a.y - mean) * (a.y - mean);
        }
      }
    }
    rstd = rsqrtf(block_sum(q, red) / D + eps);
  } else {
    rstd = rsqrtf(block_sum(s, red) / D + eps);
  }
  if (threadIdx.x == 0) {
    if (rstd_out) rstd_out[row] = rstd;
    if (LAYERNORM && mean_out) mean_out[row] = mean;
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      float wv[8], o[8], xv[8];
      load8(w + vi * 8, wv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = __bfloat1622float2(v[i].h[k]);
        xv[2 * k] = a.x;
        xv[2 * k + 1] = a.y;
      }
      if (LAYERNORM && b) {
        float bv[8];
        load8(b + vi * 8, bv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (xv[j] - mean) * rstd * wv[j] + bv[j];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (xv[j] - mean) * rstd * wv[j];
      }
      store8(y + row * ldy + vi * 8, o);
    }
  }
}

// ---------------------------------------------------------------- backward
// dx = rstd * (g - [mean(g)] - xhat * mean(g * xhat)),  g = w * dy
// dw += dy * xhat ; db += dy    (per-CTA partials, f32)
template <bool LAYERNORM>
__global__ void norm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy, const __nv_bfloat16* __restrict__ x,
                                int64_t ldx, const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean_in,
                                const float* __restrict__ rstd_in, __nv_bfloat16* __restrict__ dx, int64_t lddx,
                                const __nv_bfloat16* __restrict__ dres, int64_t lddres, float* __restrict__ dw_part,
                                float* __restrict__ db_part, int M, int D) {
  __shared__ float red[32];
  const int nvec = D / 8;
  float dwacc[VPT][8], dbacc[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwacc[i][j] = dbacc[i][j] = 0.f;
  float wv[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) load8(w + vi * 8, wv[i]);
  }
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const float rstd = rstd_in[row];
    const float mean = LAYERNORM ? mean_in[row] : 0.f;
    float xh[VPT][8], g[VPT][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = threadIdx.x + i * blockDim.x;
      if (vi < nvec) {
        float dv[8];
        load8(x + row * ldx + vi * 8, xh[i]);
        load8(dy + row * lddy + vi * 8, dv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] = (xh[i][j] - mean) * rstd;
          g[i][j] = dv[j] * wv[i][j];
          dwacc[i][j] += dv[j] * xh[i][j];
          if (LAYERNORM) dbacc[i][j] += dv[j];
          s1 += g[i][j];
          s2 += g[i][j] * xh[i][j];
        }
      }
    }
    const float c2 = block_sum(s2, red) / D;
    const float c1 = LAYERNORM ? block_sum(s1, red) / D : 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = threadIdx.x + i * blockDim.x;
      if (vi < nvec) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = rstd * (g[i][j] - c1 - xh[i][j] * c2);
        if (dres) {
          float r[8];
          load8(dres + row * lddres + vi * 8, r);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += r[j];
        }
        store8(dx + row * lddx + vi * 8, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      float* p = dw_part + (int64_t)blockIdx.x * D + vi * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) p[j] = dwacc[i][j];
      if (LAYERNORM && db_part) {
        float* q = db_part + (int64_t)blockIdx.x * D + vi * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = dbacc[i][j];
      }
    }
  }
}

// Backward for rows of up to 8192 values: one 8-element vector per thread (T = D / 8 threads, so
// twice as many warps per SM as the 4-vector kernel above), and the next row's x, dy and rstd are
// loaded before the current row's reductions so that their HBM latency overlaps the block sums.
// Same math and partial-row layout as norm_bwd_kernel.
template <bool LAYERNORM>
__global__ void __launch_bounds__(1024, 1)
    norm_bwd_v1_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy, const __nv_bfloat16* __restrict__ x,
                       int64_t ldx, const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean_in,
                       const float* __restrict__ rstd_in, __nv_bfloat16* __restrict__ dx, int64_t lddx,
                       const __nv_bfloat16* __restrict__ dres, int64_t lddres, float* __restrict__ dw_part,
                       float* __restrict__ db_part, int M, int D) {
  __shared__ float red[32];
  const int vi = threadIdx.x;
  const bool on = vi < D / 8;
  float wv[8], dwacc[8], dbacc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) dwacc[j] = dbacc[j] = wv[j] = 0.f;
  if (on) load8(w + vi * 8, wv);
  // the current and the next row's x and dy stay packed (8 bf16 in 16 bytes) until used
  const bf16x8 zero = {};
  bf16x8 xc = zero, dc = zero;
  int64_t row = blockIdx.x;
  float rstd_c = 0.f, mean_c = 0.f;
  if (row < M) {
    rstd_c = rstd_in[row];
    if (LAYERNORM) mean_c = mean_in[row];
    if (on) {
      xc = *reinterpret_cast<const bf16x8*>(x + row * ldx + vi * 8);
      dc = *reinterpret_cast<const bf16x8*>(dy + row * lddy + vi * 8);
    }
  }
  for (; row < M; row += gridDim.x) {
    const int64_t nrow = row + gridDim.x;
    bf16x8 xn = zero, dn = zero;
    float rstd_n = 0.f, mean_n = 0.f;
    if (nrow < M) {
      rstd_n = rstd_in[nrow];
      if (LAYERNORM) mean_n = mean_in[nrow];
      if (on) {
        xn = *reinterpret_cast<const bf16x8*>(x + nrow * ldx + vi * 8);
        dn = *reinterpret_cast<const bf16x8*>(dy + nrow * lddy + vi * 8);
      }
    }
    float xh[8], g[8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 xf = __bfloat1622float2(xc.h[h]), df = __bfloat1622float2(dc.h[h]);
      const float xv[2] = {xf.x, xf.y}, dv[2] = {df.x, df.y};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 2 * h + e;
        xh[j] = (xv[e] - mean_c) * rstd_c;
        g[j] = dv[e] * wv[j];
        dwacc[j] += dv[e] * xh[j];
        if (LAYERNORM) dbacc[j] += dv[e];
        s1 += g[j];
        s2 += g[j] * xh[j];
      }
    }
    const float c2 = block_sum(s2, red) / D;
    const float c1 = LAYERNORM ? block_sum(s1, red) / D : 0.f;
    if (on) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rstd_c * (g[j] - c1 - xh[j] * c2);
      if (dres) {
        float r[8];
        load8(dres + row * lddres + vi * 8, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += r[j];
      }
      store8(dx + row * lddx + vi * 8, o);
    }
    xc = xn;
    dc = dn;
    rstd_c = rstd_n;
    mean_c = mean_n;
  }
  if (on) {
    float* p = dw_part + (int64_t)blockIdx.x * D + vi * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = dwacc[j];
    if (LAYERNORM && db_part) {
      float* q = db_part + (int64_t)blockIdx.x * D + vi * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = dbacc[j];
    }
  }
}

// Backward for short rows (D <= 1024, e.g. 768 for ViT-B): one warp per row with V 8-element vectors per
// lane, so a block of 8 warps works on 8 rows at once with shuffle-only reductions (the block-per-row
// kernel above gets only D/8 threads per block at these widths). Each warp accumulates dgamma/dbeta for its
// rows; the block adds its 8 warps' sums in a fixed order into one partial row (deterministic).
template <bool LAYERNORM, int V>
__global__ void __launch_bounds__(256)
    norm_bwd_warp_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy, const __nv_bfloat16* __restrict__ x,
                         int64_t ldx, const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean_in,
                         const float* __restrict__ rstd_in, __nv_bfloat16* __restrict__ dx, int64_t lddx,
                         const __nv_bfloat16* __restrict__ dres, int64_t lddres, float* __restrict__ dw_part,
                         float* __restrict__ db_part, int M, int D) {
  extern __shared__ float wsum[];  // [8 warps][2][D]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nvec = D / 8;
  float wv[V][8], dwacc[V][8], dbacc[V][8];
#pragma unroll
  for (int v = 0; v < V; ++v) {
#pragma unroll
    for (int j = 0; j < 8; ++j) wv[v][j] = dwacc[v][j] = dbacc[v][j] = 0.f;
    const int vi = lane + 32 * v;
    if (vi < nvec) load8(w + vi * 8, wv[v]);
  }
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < M; row += (int64_t)gridDim.x * 8) {
    const float rstd = rstd_in[row];
    const float mean = LAYERNORM ? mean_in[row] : 0.f;
    float xh[V][8], g[V][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int vi = lane + 32 * v;
      float xv[8], dv[8];
      if (vi < nvec) {
        load8(x + row * ldx + vi * 8, xv);
        load8(dy + row * lddy + vi * 8, dv);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[j] = dv[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xh[v][j] = (xv[j] - mean) * rstd;
        g[v][j] = dv[j] * wv[v][j];
        dwacc[v][j] += dv[j] * xh[v][j];
        if (LAYERNORM) dbacc[v][j] += dv[j];
        s1 += g[v][j];
        s2 += g[v][j] * xh[v][j];
      }
    }
    const float c2 = warp_sum(s2) / D;
    const float c1 = LAYERNORM ? warp_sum(s1) / D : 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int vi = lane + 32 * v;
      if (vi >= nvec) continue;
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rstd * (g[v][j] - c1 - xh[v][j] * c2);
      if (dres) {
        float r[8];
        load8(dres + row * lddres + vi * 8, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += r[j];
      }
      store8(dx + row * lddx + vi * 8, o);
    }
  }
  float* mine = wsum + warp * 2 * D;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int vi = lane + 32 * v;
    if (vi < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mine[vi * 8 + j] = dwacc[v][j];
        mine[D + vi * 8 + j] = dbacc[v][j];
      }
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float sw = 0.f, sb = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      sw += wsum[k * 2 * D + d];
      sb += wsum[k * 2 * D + D + d];
    }
    dw_part[(int64_t)blockIdx.x * D + d] = sw;
    if (LAYERNORM && db_part) db_part[(int64_t)blockIdx.x * D + d] = sb;
  }
}

// out[d] (+)= sum_p part[p, d] with 8 row slices per column (block 32 x 8): each thread sums every
// 8th partial row of one column, then the 8 slice sums are added in a fixed order (deterministic).
__global__ void colsum8_kernel(const float* __restrict__ part, int P, int D, void* out, int out_f32, int accumulate) {
  __shared__ float sm[8][33];
  const int d = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (d < D)
    for (int p = threadIdx.y; p < P; p += 8) s += part[(int64_t)p * D + d];
  sm[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || d >= D) return;
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) t += sm[k][threadIdx.x];
  if (out_f32) {
    float* o = reinterpret_cast<float*>(out);
    o[d] = accumulate ? o[d] + t : t;
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
    o[d] = __float2bfloat16_rn(accumulate ? __bfloat162float(o[d]) + t : t);
  }
}

// Column sums of a bf16 matrix x [M, N] (bias gradients): block (32, 8) covers 32 column vectors of 8 and
// strides over rows with its 8 row lanes; each lane keeps 8 f32 sums, the 8 lanes are added in order and the
// block writes one f32 partial row (part[blockIdx.y, :]); colsum8_kernel then adds the partial rows.
__global__ void colsum_bf16_part_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M, int N,
                                        float* __restrict__ part) {
  __shared__ float sm[8][32 * 8 + 1];
  const int v = blockIdx.x * 32 + threadIdx.x;  // column vector
  const bool col_ok = v * 8 < N;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  if (col_ok) {
    for (int64_t r = (int64_t)blockIdx.y * 8 + threadIdx.y; r < M; r += (int64_t)gridDim.y * 8) {
      float f[8];
      load8(x + r * ldx + v * 8, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) sm[threadIdx.y][threadIdx.x * 8 + j] = acc[j];
  __syncthreads();
  // 256 threads finalise the block's 256 columns: column c = threadIdx.y * 32 + threadIdx.x
  const int c = threadIdx.y * 32 + threadIdx.x;
  const int col = blockIdx.x * 256 + c;
  if (col < N) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sm[k][c];
    part[(int64_t)blockIdx.y * N + col] = t;
  }
}

// out[d] (+)= sum_p part[p, d]; out dtype bf16 (out_f32 = 0) or f32.
__global__ void colsum_kernel(const float* __restrict__ part, int P, int D, void* out, int out_f32, int accumulate) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  for (int p = 0; p < P; ++p) s += part[(int64_t)p * D + d];
  if (out_f32) {
    float* o = reinterpret_cast<float*>(out);
    o[d] = accumulate ? o[d] + s : s;
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
    o[d] = __float2bfloat16_rn(accumulate ? __bfloat162float(o[d]) + s : s);
  }
}

int threads_for(int D) {
  int nvec = D / 8;
  int t = (nvec + VPT - 1) / VPT;
  t = ((t + 31) / 32) * 32;
  return t < 32 ? 32 : t;
}

}  // namespace

BRAIN_STATUS_READER(norms)

// kind: 0 = RMSNorm, 1 = LayerNorm.  res/sum_out optional (fused residual add).
BRAIN_API int brain_norm_fwd(int kind, const void* x, int64_t ldx, const void* res, int64_t ldres, const void* w,
                             const void* b, void* y, int64_t ldy, void* sum_out, int64_t ldsum, float* mean_out,
                             float* rstd_out, int M, int D, float eps, cudaStream_t st) {
  if (M == 0) return 0;
  if (D % 8 != 0 || D > 1024 * VPT * 8) return (int)cudaErrorInvalidValue;
  const int T = threads_for(D);
  if (T > 1024) return (int)cudaErrorInvalidValue;
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto R = reinterpret_cast<const __nv_bfloat16*>(res);
  auto W = reinterpret_cast<const __nv_bfloat16*>(w);
  auto Bp = reinterpret_cast<const __nv_bfloat16*>(b);
  auto Y = reinterpret_cast<__nv_bfloat16*>(y);
  auto S = reinterpret_cast<__nv_bfloat16*>(sum_out);
  if (kind == 0)
    norm_fwd_kernel<false><<<M, T, 0, st>>>(X, ldx, R, ldres, W, Bp, Y, ldy, S, ldsum, mean_out, rstd_out, D, eps);
  else
    norm_fwd_kernel<true><<<M, T, 0, st>>>(X, ldx, R, ldres, W, Bp, Y, ldy, S, ldsum, mean_out, rstd_out, D, eps);
  return (int)cudaGetLastError();
}

// Number of f32 partial rows brain_colsum_bf16 needs in its workspace (f32 [partials, N]).
BRAIN_API int brain_colsum_partials(int M) {
  const int p = 2 * brain_host::num_sms();
  return M < 8 * p ? (M + 7) / 8 > 0 ? (M + 7) / 8 : 1 : p;
}

// out[n] (+)= sum_m x[m, n] for bf16 x [M, N] (row stride ldx, N % 8 == 0, 16-byte aligned rows); out is
// bf16 or f32 (out_f32), accumulated when accumulate != 0. Deterministic (fixed summation order).
BRAIN_API int brain_colsum_bf16(const void* x, int64_t ldx, int M, int N, void* out, int out_f32, int accumulate,
                                float* workspace, cudaStream_t st) {
  if (N == 0) return 0;
  if (N % 8 != 0 || ldx % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15)) return (int)cudaErrorInvalidValue;
  const int P = brain_colsum_partials(M);
  if (M > 0) {
    dim3 grid((N / 8 + 31) / 32, P);
    colsum_bf16_part_kernel<<<grid, dim3(32, 8), 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, N,
                                                         workspace);
  } else {
    cudaMemsetAsync(workspace, 0, sizeof(float) * N, st);
  }
  colsum8_kernel<<<(N + 31) / 32, dim3(32, 8), 0, st>>>(workspace, M > 0 ? P : 1, N, out, out_f32, accumulate);
  return (int)cudaGetLastError();
}

// Number of f32 partial rows the backward pass needs in its workspace (per gamma/beta).
BRAIN_API int brain_norm_bwd_partials(int M) {
  int p = 2 * brain_host::num_sms();
  return M < p ? (M > 0 ? M : 1) : p;
}

// dres optional: gradient flowing into the residual stream, added to dx.
// dw/db: outputs (bf16 or f32 via dw_f32), accumulated when accumulate != 0. db may be null.
// workspace: f32 [2 * partials * D].
BRAIN_API int brain_norm_bwd(int kind, const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                             const float* mean_in, const float* rstd_in, void* dx, int64_t lddx, const void* dres,
                             int64_t lddres, void* dw, void* db, int dw_f32, int accumulate, float* workspace, int M,
                             int D, cudaStream_t st) {
  if (M == 0) return 0;
  if (D % 8 != 0 || D > 1024 * VPT * 8) return (int)cudaErrorInvalidValue;
  const int T = threads_for(D);
  const int P = brain_norm_bwd_partials(M);
  float* dwp = workspace;
  float* dbp = workspace + (int64_t)P * D;
  auto DY = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto W = reinterpret_cast<const __nv_bfloat16*>(w);
  auto DX = reinterpret_cast<__nv_bfloat16*>(dx);
  auto DR = reinterpret_cast<const __nv_bfloat16*>(dres);
  if (D <= 1024) {  // short rows: one warp per row
    const size_t sm = (size_t)8 * 2 * D * sizeof(float);
    const int vecs = (D / 8 + 31) / 32;
#define BRAIN_NORM_WARP(VV)                                                                                         \
  do {                                                                                                              \
    cudaFuncSetAttribute(norm_bwd_warp_kernel<false, VV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);   \
    cudaFuncSetAttribute(norm_bwd_warp_kernel<true, VV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);    \
    if (kind == 0)                                                                                                  \
      norm_bwd_warp_kernel<false, VV><<<P, 256, sm, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR,      \
                                                         lddres, dwp, nullptr, M, D);                              \
    else                                                                                                            \
      norm_bwd_warp_kernel<true, VV><<<P, 256, sm, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR,       \
                                                        lddres, dwp, dbp, M, D);                                   \
  } while (0)
    if (vecs <= 1) BRAIN_NORM_WARP(1);
    else if (vecs <= 2) BRAIN_NORM_WARP(2);
    else BRAIN_NORM_WARP(4);
#undef BRAIN_NORM_WARP
    colsum8_kernel<<<(D + 31) / 32, dim3(32, 8), 0, st>>>(dwp, P, D, dw, dw_f32, accumulate);
    if (kind == 1 && db) colsum8_kernel<<<(D + 31) / 32, dim3(32, 8), 0, st>>>(dbp, P, D, db, dw_f32, accumulate);
    return (int)cudaGetLastError();
  }
  if (D / 8 <= 1024) {  // one vector per thread, next-row prefetch
    const int T1 = ((D / 8 + 31) / 32) * 32;
    if (kind == 0)
      norm_bwd_v1_kernel<false><<<P, T1, 0, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR, lddres, dwp,
                                                  nullptr, M, D);
    else
      norm_bwd_v1_kernel<true><<<P, T1, 0, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR, lddres, dwp, dbp,
                                                 M, D);
    colsum8_kernel<<<(D + 31) / 32, dim3(32, 8), 0, st>>>(dwp, P, D, dw, dw_f32, accumulate);
    if (kind == 1 && db) colsum8_kernel<<<(D + 31) / 32, dim3(32, 8), 0, st>>>(dbp, P, D, db, dw_f32, accumulate);
    return (int)cudaGetLastError();
  }
  if (kind == 0)
    norm_bwd_kernel<false><<<P, T, 0, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR, lddres, dwp, nullptr, M, D);
  else
    norm_bwd_kernel<true><<<P, T, 0, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR, lddres, dwp, dbp, M, D);
  colsum_kernel<<<(D + 255) / 256, 256, 0, st>>>(dwp, P, D, dw, dw_f32, accumulate);
  if (kind == 1 && db) colsum_kernel<<<(D + 255) / 256, 256, 0, st>>>(dbp, P, D, db, dw_f32, accumulate);
  return (int)cudaGetLastError();
}

// =============================================================================================
// No-allocation variant of the normalisation backward (no counterpart in the reference; declared
// in no_alloc.h). brain_norm_bwd above takes its f32 partial-sum workspace from the caller, which
// usually means an allocation per call. Callers that must not allocate device memory while they
// run - a C or C++ host that links this library without PyTorch or any allocator, or a serving
// process that reserved the whole GPU up front under a fixed memory budget - use
// brain_norm_bwd_noalloc instead: its partial sums live in the fixed array below.
//
// Limits: the array holds 2 x 64 x 8192 floats (4 MiB, held on every GPU that loads the library
// until the process exits), so D must be <= 8192; larger D is rejected with BRAIN_NOALLOC_TOO_LARGE.
// At most 64 partial rows are used (fewer when M < 64); every partial the column sums read is
// written first by the same call, so nothing has to be cleared between calls.
// Every call shares the array: two calls that overlap on the GPU (different streams, or another
// host thread) race on it and must be serialised by the caller.
// Set-up: the first call on each device resolves the array's device address with
// cudaGetSymbolAddress while that device is current; make that first call before any stream
// capture. Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
// =============================================================================================
namespace {

constexpr int kNoAllocPartials = 64;
constexpr int kNoAllocMaxD = 8192;
static __device__ __align__(256) float g_norm_bwd_scratch[2 * kNoAllocPartials * kNoAllocMaxD];

// Device address of the array on the current device, looked up once per device. The slots are atomics:
// two host threads making their first call on the same device at once both look the address up and
// store the same value, with no data race.
float* noalloc_scratch_ptr(int* err) {
  static std::atomic<float*> ptrs[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *err = (e != cudaSuccess) ? (int)e : (int)cudaErrorInvalidDevice;
    return nullptr;
  }
  float* cached = ptrs[dev].load(std::memory_order_relaxed);
  if (!cached) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_norm_bwd_scratch);  // host-side stand-in -> device address
    if (e != cudaSuccess) {
      *err = (int)e;
      return nullptr;
    }
    cached = static_cast<float*>(p);
    ptrs[dev].store(cached, std::memory_order_relaxed);
  }
  *err = 0;
  return cached;
}

}  // namespace

// Same arguments as brain_norm_bwd without the workspace (see no_alloc.h). Returns 0, a cudaError_t
// (cudaErrorInvalidValue for M < 0, D <= 0, D not a multiple of 8 or an unknown kind), or
// BRAIN_NOALLOC_TOO_LARGE when D exceeds the fixed scratch (D > 8192).
BRAIN_API int brain_norm_bwd_noalloc(int kind, const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                                     const float* mean_in, const float* rstd_in, void* dx, int64_t lddx,
                                     const void* dres, int64_t lddres, void* dw, void* db, int dw_f32, int accumulate,
                                     int M, int D, cudaStream_t st) {
  if (M < 0 || D <= 0 || (kind != 0 && kind != 1)) return (int)cudaErrorInvalidValue;
  if (D > kNoAllocMaxD) return BRAIN_NOALLOC_TOO_LARGE;
  if (D % 8 != 0) return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  int err = 0;
  float* scratch = noalloc_scratch_ptr(&err);
  if (!scratch) return err;
  const int T = threads_for(D);
  const int P = M < kNoAllocPartials ? M : kNoAllocPartials;
  float* dwp = scratch;
  float* dbp = scratch + (int64_t)P * D;
  auto DY = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto W = reinterpret_cast<const __nv_bfloat16*>(w);
  auto DX = reinterpret_cast<__nv_bfloat16*>(dx);
  auto DR = reinterpret_cast<const __nv_bfloat16*>(dres);
  if (kind == 0)
    norm_bwd_kernel<false><<<P, T, 0, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR, lddres, dwp, nullptr, M, D);
  else
    norm_bwd_kernel<true><<<P, T, 0, st>>>(DY, lddy, X, ldx, W, mean_in, rstd_in, DX, lddx, DR, lddres, dwp, dbp, M, D);
  colsum_kernel<<<(D + 255) / 256, 256, 0, st>>>(dwp, P, D, dw, dw_f32, accumulate);
  if (kind == 1 && db) colsum_kernel<<<(D + 255) / 256, 256, 0, st>>>(dbp, P, D, db, dw_f32, accumulate);
  return (int)cudaGetLastError();
}
