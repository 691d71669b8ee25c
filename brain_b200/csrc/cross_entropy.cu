// Softmax cross-entropy over large vocabularies (e.g. 128 256 classes), bf16 logits, f32 math.
//
// Forward: one CTA per row streams the row once with 16-byte loads and an online (max, sum-exp)
// reduction, giving lse, the target logit and (for label smoothing) the row sum of logits:
//   loss = (1 - eps) * (lse - z_y) + eps * (lse - mean(z))
// Backward: one more streaming pass writes dlogits = g_row * (softmax(z) - (1 - eps) onehot - eps / V),
// optionally in place over the logits buffer (the logits are dead after the loss).
// Rows whose label equals ignore_index get zero loss and zero gradient.
//
// Reference: softmax subtracts the row max (crates/brain-core/src/tensor/special.rs:119-125);
// cross_entropy_loss (crates/brain-core/src/tensor/neural.rs:40-58); CrossEntropyLoss with label
// smoothing (crates/brain-loss/src/classification/ce.rs:16-135).
#include "common.cuh"

using namespace brain;

namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
  m = mn;
}

__global__ void __launch_bounds__(kThreads) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                                          const int64_t* __restrict__ labels, float* __restrict__ loss,
                                                          float* __restrict__ lse_out, int V, int64_t ignore_index,
                                                          float smoothing) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* z = logits + row * ld;
  float m = -INFINITY, s = 0.f, zsum = 0.f;
  const int nv = V / 8;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float v[8];
    load8(z + i * 8, v);
    float lm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ls += __expf(v[j] - lm);
      zsum += v[j];
    }
    online_merge(m, s, lm, ls);
  }
  for (int i = nv * 8 + threadIdx.x; i < V; i += kThreads) {
    const float v = __bfloat162float(z[i]);
    online_merge(m, s, v, 1.f);
    zsum += v;
  }
  // block reduction of (m, s) and zsum
  __shared__ float sm[kThreads / 32], ss[kThreads / 32], sz[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
    zsum += __shfl_xor_sync(0xffffffffu, zsum, o);
  }
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) {
    sm[w] = m;
    ss[w] = s;
    sz[w] = zsum;
  }
  __syncthreads();
  if (w == 0) {
    constexpr int NW = kThreads / 32;
    m = l < NW ? sm[l] : -INFINITY;
    s = l < NW ? ss[l] : 0.f;
    zsum = l < NW ? sz[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
      zsum += __shfl_xor_sync(0xffffffffu, zsum, o);
    }
    if (l == 0) {
      const float lse = m + __logf(s);
      const int64_t y = labels[row];
      float L = 0.f;
      if (y != ignore_index) {
        if (y < 0 || y >= V) {
          set_status(BRAIN_ERR_BOUNDS, 700);
        } else {
          const float zy = __bfloat162float(z[y]);
          L = (1.f - smoothing) * (lse - zy) + smoothing * (lse - zsum / V);
        }
      }
      loss[row] = L;
      lse_out[row] = lse;
    }
  }
}

// grad: per-row upstream gradient (f32 [M]) or, when grad_scalar_ptr is set, one f32 scalar
// multiplied by `scale` (e.g. 1/num_valid for a mean reduction).
__global__ void __launch_bounds__(kThreads) ce_bwd_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                                          const int64_t* __restrict__ labels,
                                                          const float* __restrict__ lse_in, const float* __restrict__ grad,
                                                          const float* __restrict__ grad_scalar, float scale,
                                                          __nv_bfloat16* __restrict__ dlogits, int64_t ldd, int V,
                                                          int64_t ignore_index, float smoothing) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* z = logits + row * ld;
  __nv_bfloat16* dz = dlogits + row * ldd;
  const int64_t y = labels[row];
  float g = grad_scalar ? grad_scalar[0] * scale : grad[row] * scale;
  if (y == ignore_index) g = 0.f;
  const float lse = lse_in[row];
  const float off = smoothing / V;
  const int nv = V / 8;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float v[8];
    load8(z + i * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = i * 8 + j;
      v[j] = g * (__expf(v[j] - lse) - off - (c == y ? 1.f - smoothing : 0.f));
    }
    store8(dz + i * 8, v);
  }
  for (int c = nv * 8 + threadIdx.x; c < V; c += kThreads) {
    const float v = __bfloat162float(z[c]);
    dz[c] = __float2bfloat16_rn(g * (__expf(v - lse) - off - (c == y ? 1.f - smoothing : 0.f)));
  }
}

}  // namespace

BRAIN_STATUS_READER(ce)

BRAIN_API int brain_ce_fwd(const void* logits, int64_t ld, const int64_t* labels, float* loss, float* lse, int64_t M,
                           int V, int64_t ignore_index, float smoothing, cudaStream_t st) {
  if (M == 0) return 0;
  if (ld % 8) return (int)cudaErrorInvalidValue;
  ce_fwd_kernel<<<(unsigned)M, kThreads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(logits), ld, labels, loss,
                                                   lse, V, ignore_index, smoothing);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_ce_bwd(const void* logits, int64_t ld, const int64_t* labels, const float* lse, const float* grad,
                           const float* grad_scalar, float scale, void* dlogits, int64_t ldd, int64_t M, int V,
                           int64_t ignore_index, float smoothing, cudaStream_t st) {
  if (M == 0) return 0;
  if (ld % 8 || ldd % 8) return (int)cudaErrorInvalidValue;
  ce_bwd_kernel<<<(unsigned)M, kThreads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(logits), ld, labels, lse,
                                                   grad, grad_scalar, scale,
                                                   reinterpret_cast<__nv_bfloat16*>(dlogits), ldd, V, ignore_index,
                                                   smoothing);
  return (int)cudaGetLastError();
}
