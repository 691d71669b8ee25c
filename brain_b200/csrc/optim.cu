// Fused optimizer kernels over flat parameter buffers (single pass, 16-byte vector accesses).
//
// AdamW follows the reference order exactly (crates/brain-optim/src/adam/mod.rs:128-200):
//   p -= lr * wd * p                      (decoupled decay, before the moments)
//   m  = b1 m + (1 - b1) g ; v = b2 v + (1 - b2) g^2
//   p -= lr * (m / bc1) / (sqrt(v / bc2) + eps)
// with g = grad * grad_scale (loss-scale and world-size un-scaling folded in). When `found_inf`
// (device int) is non-zero the step is skipped entirely, which is how a non-finite gradient is
// handled under dynamic loss scaling (the reference returns an error for it). The master weights
// stay f32; an optional bf16 copy (the compute weights) is written in the same pass.
#include "common.cuh"

using namespace brain;

namespace {

template <typename G>
__device__ __forceinline__ float ld_grad(const G* g, int64_t i);
template <>
__device__ __forceinline__ float ld_grad<float>(const float* g, int64_t i) { return g[i]; }
template <>
__device__ __forceinline__ float ld_grad<__nv_bfloat16>(const __nv_bfloat16* g, int64_t i) {
  return __bfloat162float(g[i]);
}

// Four consecutive gradient elements starting at element 4 * i4 (one 16-byte f32 or 8-byte bf16 load
// when the pointer allows it).
template <typename G>
__device__ __forceinline__ void ld_grad4(const G* g, int64_t i4, bool vec, float* out);
template <>
__device__ __forceinline__ void ld_grad4<float>(const float* g, int64_t i4, bool vec, float* out) {
  if (vec) {
    const float4 t = reinterpret_cast<const float4*>(g)[i4];
    out[0] = t.x; out[1] = t.y; out[2] = t.z; out[3] = t.w;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = g[i4 * 4 + j];
  }
}
template <>
__device__ __forceinline__ void ld_grad4<__nv_bfloat16>(const __nv_bfloat16* g, int64_t i4, bool vec, float* out) {
  if (vec) {
    const uint2 t = reinterpret_cast<const uint2*>(g)[i4];
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.y));
    out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = __bfloat162float(g[i4 * 4 + j]);
  }
}

struct AdamHyper {
  float lr, b1, b2, eps, wd, bc1, bc2, grad_scale;
  int amsgrad;
};

template <typename G>
__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                             float* __restrict__ vmax, const G* __restrict__ g, __nv_bfloat16* __restrict__ p16,
                             int64_t n, AdamHyper h, const int* __restrict__ found_inf,
                             const float* __restrict__ coef) {
  if (found_inf && *found_inf) return;
  if (coef) h.grad_scale *= *coef;  // global-norm clipping coefficient computed on the device
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float one_b1 = 1.f - h.b1, one_b2 = 1.f - h.b2;
  const float inv_bc1 = 1.f / h.bc1, inv_bc2 = 1.f / h.bc2;
  const float decay = 1.f - h.lr * h.wd;
  // 4 elements per thread-iteration
  const int64_t n4 = n / 4;
  const bool gvec = (reinterpret_cast<uintptr_t>(g) & (4 * sizeof(G) - 1)) == 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float gg[4];
    ld_grad4(g, i, gvec, gg);
#pragma unroll
    for (int j = 0; j < 4; ++j) gg[j] *= h.grad_scale;
    float* P = &pp.x;
    float* Mv = &mm.x;
    float* Vv = &vv.x;
    float vm[4];
    if (h.amsgrad) {
      float4 t = reinterpret_cast<float4*>(vmax)[i];
      vm[0] = t.x; vm[1] = t.y; vm[2] = t.z; vm[3] = t.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      P[j] *= decay;
      Mv[j] = h.b1 * Mv[j] + one_b1 * gg[j];
      Vv[j] = h.b2 * Vv[j] + one_b2 * gg[j] * gg[j];
      float vh = Vv[j];
      if (h.amsgrad) {
        vm[j] = fmaxf(vm[j], vh);
        vh = vm[j];
      }
      P[j] -= h.lr * (Mv[j] * inv_bc1) / (sqrtf(vh * inv_bc2) + h.eps);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (h.amsgrad) reinterpret_cast<float4*>(vmax)[i] = make_float4(vm[0], vm[1], vm[2], vm[3]);
    if (p16) {
      __nv_bfloat162 a = __floats2bfloat162_rn(pp.x, pp.y), b = __floats2bfloat162_rn(pp.z, pp.w);
      uint2 packed;
      packed.x = *reinterpret_cast<uint32_t*>(&a);
      packed.y = *reinterpret_cast<uint32_t*>(&b);
      reinterpret_cast<uint2*>(p16)[i] = packed;
    }
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gg = ld_grad(g, i) * h.grad_scale;
    float pv = p[i] * decay;
    const float mv = h.b1 * m[i] + one_b1 * gg;
    const float vv = h.b2 * v[i] + one_b2 * gg * gg;
    float vh = vv;
    if (h.amsgrad) {
      vmax[i] = fmaxf(vmax[i], vv);
      vh = vmax[i];
    }
    pv -= h.lr * (mv * inv_bc1) / (sqrtf(vh * inv_bc2) + h.eps);
    p[i] = pv;
    m[i] = mv;
    v[i] = vv;
    if (p16) p16[i] = __float2bfloat16_rn(pv);
  }
}

// SGD with optional momentum / Nesterov and (coupled) weight decay (crates/brain-optim/src/sgd/mod.rs:53-82).
template <typename G>
__global__ void sgd_kernel(float* __restrict__ p, float* __restrict__ buf, const G* __restrict__ g,
                           __nv_bfloat16* __restrict__ p16, int64_t n, float lr, float momentum, float dampening,
                           float wd, int nesterov, int first, float grad_scale, const int* __restrict__ found_inf) {
  if (found_inf && *found_inf) return;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float d = ld_grad(g, i) * grad_scale + wd * p[i];
    if (momentum != 0.f) {
      const float b = first ? d : momentum * buf[i] + (1.f - dampening) * d;
      buf[i] = b;
      d = nesterov ? d + momentum * b : b;
    }
    const float pv = p[i] - lr * d;
    p[i] = pv;
    if (p16) p16[i] = __float2bfloat16_rn(pv);
  }
}

// Sum of squares (f32 partials per CTA, then a single-CTA finish) and a non-finite flag.
template <typename G>
__global__ void sumsq_kernel(const G* __restrict__ g, int64_t n, float scale, float* __restrict__ partial,
                             int* __restrict__ found_inf) {
  float s = 0.f;
  bool bad = false;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = ld_grad(g, i) * scale;
    bad |= !isfinite(x);
    s += x * x;
  }
  s = warp_sum(s);
  __shared__ float red[32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = s;
  if (bad && found_inf) atomicExch(found_inf, 1);
  __syncthreads();
  if (w == 0) {
    float t = l < (int)(blockDim.x / 32) ? red[l] : 0.f;
    t = warp_sum(t);
    if (l == 0) partial[blockIdx.x] = t;
  }
}

__global__ void finish_sum_kernel(const float* __restrict__ partial, int P, float* __restrict__ out, int accumulate) {
  float s = 0.f;
  for (int i = threadIdx.x; i < P; i += blockDim.x) s += partial[i];
  s = warp_sum(s);
  __shared__ float red[32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = s;
  __syncthreads();
  if (w == 0) {
    float t = l < (int)(blockDim.x / 32) ? red[l] : 0.f;
    t = warp_sum(t);
    if (l == 0) *out = accumulate ? *out + t : t;
  }
}

// x *= s (f32 or bf16 flat buffer); used for gradient clipping and un-scaling.
template <typename T>
__global__ void scale_kernel(T* __restrict__ x, int64_t n, const float* __restrict__ s_ptr, float s_const) {
  const float s = s_ptr ? *s_ptr : s_const;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (std::is_same<T, float>::value) x[i] *= s;
    else x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) * s);
  }
}

// Clip coefficient from a total squared norm: coef = min(1, max_norm / (sqrt(sq) + 1e-6)).
__global__ void clip_coef_kernel(const float* sq, float max_norm, float* coef) {
  const float norm = sqrtf(*sq);
  *coef = fminf(1.f, max_norm / (norm + 1e-6f));
}

// Gradient statistics for a guarded optimizer step: per-CTA partial sums of (scale * g)^2 and a per-CTA
// non-finite flag into ws[2 * blockIdx.x + {0, 1}].
template <typename G>
__global__ void grad_stats_kernel(const G* __restrict__ g, int64_t n, float scale, float* __restrict__ ws) {
  float s = 0.f;
  float bad = 0.f;
  const int64_t n4 = n / 4;
  const bool vec = (reinterpret_cast<uintptr_t>(g) & (4 * sizeof(G) - 1)) == 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float x[4];
    ld_grad4(g, i, vec, x);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float y = x[j] * scale;
      if (!isfinite(y)) bad = 1.f;
      s += y * y;
    }
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float y = ld_grad(g, i) * scale;
    if (!isfinite(y)) bad = 1.f;
    s += y * y;
  }
  s = warp_sum(s);
  bad = warp_max(bad);
  __shared__ float red[2][32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) {
    red[0][w] = s;
    red[1][w] = bad;
  }
  __syncthreads();
  if (w == 0) {
    const bool in = l < (int)(blockDim.x / 32);
    float t = warp_sum(in ? red[0][l] : 0.f);
    float b = warp_max(in ? red[1][l] : 0.f);
    if (l == 0) {
      ws[2 * blockIdx.x] = t;
      ws[2 * blockIdx.x + 1] = b;
    }
  }
}

// stats[0] (+)= sum of the partial squares, stats[1] (+)= 1 if any partial saw a non-finite value
// (fixed summation order: the result does not depend on scheduling).
__global__ void grad_stats_finish_kernel(const float* __restrict__ ws, int P, float* __restrict__ stats,
                                         int accumulate) {
  float s = 0.f, b = 0.f;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    s += ws[2 * i];
    b = fmaxf(b, ws[2 * i + 1]);
  }
  s = warp_sum(s);
  b = warp_max(b);
  __shared__ float red[2][32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) {
    red[0][w] = s;
    red[1][w] = b;
  }
  __syncthreads();
  if (w == 0) {
    const bool in = l < (int)(blockDim.x / 32);
    float t = warp_sum(in ? red[0][l] : 0.f);
    float c = warp_max(in ? red[1][l] : 0.f);
    if (l == 0) {
      stats[0] = accumulate ? stats[0] + t : t;
      stats[1] = accumulate ? stats[1] + c : c;
    }
  }
}

// From globally reduced statistics (sum of squares, count of ranks / pieces that saw a non-finite
// value): found_inf = any non-finite (the step is skipped on every rank alike), coef = global-norm clip
// coefficient min(1, max_norm / (norm + 1e-6)) or 1 when max_norm <= 0.
__global__ void step_guard_kernel(const float* __restrict__ stats, float max_norm, int* __restrict__ found_inf,
                                  float* __restrict__ coef) {
  const float sq = stats[0];
  const bool bad = stats[1] != 0.f || !isfinite(sq);
  *found_inf = bad ? 1 : 0;
  *coef = (max_norm > 0.f && !bad) ? fminf(1.f, max_norm / (sqrtf(sq) + 1e-6f)) : 1.f;
}

// f32 -> bf16 copy
__global__ void cast_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

int grid_for(int64_t n) {
  int64_t g = (n / 4 + 255) / 256;
  int64_t cap = (int64_t)brain_host::num_sms() * 8;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

BRAIN_STATUS_READER(optim)

// grad_f32: 1 = gradient buffer is f32, 0 = bf16. vmax may be null unless amsgrad.
// found_inf (device int, may be null): skip the step when non-zero. coef (device float, may be null):
// extra factor on the gradient (global-norm clipping).
BRAIN_API int brain_adamw(float* p, float* m, float* v, float* vmax, const void* g, int grad_f32, void* p16, int64_t n,
                          float lr, float b1, float b2, float eps, float wd, float bc1, float bc2, float grad_scale,
                          int amsgrad, const int* found_inf, const float* coef, cudaStream_t st) {
  if (n == 0) return 0;
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15)
    return (int)cudaErrorInvalidValue;
  if (p16 && (reinterpret_cast<uintptr_t>(p16) & 7)) return (int)cudaErrorInvalidValue;
  AdamHyper h{lr, b1, b2, eps, wd, bc1, bc2, grad_scale, amsgrad};
  if (grad_f32)
    adamw_kernel<float><<<grid_for(n), 256, 0, st>>>(p, m, v, vmax, reinterpret_cast<const float*>(g),
                                                     reinterpret_cast<__nv_bfloat16*>(p16), n, h, found_inf, coef);
  else
    adamw_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, st>>>(p, m, v, vmax, reinterpret_cast<const __nv_bfloat16*>(g),
                                                             reinterpret_cast<__nv_bfloat16*>(p16), n, h, found_inf, coef);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_sgd(float* p, float* buf, const void* g, int grad_f32, void* p16, int64_t n, float lr,
                        float momentum, float dampening, float wd, int nesterov, int first, float grad_scale,
                        const int* found_inf, cudaStream_t st) {
  if (n == 0) return 0;
  auto P16 = reinterpret_cast<__nv_bfloat16*>(p16);
  if (grad_f32)
    sgd_kernel<float><<<grid_for(4 * n), 256, 0, st>>>(p, buf, reinterpret_cast<const float*>(g), P16, n, lr, momentum,
                                                       dampening, wd, nesterov, first, grad_scale, found_inf);
  else
    sgd_kernel<__nv_bfloat16><<<grid_for(4 * n), 256, 0, st>>>(p, buf, reinterpret_cast<const __nv_bfloat16*>(g), P16,
                                                               n, lr, momentum, dampening, wd, nesterov, first,
                                                               grad_scale, found_inf);
  return (int)cudaGetLastError();
}

// out (+)= sum(scale * g)^2 over n elements; found_inf set if any element is non-finite.
// workspace: f32 [>= 1024].
BRAIN_API int brain_sumsq(const void* g, int grad_f32, int64_t n, float scale, float* out, int accumulate,
                          int* found_inf, float* workspace, cudaStream_t st) {
  int P = grid_for(4 * n);
  if (P > 1024) P = 1024;
  if (n > 0) {
    if (grad_f32)
      sumsq_kernel<float><<<P, 256, 0, st>>>(reinterpret_cast<const float*>(g), n, scale, workspace, found_inf);
    else
      sumsq_kernel<__nv_bfloat16><<<P, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(g), n, scale, workspace,
                                                     found_inf);
  } else {
    P = 0;
  }
  finish_sum_kernel<<<1, 1024, 0, st>>>(workspace, P, out, accumulate);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_scale(void* x, int is_f32, int64_t n, const float* s_ptr, float s_const, cudaStream_t st) {
  if (n == 0) return 0;
  if (is_f32)
    scale_kernel<float><<<grid_for(4 * n), 256, 0, st>>>(reinterpret_cast<float*>(x), n, s_ptr, s_const);
  else
    scale_kernel<__nv_bfloat16><<<grid_for(4 * n), 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(x), n, s_ptr, s_const);
  return (int)cudaGetLastError();
}

// stats[0:2] (+)= (sum of (scale * g)^2, non-finite seen) over n gradient elements. workspace: f32 [>= 2048].
BRAIN_API int brain_grad_stats(const void* g, int grad_f32, int64_t n, float scale, float* stats, int accumulate,
                               float* workspace, cudaStream_t st) {
  int P = grid_for(4 * n);
  if (P > 1024) P = 1024;
  if (n > 0) {
    if (grad_f32)
      grad_stats_kernel<float><<<P, 256, 0, st>>>(reinterpret_cast<const float*>(g), n, scale, workspace);
    else
      grad_stats_kernel<__nv_bfloat16><<<P, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(g), n, scale,
                                                          workspace);
  } else {
    P = 0;
  }
  grad_stats_finish_kernel<<<1, 1024, 0, st>>>(workspace, P, stats, accumulate);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_step_guard(const float* stats, float max_norm, int* found_inf, float* coef, cudaStream_t st) {
  step_guard_kernel<<<1, 1, 0, st>>>(stats, max_norm, found_inf, coef);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_clip_coef(const float* sq, float max_norm, float* coef, cudaStream_t st) {
  clip_coef_kernel<<<1, 1, 0, st>>>(sq, max_norm, coef);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_cast_bf16(const float* x, void* y, int64_t n, cudaStream_t st) {
  if (n == 0) return 0;
  cast_bf16_kernel<<<grid_for(4 * n), 256, 0, st>>>(x, reinterpret_cast<__nv_bfloat16*>(y), n);
  return (int)cudaGetLastError();
}
