// Memory-bound elementwise kernels: SwiGLU, tanh-GELU, RoPE, embedding gather / scatter-add.
// All use 16-byte vector accesses where the layout allows and f32 math.
//
// Reference semantics:
//   SwiGLU = silu(gate) * up                  crates/brain-core/src/tensor/ops_fused.rs:127-142,
//                                             crates/brain-transformer/src/ffn/mod.rs:88-91
//   GELU   = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))   crates/brain-core/src/tensor/math.rs:284-287
//   RoPE   NeoX half-split pairs (i, i + d/2), freq_i = theta^(-2i/d)
//                                             crates/brain-transformer/src/position/rope.rs:57-142
//   Embedding gather + learned positions      crates/brain-transformer/src/embedding_layers.rs:153
#include "common.cuh"

using namespace brain;

namespace {

__device__ __forceinline__ float silu(float g) { return g / (1.f + __expf(-g)); }

// gu: [M, 2F] (gate columns [0,F), up columns [F,2F)), row stride ldgu. out [M, F].
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, int64_t ldgu, __nv_bfloat16* __restrict__ out,
                                  int64_t ldo, int64_t M, int F) {
  const int nv = F / 8;
  const int64_t total = M * nv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nv;
    const int c = (int)(i - r * nv) * 8;
    float g[8], u[8], o[8];
    load8(gu + r * ldgu + c, g);
    load8(gu + r * ldgu + F + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = silu(g[j]) * u[j];
    store8(out + r * ldo + c, o);
  }
}

// dgu[:, :F] = dy * u * silu'(g), dgu[:, F:] = dy * silu(g).  silu'(g) = s (1 + g (1 - s)), s = sigmoid(g)
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy, const __nv_bfloat16* __restrict__ gu,
                                  int64_t ldgu, __nv_bfloat16* __restrict__ dgu, int64_t lddgu, int64_t M, int F) {
  const int nv = F / 8;
  const int64_t total = M * nv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nv;
    const int c = (int)(i - r * nv) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu + r * ldgu + c, g);
    load8(gu + r * ldgu + F + c, u);
    load8(dy + r * lddy + c, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float s = 1.f / (1.f + __expf(-g[j]));
      du[j] = d[j] * g[j] * s;
      dg[j] = d[j] * u[j] * s * (1.f + g[j] * (1.f - s));
    }
    store8(dgu + r * lddgu + c, dg);
    store8(dgu + r * lddgu + F + c, du);
  }
}

// tanh-approximate GELU and its derivative with the hardware tanh (brain::gelu_tanh_fast): bf16 in and out,
// so the approximation's 2^-11 relative error is below the output rounding.
__device__ __forceinline__ float gelu_tanh(float x) { return gelu_tanh_fast(x); }
__device__ __forceinline__ float gelu_tanh_grad(float x) { return gelu_tanh_grad_fast(x); }

// Contiguous n elements (n % 8 == 0 enforced by the host wrapper; tail handled scalar).
__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  const int64_t nv = n / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float v[8];
    load8(x + i * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = gelu_tanh(v[j]);
    store8(y + i * 8, v);
  }
  for (int64_t i = nv * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(gelu_tanh(__bfloat162float(x[i])));
}
__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                __nv_bfloat16* __restrict__ dx, int64_t n) {
  const int64_t nv = n / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float v[8], d[8];
    load8(x + i * 8, v);
    load8(dy + i * 8, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = d[j] * gelu_tanh_grad(v[j]);
    store8(dx + i * 8, v);
  }
  for (int64_t i = nv * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dx[i] = __float2bfloat16_rn(__bfloat162float(dy[i]) * gelu_tanh_grad(__bfloat162float(x[i])));
}

// In-place rotary embedding on x viewed as [B, S, H, D] with element strides (sb, ss, sh), unit
// stride along D. cs: f32 table [max_pos, D] holding cos in [:, :D/2] and sin in [:, D/2:].
// pos: optional int32 [B, S] positions; otherwise position = pos_offset + s.
// sign = +1 rotates forward, -1 applies the inverse rotation (backward pass).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, int B, int S, int H, int D, int64_t sb, int64_t ss,
                            int64_t sh, const float* __restrict__ cs, const int* __restrict__ pos, int pos_offset,
                            float sign) {
  const int half = D / 2;
  const int64_t pairs = (int64_t)B * S * H * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    int64_t t = i / half;
    const int h = (int)(t % H);
    t /= H;
    const int s = (int)(t % S);
    const int b = (int)(t / S);
    const int p = pos ? pos[(int64_t)b * S + s] : pos_offset + s;
    const float c = cs[(int64_t)p * D + j];
    const float sn = sign * cs[(int64_t)p * D + half + j];
    __nv_bfloat16* base = x + b * sb + s * ss + h * sh;
    const float x1 = __bfloat162float(base[j]);
    const float x2 = __bfloat162float(base[j + half]);
    base[j] = __float2bfloat16_rn(x1 * c - x2 * sn);
    base[j + half] = __float2bfloat16_rn(x2 * c + x1 * sn);
  }
}

// Vectorised RoPE: a thread rotates 8 consecutive pairs (16-byte loads and stores of both halves,
// 32-byte loads of cos and sin); rows (b, s, h) are enumerated with 32-bit index arithmetic.
// Needs D % 16 == 0, 16-byte aligned rows and fewer than 2^31 8-pair units.
__global__ void rope_vec_kernel(__nv_bfloat16* __restrict__ x, int S, int H, int D, int64_t sb, int64_t ss, int64_t sh,
                                const float* __restrict__ cs, const int* __restrict__ pos, int pos_offset, float sign,
                                int units) {
  const int half = D / 2, U = half / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < units; i += gridDim.x * blockDim.x) {
    const int u = i % U;
    const int row = i / U;
    const int h = row % H;
    const int bsi = row / H;
    const int s = bsi % S, b = bsi / S;
    const int p = pos ? pos[bsi] : pos_offset + s;
    const int j = u * 8;
    __nv_bfloat16* base = x + b * sb + s * ss + h * sh;
    const uint4 ra = *reinterpret_cast<const uint4*>(base + j);
    const uint4 rb = *reinterpret_cast<const uint4*>(base + j + half);
    const float4* cp = reinterpret_cast<const float4*>(cs + (int64_t)p * D + j);
    const float4* sp = reinterpret_cast<const float4*>(cs + (int64_t)p * D + half + j);
    const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&ra);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&rb);
    uint4 oa, ob;
    __nv_bfloat162* oa2 = reinterpret_cast<__nv_bfloat162*>(&oa);
    __nv_bfloat162* ob2 = reinterpret_cast<__nv_bfloat162*>(&ob);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x1 = __bfloat1622float2(a2[k]), x2 = __bfloat1622float2(b2[k]);
      const float c_lo = cv[2 * k], c_hi = cv[2 * k + 1];
      const float s_lo = sign * sv[2 * k], s_hi = sign * sv[2 * k + 1];
      oa2[k] = __floats2bfloat162_rn(x1.x * c_lo - x2.x * s_lo, x1.y * c_hi - x2.y * s_hi);
      ob2[k] = __floats2bfloat162_rn(x2.x * c_lo + x1.x * s_lo, x2.y * c_hi + x1.y * s_hi);
    }
    *reinterpret_cast<uint4*>(base + j) = oa;
    *reinterpret_cast<uint4*>(base + j + half) = ob;
  }
}

// out[m, :] = W[ids[m], :] (+ P[m % S, :])   (rows of D elements, D % 8 == 0)
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ W,
                                     const __nv_bfloat16* __restrict__ P, int S, __nv_bfloat16* __restrict__ out,
                                     int64_t M, int D, int64_t V) {
  const int nv = D / 8;
  const int64_t total = M * nv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / nv;
    const int c = (int)(i - m * nv) * 8;
    int64_t id = ids[m];
    float v[8];
    if (id < 0 || id >= V) {
      set_status(BRAIN_ERR_BOUNDS, 600);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    } else {
      load8(W + id * D + c, v);
    }
    if (P) {
      float p[8];
      load8(P + (int64_t)(m % S) * D + c, p);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += p[j];
    }
    store8(out + m * D + c, v);
  }
}

// Deterministic embedding backward: ids sorted ascending (sorted_ids) with the original row of each
// (perm). One CTA per segment start sums the dy rows of its segment in f32 and adds the sum into
// dW[id] (bf16 or f32). CTAs whose position is not a segment start return at once.
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ sorted_ids, const int64_t* __restrict__ perm,
                                     const __nv_bfloat16* __restrict__ dy, void* dW, int dw_f32, int64_t M, int D,
                                     int64_t V) {
  const int64_t i = blockIdx.x;
  const int64_t id = sorted_ids[i];
  if (i > 0 && sorted_ids[i - 1] == id) return;
  if (id < 0 || id >= V) return;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s = 0.f;
    for (int64_t j = i; j < M && sorted_ids[j] == id; ++j) s += __bfloat162float(dy[perm[j] * D + c]);
    if (dw_f32) {
      float* o = reinterpret_cast<float*>(dW) + id * D + c;
      *o += s;
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(dW) + id * D + c;
      *o = __float2bfloat16_rn(__bfloat162float(*o) + s);
    }
  }
}

// Column sums of dy over rows grouped by (m % S): dP[s, :] += sum_{m: m%S==s} dy[m, :]  (learned positions)
__global__ void pos_grad_kernel(const __nv_bfloat16* __restrict__ dy, void* dP, int dp_f32, int64_t M, int S, int D) {
  const int s = blockIdx.x;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int64_t m = s; m < M; m += S) acc += __bfloat162float(dy[m * D + c]);
    if (dp_f32) {
      float* o = reinterpret_cast<float*>(dP) + (int64_t)s * D + c;
      *o += acc;
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(dP) + (int64_t)s * D + c;
      *o = __float2bfloat16_rn(__bfloat162float(*o) + acc);
    }
  }
}

int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  int64_t cap = (int64_t)brain_host::num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

BRAIN_STATUS_READER(elementwise)

BRAIN_API int brain_swiglu_fwd(const void* gu, int64_t ldgu, void* out, int64_t ldo, int64_t M, int F, cudaStream_t st) {
  if (F % 8) return (int)cudaErrorInvalidValue;
  swiglu_fwd_kernel<<<grid_for(M * (F / 8), 256), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(gu), ldgu,
                                                                reinterpret_cast<__nv_bfloat16*>(out), ldo, M, F);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_swiglu_bwd(const void* dy, int64_t lddy, const void* gu, int64_t ldgu, void* dgu, int64_t lddgu,
                               int64_t M, int F, cudaStream_t st) {
  if (F % 8) return (int)cudaErrorInvalidValue;
  swiglu_bwd_kernel<<<grid_for(M * (F / 8), 256), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy), lddy, reinterpret_cast<const __nv_bfloat16*>(gu), ldgu,
      reinterpret_cast<__nv_bfloat16*>(dgu), lddgu, M, F);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_gelu_fwd(const void* x, void* y, int64_t n, cudaStream_t st) {
  gelu_fwd_kernel<<<grid_for(n / 8 + 1, 256), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x),
                                                           reinterpret_cast<__nv_bfloat16*>(y), n);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_gelu_bwd(const void* dy, const void* x, void* dx, int64_t n, cudaStream_t st) {
  gelu_bwd_kernel<<<grid_for(n / 8 + 1, 256), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dy),
                                                           reinterpret_cast<const __nv_bfloat16*>(x),
                                                           reinterpret_cast<__nv_bfloat16*>(dx), n);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_rope(void* x, int B, int S, int H, int D, int64_t sb, int64_t ss, int64_t sh, const float* cs,
                         const int* pos, int pos_offset, float sign, cudaStream_t st) {
  if (D % 2) return (int)cudaErrorInvalidValue;
  const int64_t pairs = (int64_t)B * S * H * (D / 2);
  if (pairs == 0) return 0;
  const int64_t units = pairs / 8;
  const bool vec = D % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && sb % 8 == 0 && ss % 8 == 0 &&
                   sh % 8 == 0 && (reinterpret_cast<uintptr_t>(cs) & 15) == 0 && units < (int64_t)INT32_MAX &&
                   (int64_t)B * S < (int64_t)INT32_MAX;
  if (vec) {
    rope_vec_kernel<<<grid_for(units, 256), 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(x), S, H, D, sb, ss, sh,
                                                          cs, pos, pos_offset, sign, (int)units);
  } else {
    rope_kernel<<<grid_for(pairs, 256), 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(x), B, S, H, D, sb, ss, sh,
                                                     cs, pos, pos_offset, sign);
  }
  return (int)cudaGetLastError();
}

BRAIN_API int brain_embedding_fwd(const int64_t* ids, const void* W, const void* P, int S, void* out, int64_t M, int D,
                                  int64_t V, cudaStream_t st) {
  if (D % 8) return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  embedding_fwd_kernel<<<grid_for(M * (D / 8), 256), 256, 0, st>>>(
      ids, reinterpret_cast<const __nv_bfloat16*>(W), reinterpret_cast<const __nv_bfloat16*>(P), S,
      reinterpret_cast<__nv_bfloat16*>(out), M, D, V);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_embedding_bwd(const int64_t* sorted_ids, const int64_t* perm, const void* dy, void* dW, int dw_f32,
                                  int64_t M, int D, int64_t V, cudaStream_t st) {
  if (M == 0) return 0;
  int threads = D >= 256 ? 256 : ((D + 31) / 32) * 32;
  embedding_bwd_kernel<<<(unsigned)M, threads, 0, st>>>(sorted_ids, perm, reinterpret_cast<const __nv_bfloat16*>(dy),
                                                         dW, dw_f32, M, D, V);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_pos_grad(const void* dy, void* dP, int dp_f32, int64_t M, int S, int D, cudaStream_t st) {
  if (M == 0) return 0;
  int threads = D >= 256 ? 256 : ((D + 31) / 32) * 32;
  pos_grad_kernel<<<S, threads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dy), dP, dp_f32, M, S, D);
  return (int)cudaGetLastError();
}
