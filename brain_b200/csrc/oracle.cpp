// CPU float64 oracle kernels: plain loops in double precision for the ops the GPU kernels implement
// (GEMM, RMSNorm, LayerNorm, softmax, softmax cross-entropy, NeoX RoPE, attention with GQA and
// bottom-right causal masking). They follow the reference framework's definitions, which compute in
// f64 (crates/brain-core/src/tensor/arithmetic.rs:174-411 matmul; crates/brain-transformer/src/ops.rs
// :57-131 layer / RMS norm with biased variance and eps inside the square root, :242-290 masks;
// special.rs:119-125 max-subtracted softmax; neural.rs:40-58 cross-entropy; position/rope.rs:57-142
// NeoX half-split rotation with theta stored as f32; attention/scaled.rs:41-139 SDPA, scale
// 1/sqrt(head_dim)). They are a second, independent statement of each op next to the PyTorch float64
// restatements the tests use, written for clarity rather than speed.
#include <cmath>
#include <cstdint>
#include <vector>

#define BRAIN_API extern "C" __attribute__((visibility("default")))

// C[M, N] = A[M, K] * B[N, K]^T
BRAIN_API int brain_oracle_gemm(const double* A, const double* B, double* C, int64_t M, int64_t N, int64_t K) {
  if (!A || !B || !C || M < 0 || N < 0 || K < 0) return -10;
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      double s = 0.0;
      for (int64_t k = 0; k < K; ++k) s += A[i * K + k] * B[j * K + k];
      C[i * N + j] = s;
    }
  return 0;
}

// y = x * (mean(x^2) + eps)^-1/2 * w, rows of D
BRAIN_API int brain_oracle_rms_norm(const double* x, const double* w, double* y, int64_t M, int64_t D, double eps) {
  if (!x || !w || !y || D <= 0) return -10;
  for (int64_t i = 0; i < M; ++i) {
    double ss = 0.0;
    for (int64_t d = 0; d < D; ++d) ss += x[i * D + d] * x[i * D + d];
    const double r = 1.0 / std::sqrt(ss / (double)D + eps);
    for (int64_t d = 0; d < D; ++d) y[i * D + d] = x[i * D + d] * r * w[d];
  }
  return 0;
}

// y = (x - mean) / sqrt(var + eps) * w + b, biased variance; b may be null
BRAIN_API int brain_oracle_layer_norm(const double* x, const double* w, const double* b, double* y, int64_t M,
                                      int64_t D, double eps) {
  if (!x || !w || !y || D <= 0) return -10;
  for (int64_t i = 0; i < M; ++i) {
    double mean = 0.0;
    for (int64_t d = 0; d < D; ++d) mean += x[i * D + d];
    mean /= (double)D;
    double var = 0.0;
    for (int64_t d = 0; d < D; ++d) var += (x[i * D + d] - mean) * (x[i * D + d] - mean);
    var /= (double)D;
    const double r = 1.0 / std::sqrt(var + eps);
    for (int64_t d = 0; d < D; ++d) y[i * D + d] = (x[i * D + d] - mean) * r * w[d] + (b ? b[d] : 0.0);
  }
  return 0;
}

// row softmax with the row maximum subtracted
BRAIN_API int brain_oracle_softmax(const double* x, double* y, int64_t M, int64_t N) {
  if (!x || !y || N <= 0) return -10;
  for (int64_t i = 0; i < M; ++i) {
    double mx = -INFINITY;
    for (int64_t j = 0; j < N; ++j) mx = std::fmax(mx, x[i * N + j]);
    double s = 0.0;
    for (int64_t j = 0; j < N; ++j) s += std::exp(x[i * N + j] - mx);
    for (int64_t j = 0; j < N; ++j) y[i * N + j] = std::exp(x[i * N + j] - mx) / s;
  }
  return 0;
}

// per-row loss = logsumexp(logits) - logits[label]; rows whose label equals ignore_index get 0
BRAIN_API int brain_oracle_cross_entropy(const double* logits, const int64_t* labels, double* loss, int64_t M,
                                         int64_t V, int64_t ignore_index) {
  if (!logits || !labels || !loss || V <= 0) return -10;
  for (int64_t i = 0; i < M; ++i) {
    if (labels[i] == ignore_index) {
      loss[i] = 0.0;
      continue;
    }
    if (labels[i] < 0 || labels[i] >= V) return -10;
    double mx = -INFINITY;
    for (int64_t j = 0; j < V; ++j) mx = std::fmax(mx, logits[i * V + j]);
    double s = 0.0;
    for (int64_t j = 0; j < V; ++j) s += std::exp(logits[i * V + j] - mx);
    loss[i] = std::log(s) + mx - logits[i * V + labels[i]];
  }
  return 0;
}

// x [S, H, D] rotated in place: pairs (i, i + D/2), angle (pos) * theta^(-2i/D) with pos = s + offset;
// theta is rounded to float first, as the reference stores it
BRAIN_API int brain_oracle_rope(double* x, int64_t S, int64_t H, int64_t D, double theta, int64_t offset) {
  if (!x || D <= 0 || D % 2) return -10;
  const double th = (double)(float)theta;
  const int64_t half = D / 2;
  for (int64_t s = 0; s < S; ++s)
    for (int64_t h = 0; h < H; ++h) {
      double* v = x + (s * H + h) * D;
      for (int64_t i = 0; i < half; ++i) {
        const double ang = (double)(s + offset) * std::pow(th, -2.0 * (double)i / (double)D);
        const double c = std::cos(ang), sn = std::sin(ang);
        const double a = v[i], b = v[i + half];
        v[i] = a * c - b * sn;
        v[i + half] = b * c + a * sn;
      }
    }
  return 0;
}

// o[Sq, Hq, D] = softmax(q k^T / sqrt(D) [+ causal mask]) v, q [Sq, Hq, D], k / v [Sk, Hkv, D];
// q-head h reads kv-head h / (Hq / Hkv); causal: key j visible to query i iff j <= i + Sk - Sq
BRAIN_API int brain_oracle_attention(const double* q, const double* k, const double* v, double* o, int64_t Sq,
                                     int64_t Sk, int64_t Hq, int64_t Hkv, int64_t D, int causal) {
  if (!q || !k || !v || !o || Hkv <= 0 || Hq % Hkv || D <= 0) return -10;
  const int64_t group = Hq / Hkv;
  const double scale = 1.0 / std::sqrt((double)D);
  std::vector<double> p((size_t)Sk);
  for (int64_t h = 0; h < Hq; ++h) {
    const int64_t kh = h / group;
    for (int64_t i = 0; i < Sq; ++i) {
      double mx = -INFINITY;
      for (int64_t j = 0; j < Sk; ++j) {
        if (causal && j > i + Sk - Sq) {
          p[(size_t)j] = -INFINITY;
          continue;
        }
        double s = 0.0;
        for (int64_t d = 0; d < D; ++d) s += q[(i * Hq + h) * D + d] * k[(j * Hkv + kh) * D + d];
        p[(size_t)j] = s * scale;
        mx = std::fmax(mx, p[(size_t)j]);
      }
      double den = 0.0;
      for (int64_t j = 0; j < Sk; ++j) {
        p[(size_t)j] = std::isinf(p[(size_t)j]) ? 0.0 : std::exp(p[(size_t)j] - mx);
        den += p[(size_t)j];
      }
      for (int64_t d = 0; d < D; ++d) {
        double acc = 0.0;
        for (int64_t j = 0; j < Sk; ++j) acc += p[(size_t)j] * v[(j * Hkv + kh) * D + d];
        o[(i * Hq + h) * D + d] = den > 0.0 ? acc / den : 0.0;
      }
    }
  }
  return 0;
}
