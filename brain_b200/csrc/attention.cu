// Flash attention (forward + backward) with native GQA, causal masking and log-sum-exp output.
//
// Layout: q [B, Sq, Hq, D], k/v [B, Sk, Hkv, D] with arbitrary (batch, seq, head) element strides
// and unit stride along D, so the kernels read straight out of a fused QKV projection buffer.
// o [B, Sq, Hq, D] bf16, lse [B, Hq, Sq] f32 (natural log of sum exp(scale * q.k)).
// Causal masking is bottom-right aligned: query i may see key j iff j <= i + (Sk - Sq), which is the
// right rule for prefill against a cache and for decode. (The reference masks top-left with -1e9,
// crates/brain-transformer/src/ops.rs:242-290, which is wrong when Sq < Sk; equal lengths agree.)
// Reference attention: crates/brain-transformer/src/attention/scaled.rs:41-139 (naive SDPA, scale
// 1/sqrt(d)), flash_lite.rs:46-222 (tiled online softmax), multi_query.rs (GQA by repeat_kv; here
// the kv head is indexed directly, no repeat).
//
// Tiles: each warp owns 16 query rows (forward, dQ) or 16 key rows (dK/dV); K/V (or Q/dO) tiles of
// 64 rows stream through a cp.async double buffer in XOR-swizzled shared memory; products use the
// bf16 m16n8k16 tensor-core instruction with f32 accumulation, and the probability tile is re-used
// from registers as the next product's A operand. Backward is split in two deterministic kernels
// (no atomics): one walks query blocks for a key block (dK, dV, summed over the GQA group), the
// other walks key blocks for a query block (dQ).
#include "common.cuh"

using namespace brain;

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnParams {
  const __nv_bfloat16 *q, *k, *v;
  int64_t qb, qs, qh;  // element strides of q (batch, seq, head)
  int64_t kb, ks, kh;
  int64_t vb, vs, vh;
  __nv_bfloat16* o;
  int64_t ob, os, oh;
  float* lse;  // [B, Hq, Sq]
  const __nv_bfloat16* dout;
  int64_t db, ds, dh;
  const float* delta;  // [B, Hq, Sq]
  __nv_bfloat16 *dq, *dk, *dv;
  int64_t dqb, dqs, dqh;
  int64_t dkb, dks, dkh;
  int64_t dvb, dvs, dvh;
  int B, Hq, Hkv, Sq, Sk;
  float scale;  // softmax scale (1/sqrt(D) by default)
  int causal;
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of 16-byte chunk `c` of row `r` in a [rows, D] bf16 tile with XOR swizzle.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  constexpr int C = D / 8;
  constexpr int MASK = C >= 8 ? 7 : C - 1;
  return (uint32_t)((r * C + (c ^ (r & MASK))) * 16);
}

// Cooperative async load of `rows` rows (row stride `ld` elements) into a swizzled tile.
template <int D, int NT>
__device__ __forceinline__ void load_tile(uint32_t s, const __nv_bfloat16* g, int64_t ld, int rows, int valid_rows) {
  constexpr int C = D / 8;
  for (int i = threadIdx.x; i < rows * C; i += NT) {
    const int r = i / C, c = i % C;
    const bool ok = r < valid_rows;
    cp_async16(s + swz<D>(r, c), ok ? (const void*)(g + (int64_t)r * ld + c * 8) : (const void*)g, ok);
  }
}

// A fragment (16 rows x 16 cols) at (row0, col0) of a swizzled tile: ldmatrix x4.
template <int D>
__device__ __forceinline__ void lds_a(uint32_t s, int row0, int col0, uint32_t* a) {
  const int lane = threadIdx.x & 31;
  const int r = row0 + (lane & 15);
  const int c = (col0 >> 3) + (lane >> 4);
  ldsm_x4(s + swz<D>(r, c), a);
}
// Two B fragments (n 16 x k 16) from a tile stored [n][k] (k contiguous): b[0..1] for n 0-7, b[2..3] for n 8-15.
template <int D>
__device__ __forceinline__ void lds_b_nk(uint32_t s, int n0, int k0, uint32_t* b) {
  const int lane = threadIdx.x & 31;
  const int r = n0 + (lane & 7) + ((lane >> 4) << 3);
  const int c = (k0 >> 3) + ((lane >> 3) & 1);
  ldsm_x4(s + swz<D>(r, c), b);
}
// Two B fragments (k 16 x n 16) from a tile stored [k][n] (n contiguous): transpose load.
template <int D>
__device__ __forceinline__ void lds_b_kn(uint32_t s, int k0, int n0, uint32_t* b) {
  const int lane = threadIdx.x & 31;
  const int r = k0 + (lane & 7) + (((lane >> 3) & 1) << 3);
  const int c = (n0 >> 3) + (lane >> 4);
  ldsm_x4_t(s + swz<D>(r, c), b);
}

constexpr int BLK = 64;  // rows of the streamed tile

// =============================================================================================
// Forward
// =============================================================================================
template <int D, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) fa_fwd_kernel(AttnParams p) {
  constexpr int NT = WARPS * 32;
  constexpr int BM = 16 * WARPS;
  constexpr int TILE = BLK * D * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + BM * D * 2;  // 2 stages of K then 2 of V
  const uint32_t sV = sK + 2 * TILE;

  const int nmb = (p.Sq + BM - 1) / BM;
  const int mb = p.causal ? (nmb - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int m0 = mb * BM;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int off = p.Sk - p.Sq;

  const __nv_bfloat16* Q = p.q + (int64_t)b * p.qb + (int64_t)h * p.qh + (int64_t)m0 * p.qs;
  const __nv_bfloat16* K = p.k + (int64_t)b * p.kb + (int64_t)hk * p.kh;
  const __nv_bfloat16* V = p.v + (int64_t)b * p.vb + (int64_t)hk * p.vh;

  int kend = p.Sk;
  if (p.causal) kend = min(p.Sk, m0 + BM + off);
  const int nkb = kend > 0 ? (kend + BLK - 1) / BLK : 0;

  load_tile<D, NT>(sQ, Q, p.qs, BM, min(BM, p.Sq - m0));
  cp_commit();
  if (nkb > 0) {
    load_tile<D, NT>(sK, K, p.ks, BLK, min(BLK, p.Sk));
    load_tile<D, NT>(sV, V, p.vs, BLK, min(BLK, p.Sk));
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) lds_a<D>(sQ, warp * 16, kk * 16, qf[kk]);

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = p.scale * kLog2e;
  const int qrow0 = m0 + warp * 16 + g;

  for (int j = 0; j < nkb; ++j) {
    const int st = j & 1;
    if (j + 1 < nkb) {
      const int n1 = (j + 1) * BLK;
      load_tile<D, NT>(sK + (st ^ 1) * TILE, K + (int64_t)n1 * p.ks, p.ks, BLK, min(BLK, p.Sk - n1));
      load_tile<D, NT>(sV + (st ^ 1) * TILE, V + (int64_t)n1 * p.vs, p.vs, BLK, min(BLK, p.Sk - n1));
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t tk = sK + st * TILE, tv = sV + st * TILE;
    float s[BLK / 8][4];
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < BLK / 16; ++np) {
        uint32_t bfr[4];
        lds_b_nk<D>(tk, np * 16, kk * 16, bfr);
        mma16816(s[2 * np], qf[kk], bfr);
        mma16816(s[2 * np + 1], qf[kk], bfr + 2);
      }
    }
    // scale, mask, online softmax (rows g and g+8 of this warp's 16)
    const int n0 = j * BLK;
    float rmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = n0 + i * 8 + 2 * t + (e & 1);
        const int qi = qrow0 + (e >> 1) * 8;
        float v = s[i][e] * sl2;
        if (key >= p.Sk || (p.causal && key > qi + off)) v = -INFINITY;
        s[i][e] = v;
        rmax[e >> 1] = fmaxf(rmax[e >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rmax[r] = fmaxf(rmax[r], __shfl_xor_sync(0xffffffffu, rmax[r], 1));
      rmax[r] = fmaxf(rmax[r], __shfl_xor_sync(0xffffffffu, rmax[r], 2));
      const float mnew = fmaxf(mrow[r], rmax[r]);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      alpha[r] = exp2f(mrow[r] - muse);
      mrow[r] = mnew;
      rmax[r] = muse;
    }
    float rsum[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = exp2f(s[i][e] - rmax[e >> 1]);
        s[i][e] = pv;
        rsum[e >> 1] += pv;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + rsum[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BLK / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t bfr[4];
        lds_b_kn<D>(tv, kk * 16, np * 16, bfr);
        mma16816(o[2 * np], a, bfr);
        mma16816(o[2 * np + 1], a, bfr + 2);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  __nv_bfloat16* O = p.o + (int64_t)b * p.ob + (int64_t)h * p.oh;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qrow0 + r * 8;
    if (qi >= p.Sq) continue;
    const float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
    __nv_bfloat16* orow = O + (int64_t)qi * p.os;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<uint32_t*>(orow + i * 8 + 2 * t) = pack_bf16(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
    }
    if (t == 0 && p.lse) {
      p.lse[((int64_t)b * p.Hq + h) * p.Sq + qi] = lrow[r] > 0.f ? (mrow[r] + log2f(lrow[r])) * kLn2 : -INFINITY;
    }
  }
}

// =============================================================================================
// Backward preprocess: delta[b, h, i] = sum_d dO[b, i, h, d] * O[b, i, h, d]
// =============================================================================================
template <int D>
__global__ void fa_bwd_delta_kernel(AttnParams p) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;  // one warp per (b, h, i)
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)p.B * p.Hq * p.Sq;
  if (row >= total) return;
  const int i = (int)(row % p.Sq);
  const int bh = (int)(row / p.Sq);
  const int b = bh / p.Hq, h = bh % p.Hq;
  const __nv_bfloat16* dO = p.dout + (int64_t)b * p.db + (int64_t)h * p.dh + (int64_t)i * p.ds;
  const __nv_bfloat16* O = p.o + (int64_t)b * p.ob + (int64_t)h * p.oh + (int64_t)i * p.os;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s += __bfloat162float(dO[d]) * __bfloat162float(O[d]);
  s = warp_sum(s);
  if (lane == 0) const_cast<float*>(p.delta)[row] = s;
}

// =============================================================================================
// Backward dK/dV: CTA owns BK = 16*WARPS keys of one kv head; loops over the GQA group's q heads
// and over query blocks.  S^T = K Q^T, P^T = exp(S^T*scale - lse), dV += P^T dO,
// dP^T = V dO^T, dS^T = P^T (dP^T - delta), dK += dS^T Q * scale.
// =============================================================================================
template <int D, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) fa_bwd_dkdv_kernel(AttnParams p) {
  constexpr int NT = WARPS * 32;
  constexpr int BKEY = 16 * WARPS;
  constexpr int TILE = BLK * D * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BKEY * D * 2;
  const uint32_t sQ = sV + BKEY * D * 2;  // 2 stages
  const uint32_t sO = sQ + 2 * TILE;      // dO, 2 stages
  float* sLse = reinterpret_cast<float*>(smem + 2 * BKEY * D * 2 + 4 * TILE);  // 2 stages x BLK
  float* sDel = sLse + 2 * BLK;

  const int nkb = (p.Sk + BKEY - 1) / BKEY;
  const int kbi = blockIdx.x;
  const int bhk = blockIdx.y;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int n0 = kbi * BKEY;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int off = p.Sk - p.Sq;
  (void)nkb;

  const __nv_bfloat16* K = p.k + (int64_t)b * p.kb + (int64_t)hk * p.kh + (int64_t)n0 * p.ks;
  const __nv_bfloat16* V = p.v + (int64_t)b * p.vb + (int64_t)hk * p.vh + (int64_t)n0 * p.vs;
  load_tile<D, NT>(sK, K, p.ks, BKEY, min(BKEY, p.Sk - n0));
  load_tile<D, NT>(sV, V, p.vs, BKEY, min(BKEY, p.Sk - n0));
  cp_commit();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const float sl2 = p.scale * kLog2e;
  const int key0 = n0 + warp * 16 + g;  // this thread's keys: key0, key0 + 8
  // first query block that can see any key of this CTA (causal): q >= key - off
  const int qstart = p.causal ? max(0, ((n0 - off) / BLK) * BLK) : 0;
  const int nqb = p.Sq > qstart ? (p.Sq - qstart + BLK - 1) / BLK : 0;
  const int total = nqb * group;

  auto issue = [&](int it, int stage) {
    const int hh = hk * group + it / nqb;
    const int q0 = qstart + (it % nqb) * BLK;
    const __nv_bfloat16* Q = p.q + (int64_t)b * p.qb + (int64_t)hh * p.qh + (int64_t)q0 * p.qs;
    const __nv_bfloat16* dO = p.dout + (int64_t)b * p.db + (int64_t)hh * p.dh + (int64_t)q0 * p.ds;
    const int valid = min(BLK, p.Sq - q0);
    load_tile<D, NT>(sQ + stage * TILE, Q, p.qs, BLK, valid);
    load_tile<D, NT>(sO + stage * TILE, dO, p.ds, BLK, valid);
    const float* L = p.lse + ((int64_t)b * p.Hq + hh) * p.Sq + q0;
    const float* Dl = p.delta + ((int64_t)b * p.Hq + hh) * p.Sq + q0;
    for (int i = threadIdx.x; i < BLK; i += NT) {
      sLse[stage * BLK + i] = i < valid ? L[i] * kLog2e : INFINITY;
      sDel[stage * BLK + i] = i < valid ? Dl[i] : 0.f;
    }
  };
  if (total > 0) issue(0, 0);
  cp_commit();

  for (int it = 0; it < total; ++it) {
    const int st = it & 1;
    __syncthreads();  // previous stage fully consumed before it is refilled
    if (it + 1 < total) issue(it + 1, st ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const int q0 = qstart + (it % nqb) * BLK;
    const uint32_t tq = sQ + st * TILE, to = sO + st * TILE;
    const float* lse2 = sLse + st * BLK;
    const float* del = sDel + st * BLK;
    // S^T [16 keys x BLK queries] = K Q^T
    float s[BLK / 8][4];
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      lds_a<D>(sK, warp * 16, kk * 16, a);
#pragma unroll
      for (int np = 0; np < BLK / 16; ++np) {
        uint32_t bfr[4];
        lds_b_nk<D>(tq, np * 16, kk * 16, bfr);
        mma16816(s[2 * np], a, bfr);
        mma16816(s[2 * np + 1], a, bfr + 2);
      }
    }
    // P^T
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = i * 8 + 2 * t + (e & 1);
        const int qi = q0 + qc;
        const int key = key0 + (e >> 1) * 8;
        const float l2 = lse2[qc];
        float pv = exp2f(s[i][e] * sl2 - l2);
        if (qi >= p.Sq || key >= p.Sk || (p.causal && key > qi + off) || l2 == -INFINITY) pv = 0.f;
        s[i][e] = pv;
      }
    }
    // dV += P^T dO
#pragma unroll
    for (int kk = 0; kk < BLK / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t bfr[4];
        lds_b_kn<D>(to, kk * 16, np * 16, bfr);
        mma16816(dv[2 * np], a, bfr);
        mma16816(dv[2 * np + 1], a, bfr + 2);
      }
    }
    // dP^T [16 keys x BLK queries] = V dO^T
    float dp[BLK / 8][4];
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      lds_a<D>(sV, warp * 16, kk * 16, a);
#pragma unroll
      for (int np = 0; np < BLK / 16; ++np) {
        uint32_t bfr[4];
        lds_b_nk<D>(to, np * 16, kk * 16, bfr);
        mma16816(dp[2 * np], a, bfr);
        mma16816(dp[2 * np + 1], a, bfr + 2);
      }
    }
    // dS^T = P^T (dP^T - delta)
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = i * 8 + 2 * t + (e & 1);
        s[i][e] = s[i][e] * (dp[i][e] - del[qc]);
      }
    }
    // dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BLK / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t bfr[4];
        lds_b_kn<D>(tq, kk * 16, np * 16, bfr);
        mma16816(dk[2 * np], a, bfr);
        mma16816(dk[2 * np + 1], a, bfr + 2);
      }
    }
  }
  cp_wait<0>();
  __nv_bfloat16* dK = p.dk + (int64_t)b * p.dkb + (int64_t)hk * p.dkh;
  __nv_bfloat16* dV = p.dv + (int64_t)b * p.dvb + (int64_t)hk * p.dvh;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key0 + r * 8;
    if (key >= p.Sk) continue;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<uint32_t*>(dK + (int64_t)key * p.dks + i * 8 + 2 * t) =
          pack_bf16(dk[i][2 * r] * p.scale, dk[i][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(dV + (int64_t)key * p.dvs + i * 8 + 2 * t) = pack_bf16(dv[i][2 * r], dv[i][2 * r + 1]);
    }
  }
}

// =============================================================================================
// Backward dQ: CTA owns BM = 16*WARPS queries of one q head; loops over key blocks.
// S = Q K^T, P = exp(S*scale - lse), dP = dO V^T, dS = P (dP - delta), dQ += dS K * scale.
// =============================================================================================
template <int D, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) fa_bwd_dq_kernel(AttnParams p) {
  constexpr int NT = WARPS * 32;
  constexpr int BM = 16 * WARPS;
  constexpr int TILE = BLK * D * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sO = sQ + BM * D * 2;
  const uint32_t sK = sO + BM * D * 2;  // 2 stages
  const uint32_t sV = sK + 2 * TILE;    // 2 stages

  const int nmb = (p.Sq + BM - 1) / BM;
  const int mb = p.causal ? (nmb - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int m0 = mb * BM;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int off = p.Sk - p.Sq;

  const __nv_bfloat16* Q = p.q + (int64_t)b * p.qb + (int64_t)h * p.qh + (int64_t)m0 * p.qs;
  const __nv_bfloat16* dO = p.dout + (int64_t)b * p.db + (int64_t)h * p.dh + (int64_t)m0 * p.ds;
  const __nv_bfloat16* K = p.k + (int64_t)b * p.kb + (int64_t)hk * p.kh;
  const __nv_bfloat16* V = p.v + (int64_t)b * p.vb + (int64_t)hk * p.vh;
  int kend = p.Sk;
  if (p.causal) kend = min(p.Sk, m0 + BM + off);
  const int nkb = kend > 0 ? (kend + BLK - 1) / BLK : 0;

  const int valid = min(BM, p.Sq - m0);
  load_tile<D, NT>(sQ, Q, p.qs, BM, valid);
  load_tile<D, NT>(sO, dO, p.ds, BM, valid);
  cp_commit();
  if (nkb > 0) {
    load_tile<D, NT>(sK, K, p.ks, BLK, min(BLK, p.Sk));
    load_tile<D, NT>(sV, V, p.vs, BLK, min(BLK, p.Sk));
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();

  const int qrow0 = m0 + warp * 16 + g;
  float lse2[2], del[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qrow0 + r * 8;
    const bool ok = qi < p.Sq;
    lse2[r] = ok ? p.lse[((int64_t)b * p.Hq + h) * p.Sq + qi] * kLog2e : INFINITY;
    del[r] = ok ? p.delta[((int64_t)b * p.Hq + h) * p.Sq + qi] : 0.f;
  }
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  const float sl2 = p.scale * kLog2e;

  for (int j = 0; j < nkb; ++j) {
    const int st = j & 1;
    if (j + 1 < nkb) {
      const int n1 = (j + 1) * BLK;
      load_tile<D, NT>(sK + (st ^ 1) * TILE, K + (int64_t)n1 * p.ks, p.ks, BLK, min(BLK, p.Sk - n1));
      load_tile<D, NT>(sV + (st ^ 1) * TILE, V + (int64_t)n1 * p.vs, p.vs, BLK, min(BLK, p.Sk - n1));
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t tk = sK + st * TILE, tv = sV + st * TILE;
    float s[BLK / 8][4], dp[BLK / 8][4];
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4], ao[4];
      lds_a<D>(sQ, warp * 16, kk * 16, a);
      lds_a<D>(sO, warp * 16, kk * 16, ao);
#pragma unroll
      for (int np = 0; np < BLK / 16; ++np) {
        uint32_t bk[4], bv[4];
        lds_b_nk<D>(tk, np * 16, kk * 16, bk);
        lds_b_nk<D>(tv, np * 16, kk * 16, bv);
        mma16816(s[2 * np], a, bk);
        mma16816(s[2 * np + 1], a, bk + 2);
        mma16816(dp[2 * np], ao, bv);
        mma16816(dp[2 * np + 1], ao, bv + 2);
      }
    }
    const int n0 = j * BLK;
#pragma unroll
    for (int i = 0; i < BLK / 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = n0 + i * 8 + 2 * t + (e & 1);
        const int r = e >> 1;
        const int qi = qrow0 + r * 8;
        float pv = exp2f(s[i][e] * sl2 - lse2[r]);
        if (qi >= p.Sq || key >= p.Sk || (p.causal && key > qi + off) || lse2[r] == -INFINITY) pv = 0.f;
        s[i][e] = pv * (dp[i][e] - del[r]);
      }
    }
    // dQ += dS K
#pragma unroll
    for (int kk = 0; kk < BLK / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t bfr[4];
        lds_b_kn<D>(tk, kk * 16, np * 16, bfr);
        mma16816(dq[2 * np], a, bfr);
        mma16816(dq[2 * np + 1], a, bfr + 2);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  __nv_bfloat16* dQ = p.dq + (int64_t)b * p.dqb + (int64_t)h * p.dqh;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qrow0 + r * 8;
    if (qi >= p.Sq) continue;
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
      *reinterpret_cast<uint32_t*>(dQ + (int64_t)qi * p.dqs + i * 8 + 2 * t) =
          pack_bf16(dq[i][2 * r] * p.scale, dq[i][2 * r + 1] * p.scale);
  }
}

template <int D>
constexpr int fwd_warps() {
  return 4;
}

template <int D>
int launch_fwd(const AttnParams& p, cudaStream_t st) {
  constexpr int W = fwd_warps<D>();
  constexpr int BM = 16 * W;
  const int smem = BM * D * 2 + 4 * BLK * D * 2;
  auto kern = fa_fwd_kernel<D, W>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((p.Sq + BM - 1) / BM, p.B * p.Hq);
  kern<<<grid, W * 32, smem, st>>>(p);
  return (int)cudaGetLastError();
}

template <int D>
int launch_bwd(const AttnParams& p, cudaStream_t st) {
  {
    const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
    fa_bwd_delta_kernel<D><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(p);
  }
  constexpr int W = 4;
  {
    constexpr int BKEY = 16 * W;
    const int smem = 2 * BKEY * D * 2 + 4 * BLK * D * 2 + 4 * BLK * 4;
    auto kern = fa_bwd_dkdv_kernel<D, W>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid((p.Sk + BKEY - 1) / BKEY, p.B * p.Hkv);
    kern<<<grid, W * 32, smem, st>>>(p);
  }
  {
    constexpr int BM = 16 * W;
    const int smem = 2 * BM * D * 2 + 4 * BLK * D * 2;
    auto kern = fa_bwd_dq_kernel<D, W>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid((p.Sq + BM - 1) / BM, p.B * p.Hq);
    kern<<<grid, W * 32, smem, st>>>(p);
  }
  return (int)cudaGetLastError();
}

}  // namespace

BRAIN_STATUS_READER(attention)

// strides: int64 array of 9 (q b,s,h; k b,s,h; v b,s,h); ostr: 3 (o b,s,h).
BRAIN_API int brain_attn_fwd(const void* q, const void* k, const void* v, const int64_t* qkv_strides, void* o,
                             const int64_t* ostr, float* lse, int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale,
                             int causal, cudaStream_t st) {
  if (Hkv <= 0 || Hq % Hkv) return (int)cudaErrorInvalidValue;
  if (B * Hq == 0 || Sq == 0) return 0;
  AttnParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k = reinterpret_cast<const __nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.qb = qkv_strides[0]; p.qs = qkv_strides[1]; p.qh = qkv_strides[2];
  p.kb = qkv_strides[3]; p.ks = qkv_strides[4]; p.kh = qkv_strides[5];
  p.vb = qkv_strides[6]; p.vs = qkv_strides[7]; p.vh = qkv_strides[8];
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.ob = ostr[0]; p.os = ostr[1]; p.oh = ostr[2];
  p.lse = lse;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Sq = Sq; p.Sk = Sk; p.scale = scale; p.causal = causal;
  switch (D) {
    case 32: return launch_fwd<32>(p, st);
    case 64: return launch_fwd<64>(p, st);
    case 128: return launch_fwd<128>(p, st);
    default: return (int)cudaErrorInvalidValue;
  }
}

// strides: q,k,v (9), o (3), dout (3), dq (3), dk (3), dv (3). delta: f32 workspace [B*Hq*Sq].
BRAIN_API int brain_attn_bwd(const void* q, const void* k, const void* v, const int64_t* qkv_strides, const void* o,
                             const int64_t* ostr, const float* lse, const void* dout, const int64_t* dostr, void* dq,
                             const int64_t* dqstr, void* dk, const int64_t* dkstr, void* dv, const int64_t* dvstr,
                             float* delta, int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale, int causal,
                             cudaStream_t st) {
  if (Hkv <= 0 || Hq % Hkv) return (int)cudaErrorInvalidValue;
  if (B * Hq == 0 || Sq == 0) return 0;
  AttnParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k = reinterpret_cast<const __nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.qb = qkv_strides[0]; p.qs = qkv_strides[1]; p.qh = qkv_strides[2];
  p.kb = qkv_strides[3]; p.ks = qkv_strides[4]; p.kh = qkv_strides[5];
  p.vb = qkv_strides[6]; p.vs = qkv_strides[7]; p.vh = qkv_strides[8];
  p.o = const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(o));
  p.ob = ostr[0]; p.os = ostr[1]; p.oh = ostr[2];
  p.lse = const_cast<float*>(lse);
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout);
  p.db = dostr[0]; p.ds = dostr[1]; p.dh = dostr[2];
  p.dq = reinterpret_cast<__nv_bfloat16*>(dq);
  p.dqb = dqstr[0]; p.dqs = dqstr[1]; p.dqh = dqstr[2];
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dkb = dkstr[0]; p.dks = dkstr[1]; p.dkh = dkstr[2];
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.dvb = dvstr[0]; p.dvs = dvstr[1]; p.dvh = dvstr[2];
  p.delta = delta;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Sq = Sq; p.Sk = Sk; p.scale = scale; p.causal = causal;
  switch (D) {
    case 32: return launch_bwd<32>(p, st);
    case 64: return launch_bwd<64>(p, st);
    case 128: return launch_bwd<128>(p, st);
    default: return (int)cudaErrorInvalidValue;
  }
}
