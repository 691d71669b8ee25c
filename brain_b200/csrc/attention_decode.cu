// Decode attention over a paged KV cache (one new query token per sequence), sm_100a.
//
// Layout: K/V pools [num_blocks, block_size, Hkv, D] bf16; block_table [B, max_blocks] int32 maps
// a sequence's logical block to a pool block; seq_lens [B] int32 counts the cached tokens (the new
// token included). q [B, Hq, D] (row stride qs elements), out [B, Hq, D].
//
// Split-K flash decoding, GQA-packed: a CTA owns one (sequence, kv head) and a contiguous slice of
// the sequence's KV blocks; the G = Hq / Hkv query heads of the group form the M = 16 side of
// mma.sync tiles, so every K/V block is read from HBM once (decode is bound by reading the cache and
// the weights) and S = Q K^T and O += P V run on tensor cores. K/V chunks of 64 keys stream through
// a 3-stage cp.async ring gathered through the block table into XOR-swizzled shared memory. Each split
// writes its running (max, sum, unnormalised output); the last split CTA of a (sequence, kv head)
// (atomic ticket) merges the splits with the log-sum-exp rule. The KV append kernel applies RoPE
// (NeoX half split) to the new token's q and k and writes k / v into their paged slots.
// Reference: the contiguous, realloc-per-append KvCache::update (crates/brain-transformer/src/kv_cache.rs:83-158)
// and SDPA (attention/scaled.rs:41-139); LlamaLite::generate recomputes everything instead.
#include "common.cuh"

using namespace brain;

namespace {

constexpr int kBlock = 64;    // tokens per KV block handled per step (pool block_size must divide by it or equal it)
constexpr int kThreads = 128;
constexpr int kWarpsDec = kThreads / 32;
constexpr int kMaxG = 16;     // query heads per kv head supported (the M = 16 side of the MMA tiles)

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct DecodeArgs {
  const __nv_bfloat16* q;
  int64_t qb, qh;  // strides of q [B, Hq, D]
  const __nv_bfloat16 *kp, *vp;
  const int* table;
  int max_blocks;
  const int* seq_lens;
  int block_size;
  int B, Hq, Hkv, D;
  float scale_log2;
  int splits;
  float* part_o;   // [B, Hkv, splits, G, D]
  float* part_ml;  // [B, Hkv, splits, G, 2]
  int* tickets;    // [B, Hkv] split arrivals, zero between launches
  __nv_bfloat16* out;
  int64_t ob, oh;  // strides of out [B, Hq, D]
};

constexpr int kMaxSplitsDec = 64;

// ---- warp-level tensor-core helpers (mma.sync m16n8k16 bf16 -> f32, ldmatrix from swizzled rows)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of 16-byte unit `c` of row `r` in a [rows][D] bf16 tile whose units are XOR-swizzled
// by (r & 7), so the 8 rows an ldmatrix reads at one column hit 8 different bank groups.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

constexpr int kStages = 3;  // K/V chunks in flight per CTA

template <int D>
struct DecSmem {
  static constexpr int CHUNK = kBlock * D * 2;         // one K or V chunk
  static constexpr int STAGE = 2 * CHUNK;              // K + V
  static constexpr int Q_OFF = kStages * STAGE;        // Q tile [16][D] bf16, swizzled
  static constexpr int TOTAL = Q_OFF + kMaxG * D * 2;  // merge scratch reuses the stages
};

// One CTA = (sequence b, kv head hk, split): the GQA group's G <= 16 query heads form the M = 16 side
// of mma.sync tiles, so the 4 warps compute S = Q K^T and O += P V on tensor cores; warp w owns keys
// [16 w, 16 w + 16) of every 64-key chunk with its own online-softmax state, and the warps merge
// at the end. K/V chunks stream through a 3-stage cp.async ring gathered through the block table.
template <int D>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(DecodeArgs a) {
  using S = DecSmem<D>;
  constexpr int DU = D / 8;  // 16-byte units per row
  pdl_trigger();
  pdl_wait();
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.Hkv, hk = bh % a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int len = a.seq_lens[b];
  const int nchunks = (len + kBlock - 1) / kBlock;
  const int per = (nchunks + a.splits - 1) / a.splits;
  const int c0 = split * per, c1 = min(nchunks, c0 + per);

  extern __shared__ __align__(128) uint8_t dsmem[];
  const uint32_t sbase = smem_u32(dsmem);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

  // Q (rows >= G zero) -> swizzled smem -> A fragments held for the whole kernel
  for (int i = tid; i < kMaxG * DU; i += kThreads) {
    const int g = i / DU, c = i % DU;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (g < G) v = *reinterpret_cast<const uint4*>(a.q + (int64_t)b * a.qb + (int64_t)(hk * G + g) * a.qh + c * 8);
    *reinterpret_cast<uint4*>(dsmem + S::Q_OFF + swz<D>(g, c)) = v;
  }

  auto load_chunk = [&](int c, int stage) {
    const int tok0 = c * kBlock;
    const uint32_t ks = sbase + stage * S::STAGE, vs = ks + S::CHUNK;
    for (int i = tid; i < kBlock * DU; i += kThreads) {
      const int t = i / DU, u = i % DU;
      const int tok = tok0 + t;
      const bool ok = tok < len;
      int64_t off = 0;
      if (ok) {
        const int blk = a.table[(int64_t)b * a.max_blocks + tok / a.block_size];
        off = ((int64_t)blk * a.block_size + tok % a.block_size) * a.Hkv * D + (int64_t)hk * D + u * 8;
      }
      cp_async16(ks + swz<D>(t, u), a.kp + off, ok);
      cp_async16(vs + swz<D>(t, u), a.vp + off, ok);
    }
  };
#pragma unroll
  for (int j = 0; j < kStages - 1; ++j) {
    if (c0 + j < c1) load_chunk(c0 + j, j);
    cp_commit();
  }
  __syncthreads();
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int row = (lane & 7) + ((lane >> 3) & 1) * 8, unit = kk * 2 + (lane >> 4);
    ldsm_x4(sbase + S::Q_OFF + swz<D>(row, unit), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
  }

  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};  // rows lane/4 and lane/4 + 8
  const int kw = warp * 16;                                     // this warp's keys inside a chunk

  for (int c = c0; c < c1; ++c) {
    cp_wait<kStages - 2>();
    __syncthreads();  // chunk c landed; every warp is done with chunk c - 1's stage
    if (c + kStages - 1 < c1) load_chunk(c + kStages - 1, (c - c0 + kStages - 1) % kStages);
    cp_commit();
    const uint32_t ks = sbase + ((c - c0) % kStages) * S::STAGE, vs = ks + S::CHUNK;
    // S[16 x 16] = Q K^T over this warp's 16 keys (two n8 tiles)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t b0, b1, b2, b3;
      const int key = kw + (lane & 7) + (lane >> 4) * 8, unit = kk * 2 + ((lane >> 3) & 1);
      ldsm_x4(ks + swz<D>(key, unit), b0, b1, b2, b3);
      mma_bf16(sc[0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
      mma_bf16(sc[1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
    }
    // online softmax (base 2) for rows r0 = lane/4 and r1 = r0 + 8
    const int kbase = c * kBlock + kw + (lane & 3) * 2;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool valid = kbase + n * 8 + (j & 1) < len;
        sc[n][j] = valid ? sc[n][j] * a.scale_log2 : -INFINITY;
        mx[j >> 1] = fmaxf(mx[j >> 1], sc[n][j]);
      }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(m_r[r], mx[r]);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      alpha[r] = ex2_fast(m_r[r] - muse);
      m_r[r] = mnew;
      mx[r] = muse;
    }
    float ps[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[n][j] = ex2_fast(sc[n][j] - mx[j >> 1]);
        ps[j >> 1] += sc[n][j];
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_r[r] = l_r[r] * alpha[r] + ps[r];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // O[16 x D] += P[16 x 16] V[16 x D]; P's accumulator layout is the A fragment of k16
    const uint32_t pa0 = pack_bf16(sc[0][0], sc[0][1]), pa1 = pack_bf16(sc[0][2], sc[0][3]);
    const uint32_t pa2 = pack_bf16(sc[1][0], sc[1][1]), pa3 = pack_bf16(sc[1][2], sc[1][3]);
#pragma unroll
    for (int n2 = 0; n2 < D / 16; ++n2) {
      uint32_t b0, b1, b2, b3;
      const int key = kw + (lane & 7) + ((lane >> 3) & 1) * 8, unit = n2 * 2 + (lane >> 4);
      ldsm_x4_t(vs + swz<D>(key, unit), b0, b1, b2, b3);
      mma_bf16(o[2 * n2], pa0, pa1, pa2, pa3, b0, b1);
      mma_bf16(o[2 * n2 + 1], pa0, pa1, pa2, pa3, b2, b3);
    }
  }
  cp_wait<0>();
  __syncthreads();  // stages free: reuse them as merge scratch

  // ---- merge the 4 warps: row max over warps, rescale, sum O and l
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  float* sm = reinterpret_cast<float*>(dsmem);                 // [4 warps][16 rows] max
  float* sl = sm + kWarpsDec * kMaxG;                          // [4 warps][16 rows] sum
  float* so = sl + kWarpsDec * kMaxG;                          // [4 warps][16][D] output
  const int r0 = lane >> 2;
  if ((lane & 3) == 0) {
    sm[warp * kMaxG + r0] = m_r[0];
    sm[warp * kMaxG + r0 + 8] = m_r[1];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = r0 + 8 * r;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsDec; ++w) M = fmaxf(M, sm[w * kMaxG + row]);
    const float f = m_r[r] == -INFINITY ? 0.f : ex2_fast(m_r[r] - M);
    l_r[r] *= f;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][2 * r] *= f;
      o[n][2 * r + 1] *= f;
    }
  }
  if ((lane & 3) == 0) {
    sl[warp * kMaxG + r0] = l_r[0];
    sl[warp * kMaxG + r0 + 8] = l_r[1];
  }
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int col = n * 8 + (lane & 3) * 2;
    *reinterpret_cast<float2*>(so + (warp * kMaxG + r0) * D + col) = make_float2(o[n][0], o[n][1]);
    *reinterpret_cast<float2*>(so + (warp * kMaxG + r0 + 8) * D + col) = make_float2(o[n][2], o[n][3]);
  }
  __syncthreads();
  const int64_t base = (((int64_t)b * a.Hkv + hk) * a.splits + split) * G;
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsDec; ++w) v += so[(w * kMaxG + g) * D + d];
    a.part_o[(base + g) * D + d] = v;
  }
  if (tid < G) {
    float M = -INFINITY, L = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsDec; ++w) M = fmaxf(M, sm[w * kMaxG + tid]);
#pragma unroll
    for (int w = 0; w < kWarpsDec; ++w) L += sl[w * kMaxG + tid];
    a.part_ml[(base + tid) * 2] = M;
    a.part_ml[(base + tid) * 2 + 1] = L;
  }

  // ---- the last split CTA of (b, hk) merges all splits: out = sum_s w_s o_s / sum_s w_s l_s with
  // w_s = exp2(m_s - max_s m_s) (atomic ticket; no separate combine launch)
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(a.tickets + bh, 1);
    s_last = old == a.splits - 1;
    if (s_last) a.tickets[bh] = 0;  // ready for the next launch
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* sw = so;                             // [G][kMaxSplitsDec] split weights (merge scratch is free)
  float* sm2 = sw + kMaxG * kMaxSplitsDec;    // [G][kMaxSplitsDec] split maxima, then sums
  float* sl2 = sm2 + kMaxG * kMaxSplitsDec;
  float* sinv = sl2 + kMaxG * kMaxSplitsDec;  // [G] 1 / denominator
  const int64_t base0 = ((int64_t)b * a.Hkv + hk) * a.splits * G;
  // every (head, split) statistic is loaded at once (one L2 round trip), then reduced from smem
  for (int idx = tid; idx < G * a.splits; idx += kThreads) {
    const int sp = idx / G, g = idx % G;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + base0 + idx);
    sm2[g * kMaxSplitsDec + sp] = ml.x;
    sl2[g * kMaxSplitsDec + sp] = ml.y;
  }
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, sm2[tid * kMaxSplitsDec + sp]);
    const float muse = M == -INFINITY ? 0.f : M;
    float den = 0.f;
    for (int sp = 0; sp < a.splits; ++sp) {
      const float m = sm2[tid * kMaxSplitsDec + sp];
      const float w = m == -INFINITY ? 0.f : ex2_fast(m - muse);
      sw[tid * kMaxSplitsDec + sp] = w;
      den += w * sl2[tid * kMaxSplitsDec + sp];
    }
    sinv[tid] = den > 0.f ? 1.f / den : 0.f;
  }
  __syncthreads();
  // outputs: thread -> 4 consecutive dims of one head per pass; the splits' loads are batched 4 deep
  for (int i = tid * 4; i < G * D; i += kThreads * 4) {
    const int g = i / D, d = i % D;
    float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4* src = reinterpret_cast<const float4*>(a.part_o + (base0 + g) * D + d);
    const int64_t stride4 = (int64_t)G * D / 4;  // one split further
    int sp = 0;
    for (; sp + 4 <= a.splits; sp += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcg(src + (sp + u) * stride4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = sw[g * kMaxSplitsDec + sp + u];
        num.x += w * v[u].x;
        num.y += w * v[u].y;
        num.z += w * v[u].z;
        num.w += w * v[u].w;
      }
    }
    for (; sp < a.splits; ++sp) {
      const float4 v = __ldcg(src + sp * stride4);
      const float w = sw[g * kMaxSplitsDec + sp];
      num.x += w * v.x;
      num.y += w * v.y;
      num.z += w * v.z;
      num.w += w * v.w;
    }
    const float inv = sinv[g];
    __nv_bfloat16* o = a.out + (int64_t)b * a.ob + (int64_t)(hk * G + g) * a.oh + d;
    const __nv_bfloat162 lo = __floats2bfloat162_rn(num.x * inv, num.y * inv);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(num.z * inv, num.w * inv);
    reinterpret_cast<__nv_bfloat162*>(o)[0] = lo;
    reinterpret_cast<__nv_bfloat162*>(o)[1] = hi;
  }
}

// New token: rotate q (in place) and k, write k and v into their paged slots.
// qkv [B, (Hq + 2 Hkv) * D] (row stride ld), pos [B] int32 (position of the new token),
// cs f32 [max_pos, D] (cos | sin halves).
__global__ void kv_append_rope_kernel(__nv_bfloat16* qkv, int64_t ld, int B, int Hq, int Hkv, int D, const int* pos,
                                      const float* cs, __nv_bfloat16* kp, __nv_bfloat16* vp, const int* table,
                                      int max_blocks, int block_size) {
  const int half = D / 2;
  const int64_t total = (int64_t)B * (Hq + 2 * Hkv) * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    int64_t t = i / half;
    const int h = (int)(t % (Hq + 2 * Hkv));
    const int b = (int)(t / (Hq + 2 * Hkv));
    const int p = pos[b];
    __nv_bfloat16* row = qkv + (int64_t)b * ld + (int64_t)h * D;
    float x1 = __bfloat162float(row[j]), x2 = __bfloat162float(row[j + half]);
    if (h < Hq + Hkv) {  // q and k heads are rotated
      const float c = cs[(int64_t)p * D + j], s = cs[(int64_t)p * D + half + j];
      const float y1 = x1 * c - x2 * s, y2 = x2 * c + x1 * s;
      x1 = y1;
      x2 = y2;
      if (h < Hq) {
        row[j] = __float2bfloat16_rn(x1);
        row[j + half] = __float2bfloat16_rn(x2);
        continue;
      }
    }
    const int blk = table[(int64_t)b * max_blocks + p / block_size];
    const int hh = h < Hq + Hkv ? h - Hq : h - Hq - Hkv;
    __nv_bfloat16* dst = (h < Hq + Hkv ? kp : vp) + ((int64_t)blk * block_size + p % block_size) * Hkv * D +
                         (int64_t)hh * D;
    dst[j] = __float2bfloat16_rn(x1);
    dst[j + half] = __float2bfloat16_rn(x2);
  }
}

template <int D>
int launch_decode(const DecodeArgs& a, void* out, int64_t ob, int64_t oh, cudaStream_t st) {
  constexpr int dyn = DecSmem<D>::TOTAL;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess) return (int)e;
    // largest shared-memory carveout: two ~100 KB CTAs per SM
    e = cudaFuncSetAttribute(decode_split_kernel<D>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return (int)e;
    attr[dev & 63] = true;
  }
  const bool pdl = brain_host::g_decode_pdl != 0;
  (void)out;
  (void)ob;
  (void)oh;
  return (int)brain_host::launch(decode_split_kernel<D>, dim3(a.splits, a.B * a.Hkv), dim3(kThreads), dyn, st, pdl,
                                 a);
}

}  // namespace

BRAIN_STATUS_READER(attention_decode)

// Number of 4-byte elements of the workspace: split outputs B*Hkv*splits*G*D f32, split (max, sum)
// B*Hkv*splits*G*2 f32, then B*Hkv int32 tickets that must be zero before the first call (every call
// leaves them zero).
BRAIN_API int64_t brain_decode_workspace(int B, int Hq, int Hkv, int D, int splits) {
  return (int64_t)B * Hq * splits * (D + 2) + (int64_t)B * Hkv;
}

// Pick a split count so that B * Hkv * splits fills the GPU (about two CTAs per SM).
BRAIN_API int brain_decode_splits(int B, int Hkv, int max_len) {
  const int ctas = B * Hkv;
  int want = (2 * brain_host::num_sms()) / (ctas > 0 ? ctas : 1);  // one wave at two CTAs per SM
  const int chunks = (max_len + kBlock - 1) / kBlock;
  if (want > chunks) want = chunks;
  if (want > kMaxSplitsDec) want = kMaxSplitsDec;
  return want < 1 ? 1 : want;
}

BRAIN_API int brain_decode_attention(const void* q, int64_t qb, int64_t qh, const void* kpool, const void* vpool,
                                     const int* table, int max_blocks, const int* seq_lens, int block_size, void* out,
                                     int64_t ob, int64_t oh, float* workspace, int B, int Hq, int Hkv, int D,
                                     float scale, int splits, cudaStream_t st) {
  if (Hkv <= 0 || Hq % Hkv || Hq / Hkv > kMaxG) return (int)cudaErrorInvalidValue;
  if (D != 64 && D != 128) return (int)cudaErrorInvalidValue;
  if (B == 0) return 0;
  DecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.qb = qb; a.qh = qh;
  a.kp = reinterpret_cast<const __nv_bfloat16*>(kpool);
  a.vp = reinterpret_cast<const __nv_bfloat16*>(vpool);
  a.table = table; a.max_blocks = max_blocks; a.seq_lens = seq_lens; a.block_size = block_size;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.D = D;
  a.scale_log2 = scale * 1.4426950408889634f;
  if (splits < 1 || splits > kMaxSplitsDec) return (int)cudaErrorInvalidValue;
  a.splits = splits;
  a.part_o = workspace;
  a.part_ml = workspace + (int64_t)B * Hq * splits * D;
  a.tickets = reinterpret_cast<int*>(workspace + (int64_t)B * Hq * splits * (D + 2));
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ob = ob;
  a.oh = oh;
  if (B * Hkv > 65535) return (int)cudaErrorInvalidValue;
  return D == 64 ? launch_decode<64>(a, out, ob, oh, st) : launch_decode<128>(a, out, ob, oh, st);
}

BRAIN_API int brain_kv_append_rope(void* qkv, int64_t ld, int B, int Hq, int Hkv, int D, const int* pos,
                                   const float* cs, void* kpool, void* vpool, const int* table, int max_blocks,
                                   int block_size, cudaStream_t st) {
  const int64_t total = (int64_t)B * (Hq + 2 * Hkv) * (D / 2);
  if (total == 0) return 0;
  int grid = (int)std::min<int64_t>((total + 255) / 256, 4096);
  kv_append_rope_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(qkv), ld, B, Hq, Hkv, D, pos, cs,
                                              reinterpret_cast<__nv_bfloat16*>(kpool),
                                              reinterpret_cast<__nv_bfloat16*>(vpool), table, max_blocks, block_size);
  return (int)cudaGetLastError();
}
