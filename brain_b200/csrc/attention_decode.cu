// Decode attention over a paged KV cache (one new query token per sequence), sm_100a.
//
// Layout: K/V pools [num_blocks, block_size, Hkv, D] bf16; block_table [B, max_blocks] int32 maps
// a sequence's logical block to a pool block; seq_lens [B] int32 counts the cached tokens (the new
// token included). q [B, Hq, D] (row stride qs elements), out [B, Hq, D].
//
// Split-K flash decoding, GQA-packed: a CTA owns one (sequence, kv head) and a contiguous slice of
// the sequence's KV blocks; the G = Hq / Hkv query heads of the group are processed together, so
// every K/V block is read from HBM once (decode is bound by reading the cache and the weights).
// K/V blocks stream through a cp.async double buffer; scores and the P.V product run on CUDA cores
// in f32 (a G x 64 x 128 block is too small for tensor-core tiles to pay); each split writes its
// running (max, sum, unnormalised output) and a combine kernel merges the splits with the
// log-sum-exp rule. The KV append kernel applies RoPE (NeoX half split) to the new token's q and k
// and writes k / v into their paged slots.
// Reference: the contiguous, realloc-per-append KvCache::update (crates/brain-transformer/src/kv_cache.rs:83-158)
// and SDPA (attention/scaled.rs:41-139); LlamaLite::generate recomputes everything instead.
#include "common.cuh"

using namespace brain;

namespace {

constexpr int kBlock = 64;    // tokens per KV block handled per step (pool block_size must divide by it or equal it)
constexpr int kThreads = 128;
constexpr int kMaxG = 16;     // query heads per kv head supported

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
};

template <int D>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(DecodeArgs a) {
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.Hkv, hk = bh % a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int len = a.seq_lens[b];
  const int nchunks = (len + kBlock - 1) / kBlock;
  const int per = (nchunks + a.splits - 1) / a.splits;
  const int c0 = split * per, c1 = min(nchunks, c0 + per);

  extern __shared__ __align__(16) uint8_t dsmem[];  // K and V double buffers (2 x 2 x kBlock x D bf16)
  auto sK = reinterpret_cast<__nv_bfloat16 (*)[kBlock][D]>(dsmem);
  auto sV = reinterpret_cast<__nv_bfloat16 (*)[kBlock][D]>(dsmem + 2 * kBlock * D * 2);
  __shared__ float sQ[kMaxG][D];
  __shared__ float sP[kMaxG][kBlock];
  __shared__ float sRedMax[kMaxG][2], sRedSum[kMaxG][2];
  __shared__ float sM[kMaxG], sL[kMaxG], sAlpha[kMaxG];

  const int tid = threadIdx.x;
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    sQ[g][d] = __bfloat162float(a.q[(int64_t)b * a.qb + (int64_t)(hk * G + g) * a.qh + d]) * a.scale_log2;
  }
  if (tid < G) {
    sM[tid] = -INFINITY;
    sL[tid] = 0.f;
  }
  // output accumulator: thread owns (g = tid / (D/8) ... ) 8 consecutive dims of one head
  constexpr int DV = D / 8;              // 8-dim groups per head
  const int og = tid / DV, od = (tid % DV) * 8;
  const int outs_per_pass = kThreads / DV;  // heads covered per pass
  float acc[2][8];
#pragma unroll
  for (int p = 0; p < 2; ++p)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[p][j] = 0.f;

  auto load_chunk = [&](int c, int buf) {
    const int tok0 = c * kBlock;
    for (int i = tid; i < kBlock * (D / 8); i += kThreads) {
      const int t = i / (D / 8), dv = (i % (D / 8)) * 8;
      const int tok = tok0 + t;
      const bool ok = tok < len;
      int64_t off = 0;
      if (ok) {
        const int blk = a.table[(int64_t)b * a.max_blocks + tok / a.block_size];
        off = ((int64_t)blk * a.block_size + tok % a.block_size) * a.Hkv * D + (int64_t)hk * D + dv;
      }
      cp_async16(smem_u32(&sK[buf][t][dv]), a.kp + off, ok);
      cp_async16(smem_u32(&sV[buf][t][dv]), a.vp + off, ok);
    }
  };
  __syncthreads();
  if (c0 < c1) load_chunk(c0, 0);
  cp_commit();
  for (int c = c0; c < c1; ++c) {
    const int buf = (c - c0) & 1;
    if (c + 1 < c1) load_chunk(c + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    // scores: thread -> key (tid % 64), heads (tid / 64) * ... covering G heads in two halves
    {
      const int key = tid % kBlock;
      const int gstart = tid / kBlock;  // 0 or 1
      const bool kvalid = c * kBlock + key < len;
      for (int g = gstart; g < G; g += kThreads / kBlock) {
        float s = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; d += 8) {
          float kf[8];
          load8(&sK[buf][key][d], kf);
#pragma unroll
          for (int j = 0; j < 8; ++j) s += sQ[g][d + j] * kf[j];
        }
        sP[g][key] = kvalid ? s : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax per head (one warp per head, looping)
    {
      const int warp = tid / 32, lane = tid % 32;
      for (int g = warp; g < G; g += kThreads / 32) {
        float m = fmaxf(sP[g][lane], sP[g][lane + 32]);
        m = warp_max(m);
        const float mold = sM[g];
        const float mnew = fmaxf(mold, m);
        const float muse = mnew == -INFINITY ? 0.f : mnew;
        const float p0 = ex2_fast(sP[g][lane] - muse), p1 = ex2_fast(sP[g][lane + 32] - muse);
        sP[g][lane] = p0;
        sP[g][lane + 32] = p1;
        const float s = warp_sum(p0 + p1);
        if (lane == 0) {
          const float al = ex2_fast(mold - muse);
          sAlpha[g] = al;
          sL[g] = sL[g] * al + s;
          sM[g] = mnew;
        }
      }
    }
    __syncthreads();
    // O = alpha O + P V
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int g = og + p * outs_per_pass;
      if (g < G) {
        const float al = sAlpha[g];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[p][j] *= al;
        for (int t = 0; t < kBlock; ++t) {
          const float pv = sP[g][t];
          float vf[8];
          load8(&sV[buf][t][od], vf);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[p][j] += pv * vf[j];
        }
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  // write the split's partial state
  const int64_t base = (((int64_t)b * a.Hkv + hk) * a.splits + split) * G;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int g = og + p * outs_per_pass;
    if (g < G) {
      float* o = a.part_o + (base + g) * D + od;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = acc[p][j];
    }
  }
  if (tid < G) {
    a.part_ml[(base + tid) * 2] = sM[tid];
    a.part_ml[(base + tid) * 2 + 1] = sL[tid];
  }
}

// out[b, h, :] = sum_s w_s o_s / sum_s w_s l_s with w_s = exp2(m_s - max_s m_s)   (one warp per (b, h))
template <int D>
__global__ void decode_combine_kernel(DecodeArgs a, __nv_bfloat16* out, int64_t ob, int64_t oh) {
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (wid >= (int64_t)a.B * a.Hq) return;
  const int b = (int)(wid / a.Hq), h = (int)(wid % a.Hq);
  const int G = a.Hq / a.Hkv;
  const int hk = h / G, g = h % G;
  float mmax = -INFINITY;
  for (int s = 0; s < a.splits; ++s)
    mmax = fmaxf(mmax, a.part_ml[((((int64_t)b * a.Hkv + hk) * a.splits + s) * G + g) * 2]);
  const float muse = mmax == -INFINITY ? 0.f : mmax;
  float num[D / 32];
#pragma unroll
  for (int j = 0; j < D / 32; ++j) num[j] = 0.f;
  float den = 0.f;
  for (int s = 0; s < a.splits; ++s) {
    const int64_t idx = (((int64_t)b * a.Hkv + hk) * a.splits + s) * G + g;
    const float m = a.part_ml[idx * 2], l = a.part_ml[idx * 2 + 1];
    const float w = m == -INFINITY ? 0.f : ex2_fast(m - muse);
    den += w * l;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) num[j] += w * a.part_o[idx * D + lane + 32 * j];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
  for (int j = 0; j < D / 32; ++j)
    out[(int64_t)b * ob + (int64_t)h * oh + lane + 32 * j] = __float2bfloat16_rn(num[j] * inv);
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

}  // namespace

BRAIN_STATUS_READER(attention_decode)

// Number of f32 elements of the split workspace: o part B*Hkv*splits*G*D, ml part B*Hkv*splits*G*2.
BRAIN_API int64_t brain_decode_workspace(int B, int Hq, int Hkv, int D, int splits) {
  return (int64_t)B * Hq * splits * (D + 2);
}

// Pick a split count so that B * Hkv * splits fills the GPU (about two CTAs per SM).
BRAIN_API int brain_decode_splits(int B, int Hkv, int max_len) {
  const int ctas = B * Hkv;
  int want = (2 * brain_host::num_sms() + ctas - 1) / (ctas > 0 ? ctas : 1);
  const int chunks = (max_len + kBlock - 1) / kBlock;
  if (want > chunks) want = chunks;
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
  a.splits = splits;
  a.part_o = workspace;
  a.part_ml = workspace + (int64_t)B * Hq * splits * D;
  dim3 grid(splits, B * Hkv);
  const int64_t warps = (int64_t)B * Hq;
  const int dyn = 4 * kBlock * D * 2;
  if (D == 64) {
    decode_split_kernel<64><<<grid, kThreads, dyn, st>>>(a);
    decode_combine_kernel<64><<<(unsigned)((warps + 3) / 4), 128, 0, st>>>(a, reinterpret_cast<__nv_bfloat16*>(out), ob, oh);
  } else {
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
      cudaFuncSetAttribute(decode_split_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
      attr[dev & 63] = true;
    }
    decode_split_kernel<128><<<grid, kThreads, dyn, st>>>(a);
    decode_combine_kernel<128><<<(unsigned)((warps + 3) / 4), 128, 0, st>>>(a, reinterpret_cast<__nv_bfloat16*>(out), ob, oh);
  }
  return (int)cudaGetLastError();
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
