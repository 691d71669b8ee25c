// Decode attention over a paged KV cache (one new query token per sequence), sm_100a.
//
// Layout: K/V pools [num_blocks, block_size, Hkv, D] bf16; block_table [B, max_blocks] int32 maps
// a sequence's logical block to a pool block; seq_lens [B] int32 counts the cached tokens (the new
// token included). q [B, Hq, D] (row stride qs elements), out [B, Hq, D].
//
// Split-K flash decoding, GQA-packed: a CTA owns one (sequence, kv head) and a contiguous range of
// the sequence's tokens (16-token granules, so the splits are balanced); the G = Hq / Hkv query heads
// of the group form the M = 16 side of mma.sync tiles, so every K/V row is read from HBM once (decode
// is bound by reading the cache and the weights) and S = Q K^T and O += P V run on tensor cores.
// K/V chunks of 64 keys stream through a 3-stage ring of TMA loads (one 16-key x 64-column box per
// block-table lookup, 128-byte swizzle) completing on mbarriers. The splits of one (sequence, kv
// head) are one thread-block cluster: after the main loop every CTA pushes its running (max, sum,
// unnormalised output) into the shared memory of the CTA that owns each output slice, and after one
// cluster barrier each CTA merges its slice with the log-sum-exp rule (no global workspace, no
// atomics, no second launch). Under programmatic dependent launch the chunks that hold only tokens
// older than the newest one are requested before the kernel waits on its predecessor. The KV append
// kernel applies RoPE (NeoX half split) to the new token's q and k and writes k / v into their paged
// slots.
// Reference: the contiguous, realloc-per-append KvCache::update (crates/brain-transformer/src/kv_cache.rs:83-158)
// and SDPA (attention/scaled.rs:41-139); LlamaLite::generate recomputes everything instead.
#include "common.cuh"

using namespace brain;

namespace {

constexpr int kBlock = 64;    // keys per chunk
constexpr int kRowsBox = 16;  // keys per TMA box and granule of the split ranges (block_size must be a multiple)
constexpr int kThreads = 128;
constexpr int kWarpsDec = kThreads / 32;
constexpr int kMaxG = 16;     // query heads per kv head supported (the M = 16 side of the MMA tiles)

struct DecodeArgs {
  const __nv_bfloat16* q;
  int64_t qb, qh;  // strides of q [B, Hq, D]
  const int* table;
  int max_blocks;
  const int* seq_lens;
  int block_size;
  int B, Hq, Hkv, D;
  float scale_log2;
  int splits;      // CTAs per cluster, one cluster per (sequence, kv head)
  __nv_bfloat16* out;
  int64_t ob, oh;  // strides of out [B, Hq, D]
  unsigned long long* trace;  // optional [grid][8] per-CTA phase timestamps (globaltimer ns), else null
  int pdl_late;               // let dependents launch after the main loop instead of at the start
  const void* pf;             // optional L2 prefetch after the main loop (the next kernel's weights)
  int64_t pf_bytes;
};

constexpr int kMaxSplitsDec = 16;  // cluster size limit (non-portable above 8)

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
  static constexpr int HALF = kBlock * 128;            // 64 keys x 64 columns, rows of 128 B
  static constexpr int CHUNK = (D / 64) * HALF;        // one K or V chunk
  static constexpr int STAGE = 2 * CHUNK;              // K + V
  static constexpr int Q_OFF = kStages * STAGE;        // Q tile [16][D] bf16, swizzled
  static constexpr int BAR_OFF = Q_OFF + kMaxG * D * 2;
  static constexpr int TOTAL = BAR_OFF + kStages * 8 + 1024;  // + slack to align the base to 1 KB
  // after the main loop the stages hold the merge data
  static constexpr int WM_OFF = 0;                                    // [4 warps][16] row max
  static constexpr int WL_OFF = WM_OFF + kWarpsDec * kMaxG * 4;       // [4 warps][16] row sum
  static constexpr int WO_LD = D + 8;                                 // row stride: 8 rows of a warp's store hit 2 wavefronts
  static constexpr int WO_OFF = WL_OFF + kWarpsDec * kMaxG * 4;       // [4 warps][16][WO_LD] output
  static constexpr int RML_OFF = WO_OFF + kWarpsDec * kMaxG * WO_LD * 4;  // [split][16] (max, sum) received
  static constexpr int RO_OFF = RML_OFF + kMaxSplitsDec * kMaxG * 8;  // [split][slot][128] outputs received
  static constexpr int RO_FLOATS = kMaxG * D + kMaxSplitsDec * kThreads;
  static_assert(RO_OFF + RO_FLOATS * 4 <= Q_OFF, "merge data must fit in the stages");
};

// Byte offset of 16-byte unit `c` of key row `r` in a K/V chunk: column halves of 64 (128 B rows),
// unit index XOR (r & 7) inside each half, i.e. the TMA 128-byte swizzle of a 1 KB-aligned tile.
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
  return (uint32_t)((c >> 3) * (kBlock * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void dec_trace(const DecodeArgs& a, int slot) {
  if (a.trace != nullptr && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.trace[((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * 8 + slot] = t;
  }
}

__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_dsmem_f2(uint32_t addr, float x, float y) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(x), "f"(y) : "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// One CTA = (sequence b, kv head hk, split); the splits of (b, hk) are one cluster (cluster rank =
// split). The GQA group's G <= 16 query heads form the M = 16 side of mma.sync tiles, so the 4 warps
// compute S = Q K^T and O += P V on tensor cores; warp w owns keys [16 w, 16 w + 16) of every 64-key
// chunk with its own online-softmax state, and the warps merge at the end.
template <int D>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(const __grid_constant__ CUtensorMap tk,
                                                                const __grid_constant__ CUtensorMap tv,
                                                                DecodeArgs a) {
  using S = DecSmem<D>;
  constexpr int DU = D / 8;  // 16-byte units per row
  constexpr int NH = D / 64;  // 64-column halves
  if (!a.pdl_late) pdl_trigger();
  dec_trace(a, 0);
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.Hkv, hk = bh % a.Hkv;
  const int G = a.Hq / a.Hkv;

  extern __shared__ uint8_t dsmem_raw[];
  __shared__ int s_len;
  const uint32_t raw = smem_u32(dsmem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;  // the 128-byte swizzle repeats every 1 KB
  uint8_t* dsmem = dsmem_raw + (sbase - raw);
  const uint32_t bars = sbase + S::BAR_OFF;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

  // this split's tokens [t0, t1) of a sequence of `len` tokens, in 16-token granules
  auto range = [&](int len, int& t0, int& t1) {
    const int units = (len + kRowsBox - 1) / kRowsBox;
    t0 = min(len, (int)((int64_t)split * units / a.splits) * kRowsBox);
    t1 = min(len, (int)((int64_t)(split + 1) * units / a.splits) * kRowsBox);
  };
  // (warp 0) chunk c of the range into stage st: lane i < 4 loads key group i (16 keys, one block-table
  // lookup) of K and V, one box per 64-column half; groups past t1 are not loaded
  auto issue = [&](int t0, int t1, int c, int st) {
    const int c_start = t0 + c * kBlock;
    const int groups = min(kBlock / kRowsBox, (t1 - c_start + kRowsBox - 1) / kRowsBox);
    const uint32_t bar = bars + st * 8;
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(groups * 2 * NH * kRowsBox * 128));
    __syncwarp();
    if (lane < groups) {
      const int tok = c_start + lane * kRowsBox;
      const int blk = a.table[(int64_t)b * a.max_blocks + tok / a.block_size];
      const int y = blk * a.block_size + tok % a.block_size;
      const uint32_t ks = sbase + st * S::STAGE, vs = ks + S::CHUNK;
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const int x = hk * D + h * 64;
        tma_load_2d(&tk, ks + h * S::HALF + lane * kRowsBox * 128, bar, x, y);
        tma_load_2d(&tv, vs + h * S::HALF + lane * kRowsBox * 128, bar, x, y);
      }
    }
  };

  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) mbar_init(bars + st * 8, 1);
    fence_barrier_init();
    s_len = ld_relaxed_gpu(a.seq_lens + b);
  }
  __syncthreads();
  // Tokens older than the newest one are final while the predecessor may still run (it writes at most
  // the newest token's K/V and the lengths), so the first full chunks of the range are requested before
  // the wait, sized from a length read that may be one step stale: only chunks that end at or below
  // guess - 1 are taken, and the choice is checked against the real length after the wait.
  const int len_guess = s_len;
  int g0, g1;
  range(len_guess, g0, g1);
  int pre = 0;
  for (; pre < kStages - 1; ++pre) {
    const int end = g0 + (pre + 1) * kBlock;
    if (end > g1 || end > len_guess - 1) break;
    if (warp == 0) issue(g0, g1, pre, pre);
  }
  dec_trace(a, 1);
  pdl_wait();
  dec_trace(a, 2);
  const int len = a.seq_lens[b];
  int t0, t1;
  range(len, t0, t1);
  const int nch = (t1 - t0 + kBlock - 1) / kBlock;
  uint32_t par = 0;  // bit st: parity of the next phase of stage st's barrier
  if (pre > 0 && !(g0 == t0 && t0 + pre * kBlock <= t1 && t0 + pre * kBlock <= len - 1)) {
    // the guess was wrong: let what it fetched land, then load the range from its start
    for (int st = 0; st < pre; ++st) mbar_wait(bars + st * 8, 0, BRAIN_ERR_TIMEOUT_FULL, 241, nullptr);
    par = (1u << pre) - 1u;
    pre = 0;
  }
  for (int j = pre; j < kStages - 1 && j < nch; ++j)
    if (warp == 0) issue(t0, t1, j, j);

  // Q (rows >= G zero) -> swizzled smem -> A fragments held for the whole kernel
  for (int i = tid; i < kMaxG * DU; i += kThreads) {
    const int g = i / DU, c = i % DU;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (g < G) v = *reinterpret_cast<const uint4*>(a.q + (int64_t)b * a.qb + (int64_t)(hk * G + g) * a.qh + c * 8);
    *reinterpret_cast<uint4*>(dsmem + S::Q_OFF + swz<D>(g, c)) = v;
  }
  __syncthreads();
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int row = (lane & 7) + ((lane >> 3) & 1) * 8, unit = kk * 2 + (lane >> 4);
    ldsm_x4(sbase + S::Q_OFF + swz<D>(row, unit), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
  }
  dec_trace(a, 3);

  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};  // rows lane/4 and lane/4 + 8
  const int kw = warp * 16;                                     // this warp's keys inside a chunk

  for (int c = 0; c < nch; ++c) {
    const int st = c % kStages;
    mbar_wait(bars + st * 8, (par >> st) & 1u, BRAIN_ERR_TIMEOUT_FULL, 240, nullptr);
    par ^= 1u << st;
    const uint32_t ks = sbase + st * S::STAGE, vs = ks + S::CHUNK;
    const int c_start = t0 + c * kBlock;
    if (c_start + kBlock > t1) {
      // V rows past the range may be unloaded or hold anything (0 * NaN would poison O): zero them
      const int r0v = t1 - c_start;
      for (int i = tid; i < (kBlock - r0v) * DU; i += kThreads) {
        const int r = r0v + i / DU, u = i % DU;
        asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(vs + kv_off(r, u)), "r"(0) : "memory");
      }
    }
    __syncthreads();  // chunk c visible to every warp; every warp is done with chunk c - 1's stage
    if (c == 0) dec_trace(a, 4);
    if (warp == 0 && c + kStages - 1 < nch) issue(t0, t1, c + kStages - 1, (c + kStages - 1) % kStages);
    // S[16 x 16] = Q K^T over this warp's 16 keys (two n8 tiles)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t b0, b1, b2, b3;
      const int key = kw + (lane & 7) + (lane >> 4) * 8, unit = kk * 2 + ((lane >> 3) & 1);
      ldsm_x4(ks + kv_off(key, unit), b0, b1, b2, b3);
      mma_bf16(sc[0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
      mma_bf16(sc[1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
    }
    // online softmax (base 2) for rows r0 = lane/4 and r1 = r0 + 8
    const int kbase = c_start + kw + (lane & 3) * 2;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool valid = kbase + n * 8 + (j & 1) < t1;
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
      ldsm_x4_t(vs + kv_off(key, unit), b0, b1, b2, b3);
      mma_bf16(o[2 * n2], pa0, pa1, pa2, pa3, b0, b1);
      mma_bf16(o[2 * n2 + 1], pa0, pa1, pa2, pa3, b2, b3);
    }
  }
  __syncthreads();  // every warp is done with the stages
  if (a.pdl_late) pdl_trigger();
  // this CTA's K/V stream is done: fill L2 with its share of the next kernel's weights meanwhile
  if (tid == 0) l2_prefetch_part(a.pf, a.pf_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
  // peers may push into this CTA's stages once every CTA of the cluster has passed this point
  if (a.splits > 1) cluster_arrive_release();
  dec_trace(a, 5);

  // ---- merge the 4 warps into this split's (max, sum, output): row max over warps, rescale, sum
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  float* sm = reinterpret_cast<float*>(dsmem + S::WM_OFF);
  float* sl = reinterpret_cast<float*>(dsmem + S::WL_OFF);
  float* so = reinterpret_cast<float*>(dsmem + S::WO_OFF);
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
  constexpr int LD = S::WO_LD;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int col = n * 8 + (lane & 3) * 2;
    *reinterpret_cast<float2*>(so + (warp * kMaxG + r0) * LD + col) = make_float2(o[n][0], o[n][1]);
  }
  if (G > 8) {  // rows 8..15 are padding for groups of up to 8 heads
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      const int col = n * 8 + (lane & 3) * 2;
      *reinterpret_cast<float2*>(so + (warp * kMaxG + r0 + 8) * LD + col) = make_float2(o[n][2], o[n][3]);
    }
  }
  __syncthreads();
  // this split's output elements i = tid + 128 j (j < G*D/128), and the (max, sum) of head tid < G
  constexpr int kMaxPer = kMaxG * D / kThreads;
  const int per = (G * D + kThreads - 1) / kThreads;
  float v[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    v[j] = 0.f;
    const int i = tid + j * kThreads;
    if (j < per && i < G * D) {
      const int g = i / D, d = i % D;
#pragma unroll
      for (int w = 0; w < kWarpsDec; ++w) v[j] += so[(w * kMaxG + g) * LD + d];
    }
  }
  float Mh = -INFINITY, Lh = 0.f;
  if (tid < G) {
#pragma unroll
    for (int w = 0; w < kWarpsDec; ++w) Mh = fmaxf(Mh, sm[w * kMaxG + tid]);
#pragma unroll
    for (int w = 0; w < kWarpsDec; ++w) Lh += sl[w * kMaxG + tid];
  }

  // ---- push to the owners: element i belongs to CTA (i / 128) % splits, slot (i / 128) / splits
  const int E = (per + a.splits - 1) / a.splits;  // slots per CTA
  if (a.splits > 1) cluster_wait_acquire();       // every CTA's stages are free
  else __syncthreads();
  const uint32_t rml = sbase + S::RML_OFF, ro = sbase + S::RO_OFF;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    if (j < per) {
      const int owner = j % a.splits, slot = j / a.splits;
      st_dsmem_f32(mapa_shared(ro + (uint32_t)(((split * E + slot) * kThreads + tid) * 4), (uint32_t)owner), v[j]);
    }
  }
  if (tid < G)
    for (int p = 0; p < a.splits; ++p)
      st_dsmem_f2(mapa_shared(rml + (uint32_t)((split * kMaxG + tid) * 8), (uint32_t)p), Mh, Lh);
  if (a.splits > 1) {
    cluster_arrive_release();  // the pushes are visible to their owners after the wait
    cluster_wait_acquire();
  } else {
    __syncthreads();
  }
  dec_trace(a, 6);

  // ---- merge the owned slice: out = sum_s w_s o_s / sum_s w_s l_s with w_s = exp2(m_s - max_s m_s)
  const float* rmlp = reinterpret_cast<const float*>(dsmem + S::RML_OFF);
  const float* rop = reinterpret_cast<const float*>(dsmem + S::RO_OFF);
  for (int slot = 0; slot < E; ++slot) {
    const int j = slot * a.splits + split;  // this thread's element i = tid + 128 j
    if (j >= per) break;
    const int i = tid + j * kThreads, g = i / D, d = i % D;
    if (i >= G * D) break;
    float M = -INFINITY;
    for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, rmlp[(sp * kMaxG + g) * 2]);
    const float muse = M == -INFINITY ? 0.f : M;
    float num = 0.f, den = 0.f;
    for (int sp = 0; sp < a.splits; ++sp) {
      const float m = rmlp[(sp * kMaxG + g) * 2];
      const float w = m == -INFINITY ? 0.f : ex2_fast(m - muse);
      num += w * rop[(sp * E + slot) * kThreads + tid];
      den += w * rmlp[(sp * kMaxG + g) * 2 + 1];
    }
    a.out[(int64_t)b * a.ob + (int64_t)(hk * G + g) * a.oh + d] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
  }
  dec_trace(a, 7);
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
cudaError_t decode_attrs() {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr[dev & 63]) return cudaSuccess;
  auto kern = decode_split_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DecSmem<D>::TOTAL);
  if (e != cudaSuccess) return e;
  // largest shared-memory carveout: two ~100 KB CTAs per SM; clusters of up to 16 splits
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  attr[dev & 63] = true;
  return cudaSuccess;
}

template <int D>
cudaLaunchConfig_t decode_config(int splits, int pairs, cudaLaunchAttribute* at, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = DecSmem<D>::TOTAL;
  cfg.stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = splits;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return cfg;
}

// How many clusters of `splits` CTAs can be resident at once (0 when none fits).
template <int D>
int decode_active_clusters(int splits) {
  if (decode_attrs<D>() != cudaSuccess) return 0;
  cudaLaunchAttribute at[2];
  cudaLaunchConfig_t cfg = decode_config<D>(splits, 1, at, 0, false);
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, decode_split_kernel<D>, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return n;
}

// K or V pool [num_blocks * block_size rows, Hkv * D columns] bf16 as 16-row x 64-column boxes with the
// 128-byte swizzle.
bool encode_pool(CUtensorMap* m, const void* pool, int64_t rows, int cols) {
  uint64_t dims[2] = {(uint64_t)cols, (uint64_t)rows};
  uint64_t strides[1] = {(uint64_t)cols * 2};
  uint32_t box[2] = {64, (uint32_t)kRowsBox};
  return brain_host::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(pool), dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D>
int launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeArgs& a, cudaStream_t st) {
  cudaError_t e = decode_attrs<D>();
  if (e != cudaSuccess) return (int)e;
  cudaLaunchAttribute at[2];
  cudaLaunchConfig_t cfg = decode_config<D>(a.splits, a.B * a.Hkv, at, st, brain_host::g_decode_pdl != 0);
  return (int)cudaLaunchKernelEx(&cfg, decode_split_kernel<D>, tk, tv, a);
}

}  // namespace

BRAIN_STATUS_READER(attention_decode)

// Split count (= cluster size) for B sequences x Hkv kv heads of up to max_len tokens with head dim D:
// the largest count whose B * Hkv clusters are resident in one wave at about two CTAs per SM.
BRAIN_API int brain_decode_splits(int B, int Hkv, int D, int max_len) {
  const int pairs = B * Hkv > 0 ? B * Hkv : 1;
  const int chunks = (max_len + kBlock - 1) / kBlock;
  int c = std::min(kMaxSplitsDec, std::max(chunks, 1));
  for (; c > 1; --c) {
    if (c * pairs > 2 * brain_host::num_sms()) continue;
    if (c <= 8) break;  // portable cluster size
    const int fit = D == 64 ? decode_active_clusters<64>(c) : decode_active_clusters<128>(c);
    if (fit >= pairs) break;
  }
  return c;
}

// K/V pools are contiguous [num_blocks, block_size, Hkv, D] bf16 with block_size a multiple of 16.
BRAIN_API int brain_decode_attention(const void* q, int64_t qb, int64_t qh, const void* kpool, const void* vpool,
                                     int num_blocks, const int* table, int max_blocks, const int* seq_lens,
                                     int block_size, void* out, int64_t ob, int64_t oh, int B, int Hq, int Hkv, int D,
                                     float scale, int splits, unsigned long long* trace, const void* l2_prefetch,
                                     int64_t l2_prefetch_bytes, cudaStream_t st) {
  if (Hkv <= 0 || Hq % Hkv || Hq / Hkv > kMaxG) return (int)cudaErrorInvalidValue;
  if (D != 64 && D != 128) return (int)cudaErrorInvalidValue;
  if (block_size <= 0 || block_size % kRowsBox) return (int)cudaErrorInvalidValue;
  if (B == 0) return 0;
  if (splits < 1 || splits > kMaxSplitsDec) return (int)cudaErrorInvalidValue;
  if (B * Hkv > 65535) return (int)cudaErrorInvalidValue;
  CUtensorMap tk, tv;
  const int64_t rows = (int64_t)num_blocks * block_size;
  if (!encode_pool(&tk, kpool, rows, Hkv * D) || !encode_pool(&tv, vpool, rows, Hkv * D))
    return (int)cudaErrorInvalidValue;
  DecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.qb = qb; a.qh = qh;
  a.table = table; a.max_blocks = max_blocks; a.seq_lens = seq_lens; a.block_size = block_size;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.D = D;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.splits = splits;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ob = ob;
  a.oh = oh;
  a.trace = trace;
  a.pdl_late = brain_host::g_decode_pdl == 2;
  a.pf = (reinterpret_cast<uintptr_t>(l2_prefetch) & 15) ? nullptr : l2_prefetch;
  a.pf_bytes = l2_prefetch_bytes;
  return D == 64 ? launch_decode<64>(tk, tv, a, st) : launch_decode<128>(tk, tv, a, st);
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
