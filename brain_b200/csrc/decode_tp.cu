// Tensor-parallel decode kernels (one new token per sequence, M <= 64 tokens per step), sm_100a.
//
// 1. skinny_gemm: out[M, N] = x[M, K] * W[N, K]^T with the operands swapped on the tensor core: the
//    weight supplies the 128-row MMA M side and the tokens the N side (NT = 16 / 32 / 64), so a
//    128 x NT f32 accumulator lives in TMEM while the weight streams through a TMA ring at HBM rate
//    (decode is bound by reading the weights once per step). K is split over `splits` CTAs per
//    128-row tile so every SM streams; the partial tiles meet in an f32 workspace and the last CTA of
//    a tile (atomic ticket) sums them in split order (deterministic) and runs one of the epilogues:
//      EPI_STORE   bf16 out (+ residual)
//      EPI_PUSH    all-reduce push: the bf16 partial product goes to slot `rank` of every rank's
//                  receive buffer over NVLink; the last tile to finish publishes the step's epoch in
//                  every rank's flag word (release, system scope)
//      EPI_SWIGLU  weight rows interleaved in 64-row groups [gate 64 | up 64]; writes silu(gate) * up
//      EPI_QKV     one tile = one head of the fused [q | k | v] projection (head_dim 128): RoPE on
//                  q / k at each token's position, q to `out`, k / v straight into their paged slots
//      EPI_ARGMAX  greedy LM head: the per-token max over the tile's vocabulary rows folds into a
//                  64-bit (value, -index) key with atomicMax; the last tile pushes the keys to every
//                  rank and publishes the epoch
// 2. ar_norm: waits for the epoch flags of all ranks, sums the `world` bf16 slots of a token row in
//    f32, adds the residual stream (updated in place) and writes RMSNorm(h) * gamma for the next GEMM.
// 3. pick_embed: waits for the argmax keys of all ranks, picks the token (lowest index on ties),
//    records it, advances the positions, gathers its embedding row into the residual stream and
//    RMS-normalises it for layer 0 of the next step.
//
// Epochs live in device memory (ctrl[0]) so a whole decode step can be captured in one CUDA graph
// and replayed: the producer reads e = ctrl[0] + 1, writes slot parity e & 1, and its last tile
// stores ctrl[0] = e before it publishes e to the peers' flags; the consumer reads ctrl[0] and waits
// until every flag is >= e. Two parities suffice: a rank reaches epoch e + 2 only after every peer
// published epoch e + 1, which each peer does after it consumed epoch e. Every wait is bounded and
// reports through the status word.
//
// Reference: the reference's TensorParallelLinear::forward returns zeros
// (crates/brain-distributed/src/tensor_parallel.rs:8-27) and LlamaLite::generate re-runs the full
// prefix each step (crates/brain-transformer/src/llama_lite.rs); decoding with a KV cache follows
// KvCache::update (crates/brain-transformer/src/kv_cache.rs:83-158).
#include "common.cuh"

#include <algorithm>

using namespace brain;

namespace {

constexpr int kRows = 128;
constexpr int kBK = 64;
constexpr int kThreads = 128;
constexpr int kMaxWorld = 8;

enum Epi : int { EPI_STORE = 0, EPI_PUSH = 2, EPI_SWIGLU = 3, EPI_QKV = 4, EPI_ARGMAX = 5 };

struct SkinnyArgs {
  int M, N, K;
  int num_kb, kb_per_split, splits;
  int epi;
  float alpha;
  __nv_bfloat16* out;
  int64_t ldc;
  const __nv_bfloat16* R;
  int64_t ldr;
  float* ws;
  int* tile_cnt;
  // EPI_PUSH / EPI_ARGMAX
  int world, rank;
  int64_t slot_elems;
  int* ctrl;                 // [0] epoch, [1] finished-tile count
  unsigned long long* keys;  // EPI_ARGMAX running keys [M], zero between steps
  int64_t vocab_offset;
  void* peer_slots[kMaxWorld];
  int* peer_flags[kMaxWorld];
  // EPI_QKV
  int hq, hkv;
  const int* pos;
  const float* cs;
  __nv_bfloat16 *kpool, *vpool;
  const int* table;
  int max_blocks, block_size;
};

__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Publish epoch e: every rank's flag[rank] = e (after this CTA's and, by the ticket, all other
// tiles' pushed stores).
__device__ __forceinline__ void publish_epoch(const SkinnyArgs& a, int e) {
  a.ctrl[1] = 0;
  a.ctrl[0] = e;
  __threadfence_system();
  for (int r = 0; r < a.world; ++r) sys_st_release(a.peer_flags[r] + a.rank, e);
}

template <int NT, int STAGES>
struct SkSmem {
  static constexpr uint32_t W_BYTES = kRows * kBK * 2;
  static constexpr uint32_t X_BYTES = NT * kBK * 2;
  static constexpr uint32_t STAGE = W_BYTES + X_BYTES;
  static constexpr uint32_t BAR = STAGES * STAGE;
  static constexpr uint32_t TOTAL = BAR + (2 * STAGES + 2) * 8 + 16 + 1024;
};

template <int NT, int STAGES>
__global__ void __launch_bounds__(kThreads) skinny_gemm_kernel(const __grid_constant__ CUtensorMap tmW,
                                                               const __grid_constant__ CUtensorMap tmX,
                                                               const SkinnyArgs a) {
  using S = SkSmem<NT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + S::BAR;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
  const uint32_t done_bar = bars + 16u * STAGES;
  const uint32_t drain_bar = done_bar + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::BAR + (2 * STAGES + 2) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* ticket = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int split = blockIdx.x, tile = blockIdx.y;
  const int kb0 = split * a.kb_per_split;
  const int nkb = min(a.num_kb - kb0, a.kb_per_split);
  constexpr uint32_t kCols = NT < 32 ? 32 : NT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: weight tile [128 rows, 64 k] and token tile [NT, 64 k] per stage
    int i = 0;
    bool ok = true;
    for (; i < nkb; ++i) {
      const int s = i % STAGES;
      const uint32_t round = (uint32_t)(i / STAGES);
      if (!mbar_wait(empty_bar(s), (round & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 110, abort_flag)) {
        ok = false;
        break;
      }
      const uint32_t sw = sbase + s * S::STAGE;
      mbar_arrive_expect_tx(full_bar(s), S::STAGE);
      const int k0 = (kb0 + i) * kBK;
      tma_load_2d(&tmW, sw, full_bar(s), k0, tile * kRows);
      tma_load_2d(&tmX, sw + S::W_BYTES, full_bar(s), k0, 0);
    }
    if (!ok) {
      for (int j = i > STAGES ? i - STAGES : 0; j < i; ++j) {
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(full_bar(j % STAGES), (uint32_t)(j / STAGES) & 1) &&
               globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    constexpr uint32_t idesc = idesc_f16(kRows, NT, 1u, 0u, 0u);
    bool ok = true, issued = false;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES;
      const uint32_t round = (uint32_t)(i / STAGES);
      if (!mbar_wait(full_bar(s), round & 1, BRAIN_ERR_TIMEOUT_FULL, 111, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sw = sbase + s * S::STAGE;
      const uint32_t sx = sw + S::W_BYTES;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        tc_mma_f16(tmem_base, smem_desc_sw128(sw + kk * 32, 16, 1024), smem_desc_sw128(sx + kk * 32, 16, 1024),
                   idesc, (i > 0 || kk > 0) ? 1u : 0u);
      }
      issued = true;
      tc_commit(empty_bar(s));
    }
    if (ok) {
      tc_commit(done_bar);
    } else if (issued) {
      tc_commit(drain_bar);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain_bar, 0) && globaltimer() - t0 < 100000000ull) {
      }
    }
  }
  __syncwarp();

  // ---- accumulator -> registers (thread = weight row `row`, acc[t] = token t)
  const bool ok = mbar_wait(done_bar, 0, BRAIN_ERR_TIMEOUT_ACC, 112, abort_flag);
  tc_fence_after();
  const int row = warp * 32 + lane;
  float acc[NT];
  {
    const uint32_t taddr = tmem_base + ((uint32_t)(warp * 32) << 16);
    if (NT == 16) {
      uint32_t r[16];
      tmem_ld16(taddr, r);
      tc_wait_ld();
#pragma unroll
      for (int t = 0; t < 16; ++t) acc[t] = ok ? __uint_as_float(r[t]) : 0.f;
    } else {
#pragma unroll
      for (int c = 0; c < NT / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tc_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) acc[c * 32 + t] = ok ? __uint_as_float(r[t]) : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
  }
  if (!ok) return;

  // ---- split-K fix-up: the last CTA of the tile sums the partials in split order
  if (a.splits > 1) {
    float* part = a.ws + ((int64_t)tile * a.splits + split) * NT * kRows;
#pragma unroll
    for (int t = 0; t < NT; ++t) part[t * kRows + row] = acc[t];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int old = atomicAdd(a.tile_cnt + tile, 1);
      *ticket = (old == a.splits - 1);
      if (old == a.splits - 1) a.tile_cnt[tile] = 0;
    }
    __syncthreads();
    if (!*ticket) return;
    __threadfence();
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float* p = a.ws + ((int64_t)tile * a.splits + s) * NT * kRows;
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] += __ldcg(p + t * kRows + row);
    }
  }

  float* sx = reinterpret_cast<float*>(smem);  // stage memory is free once every MMA completed
  const int n = tile * kRows + row;
  if (a.epi == EPI_STORE) {
    if (n < a.N) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t < a.M) {
          float v = acc[t] * a.alpha;
          if (a.R) v += __bfloat162float(a.R[t * a.ldr + n]);
          a.out[t * a.ldc + n] = __float2bfloat16_rn(v);
        }
      }
    }
  } else if (a.epi == EPI_PUSH) {
    const int e = ld_volatile(a.ctrl) + 1;
    const int64_t off = ((int64_t)(e & 1) * a.world + a.rank) * a.slot_elems;
    if (n < a.N) {
      for (int r = 0; r < a.world; ++r) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.peer_slots[r]) + off;
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < a.M) dst[t * a.N + n] = __float2bfloat16_rn(acc[t] * a.alpha);
      }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int old = atomicAdd(a.ctrl + 1, 1);
      if (old == (int)gridDim.y - 1) publish_epoch(a, e);
    }
  } else if (a.epi == EPI_SWIGLU) {
    if (row >= 64) {
#pragma unroll
      for (int t = 0; t < NT; ++t) sx[t * 64 + row - 64] = acc[t];
    }
    __syncthreads();
    const int j = tile * 64 + row;
    if (row < 64 && j < a.N / 2) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t < a.M) {
          const float g = acc[t] * a.alpha, u = sx[t * 64 + row] * a.alpha;
          a.out[t * a.ldc + j] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * u);
        }
      }
    }
  } else if (a.epi == EPI_QKV) {
#pragma unroll
    for (int t = 0; t < NT; ++t) sx[t * kRows + row] = acc[t];
    __syncthreads();
    const int h = tile, d = row, dj = row & 63;
    const bool rot = h < a.hq + a.hkv;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < a.M) {
        const int p = a.pos[t];
        float x = acc[t] * a.alpha;
        if (rot) {
          const float y = sx[t * kRows + (row ^ 64)] * a.alpha;
          const float c = a.cs[(int64_t)p * kRows + dj], s = a.cs[(int64_t)p * kRows + 64 + dj];
          x = d < 64 ? x * c - y * s : x * c + y * s;
        }
        if (h < a.hq) {
          a.out[t * a.ldc + h * kRows + d] = __float2bfloat16_rn(x);
        } else {
          const int64_t slot = (int64_t)a.table[(int64_t)t * a.max_blocks + p / a.block_size] * a.block_size +
                               p % a.block_size;
          __nv_bfloat16* pool = rot ? a.kpool : a.vpool;
          const int hh = rot ? h - a.hq : h - a.hq - a.hkv;
          pool[(slot * a.hkv + hh) * kRows + d] = __float2bfloat16_rn(x);
        }
      }
    }
  } else if (a.epi == EPI_ARGMAX) {
    unsigned long long* red = reinterpret_cast<unsigned long long*>(smem);  // [4 warps][NT]
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      unsigned long long k = n < a.N ? argmax_key(acc[t] * a.alpha, a.vocab_offset + n) : 0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
        k = other > k ? other : k;
      }
      if (lane == 0) red[warp * NT + t] = k;
    }
    __syncthreads();
    if (threadIdx.x < a.M) {
      unsigned long long k = red[threadIdx.x];
      for (int w = 1; w < 4; ++w) k = red[w * NT + threadIdx.x] > k ? red[w * NT + threadIdx.x] : k;
      atomicMax(a.keys + threadIdx.x, k);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *ticket = (atomicAdd(a.ctrl + 1, 1) == (int)gridDim.y - 1);
    __syncthreads();
    if (*ticket) {
      __threadfence();
      const int e = ld_volatile(a.ctrl) + 1;
      const int64_t off = ((int64_t)(e & 1) * a.world + a.rank) * a.slot_elems;
      if (threadIdx.x < a.M) {
        const unsigned long long k = atomicExch(a.keys + threadIdx.x, 0ull);
        for (int r = 0; r < a.world; ++r)
          reinterpret_cast<unsigned long long*>(a.peer_slots[r])[off + threadIdx.x] = k;
      }
      __threadfence_system();
      __syncthreads();
      if (threadIdx.x == 0) publish_epoch(a, e);
    }
  }
}

// Wait (thread j < world) until flag j reaches the epoch in ctrl[0]; returns the epoch or -1.
__device__ int wait_epoch(const int* flags, const int* ctrl, int world, int64_t budget_ns, int where) {
  __shared__ int s_e, s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  const int e = ld_volatile(ctrl);
  if (threadIdx.x < world) {
    const uint64_t t0 = globaltimer();
    while (sys_ld_acquire(flags + threadIdx.x) < e) {
      if (globaltimer() - t0 > (uint64_t)budget_ns) {
        set_status(BRAIN_ERR_TIMEOUT_PEER, where * 16 + threadIdx.x);
        s_bad = 1;
        break;
      }
    }
  }
  if (threadIdx.x == 0) s_e = e;
  __syncthreads();
  return s_bad ? -1 : s_e;
}

constexpr int kNormThreads = 256;
constexpr int kMaxChunks = 8;  // N <= 256 * 8 * 8 = 16384

__device__ __forceinline__ float block_sum(float v) {
  __shared__ float red[kNormThreads / 32];
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) s += red[i];
  return s;
}

// residual[row] += sum_j slot_j[row]; normed[row] = rmsnorm(residual[row]) * gamma.
__global__ void __launch_bounds__(kNormThreads) ar_norm_kernel(const __nv_bfloat16* slots, const int* flags,
                                                               const int* ctrl, int world, int64_t slot_elems, int N,
                                                               __nv_bfloat16* resid, int64_t ldr,
                                                               const __nv_bfloat16* gamma, float eps,
                                                               __nv_bfloat16* normed, int64_t ldn,
                                                               int64_t budget_ns) {
  const int row = blockIdx.x;
  const int e = wait_epoch(flags, ctrl, world, budget_ns, 12);
  if (e < 0) return;
  const __nv_bfloat16* base = slots + (int64_t)(e & 1) * world * slot_elems + (int64_t)row * N;
  float h[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int i = (c * kNormThreads + threadIdx.x) * 8;
    if (i < N) {
      load8(resid + row * ldr + i, h[c]);
      for (int j = 0; j < world; ++j) {
        float f[8];
        load8(base + j * slot_elems + i, f);
#pragma unroll
        for (int u = 0; u < 8; ++u) h[c][u] += f[u];
      }
      store8(resid + row * ldr + i, h[c]);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        h[c][u] = __bfloat162float(__float2bfloat16_rn(h[c][u]));  // normalise the stored stream
        ss += h[c][u] * h[c][u];
      }
    }
  }
  const float rstd = rsqrtf(block_sum(ss) / N + eps);
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int i = (c * kNormThreads + threadIdx.x) * 8;
    if (i < N) {
      float g[8];
      load8(gamma + i, g);
#pragma unroll
      for (int u = 0; u < 8; ++u) g[u] *= h[c][u] * rstd;
      store8(normed + row * ldn + i, g);
    }
  }
}

// Greedy pick over the ranks' argmax keys, then the next step's layer-0 input.
__global__ void __launch_bounds__(kNormThreads) pick_embed_kernel(
    const unsigned long long* key_slots, const int* flags, const int* ctrl, int world, int64_t slot_elems,
    const __nv_bfloat16* emb, int64_t lde, int vocab, int N, __nv_bfloat16* resid, const __nv_bfloat16* gamma,
    float eps, __nv_bfloat16* normed, int* hist, int64_t hist_ld, int* pos, int* seq_lens, int64_t budget_ns) {
  const int row = blockIdx.x;
  const int e = wait_epoch(flags, ctrl, world, budget_ns, 13);
  if (e < 0) return;
  __shared__ int s_tok;
  if (threadIdx.x == 0) {
    unsigned long long best = 0;
    for (int j = 0; j < world; ++j) {
      const unsigned long long k = key_slots[((int64_t)(e & 1) * world + j) * slot_elems + row];
      best = k > best ? k : best;
    }
    int tok = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    if (tok < 0 || tok >= vocab) {
      set_status(BRAIN_ERR_BAD_ARG, 14);
      tok = 0;
    }
    const int p = pos[row] + 1;
    if (p < hist_ld) hist[(int64_t)row * hist_ld + p] = tok;
    else set_status(BRAIN_ERR_BOUNDS, 14);
    pos[row] = p;
    seq_lens[row] = p + 1;
    s_tok = tok;
  }
  __syncthreads();
  const __nv_bfloat16* src = emb + (int64_t)s_tok * lde;
  float h[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int i = (c * kNormThreads + threadIdx.x) * 8;
    if (i < N) {
      load8(src + i, h[c]);
      *reinterpret_cast<uint4*>(resid + (int64_t)row * N + i) = *reinterpret_cast<const uint4*>(src + i);
#pragma unroll
      for (int u = 0; u < 8; ++u) ss += h[c][u] * h[c][u];
    }
  }
  const float rstd = rsqrtf(block_sum(ss) / N + eps);
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int i = (c * kNormThreads + threadIdx.x) * 8;
    if (i < N) {
      float g[8];
      load8(gamma + i, g);
#pragma unroll
      for (int u = 0; u < 8; ++u) g[u] *= h[c][u] * rstd;
      store8(normed + (int64_t)row * N + i, g);
    }
  }
}

int nt_for(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

template <int NT, int STAGES>
int launch_skinny(const CUtensorMap& tw, const CUtensorMap& tx, const SkinnyArgs& a, int tiles, cudaStream_t st) {
  using S = SkSmem<NT, STAGES>;
  auto kern = skinny_gemm_kernel<NT, STAGES>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::TOTAL);
    if (e != cudaSuccess) return (int)e;
    attr[dev & 63] = true;
  }
  kern<<<dim3(a.splits, tiles), kThreads, S::TOTAL, st>>>(tw, tx, a);
  return (int)cudaGetLastError();
}

bool map_2d(CUtensorMap* m, const void* p, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer) {
  uint64_t dims[2] = {inner, outer};
  uint64_t strides[1] = {ld * 2};
  uint32_t box[2] = {(uint32_t)kBK, box_outer};
  return brain_host::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

BRAIN_STATUS_READER(decode_tp)

// Split count for a skinny GEMM: fill about two CTAs per SM, at least 4 k-blocks per split.
BRAIN_API int brain_skinny_splits(int M, int N, int K) {
  (void)M;
  const int tiles = (N + kRows - 1) / kRows;
  const int num_kb = (K + kBK - 1) / kBK;
  int s = std::max(1, (2 * brain_host::num_sms()) / std::max(tiles, 1));
  s = std::min(s, std::max(1, num_kb / 4));
  const int per = (num_kb + s - 1) / s;
  return (num_kb + per - 1) / per;  // no empty split
}

// f32 elements of split-K workspace for (M, N, splits).
BRAIN_API int64_t brain_skinny_workspace(int M, int N, int splits) {
  return (int64_t)((N + kRows - 1) / kRows) * splits * nt_for(M) * kRows;
}

// ext (int64[32], may be null for EPI_STORE / EPI_SWIGLU):
//   [0] world [1] rank [2] slot_elems [3] ctrl* [4] keys* [5] vocab_offset [6] hq [7] hkv [8] pos*
//   [9] cos|sin table* [10] k pool* [11] v pool* [12] block table* [13] max_blocks [14] block_size
//   [16..24) peer slot bases  [24..32) peer flag arrays
BRAIN_API int brain_skinny_gemm(const void* X, int64_t ldx, const void* W, int64_t ldw, int M, int N, int K, int epi,
                                float alpha, void* out, int64_t ldc, const void* R, int64_t ldr, int splits,
                                float* ws, int* tile_cnt, const int64_t* ext, cudaStream_t st) {
  if (M <= 0 || M > 64 || N <= 0 || K <= 0 || (K % 8) || (ldx % 8) || (ldw % 8)) return (int)cudaErrorInvalidValue;
  SkinnyArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.num_kb = (K + kBK - 1) / kBK;
  if (splits < 1) splits = 1;
  a.kb_per_split = (a.num_kb + splits - 1) / splits;
  a.splits = (a.num_kb + a.kb_per_split - 1) / a.kb_per_split;
  if (a.splits > 1 && (!ws || !tile_cnt)) return (int)cudaErrorInvalidValue;
  a.epi = epi;
  a.alpha = alpha;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ldc = ldc;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  a.ws = ws;
  a.tile_cnt = tile_cnt;
  if (epi == EPI_PUSH || epi == EPI_ARGMAX || epi == EPI_QKV) {
    if (!ext) return (int)cudaErrorInvalidValue;
    a.world = (int)ext[0];
    a.rank = (int)ext[1];
    a.slot_elems = ext[2];
    a.ctrl = reinterpret_cast<int*>(ext[3]);
    a.keys = reinterpret_cast<unsigned long long*>(ext[4]);
    a.vocab_offset = ext[5];
    a.hq = (int)ext[6];
    a.hkv = (int)ext[7];
    a.pos = reinterpret_cast<const int*>(ext[8]);
    a.cs = reinterpret_cast<const float*>(ext[9]);
    a.kpool = reinterpret_cast<__nv_bfloat16*>(ext[10]);
    a.vpool = reinterpret_cast<__nv_bfloat16*>(ext[11]);
    a.table = reinterpret_cast<const int*>(ext[12]);
    a.max_blocks = (int)ext[13];
    a.block_size = (int)ext[14];
    if (a.world < 1 || a.world > kMaxWorld) return (int)cudaErrorInvalidValue;
    for (int r = 0; r < a.world; ++r) {
      a.peer_slots[r] = reinterpret_cast<void*>(ext[16 + r]);
      a.peer_flags[r] = reinterpret_cast<int*>(ext[24 + r]);
    }
  }
  if (epi == EPI_QKV && N != (a.hq + 2 * a.hkv) * kRows) return (int)cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU && (N % kRows)) return (int)cudaErrorInvalidValue;
  if (epi == EPI_ARGMAX && !a.keys) return (int)cudaErrorInvalidValue;
  const int tiles = (N + kRows - 1) / kRows;
  const int NT = nt_for(M);
  CUtensorMap tw, tx;
  if (!map_2d(&tw, W, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kRows) ||
      !map_2d(&tx, X, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, (uint32_t)NT))
    return (int)cudaErrorInvalidValue;
  if (NT == 16) return launch_skinny<16, 6>(tw, tx, a, tiles, st);
  if (NT == 32) return launch_skinny<32, 5>(tw, tx, a, tiles, st);
  return launch_skinny<64, 4>(tw, tx, a, tiles, st);
}

BRAIN_API int brain_tp_ar_norm(const void* slots, const int* flags, const int* ctrl, int world, int64_t slot_elems,
                               int M, int N, void* resid, int64_t ldr, const void* gamma, float eps, void* normed,
                               int64_t ldn, int64_t budget_ns, cudaStream_t st) {
  if (N % 8 || N > kNormThreads * 8 * kMaxChunks || world < 1 || world > kMaxWorld) return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  ar_norm_kernel<<<M, kNormThreads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(slots), flags, ctrl, world,
                                             slot_elems, N, reinterpret_cast<__nv_bfloat16*>(resid), ldr,
                                             reinterpret_cast<const __nv_bfloat16*>(gamma), eps,
                                             reinterpret_cast<__nv_bfloat16*>(normed), ldn, budget_ns);
  return (int)cudaGetLastError();
}

BRAIN_API int brain_tp_pick_embed(const void* key_slots, const int* flags, const int* ctrl, int world,
                                  int64_t slot_elems, int M, const void* emb, int64_t lde, int vocab, int N,
                                  void* resid, const void* gamma, float eps, void* normed, int* hist, int64_t hist_ld,
                                  int* pos, int* seq_lens, int64_t budget_ns, cudaStream_t st) {
  if (N % 8 || N > kNormThreads * 8 * kMaxChunks || world < 1 || world > kMaxWorld) return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  pick_embed_kernel<<<M, kNormThreads, 0, st>>>(
      reinterpret_cast<const unsigned long long*>(key_slots), flags, ctrl, world, slot_elems,
      reinterpret_cast<const __nv_bfloat16*>(emb), lde, vocab, N, reinterpret_cast<__nv_bfloat16*>(resid),
      reinterpret_cast<const __nv_bfloat16*>(gamma), eps, reinterpret_cast<__nv_bfloat16*>(normed), hist, hist_ld,
      pos, seq_lens, budget_ns);
  return (int)cudaGetLastError();
}
