// Tensor-parallel decode kernels (one new token per sequence, M <= 64 tokens per step), sm_100a.
//
// 1. skinny_gemm: out[M, N] = x[M, K] * W[N, K]^T with the operands swapped on the tensor core: the
//    weight supplies the 128-row MMA M side and the tokens the N side (NT = 16 / 32 / 64), so a
//    128 x NT f32 accumulator lives in TMEM while the weight streams through a TMA ring at HBM rate
//    (decode is bound by reading the weights once per step). K is split over a cluster of `splits`
//    (<= 8) CTAs per 128-row tile so every SM streams. The split-K reduction runs in distributed
//    shared memory: CTA r finishes tokens [r * tper, (r + 1) * tper); every CTA stores its partials
//    for those tokens straight into CTA r's receive buffer (remote shared-memory stores), one cluster
//    barrier, then CTA r sums them in rank order (deterministic, no workspace, no atomics) and runs
//    one of the epilogues for its tokens over all 128 rows of the tile:
//      EPI_STORE   bf16 out (+ residual)
//      EPI_PUSH    all-reduce push: the bf16 partial product goes to slot `rank` of every rank's
//                  receive buffer over NVLink with plain stores; no fence or flag follows them
//      EPI_SWIGLU  weight rows interleaved in 64-row groups [gate 64 | up 64]; writes silu(gate) * up
//      EPI_QKV     one tile = one head of the fused [q | k | v] projection (head_dim 128): RoPE on
//                  q / k at each token's position, q to `out`, k / v straight into their paged slots
//      EPI_ARGMAX  greedy LM head: the per-token max over the tile's vocabulary rows folds into a
//                  64-bit (value, -index) key with atomicMax; the last CTA (ticket) pushes the keys to
//                  every rank
//    The first weight stages are requested before the kernel waits for its predecessor
//    (programmatic dependent launch), so the weight stream starts while the previous kernel ends.
// 2. ar_norm: sums the `world` bf16 slots of a token row in f32 as they arrive, adds the residual
//    stream (updated in place) and writes RMSNorm(h) * gamma for the next GEMM.
// 3. pick_embed: waits for the argmax keys of all ranks, picks the token (lowest index on ties),
//    records it, advances the positions, gathers its embedding row into the residual stream and
//    RMS-normalises it for layer 0 of the next step.
//
// Synchronisation without fences or flags ("the data is the flag"): every receive slot holds a
// sentinel until its value arrives - bf16 -0.0 for the all-reduce slots (a -0.0 result is sent as
// +0.0) and 0 for the argmax keys (never a valid key). Consumers poll their 16-byte pieces with
// relaxed system-scope loads until no sentinel is left, use them, and write the sentinel back for the
// next use of that slot parity. Epochs live in device memory so a whole decode step is one replayable
// CUDA graph: ctrl[0] = last epoch consumed (written by consumers), ctrl[1] = last epoch produced
// (written by producers), ctrl[2] = argmax ticket; a producer uses e = ctrl[0] + 1 and slot parity
// e & 1, the consumer reads e = ctrl[1]. Two parities suffice: a rank pushes epoch e + 2 only after
// it consumed epoch e + 1, which needs every peer's epoch e + 1 push, which each peer issues after
// it consumed (and reset) epoch e. Every poll is bounded and reports through the status word.
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
constexpr int kMaxSplits = 16;       // cluster size: 8 is portable, 16 needs the non-portable opt-in
constexpr unsigned short kSentinel = 0x8000;  // bf16 -0.0: "not written yet" in a receive slot

enum Epi : int { EPI_STORE = 0, EPI_PUSH = 2, EPI_SWIGLU = 3, EPI_QKV = 4, EPI_ARGMAX = 5 };

struct SkinnyArgs {
  int M, N, K;
  int num_kb, kb_per_split, splits;
  float alpha;
  __nv_bfloat16* out;
  int64_t ldc;
  const __nv_bfloat16* R;
  int64_t ldr;
  // EPI_PUSH / EPI_ARGMAX
  int world, rank;
  int64_t slot_elems;
  int* ctrl;                 // [0] epoch consumed, [1] epoch produced, [2] argmax ticket
  unsigned long long* keys;  // EPI_ARGMAX running keys [M], zero between steps
  int64_t vocab_offset;
  void* peer_slots[kMaxWorld];
  // EPI_QKV
  int hq, hkv;
  const int* pos;
  const float* cs;
  __nv_bfloat16 *kpool, *vpool;
  const int* table;
  int max_blocks, block_size;
  // optional per-CTA phase timestamps (globaltimer ns), [cta][8]; null = off
  unsigned long long* trace;
  int pdl_late;  // let dependents launch after the main loop instead of at the start
  const void* pf;  // optional L2 prefetch once the weights are consumed (the next kernels' weights)
  int64_t pf_bytes;
};

__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// f32 store to the shared memory of a CTA of this cluster (address from mapa_shared).
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v));
}

// Bulk copy of `bytes` (multiple of 16) from this CTA's shared memory to shared memory of a CTA of
// this cluster (`dst` and `bar` from mapa_shared), completing transactions on that CTA's mbarrier.
// A unicast copy between CTAs of one cluster; global memory is not involved.
__device__ __forceinline__ void bulk_s2s(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "r"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Polling load of 16 bytes that peers write over NVLink (system scope, no L1 caching).
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const void* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool has_sentinel(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  bool any = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) any |= (w[i] & 0xFFFFu) == kSentinel || (w[i] >> 16) == kSentinel;
  return any;
}

template <int NT, int STAGES>
struct SkSmem {
  static constexpr uint32_t W_BYTES = kRows * kBK * 2;
  static constexpr uint32_t X_BYTES = NT * kBK * 2;
  static constexpr uint32_t STAGE = W_BYTES + X_BYTES;
  static constexpr uint32_t RECV = STAGES * STAGE;                  // [splits][tper][128] f32
  static constexpr uint32_t RECV_BYTES = (NT + kMaxSplits) * kRows * 4;
  static constexpr uint32_t BAR = RECV + RECV_BYTES;
  static constexpr uint32_t TOTAL = BAR + (2 * STAGES + 3) * 8 + 16 + 1024;
  // after the main loop the stage memory holds the outgoing partials [M][128] f32 at 0 and the
  // epilogue scratch [tper][128] f32 at SX
  static constexpr uint32_t SX = NT * kRows * 4;
  static_assert(2 * NT * kRows * 4 <= STAGES * STAGE, "stage memory too small for the tail buffers");
};

template <int NT, int STAGES, int EPI>
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
  const uint32_t recv_bar = done_bar + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::BAR + (2 * STAGES + 3) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* ticket = reinterpret_cast<volatile int*>(tmem_slot + 2);

  if (!a.pdl_late) pdl_trigger();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int split = blockIdx.x, tile = blockIdx.y;
  unsigned long long* trace =
      a.trace && threadIdx.x == 0 ? a.trace + ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * 16 : nullptr;
  if (trace) trace[0] = globaltimer();
  const int kb0 = split * a.kb_per_split;
  const int nkb = min(a.num_kb - kb0, a.kb_per_split);
  constexpr uint32_t kCols = NT < 32 ? 32 : NT;
  // tokens finished by this CTA: [t0, t0 + nt)
  const int nsplit = a.splits;
  const int tper = (a.M + nsplit - 1) / nsplit;
  const int t0 = split * tper;
  const int nt = max(0, min(a.M - t0, tper));

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(drain_bar, 1);
    mbar_init(recv_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    // every CTA of the cluster (this one included) will copy nt tokens x 128 rows of partials here
    mbar_arrive_expect_tx(recv_bar, (uint32_t)(nsplit * nt * kRows * 4));
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
  cluster_arrive_relaxed();  // receive barriers initialised; the matching wait precedes the first copy
  if (trace) trace[1] = globaltimer();

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: weight tile [128 rows, 64 k] and token tile [NT, 64 k] per stage. The
    // weights are never written by a predecessor, so the first ring of weight tiles is requested
    // before pdl_wait(): under programmatic launch it streams while the previous kernel finishes.
    const int pre = nkb < STAGES ? nkb : STAGES;
    for (int j = 0; j < pre; ++j) {
      mbar_arrive_expect_tx(full_bar(j), S::STAGE);
      tma_load_2d(&tmW, sbase + j * S::STAGE, full_bar(j), (kb0 + j) * kBK, tile * kRows);
    }
    pdl_wait();
    if (trace) trace[2] = globaltimer();
    for (int j = 0; j < pre; ++j)
      tma_load_2d(&tmX, sbase + j * S::STAGE + S::W_BYTES, full_bar(j), (kb0 + j) * kBK, 0);
    int i = pre;
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

  // The tail below runs once per CTA, so it is written as compact rolled loops: fully unrolled
  // straight-line code here was dominated by cold instruction fetch.
  const bool ok = mbar_wait(done_bar, 0, BRAIN_ERR_TIMEOUT_ACC, 112, abort_flag);
  tc_fence_after();
  if (a.pdl_late) pdl_trigger();  // every weight tile consumed: the successor may take the SM slots
  if (threadIdx.x == 0) l2_prefetch_part(a.pf, a.pf_bytes, tile * nsplit + split, gridDim.x * gridDim.y);
  if (trace) {
    trace[3] = globaltimer();
    trace[8] = clock64();
  }
  const int row = warp * 32 + lane;
  pdl_wait();  // predecessor complete: its writes (residual, epochs, cache, outputs) are visible
  if (trace) trace[9] = clock64();

  // ---- split-K reduction: partials -> local staging [M][128] -> one bulk copy per finishing CTA
  float* stg = reinterpret_cast<float*>(smem);             // stage memory is free once every MMA completed
  float* recv = reinterpret_cast<float*>(smem + S::RECV);  // [nsplit][tper][128]
  {
    const uint32_t taddr = tmem_base + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < a.M; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + (uint32_t)c, r);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) stg[(c + j) * kRows + row] = ok ? __uint_as_float(r[j]) : 0.f;
    }
  }
  fence_proxy_async();  // staging writes visible to the bulk-copy (async) proxy
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
  }
  cluster_wait();  // every CTA of the cluster has initialised its receive barrier
  if (threadIdx.x == 0) {
    const uint32_t src0 = smem_u32(stg), dst0 = smem_u32(recv) + (uint32_t)(split * tper * kRows * 4);
    for (int d = 0; d < nsplit; ++d) {
      const int ntd = min(a.M - d * tper, tper);
      if (ntd > 0)
        bulk_s2s(mapa_shared(dst0, (uint32_t)d), src0 + (uint32_t)(d * tper * kRows * 4), (uint32_t)(ntd * kRows * 4),
                 mapa_shared(recv_bar, (uint32_t)d));
    }
    bulk_commit();
  }
  if (trace) trace[10] = clock64();
  // A CTA whose pipeline gave up still sends its (zero) partials, so the other CTAs of its cluster
  // never wait for it; the status word already records the failure.
  const bool got = mbar_wait(recv_bar, 0, BRAIN_ERR_TIMEOUT_ACC, 113, nullptr);
  if (threadIdx.x == 0) bulk_wait_read0();  // outgoing copies have read the staging buffer
  __syncthreads();
  if (trace) {
    trace[4] = globaltimer();
    trace[11] = clock64();
  }
  if (!ok || !got) return;
  auto reduced = [&](int i) {  // sum of the partials of local token i for this row, in rank order
    float part[kMaxSplits];
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r) part[r] = r < nsplit ? recv[(r * tper + i) * kRows + row] : 0.f;
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r) sum += part[r];
    return sum;
  };

  float* sx = reinterpret_cast<float*>(smem + S::SX);  // epilogue scratch [tper][128]
  const int n = tile * kRows + row;
  const int total_ctas = (int)(gridDim.x * gridDim.y);
  if constexpr (EPI == EPI_STORE) {
    if (n < a.N) {
#pragma unroll 1
      for (int i = 0; i < nt; ++i) {
        const int t = t0 + i;
        float x = reduced(i) * a.alpha;
        if (a.R) x += __bfloat162float(a.R[t * a.ldr + n]);
        a.out[t * a.ldc + n] = __float2bfloat16_rn(x);
      }
    }
  } else if constexpr (EPI == EPI_PUSH) {
    // Receive slots hold the sentinel (bf16 -0.0) until written; a -0.0 result is sent as +0.0. The
    // consumer polls the values themselves, so no fence or flag follows the stores.
    const int e = ld_volatile(a.ctrl) + 1;
    const int64_t off = ((int64_t)(e & 1) * a.world + a.rank) * a.slot_elems;
    if (n < a.N) {
#pragma unroll 1
      for (int i = 0; i < nt; ++i) {
        __nv_bfloat16 x = __float2bfloat16_rn(reduced(i) * a.alpha);
        if (__bfloat16_as_ushort(x) == kSentinel) x = __ushort_as_bfloat16((unsigned short)0);
#pragma unroll 1
        for (int r = 0; r < a.world; ++r)
          reinterpret_cast<__nv_bfloat16*>(a.peer_slots[(a.rank + 1 + r) % a.world])[off + (t0 + i) * a.N + n] = x;
      }
    }
    if (threadIdx.x == 0) a.ctrl[1] = e;  // same value from every CTA; read after this grid completes
  } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
    for (int i = 0; i < nt; ++i) sx[i * kRows + row] = reduced(i) * a.alpha;
    __syncthreads();
    const int j = tile * 64 + row;
    if (row < 64 && j < a.N / 2) {
#pragma unroll 1
      for (int i = 0; i < nt; ++i) {
        const float g = sx[i * kRows + row], u = sx[i * kRows + row + 64];
        a.out[(t0 + i) * a.ldc + j] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * u);
      }
    }
  } else if constexpr (EPI == EPI_QKV) {
#pragma unroll 1
    for (int i = 0; i < nt; ++i) sx[i * kRows + row] = reduced(i) * a.alpha;
    __syncthreads();
    const int h = tile, d = row, dj = row & 63;
    const bool rot = h < a.hq + a.hkv;
    __nv_bfloat16* pool = rot ? a.kpool : a.vpool;
    const int hh = rot ? h - a.hq : h - a.hq - a.hkv;
#pragma unroll 1
    for (int i = 0; i < nt; ++i) {
      const int t = t0 + i;
      const int p = a.pos[t];
      float x = sx[i * kRows + row];
      if (rot) {
        const float y = sx[i * kRows + (row ^ 64)];
        const float c = a.cs[(int64_t)p * kRows + dj], sn = a.cs[(int64_t)p * kRows + 64 + dj];
        x = d < 64 ? x * c - y * sn : x * c + y * sn;
      }
      if (h < a.hq) {
        a.out[t * a.ldc + h * kRows + d] = __float2bfloat16_rn(x);
      } else {
        const int64_t slot = (int64_t)a.table[(int64_t)t * a.max_blocks + p / a.block_size] * a.block_size +
                             p % a.block_size;
        pool[(slot * a.hkv + hh) * kRows + d] = __float2bfloat16_rn(x);
      }
    }
  } else if constexpr (EPI == EPI_ARGMAX) {
    unsigned long long* kred = reinterpret_cast<unsigned long long*>(smem);  // [4 warps][NT]
#pragma unroll 1
    for (int i = 0; i < nt; ++i) {
      const float x = reduced(i) * a.alpha;
      unsigned long long k = n < a.N ? argmax_key(x, a.vocab_offset + n) : 0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
        k = other > k ? other : k;
      }
      if (lane == 0) kred[warp * NT + i] = k;
    }
    __syncthreads();
    if (threadIdx.x < nt) {
      unsigned long long k = kred[threadIdx.x];
      for (int w = 1; w < 4; ++w) k = kred[w * NT + threadIdx.x] > k ? kred[w * NT + threadIdx.x] : k;
      atomicMax(a.keys + t0 + threadIdx.x, k);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *ticket = (atomicAdd(a.ctrl + 2, 1) == total_ctas - 1);
    __syncthreads();
    if (*ticket) {
      __threadfence();
      const int e = ld_volatile(a.ctrl) + 1;
      const int64_t off = ((int64_t)(e & 1) * a.world + a.rank) * a.slot_elems;
      if (threadIdx.x < a.M) {
        // a key is never 0 (the value half of a finite max is non-zero), so 0 marks an empty slot
        const unsigned long long k = atomicExch(a.keys + threadIdx.x, 0ull);
        for (int r = 0; r < a.world; ++r)
          reinterpret_cast<unsigned long long*>(a.peer_slots[r])[off + threadIdx.x] = k;
      }
      if (threadIdx.x == 0) {
        a.ctrl[2] = 0;
        a.ctrl[1] = e;
      }
    }
  }
  if (trace) {
    trace[6] = globaltimer();
    trace[15] = clock64();
  }
}

constexpr int kNormThreads = 256;
constexpr int kMaxChunks = 8;  // pick_embed: N <= 256 * 8 * 8 = 16384

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

// Wait until none of the 8 bf16 at p is the sentinel (bounded); returns the values, or zeros after
// the budget ran out (status recorded).
__device__ __forceinline__ uint4 poll_slot(const __nv_bfloat16* p, uint4 v, int64_t budget_ns, int where) {
  if (!has_sentinel(v)) return v;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    v = ld_relaxed_sys_v4(p);
    if (!has_sentinel(v)) return v;
    if ((it & 63u) == 63u && globaltimer() - t0 > (uint64_t)budget_ns) {
      set_status(BRAIN_ERR_TIMEOUT_PEER, where);
      return make_uint4(0, 0, 0, 0);
    }
  }
}

// residual[row] += sum_j slot_j[row]; normed[row] = rmsnorm(residual[row]) * gamma.
// A cluster of kArParts CTAs shares one token row (each owns N / kArParts columns, one 8-element chunk
// per thread for N = 8192); the row's sum of squares is combined through distributed shared memory.
// Each thread polls its 16-byte piece of every rank's slot until the sentinel is gone, then writes the
// sentinel back for the next use of this slot parity. The residual and gamma loads are issued first.
constexpr int kArParts = 4;
constexpr int kArChunks = 2;  // N <= kArParts * kNormThreads * 8 * kArChunks = 16384

__global__ void __launch_bounds__(kNormThreads) ar_norm_kernel(__nv_bfloat16* slots, int* ctrl, int world,
                                                               int64_t slot_elems, int N, __nv_bfloat16* resid,
                                                               int64_t ldr, const __nv_bfloat16* gamma, float eps,
                                                               __nv_bfloat16* normed, int64_t ldn, int64_t budget_ns) {
  pdl_trigger();
  pdl_wait();
  __shared__ float s_parts[kArParts];
  const int part = blockIdx.x, row = blockIdx.y;
  const int cols = N / kArParts;
  float h[kArChunks][8], g[kArChunks][8];
#pragma unroll
  for (int c = 0; c < kArChunks; ++c) {
    const int k = (c * kNormThreads + threadIdx.x) * 8;
    if (k < cols) {
      load8(resid + row * ldr + part * cols + k, h[c]);
      load8(gamma + part * cols + k, g[c]);
    }
  }
  const int e = ld_volatile(ctrl + 1);
  __nv_bfloat16* base = slots + (int64_t)(e & 1) * world * slot_elems + (int64_t)row * N + part * cols;
  const uint4 empty = make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kArChunks; ++c) {
    const int k = (c * kNormThreads + threadIdx.x) * 8;
    if (k < cols) {
      uint4 v[kMaxWorld];
#pragma unroll
      for (int j = 0; j < kMaxWorld; ++j)
        if (j < world) v[j] = ld_relaxed_sys_v4(base + j * slot_elems + k);
#pragma unroll
      for (int j = 0; j < kMaxWorld; ++j) {
        if (j < world) {
          __nv_bfloat16* p = base + j * slot_elems + k;
          v[j] = poll_slot(p, v[j], budget_ns, 12 * 16 + j);
          *reinterpret_cast<uint4*>(p) = empty;  // ready for the next use of this parity
          const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v[j]);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 f = __bfloat1622float2(b2[u]);
            h[c][2 * u] += f.x;
            h[c][2 * u + 1] += f.y;
          }
        }
      }
      store8(resid + row * ldr + part * cols + k, h[c]);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        h[c][u] = __bfloat162float(__float2bfloat16_rn(h[c][u]));  // normalise the stored stream
        ss += h[c][u] * h[c][u];
      }
    }
  }
  ss = block_sum(ss);
  // every CTA of the row's cluster stores its partial sum of squares into every CTA's s_parts; one
  // barrier, then each sums locally (no remote reads, so no second barrier before exit)
  if (threadIdx.x < kArParts) st_dsmem_f32(mapa_shared(smem_u32(&s_parts[part]), (uint32_t)threadIdx.x), ss);
  cluster_sync();
  float tot = 0.f;
#pragma unroll
  for (int r = 0; r < kArParts; ++r) tot += s_parts[r];
  if (threadIdx.x == 0) ctrl[0] = e;  // same value from every CTA; read after this grid completes
  const float rstd = rsqrtf(tot / N + eps);
#pragma unroll
  for (int c = 0; c < kArChunks; ++c) {
    const int k = (c * kNormThreads + threadIdx.x) * 8;
    if (k < cols) {
#pragma unroll
      for (int u = 0; u < 8; ++u) g[c][u] *= h[c][u] * rstd;
      store8(normed + row * ldn + part * cols + k, g[c]);
    }
  }
}

// Greedy pick over the ranks' argmax keys (each polled until non-zero, then cleared), then the next
// step's layer-0 input.
__global__ void __launch_bounds__(kNormThreads) pick_embed_kernel(
    unsigned long long* key_slots, int* ctrl, int world, int64_t slot_elems, const __nv_bfloat16* emb, int64_t lde,
    int vocab, int N, __nv_bfloat16* resid, const __nv_bfloat16* gamma, float eps, __nv_bfloat16* normed, int* hist,
    int64_t hist_ld, int* pos, int* seq_lens, int64_t budget_ns) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int e = ld_volatile(ctrl + 1);
  __shared__ int s_tok;
  if (threadIdx.x == 0) {
    unsigned long long best = 0;
    const uint64_t t0 = globaltimer();
    for (int j = 0; j < world; ++j) {
      unsigned long long* p = key_slots + ((int64_t)(e & 1) * world + j) * slot_elems + row;
      unsigned long long k = ld_relaxed_sys_u64(p);
      while (k == 0ull) {
        if (globaltimer() - t0 > (uint64_t)budget_ns) {
          set_status(BRAIN_ERR_TIMEOUT_PEER, 13 * 16 + j);
          break;
        }
        k = ld_relaxed_sys_u64(p);
      }
      *p = 0ull;
      best = k > best ? k : best;
    }
    int tok = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    if (best == 0ull || tok < 0 || tok >= vocab) {
      set_status(BRAIN_ERR_BAD_ARG, 14);
      tok = 0;
    }
    const int p = pos[row] + 1;
    if (p < hist_ld) hist[(int64_t)row * hist_ld + p] = tok;
    else set_status(BRAIN_ERR_BOUNDS, 14);
    pos[row] = p;
    seq_lens[row] = p + 1;
    s_tok = tok;
    ctrl[0] = e;
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

// Dynamic shared memory size plus the largest shared-memory carveout, so two ~100 KB CTAs fit on an
// SM (the default carveout left room for one).
template <typename K>
cudaError_t set_smem_attrs(K kern, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                              (int)cudaSharedmemCarveoutMaxShared);
}

// Whether a cluster of `splits` skinny-GEMM CTAs can be resident on this GPU at all.
template <int NT, int STAGES>
bool cluster_fits(int splits) {
  using S = SkSmem<NT, STAGES>;
  auto kern = skinny_gemm_kernel<NT, STAGES, EPI_STORE>;
  if (set_smem_attrs(kern, (int)S::TOTAL) != cudaSuccess) return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::TOTAL;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = splits;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  return cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0;
}

template <int NT, int STAGES, int EPI>
int launch_skinny(const CUtensorMap& tw, const CUtensorMap& tx, const SkinnyArgs& a, int tiles, cudaStream_t st) {
  using S = SkSmem<NT, STAGES>;
  auto kern = skinny_gemm_kernel<NT, STAGES, EPI>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = set_smem_attrs(kern, (int)S::TOTAL);
    if (e != cudaSuccess) return (int)e;
    attr[dev & 63] = true;
  }
  // grid (splits, tiles), one cluster of `splits` CTAs per 128-row tile (the split-K reduction runs
  // over distributed shared memory); programmatic dependent launch when enabled
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = a.splits;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = brain_host::g_decode_pdl ? 2 : 1;
  return (int)cudaLaunchKernelEx(&cfg, kern, tw, tx, a);
}

template <int NT, int STAGES>
int launch_by_epi(int epi, const CUtensorMap& tw, const CUtensorMap& tx, const SkinnyArgs& a, int tiles,
                  cudaStream_t st) {
  switch (epi) {
    case EPI_STORE: return launch_skinny<NT, STAGES, EPI_STORE>(tw, tx, a, tiles, st);
    case EPI_PUSH: return launch_skinny<NT, STAGES, EPI_PUSH>(tw, tx, a, tiles, st);
    case EPI_SWIGLU: return launch_skinny<NT, STAGES, EPI_SWIGLU>(tw, tx, a, tiles, st);
    case EPI_QKV: return launch_skinny<NT, STAGES, EPI_QKV>(tw, tx, a, tiles, st);
    case EPI_ARGMAX: return launch_skinny<NT, STAGES, EPI_ARGMAX>(tw, tx, a, tiles, st);
    default: return (int)cudaErrorInvalidValue;
  }
}

bool map_2d(CUtensorMap* m, const void* p, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer) {
  uint64_t dims[2] = {inner, outer};
  uint64_t strides[1] = {ld * 2};
  uint32_t box[2] = {(uint32_t)kBK, box_outer};
  return brain_host::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

namespace brain_host {
int g_decode_pdl = 2;
}

BRAIN_STATUS_READER(decode_tp)

// Programmatic dependent launch for the decode-step kernels: 0 off; 1 on, dependents may launch as soon
// as a kernel starts; 2 on, the skinny GEMM and the decode attention let them launch only after their
// main loop (their early-launched successors would otherwise take SM slots they still need). Returns
// the old value.
BRAIN_API int brain_decode_set_pdl(int on) {
  const int old = brain_host::g_decode_pdl;
  brain_host::g_decode_pdl = on;
  return old;
}

// Split count (= cluster size, at most 16) for a skinny GEMM: about two CTAs per SM in one wave (the
// ~100 KB CTAs fit two per SM; measured residency, not the occupancy API, which reports one), at least
// 4 k-blocks per split, no empty split; above 8 only where a 16-CTA cluster fits on this GPU.
BRAIN_API int brain_skinny_splits(int M, int N, int K) {
  const int tiles = (N + kRows - 1) / kRows;
  const int num_kb = (K + kBK - 1) / kBK;
  int s = std::max(1, (2 * brain_host::num_sms()) / std::max(tiles, 1));
  s = std::min(s, kMaxSplits);
  if (s > 8) {
    static int fits16[64][3];  // [device][token tile]: 0 unknown, 1 yes, 2 no
    int dev = 0;
    cudaGetDevice(&dev);
    const int NT = nt_for(M), nti = NT == 16 ? 0 : (NT == 32 ? 1 : 2);
    int& f = fits16[dev & 63][nti];
    if (f == 0) {
      const bool ok = NT == 16 ? cluster_fits<16, 5>(kMaxSplits)
                               : (NT == 32 ? cluster_fits<32, 4>(kMaxSplits) : cluster_fits<64, 3>(kMaxSplits));
      f = ok ? 1 : 2;
    }
    if (f != 1) s = 8;
  }
  s = std::min(s, std::max(1, num_kb / 4));
  const int per = (num_kb + s - 1) / s;
  return (num_kb + per - 1) / per;
}


// ext (int64[32], may be null for EPI_STORE / EPI_SWIGLU):
//   [0] world [1] rank [2] slot_elems [3] ctrl* [4] keys* [5] vocab_offset [6] hq [7] hkv [8] pos*
//   [9] cos|sin table* [10] k pool* [11] v pool* [12] block table* [13] max_blocks [14] block_size
//   [15] optional phase-timestamp buffer (uint64 [ctas][16]: globaltimer ns [0..7), SM clocks [8..16))
//   [16..24) peer slot bases  [24] optional L2-prefetch base (16-byte aligned)  [25] its size in bytes
BRAIN_API int brain_skinny_gemm(const void* X, int64_t ldx, const void* W, int64_t ldw, int M, int N, int K, int epi,
                                float alpha, void* out, int64_t ldc, const void* R, int64_t ldr, int splits,
                                const int64_t* ext, cudaStream_t st) {
  if (M <= 0 || M > 64 || N <= 0 || K <= 0 || (K % 8) || (ldx % 8) || (ldw % 8)) return (int)cudaErrorInvalidValue;
  SkinnyArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.num_kb = (K + kBK - 1) / kBK;
  if (splits < 1) splits = 1;
  if (splits > kMaxSplits) splits = kMaxSplits;
  a.kb_per_split = (a.num_kb + splits - 1) / splits;
  a.splits = (a.num_kb + a.kb_per_split - 1) / a.kb_per_split;
  a.alpha = alpha;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ldc = ldc;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  if (ext) a.trace = reinterpret_cast<unsigned long long*>(ext[15]);
  a.pdl_late = brain_host::g_decode_pdl == 2;
  if (ext && ext[24] && !(ext[24] & 15)) {
    a.pf = reinterpret_cast<const void*>(ext[24]);
    a.pf_bytes = ext[25];
  }
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
    for (int r = 0; r < a.world; ++r) a.peer_slots[r] = reinterpret_cast<void*>(ext[16 + r]);
  }
  const int tiles = (N + kRows - 1) / kRows;
  if (tiles > 65535) return (int)cudaErrorInvalidValue;
  if (epi == EPI_QKV && N != (a.hq + 2 * a.hkv) * kRows) return (int)cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU && (N % kRows)) return (int)cudaErrorInvalidValue;
  if (epi == EPI_ARGMAX && !a.keys) return (int)cudaErrorInvalidValue;
  const int NT = nt_for(M);
  CUtensorMap tw, tx;
  if (!map_2d(&tw, W, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kRows) ||
      !map_2d(&tx, X, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, (uint32_t)NT))
    return (int)cudaErrorInvalidValue;
  if (NT == 16) return launch_by_epi<16, 5>(epi, tw, tx, a, tiles, st);
  if (NT == 32) return launch_by_epi<32, 4>(epi, tw, tx, a, tiles, st);
  return launch_by_epi<64, 3>(epi, tw, tx, a, tiles, st);
}

BRAIN_API int brain_tp_ar_norm(void* slots, void* ctrl, int world, int64_t slot_elems, int M, int N, void* resid,
                               int64_t ldr, const void* gamma, float eps, void* normed, int64_t ldn, int64_t budget_ns,
                               cudaStream_t st) {
  if (N % (8 * kArParts) || N > kArParts * kNormThreads * 8 * kArChunks || world < 1 || world > kMaxWorld)
    return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kArParts, M);
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kArParts;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = brain_host::g_decode_pdl ? 2 : 1;
  return (int)cudaLaunchKernelEx(&cfg, ar_norm_kernel, reinterpret_cast<__nv_bfloat16*>(slots),
                                 reinterpret_cast<int*>(ctrl), world, slot_elems, N,
                                 reinterpret_cast<__nv_bfloat16*>(resid), ldr,
                                 reinterpret_cast<const __nv_bfloat16*>(gamma), eps,
                                 reinterpret_cast<__nv_bfloat16*>(normed), ldn, budget_ns);
}

BRAIN_API int brain_tp_pick_embed(void* key_slots, void* ctrl, int world, int64_t slot_elems, int M, const void* emb,
                                  int64_t lde, int vocab, int N, void* resid, const void* gamma, float eps,
                                  void* normed, int* hist, int64_t hist_ld, int* pos, int* seq_lens, int64_t budget_ns,
                                  cudaStream_t st) {
  if (N % 8 || N > kNormThreads * 8 * kMaxChunks || world < 1 || world > kMaxWorld) return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  return (int)brain_host::launch(
      pick_embed_kernel, dim3(M), dim3(kNormThreads), 0, st, brain_host::g_decode_pdl != 0,
      reinterpret_cast<unsigned long long*>(key_slots), reinterpret_cast<int*>(ctrl), world, slot_elems,
      reinterpret_cast<const __nv_bfloat16*>(emb), lde, vocab, N, reinterpret_cast<__nv_bfloat16*>(resid),
      reinterpret_cast<const __nv_bfloat16*>(gamma), eps, reinterpret_cast<__nv_bfloat16*>(normed), hist, hist_ld,
      pos, seq_lens, budget_ns);
}
