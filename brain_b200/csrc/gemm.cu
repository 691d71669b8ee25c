// Dense bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   C[M,N] = alpha * op(A)[M,K] * op(B)[K,N]  (+ beta * C_old) (+ bias[N]) (+ R[M,N])
//
// op(A): A stored [M,K] row-major ("K-major") or [K,M] row-major ("M-major").
// op(B): B stored [N,K] row-major ("K-major", i.e. a PyTorch Linear weight) or [K,N] ("N-major").
// These four combinations cover Linear forward (x W^T), data-gradient (dy W) and weight-gradient
// (dy^T x) without any transpose copies: the tensor core reads MN-major shared-memory tiles directly.
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: cp.async.bulk.tensor 2-D tiles (SWIZZLE_128B) into a S-stage ring.
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM
//               accumulator, tcgen05.commit frees the smem stage; TMEM is double-buffered so the
//               epilogue of tile i overlaps the main loop of tile i+1. Warp 1 also owns TMEM alloc.
//   warps 2..5  epilogue: tcgen05.ld 32x32b -> registers -> alpha/beta/bias/residual -> bf16/f32.
// Every wait is bounded (globaltimer); a timeout records a status code and all roles drain and
// return, releasing TMEM. Every TMA load fills only the issuing CTA's own shared memory.
//
// Reference parity: brain-core `matmul` / `blas::gemm` (crates/brain-core/src/tensor/arithmetic.rs:174,
// crates/brain-core/src/tensor/blas.rs:227) compute the same product in f64 on the CPU.
#include "common.cuh"

#include <mutex>
#include <unordered_map>

using namespace brain;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 B = one swizzle row
constexpr int kThreads = 192;
constexpr int kGroupM = 16;  // tile rasterisation group (L2 reuse)

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;
  void* C;
  int64_t ldc;
  int c_f32;
  int accumulate;
  float alpha, beta;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* R;
  int64_t ldr;
  // Output push over NVLink (tensor-parallel GEMM -> reduce-scatter / all-reduce): row gm goes to
  // slot `push_rank` of the receive buffer of rank gm / push_chunk_rows (mode 1) or of every rank
  // (mode 2), at row gm % push_chunk_rows (mode 1) or gm (mode 2). bf16 output only.
  int push;
  int push_world, push_rank;
  int push_chunk_rows;
  int64_t push_slot_elems;
  __nv_bfloat16* push_dst[8];
  // CTA-pair kernel: the pushed rows leave through the swizzled staging buffer, each warp writing its
  // 32 rows x 128 B with coalesced 16-byte stores (4 rows of 128 B per instruction), and tile rows are
  // visited from owner push_rank + 1 on (push_rot = that shift in tile rows), so at any time the ranks
  // push to different owners and a rank's own rows come last
  int push_stage, push_rot;
  // CTA-pair kernel: the output tile leaves through shared memory and TMA stores (tmC) instead of
  // per-thread row stores
  int tma_store;
  // NeoX RoPE on the first rope_cols output columns (q and k heads of a fused QKV projection, head dim
  // rope_hd in {64, 128}); row r is token (r % rope_S) + rope_off; rope_cs f32 [positions, rope_hd]
  // (cos | sin halves). TMA-store epilogue only.
  const float* rope_cs;
  int rope_cols, rope_hd, rope_S, rope_off;
  // Split-K (CTA-pair kernel, TMA-store epilogue): work unit t covers output tile t % (tiles_m * tiles_n)
  // over k-blocks [s * kb_split, (s + 1) * kb_split) with s = t / (tiles_m * tiles_n); its raw f32 sums go
  // to rows [s * split_rows, ...) of the workspace C, and a second kernel adds the slices in order.
  int splits, kb_split, split_rows;
  // CTA-pair TMA-store epilogue with a bf16 output: the residual tile arrives by TMA (extra map tmE) into
  // per-warp swizzled buffers one 64-column unit ahead, instead of per-row global loads. r_op 0 adds it;
  // r_op 1 multiplies the product by gelu'(R) (the data gradient of a GELU MLP's first layer, R = its
  // pre-activation)
  int r_tma, r_op;
  // dual output (CTA-pair TMA-store, bf16): C = the product (+ bias) and a second matrix (map tmE, same
  // shape) = gelu(C): the first layer of a GELU MLP keeps its pre-activation and feeds the second layer
  int dual_gelu;
  // row-wise scaled fp8 operands (CTA-pair kernel with F8 = 1): the product is multiplied by
  // row_scale[m] * col_scale[n] instead of alpha
  const float* row_scale;
  const float* col_scale;
};

template <int BN, int STAGES>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  // full[S], empty[S], tmem_full[2], tmem_empty[2], drain[1]; then tmem base + abort flag
  static constexpr int TOTAL = BAR_OFFSET + (2 * STAGES + 5) * 8 + 16 + 1024 /*alignment slack*/;
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  int group_size = kGroupM * tiles_n;
  int group = t / group_size;
  int first_m = group * kGroupM;
  int gm = min(tiles_m - first_m, kGroupM);
  int r = t - group * group_size;
  tm = first_m + r % gm;
  tn = r / gm;
}

// Work unit t -> output tile coordinates, k-block range and split index (split-K or a plain tile).
__device__ __forceinline__ void unit_coords(const GemmArgs& a, int t, int num_kb, int& tm, int& tn, int& kb0,
                                            int& kb1, int& split) {
  split = 0;
  kb0 = 0;
  kb1 = num_kb;
  if (a.splits > 1) {
    const int per = a.tiles_m * a.tiles_n;
    split = t / per;
    t -= split * per;
    kb0 = split * a.kb_split;
    kb1 = min(num_kb, kb0 + a.kb_split);
  }
  tile_coords(t, a.tiles_m, a.tiles_n, tm, tn);
  if (a.push_rot) tm = (tm + a.push_rot) % a.tiles_m;
}

__device__ __forceinline__ void store_chunk_at(const GemmArgs& args, int gm, int gn0, const uint32_t* r, void* cbase,
                                               int64_t crow);

// v[j] += bias[gn0 + j] for 32 columns: one 16-byte load per 8 columns when the row chunk is whole and
// aligned (every lane of a warp reads the same address: a broadcast), else per column within N.
__device__ __forceinline__ void add_bias32(const GemmArgs& args, int gn0, bool full, float* v) {
  const __nv_bfloat16* bp = args.bias + gn0;
  if (full && ((reinterpret_cast<uintptr_t>(bp) & 15) == 0)) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float bv[8];
      load8(bp + j, bv);
#pragma unroll
      for (int u = 0; u < 8; ++u) v[j + u] += bv[u];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (gn0 + j < args.N) v[j] += __bfloat162float(bp[j]);
  }
}

// v = acc * alpha, or acc * row_scale[gm] * col_scale[n] for row-wise scaled fp8 operands (the column
// scales as 16-byte loads when the 32 columns are whole and aligned; every lane reads the same address).
__device__ __forceinline__ void scale32(const GemmArgs& args, int gm, int gn0, const uint32_t* r, float* v) {
  if (!args.row_scale) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * args.alpha;
    return;
  }
  const float rs = gm < args.M ? __ldg(args.row_scale + gm) : 0.f;
  const float* cs = args.col_scale + gn0;
  if (gn0 + 32 <= args.N && (reinterpret_cast<uintptr_t>(cs) & 15) == 0) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + j));
      v[j] = __uint_as_float(r[j]) * rs * c4.x;
      v[j + 1] = __uint_as_float(r[j + 1]) * rs * c4.y;
      v[j + 2] = __uint_as_float(r[j + 2]) * rs * c4.z;
      v[j + 3] = __uint_as_float(r[j + 3]) * rs * c4.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gn0 + j < args.N ? __uint_as_float(r[j]) * rs * __ldg(cs + j) : 0.f;
  }
}

// alpha, bias, residual and beta * C_old for one row x 32 columns (C_old read at row gm of C).
__device__ __forceinline__ void epi_math(const GemmArgs& args, int gm, int gn0, const uint32_t* r, float* v,
                                         bool skip_r = false) {
  scale32(args, gm, gn0, r, v);
  if (gm >= args.M) return;
  const bool full = gn0 + 32 <= args.N;
  if (args.bias) add_bias32(args, gn0, full, v);
  if (args.R && !skip_r) {
    const __nv_bfloat16* rp = args.R + (int64_t)gm * args.ldr + gn0;
    if (full && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        float rv[8];
        load8(rp + j, rv);
#pragma unroll
        for (int u = 0; u < 8; ++u) v[j + u] += rv[u];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gn0 + j < args.N) v[j] += __bfloat162float(rp[j]);
    }
  }
  if (args.accumulate) {
    if (args.c_f32) {
      const float* cp = reinterpret_cast<const float*>(args.C) + (int64_t)gm * args.ldc + gn0;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (full || gn0 + j < args.N) v[j] += args.beta * cp[j];
    } else {
      const __nv_bfloat16* cp = reinterpret_cast<const __nv_bfloat16*>(args.C) + (int64_t)gm * args.ldc + gn0;
      if (full && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float old[8];
          load8(cp + j, old);
#pragma unroll
          for (int u = 0; u < 8; ++u) v[j + u] += args.beta * old[u];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (gn0 + j < args.N) v[j] += args.beta * __bfloat162float(cp[j]);
      }
    }
  }
}

// Epilogue for one row x 32 columns of f32 accumulator: alpha, bias, residual, beta * C_old, store
// (or push to the owning ranks' receive buffers).
__device__ __forceinline__ void store_chunk(const GemmArgs& args, int gm, int gn0, const uint32_t* r) {
  if (!args.push) {
    store_chunk_at(args, gm, gn0, r, args.C, gm);
    return;
  }
  if (args.push == 1) {
    const int j = gm / args.push_chunk_rows;
    store_chunk_at(args, gm, gn0, r, args.push_dst[j] + (int64_t)args.push_rank * args.push_slot_elems,
                   gm - (int64_t)j * args.push_chunk_rows);
  } else {
    for (int j = 0; j < args.push_world; ++j) {
      const int dst = (args.push_rank + 1 + j) % args.push_world;  // stagger the peers
      store_chunk_at(args, gm, gn0, r, args.push_dst[dst] + (int64_t)args.push_rank * args.push_slot_elems, gm);
    }
  }
}

__device__ __forceinline__ void store_chunk_at(const GemmArgs& args, int gm, int gn0, const uint32_t* r, void* cbase,
                                               int64_t crow) {
  float v[32];
  scale32(args, gm, gn0, r, v);
  const bool full = gn0 + 32 <= args.N;
  if (args.bias) add_bias32(args, gn0, full, v);
  if (args.R) {
    const __nv_bfloat16* rp = args.R + (int64_t)gm * args.ldr + gn0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full || gn0 + j < args.N) v[j] += __bfloat162float(rp[j]);
  }
  if (args.c_f32) {
    float* cp = reinterpret_cast<float*>(cbase) + crow * args.ldc + gn0;
    if (full && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        if (args.accumulate) {
          float4 old = *reinterpret_cast<const float4*>(cp + j);
          o.x += args.beta * old.x; o.y += args.beta * old.y; o.z += args.beta * old.z; o.w += args.beta * old.w;
        }
        *reinterpret_cast<float4*>(cp + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gn0 + j < args.N) cp[j] = v[j] + (args.accumulate ? args.beta * cp[j] : 0.f);
    }
  } else {
    __nv_bfloat16* cp = reinterpret_cast<__nv_bfloat16*>(cbase) + crow * args.ldc + gn0;
    if (full && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        if (args.accumulate) {
          float old[8];
          load8(cp + j, old);
#pragma unroll
          for (int u = 0; u < 8; ++u) v[j + u] += args.beta * old[u];
        }
        store8(cp + j, v + j);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (gn0 + j < args.N) {
          float o = v[j] + (args.accumulate ? args.beta * __bfloat162float(cp[j]) : 0.f);
          cp[j] = __float2bfloat16_rn(o);
        }
      }
    }
  }
}

template <int BN, int STAGES, int A_MN, int B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   GemmArgs args) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_base = sbase + S::BAR_OFFSET;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::BAR_OFFSET + (2 * STAGES + 5) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  constexpr uint32_t kTmemCols = 2 * BN;  // double-buffered f32 accumulator (power of two >= 32)
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (args.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, args.tiles_m, args.tiles_n, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (!mbar_wait(empty_bar(s), (round & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 10, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = sbase + s * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
          mbar_arrive_expect_tx(full_bar(s), S::STAGE_BYTES);
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(&tmA, sa + j * (64 * BK * 2), full_bar(s), m0 + 64 * j, k0);
          } else {
            tma_load_2d(&tmA, sa, full_bar(s), k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(&tmB, sb + j * (64 * BK * 2), full_bar(s), n0 + 64 * j, k0);
          } else {
            tma_load_2d(&tmB, sb, full_bar(s), k0, n0);
          }
        }
      }
      if (!ok) {
        // Drain: let the copies already issued land before the CTA exits.
        uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
        for (uint32_t j = first; j < it; ++j) {
          uint32_t s = j % STAGES, round = j / STAGES;
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full_bar(s), round & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, BN, 1u, (uint32_t)A_MN, (uint32_t)B_MN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      bool issued = false;
      for (int t = blockIdx.x; t < args.num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_round = (uint32_t)(local >> 1);
        if (!mbar_wait(tempty_bar(acc), (acc_round & 1) ^ 1, BRAIN_ERR_TIMEOUT_ACC, 20, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (!mbar_wait(full_bar(s), round & 1, BRAIN_ERR_TIMEOUT_FULL, 21, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t adesc = A_MN ? smem_desc_sw128(sa + kk * 2048, 64 * BK * 2, 1024)
                                  : smem_desc_sw128(sa + kk * 32, 16, 1024);
            uint64_t bdesc = B_MN ? smem_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                  : smem_desc_sw128(sb + kk * 32, 16, 1024);
            tc_mma_f16(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued = true;
          tc_commit(empty_bar(s));  // smem stage free once these MMAs have read it
        }
        if (!ok) break;
        tc_commit(tfull_bar(acc));  // accumulator ready for the epilogue
      }
      if (!ok && issued) {
        // Drain outstanding tensor-core work before the CTA releases TMEM.
        tc_commit(drain_bar);
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain_bar, 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ------------------------------- epilogue (warps 2..5) -------------------------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < args.num_tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_round = (uint32_t)(local >> 1);
      if (!mbar_wait(tfull_bar(acc), acc_round & 1, BRAIN_ERR_TIMEOUT_ACC, 30, abort_flag)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(t, args.tiles_m, args.tiles_n, tm, tn);
      const int gm = tm * BM + row_in_tile;
      const int n0 = tn * BN;
      const bool row_ok = gm < args.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld32(tmem_base + (uint32_t)(acc * BN + c * 32) + ((uint32_t)(q * 32) << 16), r);
        tc_wait_ld();
        const int gn0 = n0 + c * 32;
        if (row_ok && gn0 < args.N) store_chunk(args, gm, gn0, r);
        __syncwarp();
      }
      if (args.push) __threadfence_system();  // pushed rows visible to peers before the next barrier
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// CTA-pair variant: a cluster of 2 CTAs computes one 256 x 256 tile with tcgen05.mma.cta_group::2
// issued by CTA 0. Each CTA stages its own 128 rows of A and its own 128 columns of B (32 KB per
// stage), so an SM reads 8 KB of operands per 256x256x16 pair instruction instead of 12 KB per
// 128x256x16 single-CTA one; the tensor core, not shared-memory bandwidth, becomes the limit.
// Both CTAs' TMA copies complete on CTA 0's stage barrier; CTA 0's commits arrive on the stage /
// accumulator barriers of both CTAs (one commit per CTA address); each CTA's epilogue drains its
// own 128 TMEM lanes and releases the accumulator on CTA 0's barrier.
// ---------------------------------------------------------------------------------------------
constexpr int kPairStages = 5;
struct PairSmem {
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = 128 * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // output staging: per epilogue warp two 4 KB buffers of 32 rows x 128 B (128-byte swizzle); then per warp
  // two 4 KB residual buffers (same layout) filled by TMA
  static constexpr int EPI_OFFSET = kPairStages * STAGE_BYTES;
  static constexpr int EPI_BYTES = 4 * 2 * 4096;
  static constexpr int RES_OFFSET = EPI_OFFSET + EPI_BYTES;
  static constexpr int RES_BYTES = 4 * 2 * 4096;
  static constexpr int BAR_OFFSET = RES_OFFSET + RES_BYTES;
  // full[S], empty[S], tmem_full[2], tmem_empty[2], drain, res_full[4 warps][2]
  static constexpr int NBAR = 2 * kPairStages + 5 + 8;
  static constexpr int TOTAL = BAR_OFFSET + NBAR * 8 + 16 + 1024;
  static_assert(TOTAL <= 232448, "more dynamic shared memory than one CTA may use");
};

// F8 = 1: e4m3 operands (K-major only) through tcgen05.mma kind::f8f6f4. A K block is then 128 fp8 =
// the same 128-byte swizzle row as 64 bf16, and each MMA still consumes 32 bytes of K (32 fp8 instead of
// 16 bf16), so shared-memory layouts, descriptors and stage sizes are those of the bf16 kernel.
template <int A_MN, int B_MN, int F8 = 0>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmE, GemmArgs args) {
  using S = PairSmem;
  constexpr int ST = kPairStages;
  constexpr int TN = 256;  // pair tile: 256 x 256
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_base = sbase + S::BAR_OFFSET;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (ST + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * ST + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * ST + 2 + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * ST + 4);
  auto res_bar = [&](int q, int slot) { return bar_base + 8u * (2 * ST + 5 + 2 * q + slot); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::BAR_OFFSET + S::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t cta = cluster_ctarank();
  const bool leader = cta == 0;
  const int pid = blockIdx.x / 2, npairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 256);  // 128 epilogue threads of each CTA arrive on CTA 0's barrier
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < 8; ++i) mbar_init(res_bar(i / 2, i % 2), 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (args.tma_store && !args.push_stage) prefetch_tmap(&tmC);
    if (args.r_tma || args.dual_gelu) prefetch_tmap(&tmE);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before anyone signals a peer
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  static_assert(!F8 || (A_MN == 0 && B_MN == 0), "fp8 operands are K-major");
  constexpr int KE = F8 ? 2 * BK : BK;  // elements per K block (128 bytes either way)
  const int num_kb = (args.K + KE - 1) / KE;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs): own A rows and own B columns
      uint32_t it = 0;
      bool ok = true;
      for (int t = pid; t < args.num_tiles && ok; t += npairs) {
        int tm, tn, kb0, kb1, split;
        unit_coords(args, t, num_kb, tm, tn, kb0, kb1, split);
        const int m0 = tm * 256 + (int)cta * 128, n0 = tn * TN + (int)cta * 128;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % ST;
          const uint32_t round = it / ST;
          if (!mbar_wait(empty_bar(s), (round & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 40, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = sbase + s * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
          const uint32_t fb = mapa_shared(full_bar(s), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * S::STAGE_BYTES);
          const int k0 = kb * KE;
          if (A_MN) {
            tma_load_2d_pair(&tmA, sa, fb, m0, k0);
            tma_load_2d_pair(&tmA, sa + 64 * BK * 2, fb, m0 + 64, k0);
          } else {
            tma_load_2d_pair(&tmA, sa, fb, k0, m0);
          }
          if (B_MN) {
            tma_load_2d_pair(&tmB, sb, fb, n0, k0);
            tma_load_2d_pair(&tmB, sb + 64 * BK * 2, fb, n0 + 64, k0);
          } else {
            tma_load_2d_pair(&tmB, sb, fb, k0, n0);
          }
        }
      }
      if (!ok && leader) {
        uint32_t first = it > (uint32_t)ST ? it - ST : 0;
        for (uint32_t j = first; j < it; ++j) {
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full_bar(j % ST), (j / ST) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (CTA 0 only)
      constexpr uint32_t idesc = F8 ? idesc_f8(256, TN, 0u, 0u, 0u, 0u)
                                    : idesc_f16(256, TN, 1u, (uint32_t)A_MN, (uint32_t)B_MN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true, issued = false;
      for (int t = pid; t < args.num_tiles && ok; t += npairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_round = (uint32_t)(local >> 1);
        if (!mbar_wait(tempty_bar(acc), (acc_round & 1) ^ 1, BRAIN_ERR_TIMEOUT_ACC, 50, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * TN);
        int tm_, tn_, kb0, kb1, split_;
        unit_coords(args, t, num_kb, tm_, tn_, kb0, kb1, split_);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % ST;
          if (!mbar_wait(full_bar(s), (it / ST) & 1, BRAIN_ERR_TIMEOUT_FULL, 51, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t adesc = A_MN ? smem_desc_sw128(sa + kk * 2048, 64 * BK * 2, 1024)
                                  : smem_desc_sw128(sa + kk * 32, 16, 1024);
            uint64_t bdesc = B_MN ? smem_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                  : smem_desc_sw128(sb + kk * 32, 16, 1024);
            if constexpr (F8)
              tc_mma_f8_pair(d_tmem, adesc, bdesc, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
            else
              tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          issued = true;
          tc_commit_pair(empty_bar(s));
          tc_commit_pair(mapa_shared(empty_bar(s), 1));
        }
        if (!ok) break;
        tc_commit_pair(tfull_bar(acc));
        tc_commit_pair(mapa_shared(tfull_bar(acc), 1));
      }
      if (!ok && issued) {
        tc_commit_pair(drain_bar);
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain_bar, 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs)
    const int q = warp & 3;
    const int row_in_tile = (int)cta * 128 + q * 32 + lane;
    const uint32_t stg = sbase + S::EPI_OFFSET + (uint32_t)q * 8192u;  // this warp's two staging buffers
    int ebuf = 0;
    int local = 0;
    // residual by TMA: this warp's stream of (tile, 64-column unit) boxes, loaded one unit ahead into two
    // slots; rc units consumed, r_issued units requested
    const uint32_t rbase = sbase + S::RES_OFFSET + (uint32_t)q * 8192u;
    int rc = 0, r_issued = 0, r_done = 0;
    bool r_ok = true;
    auto res_units = [&](int tt) {
      int tm_, tn_, k0_, k1_, sp_;
      unit_coords(args, tt, num_kb, tm_, tn_, k0_, k1_, sp_);
      return min(TN / 64, (args.N - tn_ * TN + 63) / 64);
    };
    auto res_issue = [&](int tt, int uu) {  // lane 0
      int tm_, tn_, k0_, k1_, sp_;
      unit_coords(args, tt, num_kb, tm_, tn_, k0_, k1_, sp_);
      const int slot = r_issued & 1;
      mbar_arrive_expect_tx(res_bar(q, slot), 4096);
      tma_load_2d(&tmE, rbase + (uint32_t)slot * 4096u, res_bar(q, slot), tn_ * TN + uu * 64,
                  tm_ * 256 + (int)cta * 128 + q * 32);
    };
    if (args.r_tma && pid < args.num_tiles) {
      if (lane == 0) res_issue(pid, 0);
      ++r_issued;
    }
    for (int t = pid; t < args.num_tiles; t += npairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_round = (uint32_t)(local >> 1);
      if (!mbar_wait(tfull_bar(acc), acc_round & 1, BRAIN_ERR_TIMEOUT_ACC, 60, abort_flag)) break;
      tc_fence_after();
      int tm, tn, kb0_, kb1_, split;
      unit_coords(args, t, num_kb, tm, tn, kb0_, kb1_, split);
      const int gm = tm * 256 + row_in_tile;
      const int n0 = tn * TN;
      const bool row_ok = gm < args.M;
      const uint32_t tm_row = tmem_base + (uint32_t)(acc * TN) + ((uint32_t)(q * 32) << 16);
      if (args.tma_store) {
        // 128 B of this row per unit (64 bf16 or 32 f32 columns): registers -> swizzled staging buffer
        // -> one TMA store of the warp's 32 rows; the two buffers alternate, and a buffer is rewritten
        // only after the store issued from it two units earlier has read it.
        const int cols = args.c_f32 ? 32 : 64;
        const int row0 = split * args.split_rows + tm * 256 + (int)cta * 128 + q * 32;
        const int rpos = args.rope_cs && row_ok ? gm % args.rope_S + args.rope_off : 0;
        // RoPE: rotate 32 pairs (x1 at TMEM column c1, x2 at c2; pair index j0 in the head) into bf16 words
        auto rope32 = [&](int c1, int c2, int j0, uint32_t* w1, uint32_t* w2) {
          uint32_t r1[32], r2[32];
          tmem_ld32(tm_row + (uint32_t)c1, r1);
          tmem_ld32(tm_row + (uint32_t)c2, r2);
          tc_wait_ld();
          float v1[32], v2[32];
          epi_math(args, gm, n0 + c1, r1, v1);
          epi_math(args, gm, n0 + c2, r2, v2);
          const float4* cp = reinterpret_cast<const float4*>(args.rope_cs + (int64_t)rpos * args.rope_hd + j0);
          const float4* sp = reinterpret_cast<const float4*>(args.rope_cs + (int64_t)rpos * args.rope_hd +
                                                             args.rope_hd / 2 + j0);
#pragma unroll
          for (int k4 = 0; k4 < 8; ++k4) {
            const float4 c4 = __ldg(cp + k4), s4 = __ldg(sp + k4);
            const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
              const int k = k4 * 4 + e;
              const float a0 = v1[k] * cv[e] - v2[k] * sv[e], a1 = v1[k + 1] * cv[e + 1] - v2[k + 1] * sv[e + 1];
              const float b0 = v2[k] * cv[e] + v1[k] * sv[e], b1 = v2[k + 1] * cv[e + 1] + v1[k + 1] * sv[e + 1];
              __nv_bfloat162 ha = __floats2bfloat162_rn(a0, a1), hb = __floats2bfloat162_rn(b0, b1);
              w1[k / 2] = *reinterpret_cast<uint32_t*>(&ha);
              w2[k / 2] = *reinterpret_cast<uint32_t*>(&hb);
            }
          }
        };
        auto stage_chunks = [&](uint32_t buf, int c0, const uint32_t* w16) {  // 4 chunks of 16 B from chunk c0
#pragma unroll
          for (int c = 0; c < 4; ++c)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(buf + (uint32_t)lane * 128u +
                                                                             (uint32_t)(((c0 + c) ^ (lane & 7)) << 4)),
                         "r"(w16[4 * c]), "r"(w16[4 * c + 1]), "r"(w16[4 * c + 2]), "r"(w16[4 * c + 3])
                         : "memory");
        };
#pragma unroll 1
        for (int u = 0; u < TN / cols; ++u) {
          if (n0 + u * cols >= args.N) break;
          if (args.rope_cs && n0 + u * cols < args.rope_cols) {
            // a rotated head: pairs (d, d + hd/2) meet in registers before the store
            const uint32_t bufA = stg + (uint32_t)ebuf * 4096u, bufB = stg + (uint32_t)(ebuf ^ 1) * 4096u;
            uint32_t w1[16], w2[16];
            if (args.rope_hd == 128) {  // units u (first half) and u + 1 (second half) of one head
              if (lane == 0) tma_store_wait_read<0>();
              __syncwarp();
#pragma unroll 1
              for (int h2 = 0; h2 < 2; ++h2) {
                rope32(u * 64 + h2 * 32, u * 64 + 64 + h2 * 32, h2 * 32, w1, w2);
                stage_chunks(bufA, h2 * 4, w1);
                stage_chunks(bufB, h2 * 4, w2);
              }
              fence_proxy_async();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmC, bufA, n0 + u * 64, row0);
                tma_store_commit();
                tma_store_2d(&tmC, bufB, n0 + (u + 1) * 64, row0);
                tma_store_commit();
              }
              ++u;  // the head's second unit is done too; ebuf is unchanged (both buffers used once)
            } else {  // head dim 64: one unit, halves of 32 columns
              rope32(u * 64, u * 64 + 32, 0, w1, w2);
              if (lane == 0) tma_store_wait_read<1>();
              __syncwarp();
              stage_chunks(bufA, 0, w1);
              stage_chunks(bufA, 4, w2);
              fence_proxy_async();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmC, bufA, n0 + u * 64, row0);
                tma_store_commit();
              }
              ebuf ^= 1;
            }
            continue;
          }
          uint32_t w[32];
          if (args.c_f32) {
            uint32_t r[32];
            tmem_ld32(tm_row + (uint32_t)(u * 32), r);
            tc_wait_ld();
            float v[32];
            epi_math(args, gm, n0 + u * 32, r, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j]);
          } else {
            uint32_t rslot = 0;
            if (args.r_tma) {
              // request the next unit's residual box (this tile's next unit or the next tile's first) into
              // the other slot, whose previous box every lane has read by now
              int nt = t, nu = u + 1;
              if (nu >= res_units(t)) {
                nt = t + npairs;
                nu = 0;
              }
              __syncwarp();
              if (nt < args.num_tiles && r_ok) {
                if (lane == 0) {
                  fence_proxy_async();
                  res_issue(nt, nu);
                }
                ++r_issued;
              }
              rslot = rbase + (uint32_t)(rc & 1) * 4096u;
              if (r_ok) r_ok = mbar_wait(res_bar(q, rc & 1), (rc >> 1) & 1, BRAIN_ERR_TIMEOUT_FULL, 61, abort_flag);
              if (r_ok) r_done = rc + 1;
              ++rc;
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t r[32];
              tmem_ld32(tm_row + (uint32_t)(u * 64 + h * 32), r);
              tc_wait_ld();
              float v[32];
              epi_math(args, gm, n0 + u * 64 + h * 32, r, v, args.r_tma != 0);
              if (args.r_tma) {
                // this row's 32 residual columns: 4 swizzled 16-byte pieces of the 128-byte row
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                  uint32_t x0, x1, x2, x3;
                  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                               : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3)
                               : "r"(rslot + (uint32_t)lane * 128u + (uint32_t)(((h * 4 + cc) ^ (lane & 7)) << 4)));
                  const uint32_t xs[4] = {x0, x1, x2, x3};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xs[e]));
                    if (args.r_op == 0) {
                      v[cc * 8 + 2 * e] += f.x;
                      v[cc * 8 + 2 * e + 1] += f.y;
                    } else {
                      v[cc * 8 + 2 * e] *= gelu_tanh_grad_fast(f.x);
                      v[cc * 8 + 2 * e + 1] *= gelu_tanh_grad_fast(f.y);
                    }
                  }
                }
              }
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                w[h * 16 + j] = *reinterpret_cast<uint32_t*>(&b2);
              }
              if (args.dual_gelu) {
                // gelu of the bf16-rounded pre-activation (what the backward pass reads back), staged in
                // this unit's slot of the residual buffers and stored by a second TMA store
                uint32_t g[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[h * 16 + j]));
                  __nv_bfloat162 b2 = __floats2bfloat162_rn(gelu_tanh_fast(f.x), gelu_tanh_fast(f.y));
                  g[j] = *reinterpret_cast<uint32_t*>(&b2);
                }
                if (h == 0 && lane == 0) tma_store_wait_read<1>();
                __syncwarp();
                const uint32_t gb = rbase + (uint32_t)ebuf * 4096u + (uint32_t)lane * 128u;
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(gb + (uint32_t)(((h * 4 + c) ^ (lane & 7)) << 4)),
                               "r"(g[4 * c]), "r"(g[4 * c + 1]), "r"(g[4 * c + 2]), "r"(g[4 * c + 3])
                               : "memory");
              }
            }
          }
          if (lane == 0 && !args.push_stage) tma_store_wait_read<1>();
          __syncwarp();
          const uint32_t sb = stg + (uint32_t)ebuf * 4096u + (uint32_t)lane * 128u;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sb + (uint32_t)((c ^ (lane & 7)) << 4)),
                         "r"(w[4 * c]), "r"(w[4 * c + 1]), "r"(w[4 * c + 2]), "r"(w[4 * c + 3])
                         : "memory");
          if (args.push_stage) {
            // the warp's 32 staged rows to their owners: lane l takes 16-byte piece l % 8 of rows l / 8 + 4 i
            __syncwarp();
            const uint32_t buf = stg + (uint32_t)ebuf * 4096u;
            const int gn = n0 + u * cols + (lane & 7) * 8;
#pragma unroll 2
            for (int i = 0; i < 8; ++i) {
              const int rr = i * 4 + (lane >> 3);
              const int gmr = row0 + rr;
              if (gmr >= args.M || gn >= args.N) continue;
              uint32_t x0, x1, x2, x3;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3)
                           : "r"(buf + (uint32_t)rr * 128u + (uint32_t)((((lane & 7) ^ (rr & 7))) << 4)));
              const uint4 v4 = make_uint4(x0, x1, x2, x3);
              if (args.push == 1) {
                const int j = gmr / args.push_chunk_rows;
                __nv_bfloat16* d = args.push_dst[j] + (int64_t)args.push_rank * args.push_slot_elems +
                                   (int64_t)(gmr - j * args.push_chunk_rows) * args.ldc + gn;
                *reinterpret_cast<uint4*>(d) = v4;
              } else {
                for (int jj = 0; jj < args.push_world; ++jj) {
                  const int dd = (args.push_rank + 1 + jj) % args.push_world;
                  __nv_bfloat16* d = args.push_dst[dd] + (int64_t)args.push_rank * args.push_slot_elems +
                                     (int64_t)gmr * args.ldc + gn;
                  *reinterpret_cast<uint4*>(d) = v4;
                }
              }
            }
            __syncwarp();  // every lane has read the buffer before a later unit rewrites it
            ebuf ^= 1;
            continue;
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, stg + (uint32_t)ebuf * 4096u, n0 + u * cols, row0);
            if (args.dual_gelu) tma_store_2d(&tmE, rbase + (uint32_t)ebuf * 4096u, n0 + u * cols, row0);
            tma_store_commit();
          }
          ebuf ^= 1;
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < TN / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(tm_row + (uint32_t)(c * 32), r);
          tc_wait_ld();
          const int gn0 = n0 + c * 32;
          if (row_ok && gn0 < args.N) store_chunk(args, gm, gn0, r);
          __syncwarp();
        }
      }
      if (args.push) __threadfence_system();
      tc_fence_before();
      mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
    }
    if (args.tma_store && lane == 0) tma_store_wait_all();
    // residual boxes requested and not consumed (an abort): let them land before the CTA exits
    for (int j = r_done; j < r_issued; ++j) {
      uint64_t t0 = globaltimer();
      while (!mbar_try_wait(res_bar(q, j & 1), (j >> 1) & 1) && globaltimer() - t0 < 100000000ull) {
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its pair partner may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// Tensor-map cache: encoding is cheap but not free, and training re-uses the same operands.
struct MapKey {
  uintptr_t ptr;
  uint64_t d0, d1, s1;
  uint32_t b0, b1;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && d0 == o.d0 && d1 == o.d1 && s1 == o.s1 && b0 == o.b0 && b1 == o.b1;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = k.ptr * 0x9E3779B97F4A7C15ull;
    h ^= (k.d0 + 0x632BE59BD9B4E019ull + (h << 6) + (h >> 2));
    h ^= (k.d1 * 31 + k.s1 * 131 + k.b0 * 7 + k.b1 + (h << 6) + (h >> 2));
    return h;
  }
};

bool get_map_2d(CUtensorMap* out, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                uint32_t box_inner, uint32_t box_outer, CUtensorMapDataType dt, int elem_bytes) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{reinterpret_cast<uintptr_t>(ptr) ^ ((uintptr_t)dev << 56) ^ ((uintptr_t)dt << 48), inner, outer, ld_elems,
             box_inner, box_outer};
  {
    std::lock_guard<std::mutex> g(mu);
    auto itr = cache.find(key);
    if (itr != cache.end()) {
      *out = itr->second;
      return true;
    }
  }
  uint64_t dims[2] = {inner, outer};
  uint64_t strides[1] = {ld_elems * (uint64_t)elem_bytes};
  uint32_t box[2] = {box_inner, box_outer};
  if (!brain_host::encode_tiled(out, dt, 2, const_cast<void*>(ptr), dims, strides, box,
                                CU_TENSOR_MAP_SWIZZLE_128B))
    return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache[key] = *out;
  return true;
}

// Tensor map of the output C [M, N] (row stride ldc) as boxes of 32 rows x 128 B for the TMA-store
// epilogue; false when that epilogue cannot be used (push modes, unaligned base or row stride).
bool output_map(CUtensorMap* out, const GemmArgs& a) {
  if (a.push) return false;
  const int esz = a.c_f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(a.C) & 15) || ((a.ldc * esz) % 16) || a.ldc < a.N) return false;
  return get_map_2d(out, a.C, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.ldc, (uint32_t)(128 / esz), 32,
                    a.c_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, esz);
}

template <int BN, int STAGES, int A_MN, int B_MN>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, cudaStream_t st) {
  using S = Smem<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, A_MN, B_MN>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL);
    attr_set[dev & 63] = true;
  }
  int grid = std::min(a.num_tiles, brain_host::num_sms());
  kern<<<grid, kThreads, S::TOTAL, st>>>(ta, tb, a);
  return (int)cudaGetLastError();
}

template <int A_MN, int B_MN, int F8 = 0>
int launch_tc2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& a,
               cudaStream_t st, const CUtensorMap* tr = nullptr) {
  static const CUtensorMap no_map{};
  auto kern = gemm_tc2_kernel<A_MN, B_MN, F8>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PairSmem::TOTAL);
    attr_set[dev & 63] = true;
  }
  int pairs = std::min(a.num_tiles, brain_host::num_sms() / 2);
  kern<<<2 * pairs, kThreads, PairSmem::TOTAL, st>>>(ta, tb, tc, tr ? *tr : no_map, a);
  return (int)cudaGetLastError();
}

// Simple SIMT fallback for shapes the TMA path cannot describe (unaligned strides). f32 accumulate.
__global__ void gemm_simt_kernel(const __nv_bfloat16* A, int64_t lda, int a_mn, const __nv_bfloat16* B,
                                 int64_t ldb, int b_mn, GemmArgs args) {
  __shared__ float As[32][33];
  __shared__ float Bs[32][33];
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // 32 x 8 threads
  const int m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < args.K; k0 += 32) {
    for (int i = ty; i < 32; i += 8) {
      int m = m0 + i, k = k0 + tx;
      float av = 0.f;
      if (m < args.M && k < args.K) av = __bfloat162float(a_mn ? A[(int64_t)k * lda + m] : A[(int64_t)m * lda + k]);
      As[i][tx] = av;
      int n = n0 + i;
      float bv = 0.f;
      if (n < args.N && k < args.K) bv = __bfloat162float(b_mn ? B[(int64_t)k * ldb + n] : B[(int64_t)n * ldb + k]);
      Bs[i][tx] = bv;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      float b = Bs[tx][kk];
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] += As[ty + 8 * r][kk] * b;
    }
    __syncthreads();
  }
  const int n = n0 + tx;
  if (n >= args.N) return;
  for (int r = 0; r < 4; ++r) {
    int m = m0 + ty + 8 * r;
    if (m >= args.M) continue;
    float v = acc[r] * args.alpha;
    if (args.bias) v += __bfloat162float(args.bias[n]);
    if (args.R) v += __bfloat162float(args.R[(int64_t)m * args.ldr + n]);
    if (args.c_f32) {
      float* cp = reinterpret_cast<float*>(args.C) + (int64_t)m * args.ldc + n;
      *cp = v + (args.accumulate ? args.beta * *cp : 0.f);
    } else {
      __nv_bfloat16* cp = reinterpret_cast<__nv_bfloat16*>(args.C) + (int64_t)m * args.ldc + n;
      *cp = __float2bfloat16_rn(v + (args.accumulate ? args.beta * __bfloat162float(*cp) : 0.f));
    }
  }
}

// Split-K epilogue: C = alpha * sum_s ws[s] (+ bias) (+ R) (+ beta * C), the slices added in index order
// (deterministic). ws slices are f32 [rows >= M, N] with row stride N; four columns per thread.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int64_t slice, int M, int N, void* C,
                                     int64_t ldc, int c_f32, float alpha, int accumulate, float beta,
                                     const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ R,
                                     int64_t ldr) {
  const int n4 = N / 4;
  const int64_t total = (int64_t)M * n4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / n4), n = (int)(i % n4) * 4;
    const float* src = ws + (int64_t)m * N + n;
    float4 acc = *reinterpret_cast<const float4*>(src);
    for (int sp = 1; sp < splits; ++sp) {
      const float4 v = *reinterpret_cast<const float4*>(src + sp * slice);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    float v[4] = {acc.x * alpha, acc.y * alpha, acc.z * alpha, acc.w * alpha};
    if (bias) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] += __bfloat162float(bias[n + j]);
    }
    if (R) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] += __bfloat162float(R[(int64_t)m * ldr + n + j]);
    }
    if (c_f32) {
      float* cp = reinterpret_cast<float*>(C) + (int64_t)m * ldc + n;
#pragma unroll
      for (int j = 0; j < 4; ++j) cp[j] = v[j] + (accumulate ? beta * cp[j] : 0.f);
    } else {
      __nv_bfloat16* cp = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)m * ldc + n;
#pragma unroll
      for (int j = 0; j < 4; ++j) cp[j] = __float2bfloat16_rn(v[j] + (accumulate ? beta * __bfloat162float(cp[j]) : 0.f));
    }
  }
}

}  // namespace

BRAIN_STATUS_READER(gemm)

namespace {
int g_pair_mode = 1;   // 1: CTA-pair kernel for M, N >= 256; 0: single-CTA kernel only
int g_push_stage = 1;  // 1: pushed GEMM rows leave through shared-memory staging (coalesced); 0: per-row stores
}

// Select how the CTA-pair kernel pushes rows to peers (tests compare both); returns the previous mode.
BRAIN_API int brain_gemm_set_push_stage(int mode) {
  const int old = g_push_stage;
  g_push_stage = mode;
  return old;
}

// Select the GEMM kernel family (tests exercise both); returns the previous mode.
BRAIN_API int brain_gemm_set_pair_mode(int mode) {
  const int old = g_pair_mode;
  g_pair_mode = mode;
  return old;
}


namespace {
// A / B tensor maps of the CTA-pair kernel (each CTA stages 128 rows of A and 128 columns of B per k-block).
bool pair_maps(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, int M, int N, int K,
               CUtensorMap* ta, CUtensorMap* tb) {
  bool ok = a_mn ? get_map_2d(ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, BK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2)
                 : get_map_2d(ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, 128, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
  return ok && (b_mn ? get_map_2d(tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK,
                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2)
                     : get_map_2d(tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, 128,
                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2));
}

bool pair_aligned(const void* A, int64_t lda, const void* B, int64_t ldb, int K) {
  return (lda % 8 == 0) && (ldb % 8 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0) &&
         ((reinterpret_cast<uintptr_t>(B) & 15) == 0) && K >= 16;
}
}  // namespace

// Split-K plan for the CTA-pair kernel: returns the number of K slices (1 = no split) and the k-blocks per
// slice. Splitting pays when the output has fewer 256 x 256 tiles than there are SM pairs (weight gradients
// of narrow layers: dW [768, 768] over 12k tokens has 9 tiles for 74 pairs). The cost model counts waves of
// k-block steps (about 0.42 us per 256 x 256 x 64 step on one pair) plus the reduction's launch and its f32
// traffic (each slice written once and read once).
BRAIN_API int brain_gemm_splitk_plan(int M, int N, int K, int* kb_split) {
  const int pairs = brain_host::num_sms() / 2;
  const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
  const int num_kb = (K + BK - 1) / BK;
  if (kb_split) *kb_split = num_kb;
  if (M < 256 || N < 256 || N % 4 != 0 || tiles >= pairs || num_kb < 16) return 1;
  const double step_us = 0.42;
  double best = (double)num_kb * step_us;
  int best_s = 1;
  for (int sp = 2; sp <= 16 && num_kb / sp >= 4; ++sp) {
    const int per = (num_kb + sp - 1) / sp;
    const int used = (num_kb + per - 1) / per;  // slices actually non-empty
    const int waves = (tiles * used + pairs - 1) / pairs;
    const double red_us = 3.0 + 2.0 * used * (double)((M + 255) / 256 * 256) * N * 4 / 6.0e6;
    const double cost = waves * per * step_us + red_us;
    if (cost < best * 0.9) {
      best = cost;
      best_s = used;
      if (kb_split) *kb_split = per;
    }
  }
  if (best_s == 1 && kb_split) *kb_split = num_kb;
  return best_s;
}

namespace {
int gemm_bf16_impl(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, void* C, int64_t ldc,
                   int c_f32, int M, int N, int K, float alpha, int accumulate, float beta, const void* bias,
                   const void* R, int64_t ldr, int force_simt, float* ws, int64_t ws_elems, cudaStream_t stream);
}  // namespace

// C = alpha * op(A) op(B) (+ beta*C if accumulate) (+ bias) (+ R).
//   a_mn = 0: A is [M,K] with row stride lda; a_mn = 1: A is [K,M] with row stride lda.
//   b_mn = 0: B is [N,K] with row stride ldb; b_mn = 1: B is [K,N] with row stride ldb.
//   force_simt: 1 = use the SIMT fallback (tests), 0 = tensor cores when the layout allows.
BRAIN_API int brain_gemm_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, void* C,
                              int64_t ldc, int c_f32, int M, int N, int K, float alpha, int accumulate, float beta,
                              const void* bias, const void* R, int64_t ldr, int force_simt, cudaStream_t stream) {
  return gemm_bf16_impl(A, lda, a_mn, B, ldb, b_mn, C, ldc, c_f32, M, N, K, alpha, accumulate, beta, bias, R, ldr,
                        force_simt, nullptr, 0, stream);
}

// brain_gemm_bf16 with an f32 split-K workspace of ws_elems elements (at least splits * round_up(M, 256) * N
// for the plan of brain_gemm_splitk_plan); without room it runs unsplit.
BRAIN_API int brain_gemm_bf16_ws(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, void* C,
                                 int64_t ldc, int c_f32, int M, int N, int K, float alpha, int accumulate, float beta,
                                 const void* bias, const void* R, int64_t ldr, float* ws, int64_t ws_elems,
                                 cudaStream_t stream) {
  return gemm_bf16_impl(A, lda, a_mn, B, ldb, b_mn, C, ldc, c_f32, M, N, K, alpha, accumulate, beta, bias, R, ldr, 0,
                        ws, ws_elems, stream);
}

namespace {
int gemm_bf16_impl(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn, void* C, int64_t ldc,
                   int c_f32, int M, int N, int K, float alpha, int accumulate, float beta, const void* bias,
                   const void* R, int64_t ldr, int force_simt, float* ws, int64_t ws_elems, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.C = C; a.ldc = ldc; a.c_f32 = c_f32; a.accumulate = accumulate;
  a.alpha = alpha; a.beta = beta;
  a.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  const bool aligned = (lda % 8 == 0) && (ldb % 8 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0) &&
                       ((reinterpret_cast<uintptr_t>(B) & 15) == 0) && K >= 16;
  if (K <= 0) {
    // Degenerate K: result is the epilogue of a zero product; use the SIMT kernel (loops zero times).
    force_simt = 1;
  }
  if (force_simt || !aligned) {
    dim3 grid((N + 31) / 32, (M + 31) / 32);
    gemm_simt_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(A), lda, a_mn,
                                              reinterpret_cast<const __nv_bfloat16*>(B), ldb, b_mn, a);
    return (int)cudaGetLastError();
  }
  if (g_pair_mode && M >= 256 && N >= 256) {
    // CTA-pair kernel: 256 x 256 tiles, each CTA stages 128 rows of A and 128 columns of B
    a.tiles_m = (M + 255) / 256;
    a.tiles_n = (N + 255) / 256;
    a.num_tiles = a.tiles_m * a.tiles_n;
    CUtensorMap ta, tb;
    bool ok = a_mn ? get_map_2d(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, BK,
                                CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2)
                   : get_map_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, 128,
                                CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
    ok = ok && (b_mn ? get_map_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK,
                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2)
                     : get_map_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, 128,
                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2));
    if (!ok) return (int)cudaErrorInvalidValue;
    CUtensorMap tc{};
    int kbs = 0;
    const int splits = ws ? brain_gemm_splitk_plan(M, N, K, &kbs) : 1;
    const int rows = a.tiles_m * 256;
    if (splits > 1 && (int64_t)splits * rows * N <= ws_elems && (reinterpret_cast<uintptr_t>(ws) & 15) == 0) {
      // raw partial sums into the workspace slices, then alpha / bias / residual / beta * C in the reduction
      GemmArgs p = a;
      p.C = ws; p.ldc = N; p.c_f32 = 1; p.accumulate = 0; p.alpha = 1.f; p.beta = 0.f;
      p.bias = nullptr; p.R = nullptr;
      p.M = splits * rows;  // the map spans every slice
      if (output_map(&tc, p)) {
        p.M = M;
        p.tma_store = 1;
        p.splits = splits; p.kb_split = kbs; p.split_rows = rows;
        p.num_tiles = a.num_tiles * splits;
        int rc;
        if (a_mn == 0 && b_mn == 0) rc = launch_tc2<0, 0>(ta, tb, tc, p, stream);
        else if (a_mn == 0 && b_mn == 1) rc = launch_tc2<0, 1>(ta, tb, tc, p, stream);
        else if (a_mn == 1 && b_mn == 0) rc = launch_tc2<1, 0>(ta, tb, tc, p, stream);
        else rc = launch_tc2<1, 1>(ta, tb, tc, p, stream);
        if (rc) return rc;
        const int64_t work = (int64_t)M * (N / 4);
        const int grid = (int)std::min<int64_t>((work + 255) / 256, (int64_t)brain_host::num_sms() * 8);
        splitk_reduce_kernel<<<grid, 256, 0, stream>>>(ws, splits, (int64_t)rows * N, M, N, C, ldc, c_f32, alpha,
                                                       accumulate, beta, a.bias, a.R, ldr);
        return (int)cudaGetLastError();
      }
    }
    a.tma_store = output_map(&tc, a) ? 1 : 0;
    CUtensorMap tr{};
    if (a.tma_store && a.R && !c_f32 && ldr % 8 == 0 && (reinterpret_cast<uintptr_t>(R) & 15) == 0 &&
        get_map_2d(&tr, R, (uint64_t)N, (uint64_t)M, (uint64_t)ldr, 64, 32, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2))
      a.r_tma = 1;
    const CUtensorMap* trp = a.r_tma ? &tr : nullptr;
    if (a_mn == 0 && b_mn == 0) return launch_tc2<0, 0>(ta, tb, tc, a, stream, trp);
    if (a_mn == 0 && b_mn == 1) return launch_tc2<0, 1>(ta, tb, tc, a, stream, trp);
    if (a_mn == 1 && b_mn == 0) return launch_tc2<1, 0>(ta, tb, tc, a, stream, trp);
    return launch_tc2<1, 1>(ta, tb, tc, a, stream, trp);
  }
  const int BN = (N <= 128) ? 128 : 256;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_n = (N + BN - 1) / BN;
  a.num_tiles = a.tiles_m * a.tiles_n;
  CUtensorMap ta, tb;
  bool ok;
  // A operand
  if (a_mn) ok = get_map_2d(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, BK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
  else ok = get_map_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, BM, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
  if (!ok) return (int)cudaErrorInvalidValue;
  if (b_mn) ok = get_map_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
  else ok = get_map_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, (uint32_t)BN, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
  if (!ok) return (int)cudaErrorInvalidValue;
#define BRAIN_GEMM_CASE(BN_, ST_)                                                   \
  if (a_mn == 0 && b_mn == 0) return launch_tc<BN_, ST_, 0, 0>(ta, tb, a, stream); \
  if (a_mn == 0 && b_mn == 1) return launch_tc<BN_, ST_, 0, 1>(ta, tb, a, stream); \
  if (a_mn == 1 && b_mn == 0) return launch_tc<BN_, ST_, 1, 0>(ta, tb, a, stream); \
  return launch_tc<BN_, ST_, 1, 1>(ta, tb, a, stream);
  if (BN == 128) {
    BRAIN_GEMM_CASE(128, 6)
  } else {
    BRAIN_GEMM_CASE(256, 4)
  }
#undef BRAIN_GEMM_CASE
}
}  // namespace

// C [M, N] bf16 = A [M, K] B [N, K]^T with NeoX RoPE applied to the first rope_cols columns in the
// epilogue (a fused QKV projection: q and k heads rotated, v heads stored as they are). Row r is token
// (r % S) + pos_offset; cs f32 [positions, head_dim] (cos | sin halves). Returns cudaErrorNotSupported
// when the CTA-pair TMA-store path cannot run (M or N < 256, N % 256, head_dim not 64/128, alignment);
// the caller then applies the rotation separately.
BRAIN_API int brain_gemm_bf16_rope(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                                   int M, int N, int K, const float* cs, int rope_cols, int head_dim, int S,
                                   int pos_offset, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  if (!g_pair_mode || M < 256 || N < 256 || N % 256 || (head_dim != 64 && head_dim != 128) || rope_cols % 256 ||
      S <= 0 || K < 16 || (lda % 8) || (ldb % 8) || (reinterpret_cast<uintptr_t>(cs) & 15) ||
      ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15))
    return (int)cudaErrorNotSupported;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.C = C; a.ldc = ldc; a.c_f32 = 0; a.accumulate = 0;
  a.alpha = 1.f; a.beta = 0.f;
  a.tiles_m = (M + 255) / 256;
  a.tiles_n = (N + 255) / 256;
  a.num_tiles = a.tiles_m * a.tiles_n;
  a.rope_cs = cs;
  a.rope_cols = rope_cols;
  a.rope_hd = head_dim;
  a.rope_S = S;
  a.rope_off = pos_offset;
  CUtensorMap ta, tb, tc{};
  if (!get_map_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, 128, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2) ||
      !get_map_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, 128, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2) ||
      !output_map(&tc, a))
    return (int)cudaErrorNotSupported;
  a.tma_store = 1;
  return launch_tc2<0, 0>(ta, tb, tc, a, stream);
}

// Tensor-parallel GEMM with the communication in its epilogue, C = A B^T (A [M, K] K-major; B [N, K],
// or [K, N] with b_mn = 1):
//   push_mode 1 : row gm of C goes to slot push_rank of rank (gm / push_chunk_rows)'s receive buffer
//                 push_peers[j] (slot stride push_slot_elems, row gm % push_chunk_rows, stride ldc):
//                 GEMM -> reduce-scatter fusion. push_mode 2: every rank receives every row (-> all-reduce).
//   push_mode 0 : C written locally.
// The epilogue stores go straight to the peers' memory over NVLink; the receive side reduces its slots
// after a peer barrier (parallel/tensor_parallel.py). Operands are always this GPU's own memory.
BRAIN_API int brain_gemm_bf16_tp(const void* A, int64_t lda, const void* B, int64_t ldb, int b_mn, void* C,
                                 int64_t ldc, const int64_t* push_peers, int push_mode, int push_rank, int push_world,
                                 int push_chunk_rows, int64_t push_slot_elems, const void* R, int64_t ldr, int M, int N,
                                 int K, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  if (push_world > 8) return (int)cudaErrorInvalidValue;
  if ((lda % 8) || (ldb % 8) || K < 16) return (int)cudaErrorInvalidValue;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.C = C; a.ldc = ldc; a.c_f32 = 0; a.accumulate = 0;
  a.alpha = 1.f; a.beta = 0.f;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  a.push = push_mode;
  a.push_world = push_world;
  a.push_rank = push_rank;
  a.push_chunk_rows = push_chunk_rows > 0 ? push_chunk_rows : M;
  a.push_slot_elems = push_slot_elems;
  for (int j = 0; j < push_world && push_peers; ++j) a.push_dst[j] = reinterpret_cast<__nv_bfloat16*>(push_peers[j]);
  if (g_pair_mode && M >= 256 && N >= 256) {
    a.tiles_m = (M + 255) / 256;
    a.tiles_n = (N + 255) / 256;
    a.num_tiles = a.tiles_m * a.tiles_n;
    CUtensorMap ta, tb;
    bool ok = get_map_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, 128, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
    ok = ok && (b_mn ? get_map_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK,
                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2)
                     : get_map_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, 128,
                                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2));
    if (!ok) return (int)cudaErrorInvalidValue;
    CUtensorMap tc{};
    a.tma_store = output_map(&tc, a) ? 1 : 0;
    if (a.push && g_push_stage && N % 8 == 0 && ldc % 8 == 0) {
      // staged push (no TMA store: tc stays unused)
      a.tma_store = 1;
      a.push_stage = 1;
      if (a.push == 1 && a.push_chunk_rows % 256 == 0 && a.push_chunk_rows < M)
        a.push_rot = ((push_rank + 1) * (a.push_chunk_rows / 256)) % a.tiles_m;
    }
    return b_mn ? launch_tc2<0, 1>(ta, tb, tc, a, stream) : launch_tc2<0, 0>(ta, tb, tc, a, stream);
  }
  const int BN = (N <= 128) ? 128 : 256;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_n = (N + BN - 1) / BN;
  a.num_tiles = a.tiles_m * a.tiles_n;
  CUtensorMap ta, tb;
  bool ok = get_map_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, BM, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
  if (ok)
    ok = b_mn ? get_map_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2)
              : get_map_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, (uint32_t)BN,
                           CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2);
  if (!ok) return (int)cudaErrorInvalidValue;
  if (BN == 128) return b_mn ? launch_tc<128, 6, 0, 1>(ta, tb, a, stream) : launch_tc<128, 6, 0, 0>(ta, tb, a, stream);
  return b_mn ? launch_tc<256, 4, 0, 1>(ta, tb, a, stream) : launch_tc<256, 4, 0, 0>(ta, tb, a, stream);
}

// GELU MLP first layer: C = A B^T (+ bias) and C2 = gelu(C), both bf16 [M, N] (A [M, K], B [N, K] row-major),
// in one CTA-pair GEMM with two TMA stores per output unit. cudaErrorNotSupported (nothing launched) when the
// pair path cannot run (M or N < 256, misaligned operands or outputs); the caller then runs the GEMM and the
// activation separately.
BRAIN_API int brain_gemm_bf16_gelu_dual(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                                        void* C2, int64_t ldc2, int M, int N, int K, const void* bias,
                                        cudaStream_t stream) {
  if (!g_pair_mode || M < 256 || N < 256 || !pair_aligned(A, lda, B, ldb, K)) return (int)cudaErrorNotSupported;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.C = C; a.ldc = ldc; a.alpha = 1.f;
  a.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.tiles_m = (M + 255) / 256;
  a.tiles_n = (N + 255) / 256;
  a.num_tiles = a.tiles_m * a.tiles_n;
  CUtensorMap ta, tb, tc, t2;
  if (!pair_maps(A, lda, 0, B, ldb, 0, M, N, K, &ta, &tb) || !output_map(&tc, a)) return (int)cudaErrorNotSupported;
  GemmArgs a2 = a;
  a2.C = C2; a2.ldc = ldc2;
  if (!output_map(&t2, a2)) return (int)cudaErrorNotSupported;
  a.tma_store = 1;
  a.dual_gelu = 1;
  return launch_tc2<0, 0>(ta, tb, tc, a, stream, &t2);
}

// GELU MLP data gradient through the activation: C = (A op(B)) * gelu'(H), bf16 [M, N]; A [M, K] row-major,
// B [K, N] (b_mn = 1, the second layer's weight read in place) or [N, K]; H [M, N] the saved pre-activation
// (row stride ldh). cudaErrorNotSupported as above.
BRAIN_API int brain_gemm_bf16_gelu_grad(const void* A, int64_t lda, const void* B, int64_t ldb, int b_mn, void* C,
                                        int64_t ldc, const void* H, int64_t ldh, int M, int N, int K,
                                        cudaStream_t stream) {
  if (!g_pair_mode || M < 256 || N < 256 || !pair_aligned(A, lda, B, ldb, K) || ldh % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(H) & 15))
    return (int)cudaErrorNotSupported;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.C = C; a.ldc = ldc; a.alpha = 1.f;
  a.tiles_m = (M + 255) / 256;
  a.tiles_n = (N + 255) / 256;
  a.num_tiles = a.tiles_m * a.tiles_n;
  CUtensorMap ta, tb, tc, th;
  if (!pair_maps(A, lda, 0, B, ldb, b_mn, M, N, K, &ta, &tb) || !output_map(&tc, a) ||
      !get_map_2d(&th, H, (uint64_t)N, (uint64_t)M, (uint64_t)ldh, 64, 32, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2))
    return (int)cudaErrorNotSupported;
  a.tma_store = 1;
  a.R = reinterpret_cast<const __nv_bfloat16*>(H);  // read only through the map (r_tma)
  a.ldr = ldh;
  a.r_tma = 1;
  a.r_op = 1;
  return b_mn ? launch_tc2<0, 1>(ta, tb, tc, a, stream, &th) : launch_tc2<0, 0>(ta, tb, tc, a, stream, &th);
}

// Row-wise scaled fp8 GEMM on the CTA pair: C [M, N] bf16 = (Aq [M, K] . Bq [N, K]^T) * sa[m] * sb[n] (+ R),
// e4m3 operands K-major (row strides lda / ldb in bytes), f32 scales sa [M], sb [N]. 256 x 256 tiles,
// kind::f8f6f4 with the bf16 kernel's pipeline and TMA-store epilogue. Returns cudaErrorNotSupported
// when the pair path cannot run (M or N < 256, pair mode off, unaligned output): the caller then uses
// the single-CTA row-wise kernel.
BRAIN_API int brain_fp8_gemm_rowwise_pair(const void* A, int64_t lda, const void* B, int64_t ldb, const float* sa,
                                          const float* sb, void* C, int64_t ldc, const void* R, int64_t ldr, int M,
                                          int N, int K, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0 || K % 16 || lda % 16 || ldb % 16 ||
      ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) || !sa || !sb)
    return (int)cudaErrorInvalidValue;
  if (!g_pair_mode || M < 256 || N < 256) return (int)cudaErrorNotSupported;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.C = C; a.ldc = ldc; a.c_f32 = 0;
  a.alpha = 1.f;
  a.row_scale = sa; a.col_scale = sb;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  a.tiles_m = (M + 255) / 256;
  a.tiles_n = (N + 255) / 256;
  a.num_tiles = a.tiles_m * a.tiles_n;
  CUtensorMap ta, tb, tc{};
  if (!get_map_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 2 * BK, 128, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1) ||
      !get_map_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 2 * BK, 128, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1))
    return (int)cudaErrorInvalidValue;
  if (!output_map(&tc, a)) return (int)cudaErrorNotSupported;
  a.tma_store = 1;
  CUtensorMap tr{};
  if (a.R && ldr % 8 == 0 && (reinterpret_cast<uintptr_t>(R) & 15) == 0 &&
      get_map_2d(&tr, R, (uint64_t)N, (uint64_t)M, (uint64_t)ldr, 64, 32, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2))
    a.r_tma = 1;
  return launch_tc2<0, 0, 1>(ta, tb, tc, a, stream, a.r_tma ? &tr : nullptr);
}
