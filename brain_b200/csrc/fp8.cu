// Block-scaled FP8 (E4M3) GEMM on tcgen05 and the activation quantiser, sm_100a.
//
//   C[M,N] (bf16) = sum_kb  (Aq[M, kb] . Bq[N, kb]^T) * sa[m, kb] * sb[n / 128, kb]
// with 1 x 128 activation scales sa [M, K/128] and 128 x 128 weight-block scales sb [N/128, K/128]
// (f32). These are general f32 scales, not power-of-two MX scales, so the scaling cannot ride on the
// tensor core's block-scale path: each 128-wide K block is accumulated by tcgen05.mma kind::f8f6f4
// into one of four TMEM partial buffers (4 x 128 columns = all of TMEM), and the epilogue warps promote
// it in registers (acc += partial * sa * sb) while the tensor core runs up to three blocks ahead. Roles (10 warps, persistent): warp 0 TMA (SWIZZLE_128B, 128 B = 128 fp8 per row), warp 1
// single-thread MMA issuer, warps 2..9 promotion + bf16 epilogue: two warps per TMEM lane quadrant, each
// thread one output row and 64 of the tile's 128 columns, so a K block's promotion (128 x 128 loads and
// FMAs) keeps up with its 256-cycle MMA. Waits are bounded and report through the status word.
//
// Reference: the FP8E4M3 / FP8E5M2 dtypes are declared without arithmetic
// (crates/brain-quantization/src/core.rs:19-31); group-wise scaling mirrors BlockQuantizer
// (block_quant.rs:30-70) with blocks of 128.
#include "common.cuh"

using namespace brain;

namespace {

constexpr int kThreads = 320;
constexpr int kPromoThreads = 256;  // warps 2..9
constexpr int TM = 128, TN = 128, TK = 128;  // tile and scale-block sizes
constexpr int STAGES = 4;
constexpr int OP_BYTES = TM * TK;  // 16 KB of fp8 per operand per stage
constexpr int NPART = 4;            // TMEM partial buffers

struct Fp8Args {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;
  const float* sa;  // [M, K/128]
  const float* sb;  // [ceil(N/128), K/128]
  int ksb;          // K / 128 (scale columns)
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* R;  // optional residual [M, N]
  int64_t ldr;
};

__device__ __forceinline__ void fp8_tile(int t, int tiles_m, int& tm, int& tn) {
  // column-major over tiles_m so consecutive CTAs share the B (weight) tile in L2
  tm = t % tiles_m;
  tn = t / tiles_m;
}

__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Fp8Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + STAGES * 2 * OP_BYTES;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (STAGES + s); };
  auto pfull = [&](int b) { return bars + 8u * (2 * STAGES + b); };
  auto pempty = [&](int b) { return bars + 8u * (2 * STAGES + NPART + b); };
  const uint32_t drain = bars + 8u * (2 * STAGES + 2 * NPART);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + STAGES * 2 * OP_BYTES + (2 * STAGES + 2 * NPART + 1) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < NPART; ++b) {
      mbar_init(pfull(b), 1);
      mbar_init(pempty(b), kPromoThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 128 * NPART);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // partial buffer b at columns [b*128, b*128 + 128)
  const int nkb = (a.K + TK - 1) / TK;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        fp8_tile(t, a.tiles_m, tm, tn);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(empty(s), ((it / STAGES) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 310, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa_ = sbase + s * 2 * OP_BYTES;
          mbar_arrive_expect_tx(full(s), 2 * OP_BYTES);
          tma_load_2d(&tmA, sa_, full(s), kb * TK, tm * TM);
          tma_load_2d(&tmB, sa_ + OP_BYTES, full(s), kb * TK, tn * TN);
        }
      }
      if (!ok) {
        for (uint32_t j = it > (uint32_t)STAGES ? it - STAGES : 0; j < it; ++j) {
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full(j % STAGES), (j / STAGES) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f8(TM, TN, 0u, 0u, 0u, 0u);
      uint32_t it = 0, pb = 0;  // pb: global K-block counter (partial buffer = pb % NPART)
      bool ok = true, issued = false;
      for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb, ++it, ++pb) {
          const int s = it % STAGES;
          const int b = pb % NPART;
          if (!mbar_wait(pempty(b), ((pb / NPART) & 1) ^ 1, BRAIN_ERR_TIMEOUT_ACC, 320, abort_flag) ||
              !mbar_wait(full(s), (it / STAGES) & 1, BRAIN_ERR_TIMEOUT_FULL, 321, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa_ = sbase + s * 2 * OP_BYTES;
#pragma unroll
          for (int kk = 0; kk < TK / 32; ++kk)  // K = 32 fp8 per instruction = 32 bytes
            tc_mma_f8(tmem + (uint32_t)(b * 128), smem_desc_sw128(sa_ + kk * 32, 16, 1024),
                      smem_desc_sw128(sa_ + OP_BYTES + kk * 32, 16, 1024), idesc, kk > 0 ? 1u : 0u);
          issued = true;
          tc_commit(empty(s));
          tc_commit(pfull(b));
        }
      }
      if (!ok && issued) {
        tc_commit(drain);
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    constexpr int HC = TN / 2;  // columns per promotion thread
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    uint32_t pb = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x) {
      int tm, tn;
      fp8_tile(t, a.tiles_m, tm, tn);
      const int gm = tm * TM + r;
      const bool row_ok = gm < a.M;
      float acc[HC];
#pragma unroll
      for (int j = 0; j < HC; ++j) acc[j] = 0.f;
      const float* sarow = a.sa + (int64_t)(row_ok ? gm : 0) * a.ksb;
      const float* sbrow = a.sb + (int64_t)tn * a.ksb;
      auto scale_of = [&](int kb) { return (row_ok && kb < nkb) ? __ldg(sarow + kb) * __ldg(sbrow + kb) : 0.f; };
      float s1 = scale_of(0), s2 = scale_of(1), s3 = scale_of(2);  // scales loaded three blocks ahead
      for (int kb = 0; kb < nkb; ++kb, ++pb) {
        const int b = pb % NPART;
        const float scale = s1;
        s1 = s2;
        s2 = s3;
        s3 = scale_of(kb + 3);
        if (!mbar_wait(pfull(b), (pb / NPART) & 1, BRAIN_ERR_TIMEOUT_ACC, 330, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t v0[32], v1[32];
        const uint32_t ta = tmem + (uint32_t)(b * 128 + half * HC) + lane_addr;
        tmem_ld32(ta, v0);
        tmem_ld32(ta + 32, v1);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(pempty(b));  // the partial is in registers: the tensor core may refill the buffer
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          acc[j] = fmaf(scale, __uint_as_float(v0[j]), acc[j]);
          acc[32 + j] = fmaf(scale, __uint_as_float(v1[j]), acc[32 + j]);
        }
      }
      if (!ok) break;
      if (row_ok) {
        const int n0 = tn * TN + half * HC;
        __nv_bfloat16* crow = a.C + (int64_t)gm * a.ldc;
        if (n0 + HC <= a.N) {
          if (a.R) {
            const __nv_bfloat16* rrow = a.R + (int64_t)gm * a.ldr + n0;
#pragma unroll
            for (int j = 0; j < HC; j += 8) {
              float rv[8];
              load8(rrow + j, rv);
#pragma unroll
              for (int u = 0; u < 8; ++u) acc[j + u] += rv[u];
            }
          }
#pragma unroll
          for (int j = 0; j < HC; j += 8) store8(crow + n0 + j, acc + j);
        } else {
#pragma unroll
          for (int j = 0; j < HC; ++j)
            if (n0 + j < a.N)
              crow[n0 + j] = __float2bfloat16_rn(acc[j] + (a.R ? __bfloat162float(a.R[(int64_t)gm * a.ldr + n0 + j]) : 0.f));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128 * NPART);
  }
}

// ------------------------------------------------------------------ row-wise scaled FP8 GEMM
//   C[M,N] (bf16) = (Aq[M,K] . Bq[N,K]^T) * sa[m] * sb[n]  (+ R)
// One f32 scale per activation row (token) and one per weight row (output channel), so the whole K
// reduction accumulates in TMEM at the tensor core's fp8 rate and the scales are applied once in the
// epilogue: no per-block promotion on the CUDA cores. 128 x 256 tiles (kind::f8f6f4, N = 256), 4-stage
// TMA ring of 48 KB stages, two 256-column TMEM accumulators so the epilogue of one tile overlaps the
// MMAs of the next. Warp 0 TMA, warp 1 single-thread MMA issuer, warps 2..9 epilogue (two warps per
// TMEM lane quadrant, each thread one row and 128 of the 256 columns).
constexpr int RW_TN = 256;
constexpr int RW_STAGES = 4;
constexpr int RW_A_BYTES = TM * TK;       // 16 KB
constexpr int RW_B_BYTES = RW_TN * TK;    // 32 KB
constexpr int RW_STAGE_BYTES = RW_A_BYTES + RW_B_BYTES;
constexpr int RW_NBAR = 2 * RW_STAGES + 4 + 1;
constexpr int RW_SMEM = RW_STAGES * RW_STAGE_BYTES + RW_NBAR * 8 + 16 + 1024;

struct Fp8RwArgs {
  int M, N, K;
  int tiles_m, num_tiles;
  const float* sa;  // [M]
  const float* sb;  // [N]
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* R;
  int64_t ldr;
};

__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_rw_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Fp8RwArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + RW_STAGES * RW_STAGE_BYTES;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (RW_STAGES + s); };
  auto afull = [&](int b) { return bars + 8u * (2 * RW_STAGES + b); };
  auto aempty = [&](int b) { return bars + 8u * (2 * RW_STAGES + 2 + b); };
  const uint32_t drain = bars + 8u * (2 * RW_STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + RW_STAGES * RW_STAGE_BYTES + RW_NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RW_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(afull(b), 1);
      mbar_init(aempty(b), kPromoThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 2 * RW_TN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // accumulator b at columns [b*256, b*256 + 256)
  const int nkb = (a.K + TK - 1) / TK;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        fp8_tile(t, a.tiles_m, tm, tn);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % RW_STAGES;
          if (!mbar_wait(empty(s), ((it / RW_STAGES) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 350, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + s * RW_STAGE_BYTES;
          mbar_arrive_expect_tx(full(s), RW_STAGE_BYTES);
          tma_load_2d(&tmA, st, full(s), kb * TK, tm * TM);
          tma_load_2d(&tmB, st + RW_A_BYTES, full(s), kb * TK, tn * RW_TN);
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        for (uint32_t j = it > (uint32_t)RW_STAGES ? it - RW_STAGES : 0; j < it; ++j) {
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full(j % RW_STAGES), (j / RW_STAGES) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f8(TM, RW_TN, 0u, 0u, 0u, 0u);
      uint32_t it = 0, tc = 0;  // tc: tiles issued by this CTA (accumulator = tc & 1)
      bool ok = true, issued = false;
      for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x, ++tc) {
        const int b = tc & 1;
        if (!mbar_wait(aempty(b), ((tc >> 1) & 1) ^ 1, BRAIN_ERR_TIMEOUT_ACC, 360, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * RW_TN);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % RW_STAGES;
          if (!mbar_wait(full(s), (it / RW_STAGES) & 1, BRAIN_ERR_TIMEOUT_FULL, 361, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + s * RW_STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < TK / 32; ++kk)
            tc_mma_f8(acc, smem_desc_sw128(st + kk * 32, 16, 1024), smem_desc_sw128(st + RW_A_BYTES + kk * 32, 16, 1024),
                      idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          issued = true;
          tc_commit(empty(s));
        }
        if (!ok) break;
        tc_commit(afull(b));
      }
      if (!ok && issued) {
        tc_commit(drain);
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    constexpr int HC = RW_TN / 2;  // 128 columns per thread
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x, ++tc) {
      int tm, tn;
      fp8_tile(t, a.tiles_m, tm, tn);
      const int b = tc & 1;
      const int gm = tm * TM + r;
      const bool row_ok = gm < a.M;
      const float s_row = row_ok ? __ldg(a.sa + gm) : 0.f;
      if (!mbar_wait(afull(b), (tc >> 1) & 1, BRAIN_ERR_TIMEOUT_ACC, 370, abort_flag)) break;
      tc_fence_after();
      const int n_base = tn * RW_TN + half * HC;
      __nv_bfloat16* crow = a.C + (int64_t)gm * a.ldc;
#pragma unroll 1
      for (int c0 = 0; c0 < HC; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + (uint32_t)(b * RW_TN + half * HC + c0) + lane_addr, v);
        tc_wait_ld();
        if (c0 + 32 == HC) {  // the whole accumulator slice is in registers: hand the buffer back
          tc_fence_before();
          mbar_arrive(aempty(b));
        }
        const int n0 = n_base + c0;
        if (!row_ok || n0 >= a.N) continue;
        float o[32];
        if (n0 + 32 <= a.N) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 sb4 = __ldg(reinterpret_cast<const float4*>(a.sb + n0 + j));
            o[j] = __uint_as_float(v[j]) * s_row * sb4.x;
            o[j + 1] = __uint_as_float(v[j + 1]) * s_row * sb4.y;
            o[j + 2] = __uint_as_float(v[j + 2]) * s_row * sb4.z;
            o[j + 3] = __uint_as_float(v[j + 3]) * s_row * sb4.w;
          }
          if (a.R) {
            const __nv_bfloat16* rrow = a.R + (int64_t)gm * a.ldr + n0;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              float rv[8];
              load8(rrow + j, rv);
#pragma unroll
              for (int u = 0; u < 8; ++u) o[j + u] += rv[u];
            }
          }
#pragma unroll
          for (int j = 0; j < 32; j += 8) store8(crow + n0 + j, o + j);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (n0 + j < a.N) {
              float x = __uint_as_float(v[j]) * s_row * __ldg(a.sb + n0 + j);
              if (a.R) x += __bfloat162float(a.R[(int64_t)gm * a.ldr + n0 + j]);
              crow[n0 + j] = __float2bfloat16_rn(x);
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * RW_TN);
  }
}

// Row-wise quantiser over whole rows: s[m] = amax(|x[m, :]|) / 448, q = e4m3(x / s). One warp per row,
// 16-byte loads (8 bf16 per lane per step); the second pass re-reads the row from L1/L2.
__global__ void quant_fp8_rowwise_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_fp8_e4m3* __restrict__ q,
                                         int64_t ldq, float* __restrict__ s, int M, int K) {
  const int64_t m = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (m >= M) return;
  const __nv_bfloat16* row = x + m * ldx;
  float amax = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    float v[8];
    load8(row + k, v);
#pragma unroll
    for (int u = 0; u < 8; ++u) amax = fmaxf(amax, fabsf(v[u]));
  }
  amax = warp_max(amax);
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / scale;
  __nv_fp8_e4m3* qrow = q + m * ldq;
  for (int k = lane * 8; k < K; k += 256) {
    float v[8];
    load8(row + k, v);
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      __nv_fp8x4_e4m3 p4(make_float4(v[4 * h] * inv, v[4 * h + 1] * inv, v[4 * h + 2] * inv, v[4 * h + 3] * inv));
      w[h] = *reinterpret_cast<uint32_t*>(&p4);
    }
    *reinterpret_cast<uint2*>(qrow + k) = make_uint2(w[0], w[1]);
  }
  if (lane == 0) s[m] = scale;
}

// Row-wise 1 x 128 quantiser: q = e4m3(x / s), s = amax(|x| over 128) / 448 (one warp per block of 128).
__global__ void quant_fp8_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_fp8_e4m3* __restrict__ q,
                                      int64_t ldq, float* __restrict__ s, int M, int K) {
  const int kblocks = K / 128;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (wid >= (int64_t)M * kblocks) return;
  const int m = (int)(wid / kblocks), kb = (int)(wid % kblocks);
  const __nv_bfloat16* p = x + (int64_t)m * ldx + kb * 128 + lane * 4;
  float v[4];
  __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(p);
  __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(p + 2);
  v[0] = __low2float(h0); v[1] = __high2float(h0); v[2] = __low2float(h1); v[3] = __high2float(h1);
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / scale;
  __nv_fp8_e4m3* qp = q + (int64_t)m * ldq + kb * 128 + lane * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) qp[i] = __nv_fp8_e4m3(v[i] * inv);
  if (lane == 0) s[(int64_t)m * kblocks + kb] = scale;
}

bool map_fp8(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t ld, uint32_t box_rows = 128) {
  uint64_t dims[2] = {(uint64_t)inner, (uint64_t)outer};
  uint64_t strides[1] = {(uint64_t)ld};
  uint32_t box[2] = {128, box_rows};
  return brain_host::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

BRAIN_STATUS_READER(fp8)

// Aq [M, K] e4m3 (row stride lda bytes), Bq [N, K] e4m3 (ldb), sa [M, K/128], sb [ceil(N/128), K/128],
// C [M, N] bf16 (ldc elements), R optional residual. K must be a multiple of 128, lda/ldb of 16.
BRAIN_API int brain_fp8_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, const float* sa, const float* sb,
                             void* C, int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, cudaStream_t st) {
  if (M <= 0 || N <= 0) return 0;
  if (K % 128 || lda % 16 || ldb % 16 || ((uintptr_t)A & 15) || ((uintptr_t)B & 15)) return (int)cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  if (!map_fp8(&ta, A, K, M, lda) || !map_fp8(&tb, B, K, N, ldb)) return (int)cudaErrorInvalidValue;
  Fp8Args a;
  a.M = M; a.N = N; a.K = K;
  a.tiles_m = (M + TM - 1) / TM;
  a.tiles_n = (N + TN - 1) / TN;
  a.num_tiles = a.tiles_m * a.tiles_n;
  a.sa = sa; a.sb = sb; a.ksb = K / 128;
  a.C = reinterpret_cast<__nv_bfloat16*>(C);
  a.ldc = ldc;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  const int smem = STAGES * 2 * OP_BYTES + (2 * STAGES + 2 * NPART + 1) * 8 + 16 + 1024;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(fp8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr[dev & 63] = true;
  }
  const int grid = std::min(a.num_tiles, brain_host::num_sms());
  fp8_gemm_kernel<<<grid, kThreads, smem, st>>>(ta, tb, a);
  return (int)cudaGetLastError();
}

// x [M, K] bf16 -> q [M, K] e4m3, s [M, K/128] (K % 128 == 0).
BRAIN_API int brain_fp8_quant_rows(const void* x, int64_t ldx, void* q, int64_t ldq, float* s, int M, int K,
                                   cudaStream_t st) {
  if (K % 128) return (int)cudaErrorInvalidValue;
  const int64_t warps = (int64_t)M * (K / 128);
  if (warps == 0) return 0;
  quant_fp8_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<__nv_fp8_e4m3*>(q), ldq, s, M, K);
  return (int)cudaGetLastError();
}

// Row-wise scaled FP8 GEMM: Aq [M, K] e4m3 (lda bytes), Bq [N, K] e4m3 (ldb), sa [M], sb [N] f32 (sb must be
// 16-byte aligned), C [M, N] bf16 (ldc elements, 16-byte aligned rows when N % 8 == 0), R optional residual.
// K and lda/ldb multiples of 16.
BRAIN_API int brain_fp8_gemm_rowwise(const void* A, int64_t lda, const void* B, int64_t ldb, const float* sa,
                                     const float* sb, void* C, int64_t ldc, const void* R, int64_t ldr, int M, int N,
                                     int K, cudaStream_t st) {
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0 || K % 16 || lda % 16 || ldb % 16 || ((uintptr_t)A & 15) || ((uintptr_t)B & 15) ||
      ((uintptr_t)sb & 15) || ldc % 8 || ((uintptr_t)C & 15) || (R && (ldr % 8 || ((uintptr_t)R & 15))))
    return (int)cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  if (!map_fp8(&ta, A, K, M, lda) || !map_fp8(&tb, B, K, N, ldb, RW_TN)) return (int)cudaErrorInvalidValue;
  Fp8RwArgs a;
  a.M = M; a.N = N; a.K = K;
  a.tiles_m = (M + TM - 1) / TM;
  a.num_tiles = a.tiles_m * ((N + RW_TN - 1) / RW_TN);
  a.sa = sa; a.sb = sb;
  a.C = reinterpret_cast<__nv_bfloat16*>(C);
  a.ldc = ldc;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(fp8_gemm_rw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RW_SMEM);
    attr[dev & 63] = true;
  }
  const int grid = std::min(a.num_tiles, brain_host::num_sms());
  fp8_gemm_rw_kernel<<<grid, kThreads, RW_SMEM, st>>>(ta, tb, a);
  return (int)cudaGetLastError();
}

// x [M, K] bf16 -> q [M, K] e4m3, s [M] (K % 8 == 0, 16-byte aligned rows).
BRAIN_API int brain_fp8_quant_rowwise(const void* x, int64_t ldx, void* q, int64_t ldq, float* s, int M, int K,
                                      cudaStream_t st) {
  if (M <= 0) return 0;
  if (K % 8 || ldx % 8 || ldq % 8 || ((uintptr_t)x & 15) || ((uintptr_t)q & 7)) return (int)cudaErrorInvalidValue;
  quant_fp8_rowwise_kernel<<<(unsigned)((M + 7) / 8), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<__nv_fp8_e4m3*>(q), ldq, s, M, K);
  return (int)cudaGetLastError();
}
