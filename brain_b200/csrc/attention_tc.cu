// Flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// One CTA computes 128 query rows of one (batch, q-head) against all visible keys, 128 keys per
// step. Roles (10 warps):
//   warp 0      TMA producer: Q once, then K and V blocks (4-D tensor maps over [B, S, H, D] with the
//               caller's strides, SWIZZLE_128B, CTA-local) into a 2-4 stage ring whose K and V halves
//               are released separately: K_j right after S_j, V_j after PV_j, so the K of the next
//               block (needed one block early, for S_{j+1}) is not held up by PV_j.
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM S buffers (128 cols
//               each, f32), then O += P_j V_j into the TMEM O accumulator once softmax has written
//               P_j; V is consumed as an MN-major operand straight from its [keys, D] tile.
//   warps 2..9  softmax: two warps per TMEM lane quadrant, thread = (query row, half of the 128 keys);
//               the pair exchanges its partial row maxima through shared memory once per block.
//               tcgen05.ld of S, causal/length mask, online max with lazy rescaling (O is only
//               rescaled when the running max grows by more than 2^8), exp2, P packed to bf16 into a
//               SWIZZLE_128B K-major smem tile, and the final O / l epilogue with the log-sum-exp.
// S_{j+1} is computed while softmax works on S_j, and PV_j runs while softmax computes the
// exponentials of S_{j+1}. All waits are bounded (globaltimer) and report through the status word.
//
// Semantics match the mma.sync kernels in attention.cu (bottom-right causal alignment, GQA by head
// index, natural-log LSE) and the reference SDPA (crates/brain-transformer/src/attention/scaled.rs:41-139).
#include "common.cuh"

using namespace brain;

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P values stay <= 256 between rescales
constexpr int kThreads = 320;
constexpr int kSmThreads = 256;  // softmax threads (warps 2..9)
constexpr int SUB = 128 * 64 * 2;  // one SW128 sub-tile: 128 rows x 64 bf16

struct FwdArgs {
  __nv_bfloat16* o;
  int64_t ob, os, oh;
  float* lse;
  int B, Hq, Hkv, Sq, Sk;
  float scale_log2;
  int causal;
};

template <int D>
struct FwdLayout {
  static constexpr int NSUB = D / 64;
  static constexpr int STAGES = D == 64 ? 4 : 2;
  static constexpr int Q_OFF = 0;
  static constexpr int P_OFF = NSUB * SUB;
  static constexpr int KV_OFF = P_OFF + 2 * SUB;
  static constexpr int K_BYTES = NSUB * SUB;
  static constexpr int STAGE_BYTES = 2 * K_BYTES;
  static constexpr int X_OFF = KV_OFF + STAGES * STAGE_BYTES;  // [2 parities][2 halves][128] partial maxima
  static constexpr int BAR_OFF = X_OFF + 2 * 2 * 128 * 4;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], s_free[2], p_full, o_done, drain
  static constexpr int NBAR = 1 + 4 * STAGES + 4 + 3;
  static constexpr int TOTAL = BAR_OFF + NBAR * 8 + 16 + 1024;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, FwdArgs a) {
  using L = FwdLayout<D>;
  constexpr int ST = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + L::Q_OFF, sP = sbase + L::P_OFF, sKV = sbase + L::KV_OFF;
  const uint32_t bars = sbase + L::BAR_OFF;
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (1 + ST + s); };
  auto v_full = [&](int s) { return bars + 8u * (1 + 2 * ST + s); };
  auto v_empty = [&](int s) { return bars + 8u * (1 + 3 * ST + s); };
  auto s_full = [&](int b) { return bars + 8u * (1 + 4 * ST + b); };
  auto s_free = [&](int b) { return bars + 8u * (3 + 4 * ST + b); };
  const uint32_t p_full = bars + 8u * (5 + 4 * ST);
  const uint32_t o_done = bars + 8u * (6 + 4 * ST);
  const uint32_t drain = bars + 8u * (7 + 4 * ST);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nmb = (a.Sq + 127) / 128;
  const int mb = a.causal ? (nmb - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.Hq, h = bh % a.Hq;
  const int hk = h / (a.Hq / a.Hkv);
  const int m0 = mb * 128;
  const int off = a.Sk - a.Sq;
  int kend = a.Sk;
  if (a.causal) kend = min(a.Sk, m0 + 128 + off);
  const int nkb = kend > 0 ? (kend + 127) / 128 : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), kSmThreads);
    }
    mbar_init(p_full, kSmThreads);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0: [0,128)  S1: [128,256)  O: [256, 256 + D)

  if (warp == 0) {
    if (lane == 0 && nkb > 0) {
      // ---------------- TMA producer
      mbar_arrive_expect_tx(q_full, L::NSUB * SUB);
      for (int c = 0; c < L::NSUB; ++c) tma_load_4d(&tmQ, sQ + c * SUB, q_full, c * 64, m0, h, b);
      // K_j, then V_{j-1}: the K ring runs one block ahead of the V ring
      int nk = 0, nv = 0;  // blocks issued
      bool ok = true;
      for (int j = 0; ok && j <= nkb; ++j) {
        if (j < nkb) {
          const int s = j % ST;
          if (!mbar_wait(k_empty(s), ((j / ST) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 110, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t kb = sKV + s * L::STAGE_BYTES;
          mbar_arrive_expect_tx(k_full(s), L::K_BYTES);
          for (int c = 0; c < L::NSUB; ++c) tma_load_4d(&tmK, kb + c * SUB, k_full(s), c * 64, j * 128, hk, b);
          ++nk;
        }
        if (j > 0) {
          const int jv = j - 1, s = jv % ST;
          if (!mbar_wait(v_empty(s), ((jv / ST) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 111, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t vb = sKV + s * L::STAGE_BYTES + L::K_BYTES;
          mbar_arrive_expect_tx(v_full(s), L::K_BYTES);
          for (int c = 0; c < L::NSUB; ++c) tma_load_4d(&tmV, vb + c * SUB, v_full(s), c * 64, jv * 128, hk, b);
          ++nv;
        }
      }
      if (!ok) {  // aborted: let issued copies land
        for (int i = max(0, nk - ST); i < nk; ++i) {
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(k_full(i % ST), (i / ST) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
        for (int i = max(0, nv - ST); i < nv; ++i) {
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(v_full(i % ST), (i / ST) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkb > 0) {
      // ---------------- MMA issuer
      constexpr uint32_t IDESC_S = idesc_f16(128, 128, 1u, 0u, 0u);
      constexpr uint32_t IDESC_O = idesc_f16(128, D, 1u, 0u, 1u);
      bool ok = mbar_wait(q_full, 0, BRAIN_ERR_TIMEOUT_FULL, 120, abort_flag);
      bool issued = false;
      auto issue_s = [&](int jj) {
        const uint32_t kb = sKV + (jj % ST) * L::STAGE_BYTES;
        const uint32_t d = tmem + (uint32_t)((jj & 1) * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk / 4) * SUB + (kk % 4) * 32;
          tc_mma_f16(d, smem_desc_sw128(sQ + o, 16, 1024), smem_desc_sw128(kb + o, 16, 1024), IDESC_S,
                     kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full(jj & 1));
        tc_commit(k_empty(jj % ST));
      };
      if (ok) ok = mbar_wait(k_full(0), 0, BRAIN_ERR_TIMEOUT_FULL, 121, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        issued = true;
      }
      for (int j = 0; ok && j < nkb; ++j) {
        if (j + 1 < nkb) {
          const int jn = j + 1;
          if (!mbar_wait(k_full(jn % ST), (jn / ST) & 1, BRAIN_ERR_TIMEOUT_FULL, 122, abort_flag) ||
              !mbar_wait(s_free(jn & 1), ((jn / 2) & 1) ^ 1, BRAIN_ERR_TIMEOUT_ACC, 123, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(jn);
        }
        if (!mbar_wait(p_full, j & 1, BRAIN_ERR_TIMEOUT_ACC, 124, abort_flag) ||
            !mbar_wait(v_full(j % ST), (j / ST) & 1, BRAIN_ERR_TIMEOUT_FULL, 125, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vb = sKV + (j % ST) * L::STAGE_BYTES + L::K_BYTES;
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(sP + (kk / 4) * SUB + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(vb + kk * 2048, SUB, 1024);
          tc_mma_f16(tmem + 256, ad, bd, IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(o_done);
        tc_commit(v_empty(j % ST));
      }
      if (!ok && issued) {
        tc_commit(drain);
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- softmax warps (2..9): quadrant q of the TMEM lanes, key half hc
    const int q = warp & 3;
    const int hc = (warp - 2) >> 2;
    const int r = q * 32 + lane;  // row within the tile == TMEM lane
    const int qi = m0 + r;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const int limit = a.causal ? min(qi + off, a.Sk - 1) : a.Sk - 1;
    float* xmax = reinterpret_cast<float*>(smem + L::X_OFF);
    float m_used = -INFINITY, l = 0.f;  // l: this thread's partial row sum (its 64 keys of every block)
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      if (ok && !mbar_wait(s_full(j & 1), (j / 2) & 1, BRAIN_ERR_TIMEOUT_ACC, 130, abort_flag)) ok = false;
      tc_fence_after();
      float s[64];
      if (ok) {
#pragma unroll
        for (int c = 0; c < 2; ++c) tmem_ld32(tmem + (uint32_t)((j & 1) * 128 + hc * 64 + c * 32) + lane_addr,
                                              reinterpret_cast<uint32_t*>(s + c * 32));
        tc_wait_ld();
      } else {
#pragma unroll
        for (int k = 0; k < 64; ++k) s[k] = 0.f;
      }
      tc_fence_before();
      mbar_arrive(s_free(j & 1));
      const int n0 = j * 128 + hc * 64;  // this thread's first key
      const bool need_mask = (n0 + 63 > a.Sk - 1) || (a.causal && n0 + 63 > m0 + off);
      // Row max and row sum use 8 independent partial accumulators (no single long dependency chain).
      float mxp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mxp[u] = -INFINITY;
      if (need_mask) {
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          s[k] = (n0 + k > limit) ? -INFINITY : s[k] * a.scale_log2;
          mxp[k & 7] = fmaxf(mxp[k & 7], s[k]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          s[k] *= a.scale_log2;
          mxp[k & 7] = fmaxf(mxp[k & 7], s[k]);
        }
      }
      float* xm = xmax + (j & 1) * 256;
      xm[hc * 128 + r] = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                               fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      // the pair's partial maxima; the barrier also makes a give-up uniform (every thread arrives after
      // bounded waits, and all leave the loop together)
      if (!bar_sync_and(1, kSmThreads, ok)) {
        ok = false;
        break;
      }
      const float mx = fmaxf(xm[r], xm[128 + r]);
      float alpha = 1.f;
      if (mx > m_used + kRescaleThreshold || (m_used == -INFINITY && mx > -INFINITY)) {
        alpha = exp2f(m_used - mx);  // 0 when m_used == -inf
        m_used = mx;
      }
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      float sp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) sp[u] = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int k = 0; k < 64; k += 2) {
        const float p0 = ex2_fast(s[k] - mu), p1 = ex2_fast(s[k + 1] - mu);
        sp[(k >> 1) & 7] += p0 + p1;
        __nv_bfloat162 hv = __floats2bfloat162_rn(p0, p1);
        pk[k / 2] = *reinterpret_cast<uint32_t*>(&hv);
      }
      const float sum = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      l = l * alpha + sum;
      // P buffer and O are free once PV_{j-1} has completed
      if (j > 0 && !mbar_wait(o_done, (j - 1) & 1, BRAIN_ERR_TIMEOUT_ACC, 131, abort_flag)) ok = false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // this thread's 8 chunks of 8 keys: sub-tile hc of P
        const uint32_t addr = sP + hc * SUB + r * 128 + ((c ^ (r % 8)) * 16);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * c]), "r"(pk[4 * c + 1]),
                     "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                     : "memory");
      }
      if (ok && j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = hc * (D / 64); c < (hc + 1) * (D / 64); ++c) {  // this warp's half of O's columns
          uint32_t ov[32];
          const uint32_t ta = tmem + 256 + (uint32_t)(c * 32) + lane_addr;
          tmem_ld32(ta, ov);
          tc_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) ov[k] = __float_as_uint(__uint_as_float(ov[k]) * alpha);
          tmem_st32(ta, ov);
        }
        tc_wait_st();
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // the pair's partial row sums (the maxima slots are free once every thread passed the last exchange)
    bar_sync_and(1, kSmThreads, true);
    xmax[hc * 128 + r] = l;
    bar_sync_and(1, kSmThreads, true);
    l += xmax[(1 - hc) * 128 + r];
    // epilogue
    float inv = 0.f;
    bool have = ok && nkb > 0;
    if (have && !mbar_wait(o_done, (nkb - 1) & 1, BRAIN_ERR_TIMEOUT_ACC, 132, abort_flag)) have = false;
    tc_fence_after();
    if (l > 0.f) inv = 1.f / l;
    __nv_bfloat16* orow = a.o + (int64_t)b * a.ob + (int64_t)h * a.oh + (int64_t)qi * a.os;
#pragma unroll 1
    for (int c = hc * (D / 64); c < (hc + 1) * (D / 64); ++c) {
      uint32_t ov[32];
      if (have) {
        tmem_ld32(tmem + 256 + (uint32_t)(c * 32) + lane_addr, ov);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) ov[k] = 0u;
      }
      if (qi < a.Sq) {
        float v[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(ov[k]) * inv;
#pragma unroll
        for (int k = 0; k < 32; k += 8) store8(orow + c * 32 + k, v + k);
      }
    }
    if (hc == 0 && qi < a.Sq && a.lse)
      a.lse[((int64_t)b * a.Hq + h) * a.Sq + qi] = l > 0.f ? (m_used + log2f(l)) * kLn2 : -INFINITY;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool make_map(CUtensorMap* m, const void* base, int D, int S, int H, int B, int64_t ss, int64_t sh, int64_t sb) {
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)ss * 2, (uint64_t)sh * 2, (uint64_t)sb * 2};
  uint32_t box[4] = {64, 128, 1, 1};
  return brain_host::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D>
int launch(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const FwdArgs& a, cudaStream_t st) {
  using L = FwdLayout<D>;
  auto kern = fa_fwd_tc_kernel<D>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
  dim3 grid((a.Sq + 127) / 128, a.B * a.Hq);
  kern<<<grid, kThreads, L::TOTAL, st>>>(q, k, v, a);
  return (int)cudaGetLastError();
}

}  // namespace

BRAIN_STATUS_READER(attention_tc)

// Returns cudaErrorNotSupported (without launching) when the layout is outside what the tensor-core
// path handles (D not 64/128, strides not 16-byte multiples, misaligned bases); callers then use the
// mma.sync kernel.
BRAIN_API int brain_attn_fwd_tc(const void* q, const void* k, const void* v, const int64_t* s9, void* o,
                                const int64_t* ostr, float* lse, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                                float scale, int causal, cudaStream_t st) {
  if (Hkv <= 0 || Hq % Hkv) return (int)cudaErrorInvalidValue;
  if ((D != 64 && D != 128)) return (int)cudaErrorNotSupported;
  for (int i = 0; i < 9; ++i)
    if ((s9[i] * 2) % 16) return (int)cudaErrorNotSupported;
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15) return (int)cudaErrorNotSupported;
  if (ostr[1] % 8 || ostr[0] % 8 || ostr[2] % 8) return (int)cudaErrorNotSupported;
  if (B * Hq == 0 || Sq == 0) return 0;
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, q, D, Sq, Hq, B, s9[1], s9[2], s9[0]) || !make_map(&tk, k, D, Sk, Hkv, B, s9[4], s9[5], s9[3]) ||
      !make_map(&tv, v, D, Sk, Hkv, B, s9[7], s9[8], s9[6]))
    return (int)cudaErrorNotSupported;
  FwdArgs a;
  a.o = reinterpret_cast<__nv_bfloat16*>(o);
  a.ob = ostr[0]; a.os = ostr[1]; a.oh = ostr[2];
  a.lse = lse;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.Sq = Sq; a.Sk = Sk;
  a.scale_log2 = scale * kLog2e;
  a.causal = causal;
  return D == 64 ? launch<64>(tq, tk, tv, a, st) : launch<128>(tq, tk, tv, a, st);
}
