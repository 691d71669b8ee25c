// Flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// One CTA computes two 128-row query tiles (A: rows m0..m0+127, B: rows m0+128..m0+255) of one
// (batch, q-head) against all visible keys, 128 keys per step; both tiles share every K/V block the TMA
// brings in. Roles (12 warps, three warpgroups; setmaxnreg moves registers from warpgroup 0, which only
// issues copies and MMAs, to the softmax warpgroups: 4 x 32 x 72 + 8 x 32 x 216 = 384 x 168, the launch
// budget):
//   warp 0      TMA producer: Q_A and Q_B once, then K and V blocks (4-D tensor maps over [B, S, H, D]
//               with the caller's strides, SWIZZLE_128B, CTA-local) into a 2-stage ring whose K and V
//               halves are released separately (K_j after both score MMAs, V_j after both PV MMAs).
//   warp 1      MMA issuer (one thread), polling its barriers and issuing whatever is ready: for tile
//               t and key block j, O_t += P_t(j) V_j once softmax has written P_t(j), and S_t(j+1) =
//               Q_t K_{j+1}^T once that PV MMA has completed (S_t(j+1) overwrites the TMEM columns
//               P_t(j) is read from; tcgen05.mma orders only MMAs on the same accumulator, so the
//               completion is waited for explicitly). One tile's softmax runs while the tensor core
//               works on the other tile's MMAs.
//   warps 4..7  softmax of tile A, warps 8..11 softmax of tile B: thread = one query row (TMEM lane)
//               and all 128 keys of the block: tcgen05.ld of S, causal/length mask, row max, lazy
//               rescale of O (only when the running max grows by more than 2^8), exp2, and P packed to
//               bf16 and stored back over the first 64 columns of S (tcgen05.st). The PV MMA reads P
//               from TMEM as its A operand; V is the MN-major B operand straight from its [keys, D] tile.
// TMEM: S_A [0,128), S_B [128,256), O_A [256, 256 + D), O_B [384, 384 + D).
// O_t is final for softmax step j once S_t(j) has completed (S_t(j) is issued after PV_t(j-1) completed).
// All waits are bounded (globaltimer) and report through the status word.
//
// Semantics match the mma.sync kernels in attention.cu (bottom-right causal alignment, GQA by head
// index, natural-log LSE) and the reference SDPA (crates/brain-transformer/src/attention/scaled.rs:41-139).
#include "common.cuh"

using namespace brain;

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P values stay <= 256 between rescales
constexpr int kThreads = 384;
constexpr int SUB = 128 * 64 * 2;  // one SW128 sub-tile: 128 rows x 64 bf16

struct FwdArgs {
  __nv_bfloat16* o;
  int64_t ob, os, oh;
  float* lse;
  int B, Hq, Hkv, Sq, Sk;
  float scale_log2;
  int causal;
  // optional (BIAS kernels): key padding mask [B, Sk] (non-zero = attend), and an additive bias that depends
  // only on the key-query offset, per q head: relb[h, (k - q) + Sq - 1], float32 natural-log units
  // (ALiBi, T5 relative buckets); null when absent
  const uint8_t* kmask;
  const float* relb;
};

template <int D>
struct FwdLayout {
  static constexpr int NSUB = D / 64;
  static constexpr int STAGES = D == 64 ? 4 : 2;
  static constexpr int QBUF = D == 64 ? 2 : 1;  // query buffers: the next item's Q loads during this one
  static constexpr int Q_BYTES = NSUB * SUB;    // one 128-row query tile
  static constexpr int Q_OFF = 0;               // QBUF x (Q_A, Q_B)
  static constexpr int KV_OFF = QBUF * 2 * Q_BYTES;
  static constexpr int K_BYTES = NSUB * SUB;
  static constexpr int STAGE_BYTES = 2 * K_BYTES;
  static constexpr int BAR_OFF = KV_OFF + STAGES * STAGE_BYTES;
  // q_full[QBUF], q_empty[QBUF], k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2],
  // o_final[2], pv_done[2], drain
  static constexpr int NBAR = 2 * QBUF + 4 * STAGES + 8 + 1;
  static constexpr int TOTAL = BAR_OFF + NBAR * 8 + 16 + 1024;
};

// Key blocks that query tile `t` (rows m0 + 128 t ..) needs: 0 if the tile has no row.
__device__ __forceinline__ int tile_blocks(const FwdArgs& a, int m0, int t) {
  const int r0 = m0 + 128 * t;
  if (r0 >= a.Sq) return 0;
  int kend = a.Sk;
  if (a.causal) kend = min(a.Sk, r0 + 128 + (a.Sk - a.Sq));
  return kend > 0 ? (kend + 127) / 128 : 0;
}

// One work item = 256 query rows (two 128-row tiles A and B) of one (batch, head). Items are numbered with
// the query block slowest, heaviest first under a causal mask, and CTAs take them round-robin.
struct FwdItem {
  int m0, b, h, hk, nA, nB;
};
__device__ __forceinline__ FwdItem fwd_item(const FwdArgs& a, int w) {
  const int nmb = (a.Sq + 255) / 256;
  const int BH = a.B * a.Hq;
  const int mbi = w / BH, bh = w - mbi * BH;
  FwdItem it;
  it.m0 = (a.causal ? nmb - 1 - mbi : mbi) * 256;
  it.b = bh / a.Hq;
  it.h = bh % a.Hq;
  it.hk = it.h / (a.Hq / a.Hkv);
  it.nA = tile_blocks(a, it.m0, 0);
  it.nB = tile_blocks(a, it.m0, 1);
  return it;
}

// Persistent flash-attention forward: one CTA per SM loops over work items. Roles: warp 0 issues TMA
// copies (Q of an item into one of QBUF buffers, then its K and V blocks through a ring shared by all
// items), warp 1 issues the MMAs from an event loop, warps 4-7 / 8-11 run the online softmax of tiles A / B
// with one thread per query row. S_t = Q_t K^T lands in TMEM columns [128 t, 128 t + 128); P_t (bf16)
// overwrites its first 64 columns and is read from TMEM as the A operand of O_t += P_t V (O_t at column
// 256 + 128 t). Counters of every barrier run across items, so the next item's copies and its first S
// MMAs proceed while the softmax warps finish the current item's output.
template <int D, bool BIAS>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, FwdArgs a) {
  using L = FwdLayout<D>;
  constexpr int ST = L::STAGES;
  constexpr int QB = L::QBUF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + L::Q_OFF, sKV = sbase + L::KV_OFF;
  const uint32_t bars = sbase + L::BAR_OFF;
  auto q_full = [&](int i) { return bars + 8u * i; };
  auto q_empty = [&](int i) { return bars + 8u * (QB + i); };
  constexpr int KB0 = 2 * QB;
  auto k_full = [&](int s) { return bars + 8u * (KB0 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (KB0 + ST + s); };
  auto v_full = [&](int s) { return bars + 8u * (KB0 + 2 * ST + s); };
  auto v_empty = [&](int s) { return bars + 8u * (KB0 + 3 * ST + s); };
  auto s_full = [&](int t) { return bars + 8u * (KB0 + 4 * ST + t); };
  auto p_full = [&](int t) { return bars + 8u * (KB0 + 2 + 4 * ST + t); };
  auto o_final = [&](int t) { return bars + 8u * (KB0 + 4 + 4 * ST + t); };
  auto pv_done = [&](int t) { return bars + 8u * (KB0 + 6 + 4 * ST + t); };
  const uint32_t drain = bars + 8u * (KB0 + 8 + 4 * ST);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int items = ((a.Sq + 255) / 256) * a.B * a.Hq;
  const int off = a.Sk - a.Sq;

  if (threadIdx.x == 0) {
    for (int i = 0; i < QB; ++i) {
      mbar_init(q_full(i), 1);
      mbar_init(q_empty(i), 1);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(p_full(t), 128);
      mbar_init(o_final(t), 1);
      mbar_init(pv_done(t), 1);
    }
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
  const uint32_t tmem = *tmem_slot;
  if (warp < 4) {
    // warpgroup 0: copies and MMAs (the register hand-over is per warpgroup and dominates each role's code)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;");
  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int g = 0;             // K/V blocks of earlier items (ring position)
      int qn = 0;            // items with work so far (query buffer position)
      int nk = 0, nv = 0;    // blocks issued
      bool ok = true;
      for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
        const FwdItem it = fwd_item(a, w);
        const int nK = max(it.nA, it.nB);
        if (nK == 0) continue;
        const int qb = qn % QB;
        if (!mbar_wait(q_empty(qb), ((qn / QB) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 109, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full(qb), 2 * L::Q_BYTES);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < L::NSUB; ++c)
            tma_load_4d(&tmQ, sQ + (qb * 2 + t) * L::Q_BYTES + c * SUB, q_full(qb), c * 64, it.m0 + 128 * t, it.h,
                        it.b);
        ++qn;
        // K_j, then V_{j-1}: the K ring runs one block ahead of the V ring
        for (int j = 0; ok && j <= nK; ++j) {
          if (j < nK) {
            const int gj = g + j, s = gj % ST;
            if (!mbar_wait(k_empty(s), ((gj / ST) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 110, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t kb = sKV + s * L::STAGE_BYTES;
            mbar_arrive_expect_tx(k_full(s), L::K_BYTES);
            for (int c = 0; c < L::NSUB; ++c)
              tma_load_4d(&tmK, kb + c * SUB, k_full(s), c * 64, j * 128, it.hk, it.b);
            ++nk;
          }
          if (j > 0) {
            const int gv = g + j - 1, s = gv % ST;
            if (!mbar_wait(v_empty(s), ((gv / ST) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 111, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t vb = sKV + s * L::STAGE_BYTES + L::K_BYTES;
            mbar_arrive_expect_tx(v_full(s), L::K_BYTES);
            for (int c = 0; c < L::NSUB; ++c)
              tma_load_4d(&tmV, vb + c * SUB, v_full(s), c * 64, (j - 1) * 128, it.hk, it.b);
            ++nv;
          }
        }
        g += nK;
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
        if (qn > 0) {
          const int i = qn - 1;
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(q_full(i % QB), (i / QB) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t IDESC_S = idesc_f16(128, 128, 1u, 0u, 0u);
      constexpr uint32_t IDESC_O = idesc_f16(128, D, 1u, 0u, 1u);
      bool ok = true, issued = false;
      int g = 0, qn = 0;
      int base[2] = {0, 0};     // blocks of tile t in earlier items (S, P and PV barrier phases)
      int pv_seen[2] = {0, 0};  // PV MMAs of tile t known complete (global count)
      for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
        const FwdItem it = fwd_item(a, w);
        const int nA = it.nA, nB = it.nB;
        const int nK = max(nA, nB);
        if (nK == 0) continue;
        const int qb = qn % QB;
        if (!mbar_wait(q_full(qb), (qn / QB) & 1, BRAIN_ERR_TIMEOUT_FULL, 120, abort_flag)) {
          ok = false;
          break;
        }
        auto issue_s = [&](int t, int jj) {  // S_t = Q_t K_jj^T into TMEM columns [128 t, 128 t + 128)
          const uint32_t kb = sKV + ((g + jj) % ST) * L::STAGE_BYTES;
          const uint32_t qbuf = sQ + (qb * 2 + t) * L::Q_BYTES;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t o = (kk / 4) * SUB + (kk % 4) * 32;
            tc_mma_f16(tmem + 128u * t, smem_desc_sw128(qbuf + o, 16, 1024), smem_desc_sw128(kb + o, 16, 1024),
                       IDESC_S, kk > 0 ? 1u : 0u);
          }
          tc_commit(s_full(t));
        };
        auto issue_pv = [&](int t, int jj) {  // O_t += P_t V_jj, P_t (bf16) from TMEM columns [128 t, 128 t + 64)
          const uint32_t vb = sKV + ((g + jj) % ST) * L::STAGE_BYTES + L::K_BYTES;
#pragma unroll
          for (int kk = 0; kk < 128 / 16; ++kk)
            tc_mma_f16_ts(tmem + 256 + 128u * t, tmem + 128u * t + (uint32_t)(kk * 8),
                          smem_desc_sw128(vb + kk * 2048, SUB, 1024), IDESC_O, (jj > 0 || kk > 0) ? 1u : 0u);
          if (jj == (t == 0 ? nA : nB) - 1) tc_commit(o_final(t));
        };
        int s_n[2] = {0, 0}, pv_n[2] = {0, 0};  // S / PV issued for this item
        int k_rel = 0, v_rel = 0;               // K / V blocks of this item released to the producer
        uint64_t t0 = globaltimer();
        uint32_t idle = 0;
        while (ok && (pv_n[0] < nA || pv_n[1] < nB)) {
          bool progress = false;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int nt = t == 0 ? nA : nB;
            const int j = pv_n[t];
            if (j < nt && s_n[t] == j + 1 && mbar_test_wait(p_full(t), (base[t] + j) & 1) &&
                mbar_test_wait(v_full((g + j) % ST), ((g + j) / ST) & 1)) {
              tc_fence_after();
              issue_pv(t, j);
              tc_commit(pv_done(t));
              pv_n[t] = j + 1;
              issued = true;
              progress = true;
            }
            // S_t(j1) overwrites the columns that the last PV of tile t reads: wait for that PV first
            const int j1 = s_n[t];
            if (j1 < nt && pv_n[t] == j1) {
              const int pv_all = base[t] + j1;  // PV MMAs of tile t issued so far
              if (pv_seen[t] < pv_all && mbar_test_wait(pv_done(t), (pv_all - 1) & 1)) pv_seen[t] = pv_all;
              if (pv_seen[t] == pv_all && mbar_test_wait(k_full((g + j1) % ST), ((g + j1) / ST) & 1)) {
                tc_fence_after();
                issue_s(t, j1);
                s_n[t] = j1 + 1;
                issued = true;
                progress = true;
              }
            }
          }
          // hand K / V stages back once every tile that needs the block has issued its MMA on it
          while (k_rel < nK && (s_n[0] > k_rel || k_rel >= nA) && (s_n[1] > k_rel || k_rel >= nB)) {
            tc_commit(k_empty((g + k_rel) % ST));
            ++k_rel;
          }
          while (v_rel < nK && (pv_n[0] > v_rel || v_rel >= nA) && (pv_n[1] > v_rel || v_rel >= nB)) {
            tc_commit(v_empty((g + v_rel) % ST));
            ++v_rel;
          }
          if (progress) {
            idle = 0;
            t0 = globaltimer();
          } else if ((++idle & 255u) == 0) {
            if (*abort_flag) {
              ok = false;
            } else if (globaltimer() - t0 > kWaitBudgetNs) {
              set_status(BRAIN_ERR_TIMEOUT_ACC, 126);
              *abort_flag = 1;
              ok = false;
            }
          }
        }
        if (!ok) break;
        tc_commit(q_empty(qb));  // the item's S MMAs were all issued: its query buffer frees when they finish
        ++qn;
        g += nK;
        base[0] += nA;
        base[1] += nB;
      }
      if (!ok && issued) {
        tc_commit(drain);
        uint64_t t1 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t1 < 100000000ull) {
        }
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;");
    // ---------------- softmax warpgroups: tile t, TMEM lane quadrant q, thread = one query row
    const int t = (warp - 4) >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const uint32_t sbuf = tmem + 128u * t + lane_addr;
    const uint32_t obuf = tmem + 256 + 128u * t + lane_addr;
    bool ok = true;
    int base = 0, nfin = 0;  // blocks of this tile in earlier items; items of this tile with output in TMEM
    for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
      const FwdItem it = fwd_item(a, w);
      const int n = t == 0 ? it.nA : it.nB;
      const int qi = it.m0 + 128 * t + r;
      const int b = it.b, h = it.h;
      const int limit = a.causal ? min(qi + off, a.Sk - 1) : a.Sk - 1;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        if (ok && !mbar_wait(s_full(t), (base + j) & 1, BRAIN_ERR_TIMEOUT_ACC, 130, abort_flag)) ok = false;
        // a give-up is made uniform per warp (tcgen05.ld is warp-collective); the other warps of the
        // warpgroup then time out or see the abort flag in their own waits
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(sbuf + (uint32_t)(c * 32), reinterpret_cast<uint32_t*>(s + c * 32));
        tc_wait_ld();
        const int n0 = j * 128;
        const bool need_mask = __any_sync(0xffffffffu, n0 + 127 > limit);
        float mxp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = -INFINITY;
        if constexpr (BIAS) {
          // scores in log2 units with the bias added, -inf where masked: t = s c + bias log2(e)
          uint32_t kbits[4] = {~0u, ~0u, ~0u, ~0u};  // key n0 + 4 i + t is attended iff bit i of kbits[t]
          if (a.kmask) {
            const uint8_t* km = a.kmask + (int64_t)b * a.Sk;
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
              const int key = n0 + 4 * lane + t4;
              kbits[t4] = __ballot_sync(0xffffffffu, key < a.Sk && km[key] != 0);
            }
          }
          const bool row_ok = qi < a.Sq;
          const float* rb = a.relb ? a.relb + (int64_t)h * (a.Sq + a.Sk - 1) + (n0 - qi + a.Sq - 1) : nullptr;
#pragma unroll
          for (int k = 0; k < 128; ++k) {
            const bool valid = n0 + k <= limit && ((kbits[k & 3] >> (k >> 2)) & 1u);
            const float bias = (rb && valid && row_ok) ? __ldg(rb + k) * kLog2e : 0.f;
            s[k] = valid ? fmaf(s[k], a.scale_log2, bias) : -INFINITY;
            mxp[k & 7] = fmaxf(mxp[k & 7], s[k]);
          }
        } else if (need_mask) {
#pragma unroll
          for (int k = 0; k < 128; ++k) {
            if (n0 + k > limit) s[k] = -INFINITY;
            mxp[k & 7] = fmaxf(mxp[k & 7], s[k]);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 128; ++k) mxp[k & 7] = fmaxf(mxp[k & 7], s[k]);
        }
        // BIAS: the scores are already scaled; otherwise raw scores, and the log2-domain scale (> 0) is
        // applied in the exponent's FFMA: max(c s) = c max(s)
        const float mx = (BIAS ? 1.f : a.scale_log2) * fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                                             fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
        float alpha = 1.f;
        if (mx > m_used + kRescaleThreshold || (m_used == -INFINITY && mx > -INFINITY)) {
          alpha = exp2f(m_used - mx);  // 0 when m_used == -inf
          m_used = mx;
        }
        const float mu = m_used == -INFINITY ? 0.f : m_used;
        // O is final for step j-1 (S_t(j) was issued after PV_t(j-1) completed); rescale it before P_t(j)
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t ov[32];
            tmem_ld32(obuf + (uint32_t)(c * 32), ov);
            tc_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) ov[k] = __float_as_uint(__uint_as_float(ov[k]) * alpha);
            tmem_st32(obuf + (uint32_t)(c * 32), ov);
          }
        }
        float sp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) sp[u] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 32 keys -> 16 packed columns of P over S
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float p0 = BIAS ? ex2_fast(s[c * 32 + k] - mu) : ex2_fast(fmaf(s[c * 32 + k], a.scale_log2, -mu));
            const float p1 = BIAS ? ex2_fast(s[c * 32 + k + 1] - mu)
                                  : ex2_fast(fmaf(s[c * 32 + k + 1], a.scale_log2, -mu));
            sp[(k >> 1) & 7] += p0 + p1;
            pk[k / 2] = pack_bf16x2(p0, p1);
          }
          tmem_st16(sbuf + (uint32_t)(c * 16), pk);
        }
        l = l * alpha + (((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7])));
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(p_full(t));
      }
      if (!ok) break;
      base += n;
      // epilogue
      float inv = 0.f;
      bool have = n > 0;
      if (have) {
        if (!mbar_wait(o_final(t), nfin & 1, BRAIN_ERR_TIMEOUT_ACC, 132, abort_flag)) ok = false;
        ++nfin;
        // tcgen05.ld is warp-collective: decide per warp
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
      }
      if (l > 0.f) inv = 1.f / l;
      __nv_bfloat16* orow = a.o + (int64_t)b * a.ob + (int64_t)h * a.oh + (int64_t)qi * a.os;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        if (have) {
          tmem_ld32(obuf + (uint32_t)(c * 32), ov);
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
      if (qi < a.Sq && a.lse)
        a.lse[((int64_t)b * a.Hq + h) * a.Sq + qi] = l > 0.f ? (m_used + log2f(l)) * kLn2 : -INFINITY;
      // the output columns were read: the next item's first PV (issued after this warpgroup's p_full
      // arrival) may overwrite them
      tc_fence_before();
    }
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

template <int D, bool BIAS>
int launch(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const FwdArgs& a, cudaStream_t st) {
  using L = FwdLayout<D>;
  auto kern = fa_fwd_tc_kernel<D, BIAS>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
  const int items = ((a.Sq + 255) / 256) * a.B * a.Hq;
  const int grid = std::min(items, brain_host::num_sms());  // persistent: CTAs loop over work items
  kern<<<grid, kThreads, L::TOTAL, st>>>(q, k, v, a);
  return (int)cudaGetLastError();
}

}  // namespace

BRAIN_STATUS_READER(attention_tc)

namespace {
int fwd_tc(const void* q, const void* k, const void* v, const int64_t* s9, void* o, const int64_t* ostr, float* lse,
           int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale, int causal, const uint8_t* kmask,
           const float* relb, cudaStream_t st) {
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
  a.kmask = kmask;
  a.relb = relb;
  if (kmask || relb) return D == 64 ? launch<64, true>(tq, tk, tv, a, st) : launch<128, true>(tq, tk, tv, a, st);
  return D == 64 ? launch<64, false>(tq, tk, tv, a, st) : launch<128, false>(tq, tk, tv, a, st);
}
}  // namespace

// Returns cudaErrorNotSupported (without launching) when the layout is outside what the tensor-core
// path handles (D not 64/128, strides not 16-byte multiples, misaligned bases); callers then use the
// mma.sync kernel.
BRAIN_API int brain_attn_fwd_tc(const void* q, const void* k, const void* v, const int64_t* s9, void* o,
                                const int64_t* ostr, float* lse, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                                float scale, int causal, cudaStream_t st) {
  return fwd_tc(q, k, v, s9, o, ostr, lse, B, Hq, Hkv, Sq, Sk, D, scale, causal, nullptr, nullptr, st);
}

// Same, with a key padding mask kmask [B, Sk] (uint8, non-zero = attend; may be null) and an additive bias
// relb [Hq, Sq + Sk - 1] (float32, natural-log units; element (k - q) + Sq - 1 is added to score (q, k);
// may be null). Query rows whose keys are all masked get a zero output and lse = -inf.
BRAIN_API int brain_attn_fwd_tc_masked(const void* q, const void* k, const void* v, const int64_t* s9, void* o,
                                       const int64_t* ostr, float* lse, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                                       float scale, int causal, const uint8_t* kmask, const float* relb,
                                       cudaStream_t st) {
  return fwd_tc(q, k, v, s9, o, ostr, lse, B, Hq, Hkv, Sq, Sk, D, scale, causal, kmask, relb, st);
}
