// Flash-attention backward on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Two deterministic passes built from one templated kernel (no atomics):
//   DKDV: a CTA owns 128 keys of one kv head and streams 64-query blocks of every q head of the
//         GQA group:   S^T = K Q^T,  dP^T = V dO^T            (TMEM, double-buffered)
//                      P^T = exp2(S^T * c - lse[q]),  dS^T = P^T (dP^T - delta[q])   (CUDA cores)
//                      dV += P^T dO,  dK += dS^T Q            (TMEM accumulators)
//   DQ:   a CTA owns 128 queries of one q head and streams 64-key blocks:
//                      S = Q K^T, dP = dO V^T,  P = exp2(S * c - lse[row]),  dS = P (dP - delta[row])
//                      dQ += dS K
// Roles per CTA (10 warps): warp 0 TMA (4-D tensor maps over the caller's strides, SWIZZLE_128B,
// CTA-local destinations), warp 1 single-thread MMA issuer, warps 2..9 elementwise: two warps per TMEM
// lane quadrant (thread = row), each taking 32 of a block's 64 columns, so two warps per scheduler hide
// each other's TMEM-load and exponential latency. They write P/dS as bf16 K-major tiles that the
// accumulate MMAs read from shared memory; the tiles are double-buffered, so the elementwise warps store
// block i+1 while the accumulate MMAs of block i still read theirs. The
// streamed operand is read a second time as an MN-major B operand, so nothing is transposed.
// Bounded waits report through the status word. Reference: the Value-graph attention VJPs
// (crates/brain-autograd/src/grad_fns/mod.rs:327-420); mask/scale conventions as in attention_tc.cu.
#include "common.cuh"

using namespace brain;

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kThreads = 320;
constexpr int kEwThreads = 256;  // elementwise threads (warps 2..9)
constexpr int SUB128 = 128 * 128;  // 128 rows x 64 bf16 (16 KB)
constexpr int SUB64 = 64 * 128;    // 64 rows x 64 bf16 (8 KB)

enum { DKDV = 0, DQ = 1 };

struct BwdArgs {
  const float* lse;    // [B, Hq, Sq] natural log
  const float* delta;  // [B, Hq, Sq]
  __nv_bfloat16 *out1, *out2;  // DKDV: dV, dK   DQ: dQ
  int64_t o1b, o1s, o1h, o2b, o2s, o2h;
  int B, Hq, Hkv, Sq, Sk;
  float scale, scale_log2;
  int causal;
  // optional (BIAS kernels), as in the forward: key padding mask [B, Sk] and relative bias relb[Hq, Sq + Sk - 1]
  const uint8_t* kmask;
  const float* relb;
};

template <int D, int MODE>
struct BwdLayout {
  static constexpr int NSUB = D / 64;
  static constexpr int STAGES = D == 64 ? 4 : 3;
  static constexpr int A_BYTES = NSUB * SUB128;  // one row operand [128, D]
  static constexpr int B_BYTES = NSUB * SUB64;   // one streamed operand [64, D]
  static constexpr int ABUF = D == 64 ? 2 : 1;   // row-operand buffers: the next item's load overlaps this one
  static constexpr int A_OFF = 0;                // ABUF x (A1, A2)
  static constexpr int B_OFF = ABUF * 2 * A_BYTES;  // stages of (B1, B2)
  static constexpr int STAGE_BYTES = 2 * B_BYTES;
  static constexpr int NC = MODE == DKDV ? 2 : 1;  // C tiles (P^T, dS^T) or (dS)
  static constexpr int C_OFF = B_OFF + STAGES * STAGE_BYTES;
  static constexpr int C_BYTES = NC * SUB128;  // one buffer of C tiles; two buffers
  static constexpr int LD_OFF = C_OFF + 2 * C_BYTES;  // DKDV: per block lse*log2e and delta, 2 buffers
  static constexpr int BAR_OFF = LD_OFF + 2 * 128 * 4;
  // TMEM S/dP buffers (double-buffered: the scores of block i+1 are computed while the elementwise warps
  // work on block i); the accumulators follow them
  static constexpr int NBUF = 2;
  static constexpr int ACC = NBUF * 128;  // first accumulator column
  // a_full[ABUF], a_empty[ABUF], b_full[S], b_empty[S], sd_full[3], sd_free[3], c_full[2], c_free[2], acc_done,
  // drain, st_free[2]
  static constexpr int NBAR = 2 * ABUF + 2 * STAGES + 6 + 6 + 2;
  static constexpr int TOTAL = BAR_OFF + NBAR * 8 + 16 + 1024;
  static_assert(TOTAL <= 232448, "more dynamic shared memory than one CTA may use");
};

template <int D, int MODE, bool BIAS>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap mA1, const __grid_constant__ CUtensorMap mA2,
                     const __grid_constant__ CUtensorMap mB1, const __grid_constant__ CUtensorMap mB2, BwdArgs a) {
  using L = BwdLayout<D, MODE>;
  constexpr int ST = L::STAGES;
  constexpr int AB = L::ABUF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sB = sbase + L::B_OFF, sCb = sbase + L::C_OFF;
  const uint32_t bars = sbase + L::BAR_OFF;
  auto a_full = [&](int i) { return bars + 8u * i; };
  auto a_empty = [&](int i) { return bars + 8u * (AB + i); };
  constexpr int B0 = 2 * AB;
  auto b_full = [&](int s) { return bars + 8u * (B0 + s); };
  auto b_empty = [&](int s) { return bars + 8u * (B0 + ST + s); };
  constexpr int NB = L::NBUF;
  auto sd_full = [&](int i) { return bars + 8u * (B0 + 2 * ST + i); };
  auto sd_free = [&](int i) { return bars + 8u * (B0 + 3 + 2 * ST + i); };
  auto c_full = [&](int i) { return bars + 8u * (B0 + 6 + 2 * ST + i); };
  auto c_free = [&](int i) { return bars + 8u * (B0 + 8 + 2 * ST + i); };
  const uint32_t acc_done = bars + 8u * (B0 + 10 + 2 * ST);
  const uint32_t drain = bars + 8u * (B0 + 11 + 2 * ST);
  // DKDV: a group's statistics slot may be rewritten once all its threads have read it for the previous block
  auto st_free = [&](int grp) { return bars + 8u * (B0 + 12 + 2 * ST + grp); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + L::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int group = a.Hq / a.Hkv;
  const int off = a.Sk - a.Sq;

  // ---- work items: one 128-row block of the row operand (keys for DKDV, queries for DQ) of one head;
  // the block index is the slow coordinate, heaviest blocks first under a causal mask; CTAs take items
  // round-robin and every barrier's phase count runs on across items
  const int nrb = MODE == DKDV ? (a.Sk + 127) / 128 : (a.Sq + 127) / 128;
  const int BHr = MODE == DKDV ? a.B * a.Hkv : a.B * a.Hq;
  const int items = nrb * BHr;
  int b, hrow;      // batch and head of the row operand (kv head for DKDV, q head for DQ)
  int r0;           // first row (key for DKDV, query for DQ)
  int first_blk;    // first streamed 64-block index
  int nblk;         // streamed blocks per head
  int niter;        // total iterations (DKDV: x group)
  auto decomp = [&](int w) {
    const int rbi = w / BHr, bh = w - rbi * BHr;
    if (MODE == DKDV) {
      b = bh / a.Hkv;
      hrow = bh % a.Hkv;
      r0 = rbi * 128;
      int qstart = 0;
      if (a.causal) qstart = max(0, r0 - off);
      first_blk = qstart / 64;
      const int tot = (a.Sq + 63) / 64;
      nblk = max(0, tot - first_blk);
      niter = nblk * group;
    } else {
      const int mb = a.causal ? (nrb - 1 - rbi) : rbi;
      b = bh / a.Hq;
      hrow = bh % a.Hq;
      r0 = mb * 128;
      first_blk = 0;
      int kend = a.Sk;
      if (a.causal) kend = min(a.Sk, r0 + 128 + off);
      nblk = kend > 0 ? (kend + 63) / 64 : 0;
      niter = nblk;
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < AB; ++i) {
      mbar_init(a_full(i), 1);
      mbar_init(a_empty(i), 1);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(b_full(s), 1);
      mbar_init(b_empty(s), 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(sd_full(i), 1);
      mbar_init(sd_free(i), kEwThreads / 2);  // read by one group of elementwise warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(c_full(i), kEwThreads / 2);
      mbar_init(c_free(i), 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    mbar_init(st_free(0), kEwThreads / 2);
    mbar_init(st_free(1), kEwThreads / 2);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // buf b: S at b*128, dP at b*128+64; acc1 at 256; acc2 at 256 + D

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int g = 0;   // streamed blocks issued (ring position)
      int an = 0;  // items with work so far (row-operand buffer position)
      bool ok = true;
      for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
        decomp(w);
        if (niter == 0) continue;
        const int ab = an % AB;
        if (!mbar_wait(a_empty(ab), ((an / AB) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 209, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t sA1 = sbase + L::A_OFF + ab * 2 * L::A_BYTES, sA2 = sA1 + L::A_BYTES;
        mbar_arrive_expect_tx(a_full(ab), 2 * L::A_BYTES);
        for (int c = 0; c < L::NSUB; ++c) {
          tma_load_4d(&mA1, sA1 + c * SUB128, a_full(ab), c * 64, r0, hrow, b);
          tma_load_4d(&mA2, sA2 + c * SUB128, a_full(ab), c * 64, r0, hrow, b);
        }
        ++an;
        for (int i = 0; i < niter; ++i, ++g) {
          const int s = g % ST;
          if (!mbar_wait(b_empty(s), ((g / ST) & 1) ^ 1, BRAIN_ERR_TIMEOUT_EMPTY, 210, abort_flag)) {
            ok = false;
            break;
          }
          int hb, row;
          if (MODE == DKDV) {
            hb = hrow * group + i / nblk;
            row = (first_blk + i % nblk) * 64;
          } else {
            hb = hrow / group;
            row = i * 64;
          }
          const uint32_t st = sB + s * L::STAGE_BYTES;
          mbar_arrive_expect_tx(b_full(s), L::STAGE_BYTES);
          for (int c = 0; c < L::NSUB; ++c) {
            tma_load_4d(&mB1, st + c * SUB64, b_full(s), c * 64, row, hb, b);
            tma_load_4d(&mB2, st + L::B_BYTES + c * SUB64, b_full(s), c * 64, row, hb, b);
          }
        }
      }
      if (!ok) {  // aborted: let the copies still in flight land (the last ST streamed blocks, the last rows)
        for (int j = max(0, g - ST); j < g; ++j) {
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(b_full(j % ST), (j / ST) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
        if (an > 0) {
          const int j = an - 1;
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(a_full(j % AB), (j / AB) & 1) && globaltimer() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t IDESC_S = idesc_f16(128, 64, 1u, 0u, 0u);
      constexpr uint32_t IDESC_ACC = idesc_f16(128, D, 1u, 0u, 1u);
      bool ok = true, issued = false;
      int g = 0, an = 0;
      for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
        decomp(w);
        if (niter == 0) continue;
        const int ab = an % AB;
        const uint32_t sA1 = sbase + L::A_OFF + ab * 2 * L::A_BYTES, sA2 = sA1 + L::A_BYTES;
        if (!mbar_wait(a_full(ab), (an / AB) & 1, BRAIN_ERR_TIMEOUT_FULL, 220, abort_flag)) {
          ok = false;
          break;
        }
        auto issue_scores = [&](int i) {
          const int gi = g + i;
          const uint32_t st = sB + (gi % ST) * L::STAGE_BYTES;
          const uint32_t d = tmem + (uint32_t)((gi % NB) * 128);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = (kk / 4) * SUB128 + (kk % 4) * 32;
            const uint32_t ob = (kk / 4) * SUB64 + (kk % 4) * 32;
            tc_mma_f16(d, smem_desc_sw128(sA1 + oa, 16, 1024), smem_desc_sw128(st + ob, 16, 1024), IDESC_S,
                       kk > 0 ? 1u : 0u);
            tc_mma_f16(d + 64, smem_desc_sw128(sA2 + oa, 16, 1024),
                       smem_desc_sw128(st + L::B_BYTES + ob, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
          }
          tc_commit(sd_full(gi % NB));
        };
        // score block i waits for its streamed operands and for its TMEM buffer (freed by the elementwise
        // warps' reads of global block gi - NB)
        auto wait_scores = [&](int i) {
          const int gi = g + i;
          return mbar_wait(b_full(gi % ST), (gi / ST) & 1, BRAIN_ERR_TIMEOUT_FULL, 222, abort_flag) &&
                 mbar_wait(sd_free(gi % NB), ((gi / NB) & 1) ^ 1, BRAIN_ERR_TIMEOUT_ACC, 223, abort_flag);
        };
        // the first NB-1 score blocks go out before the loop; block i+NB-1 then goes out in iteration i
        for (int in = 0; ok && in < NB - 1 && in < niter; ++in) {
          if (!wait_scores(in)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_scores(in);
          issued = true;
        }
        for (int i = 0; ok && i < niter; ++i) {
          if (i + NB - 1 < niter) {
            const int in = i + NB - 1;
            if (!wait_scores(in)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_scores(in);
          }
          const int gi = g + i;
          if (!mbar_wait(c_full(gi & 1), (gi / 2) & 1, BRAIN_ERR_TIMEOUT_ACC, 224, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sB + (gi % ST) * L::STAGE_BYTES;
          const uint32_t sC = sCb + (gi & 1) * L::C_BYTES;
#pragma unroll
          for (int kk = 0; kk < 64 / 16; ++kk) {
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            const uint64_t c0 = smem_desc_sw128(sC + kk * 32, 16, 1024);
            if (MODE == DKDV) {
              const uint64_t c1 = smem_desc_sw128(sC + SUB128 + kk * 32, 16, 1024);
              // dV += P^T dO   (dO = B2, MN-major);  dK += dS^T Q   (Q = B1, MN-major)
              tc_mma_f16(tmem + L::ACC, c0, smem_desc_sw128(st + L::B_BYTES + kk * 2048, SUB64, 1024), IDESC_ACC,
                         acc);
              tc_mma_f16(tmem + L::ACC + D, c1, smem_desc_sw128(st + kk * 2048, SUB64, 1024), IDESC_ACC, acc);
            } else {
              // dQ += dS K   (K = B1, MN-major)
              tc_mma_f16(tmem + L::ACC, c0, smem_desc_sw128(st + kk * 2048, SUB64, 1024), IDESC_ACC, acc);
            }
          }
          tc_commit(c_free(gi & 1));
          tc_commit(b_empty(gi % ST));
        }
        if (!ok) break;
        tc_commit(a_empty(ab));  // every score MMA of the item was issued: its row operands free when done
        tc_commit(acc_done);
        ++an;
        g += niter;
      }
      if (!ok && issued) {
        tc_commit(drain);
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- elementwise warps (2..9): quadrant q of the TMEM lanes. Two groups of four warps
    // take alternate blocks (group hc the blocks of global index parity hc, so each TMEM score buffer, C tile
    // and statistics slot has one owner): while one group waits for its next scores the other computes.
    // Each thread covers its row's 64 columns of a block in two chunks of 32.
    const int q = warp & 3;
    const int hc = (warp - 2) >> 2;                  // group; also the column half of the epilogue
    const int et = (warp - 2 - 4 * hc) * 32 + lane;  // 0..127 within the group
    const int r = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    bool ok = true;
    int g = 0, nacc = 0;  // streamed blocks of earlier items; items whose accumulators were read
    for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
    decomp(w);
    const int row = r0 + r;
    float row_lse2 = 0.f, row_delta = 0.f;
    if (MODE == DQ && row < a.Sq) {
      const int64_t idx = ((int64_t)b * a.Hq + hrow) * a.Sq + row;
      row_lse2 = a.lse[idx] * kLog2e;
      row_delta = a.delta[idx];
    }
    const bool row_valid_q = MODE == DQ ? (row < a.Sq) : true;
    // DKDV: the 64 query statistics (lse * log2e, delta) of block i, one per thread et < 128, loaded
    // one iteration ahead so that their L2 latency hides behind the previous block's work
    auto stat = [&](int i) -> float {
      if (MODE != DKDV || i >= niter) return 0.f;
      const int hc_ = hrow * group + i / nblk;
      const int qi = (first_blk + i % nblk) * 64 + (et & 63);
      if (qi >= a.Sq) return 0.f;
      const int64_t base = ((int64_t)b * a.Hq + hc_) * a.Sq + qi;
      return et < 64 ? __ldg(a.lse + base) * kLog2e : __ldg(a.delta + base);
    };
    const int i0 = (hc ^ g) & 1;  // this group's first block of the item
    float v_next = stat(i0);
    auto tbuf = [&](int gi, int h) { return tmem + (uint32_t)((gi % NB) * 128 + h * 32) + lane_addr; };
    // DKDV leaves the loop only through its per-iteration group barrier (the group's threads together); DQ
    // has no barrier in the loop
    for (int i = i0; i < niter && (MODE == DKDV || ok); i += 2) {
      const int gi = g + i;
      int col0;
      if (MODE == DKDV) col0 = (first_blk + i % nblk) * 64;
      else col0 = i * 64;
      float* sld = reinterpret_cast<float*>(smem + L::LD_OFF) + (gi & 1) * 128;
      float s[32], dp[32];
      if (MODE == DKDV) {
        // the block's statistics go through shared memory (read back as broadcasts) instead of every
        // thread loading all 64. The barrier also makes the give-up decision uniform: every thread
        // reaches it after bounded waits and all of them leave the loop together when any wait gave up.
        const float v = v_next;
        v_next = stat(i + 2);
        if (ok) ok = mbar_wait(sd_full(gi % NB), (gi / NB) & 1, BRAIN_ERR_TIMEOUT_ACC, 230, abort_flag);
        // the group's slot held the statistics of its previous block (k - 1): wait until every thread of
        // the group has read them
        const int k = gi >> 1;
        if (ok && k > 0) ok = mbar_wait(st_free(hc), (k - 1) & 1, BRAIN_ERR_TIMEOUT_ACC, 233, abort_flag);
        sld[et] = v;
        if (!bar_sync_and(1 + hc, kEwThreads / 2, ok)) {
          ok = false;
          break;
        }
      } else {
        if (!mbar_wait(sd_full(gi % NB), (gi / NB) & 1, BRAIN_ERR_TIMEOUT_ACC, 230, abort_flag)) {
          ok = false;
          break;
        }
      }
      // C buffer gi&1 was last read by the accumulate MMAs of global block gi-2 (this group's previous one)
      const uint32_t sC = sCb + (gi & 1) * L::C_BYTES;
      if (gi > 1 && !mbar_wait(c_free(gi & 1), ((gi - 2) / 2) & 1, BRAIN_ERR_TIMEOUT_ACC, 231, abort_flag)) {
        ok = false;
        if (MODE == DKDV) continue;  // leaves at the next barrier, together with the group's other threads
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
      tmem_ld32(tbuf(gi, h), reinterpret_cast<uint32_t*>(s));
      tmem_ld32(tbuf(gi, h) + 64, reinterpret_cast<uint32_t*>(dp));
      tc_wait_ld();
      if (h == 1) {  // both chunks are in registers: the score buffer may take the next block
        tc_fence_before();
        mbar_arrive(sd_free(gi % NB));
      }
      const int cb = h * 32;  // this chunk's first column of the block
      uint32_t pk[16], dk[16];
      if (MODE == DKDV) {
        const int key = row;
        // masking only where this warp's 32 queries reach past Sq or across the causal diagonal: one
        // warp-uniform branch around a separate loop, so the common path has no per-element tests
        const bool all_valid = col0 + cb + 31 < a.Sq && !(a.causal && key > col0 + cb + off);
        const float4* l2v = reinterpret_cast<const float4*>(sld + cb);        // broadcast reads
        const float4* dev = reinterpret_cast<const float4*>(sld + 64 + cb);
        float pv[32];
        if constexpr (BIAS) {
          // this thread's key: padding mask and the bias per query column, every test per element
          const int hcol = hrow * group + i / nblk;
          const bool key_ok = key < a.Sk && (!a.kmask || a.kmask[(int64_t)b * a.Sk + key] != 0);
          const float* rb = a.relb ? a.relb + (int64_t)hcol * (a.Sq + a.Sk - 1) + (key - col0 - cb + a.Sq - 1) : nullptr;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int qi = col0 + cb + c;
            const bool valid = key_ok && qi < a.Sq && !(a.causal && key > qi + off);
            const float bias = (rb && valid) ? __ldg(rb - c) * kLog2e : 0.f;
            pv[c] = valid ? ex2_fast(fmaf(s[c], a.scale_log2, bias - sld[cb + c])) : 0.f;
          }
        } else {
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 l4 = l2v[c4];
          pv[4 * c4] = ex2_fast(fmaf(s[4 * c4], a.scale_log2, -l4.x));
          pv[4 * c4 + 1] = ex2_fast(fmaf(s[4 * c4 + 1], a.scale_log2, -l4.y));
          pv[4 * c4 + 2] = ex2_fast(fmaf(s[4 * c4 + 2], a.scale_log2, -l4.z));
          pv[4 * c4 + 3] = ex2_fast(fmaf(s[4 * c4 + 3], a.scale_log2, -l4.w));
        }
        }
        if (!BIAS && __any_sync(0xffffffffu, !all_valid)) {
          const int lim = a.causal ? key - off : -0x40000000;  // queries below lim are masked (causal)
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int qi = col0 + cb + c;
            pv[c] = (qi >= a.Sq || qi < lim) ? 0.f : pv[c];
          }
        }
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 d4 = dev[c4];
          const float d0 = pv[4 * c4] * (dp[4 * c4] - d4.x), d1 = pv[4 * c4 + 1] * (dp[4 * c4 + 1] - d4.y);
          const float d2 = pv[4 * c4 + 2] * (dp[4 * c4 + 2] - d4.z), d3 = pv[4 * c4 + 3] * (dp[4 * c4 + 3] - d4.w);
          pk[2 * c4] = pack_bf16x2(pv[4 * c4], pv[4 * c4 + 1]);
          pk[2 * c4 + 1] = pack_bf16x2(pv[4 * c4 + 2], pv[4 * c4 + 3]);
          dk[2 * c4] = pack_bf16x2(d0, d1);
          dk[2 * c4 + 1] = pack_bf16x2(d2, d3);
        }
      } else {
        const bool all_valid = row_valid_q && col0 + cb + 31 < a.Sk && !(a.causal && col0 + cb + 31 > row + off);
        float pv[32];
        if constexpr (BIAS) {
          uint32_t kbits[2] = {~0u, ~0u};  // key col0 + 2 i + t of the block is attended iff bit i of kbits[t]
          if (a.kmask) {
            const uint8_t* km = a.kmask + (int64_t)b * a.Sk;
#pragma unroll
            for (int t2 = 0; t2 < 2; ++t2) {
              const int key = col0 + 2 * lane + t2;
              kbits[t2] = __ballot_sync(0xffffffffu, key < a.Sk && km[key] != 0);
            }
          }
          const float* rb = a.relb ? a.relb + (int64_t)hrow * (a.Sq + a.Sk - 1) + (col0 + cb - row + a.Sq - 1) : nullptr;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int key = col0 + cb + c, idx = cb + c;
            const bool valid = row_valid_q && key < a.Sk && !(a.causal && key > row + off) &&
                               ((kbits[idx & 1] >> (idx >> 1)) & 1u);
            const float bias = (rb && valid) ? __ldg(rb + c) * kLog2e : 0.f;
            pv[c] = valid ? ex2_fast(fmaf(s[c], a.scale_log2, bias - row_lse2)) : 0.f;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) pv[c] = ex2_fast(fmaf(s[c], a.scale_log2, -row_lse2));
        }
        if (!BIAS && __any_sync(0xffffffffu, !all_valid)) {
          const int lim = !row_valid_q ? -1 : (a.causal ? min(row + off, a.Sk - 1) : a.Sk - 1);  // last visible key
#pragma unroll
          for (int c = 0; c < 32; ++c) pv[c] = (col0 + cb + c > lim) ? 0.f : pv[c];
        }
#pragma unroll
        for (int c = 0; c < 32; c += 2)
          dk[c / 2] = pack_bf16x2(pv[c] * (dp[c] - row_delta), pv[c + 1] * (dp[c + 1] - row_delta));
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {  // this chunk's 4 pieces of 8 columns (of 8 per 128 B row)
        const int c = h * 4 + cc;
        const uint32_t o = r * 128 + ((c ^ (r % 8)) * 16);
        if (MODE == DKDV) {
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sC + o), "r"(pk[4 * cc]),
                       "r"(pk[4 * cc + 1]), "r"(pk[4 * cc + 2]), "r"(pk[4 * cc + 3])
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sC + SUB128 + o), "r"(dk[4 * cc]),
                       "r"(dk[4 * cc + 1]), "r"(dk[4 * cc + 2]), "r"(dk[4 * cc + 3])
                       : "memory");
        } else {
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sC + o), "r"(dk[4 * cc]),
                       "r"(dk[4 * cc + 1]), "r"(dk[4 * cc + 2]), "r"(dk[4 * cc + 3])
                       : "memory");
        }
      }
      }
      if (MODE == DKDV) mbar_arrive(st_free(hc));  // this thread's reads of the statistics slot are done
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(c_full(gi & 1));
    }
    ok = bar_sync_and(3, kEwThreads, ok);  // a give-up in the last block: all threads leave together
    if (!ok) break;
    g += niter;
    bool have = niter > 0;
    if (have) {
      if (!mbar_wait(acc_done, nacc & 1, BRAIN_ERR_TIMEOUT_ACC, 232, abort_flag)) ok = false;
      ++nacc;
      // the next item's first accumulate MMA (issued after every thread's c_full arrival) overwrites the
      // accumulators: all threads leave together when a wait gave up
      ok = bar_sync_and(3, kEwThreads, ok);
      if (!ok) break;
      tc_fence_after();
    }
    // epilogue: DKDV writes dV (acc1) and dK * scale (acc2); DQ writes dQ * scale (acc1)
    const bool store = MODE == DKDV ? (row < a.Sk) : (row < a.Sq);
#pragma unroll 1
    for (int which = 0; which < (MODE == DKDV ? 2 : 1); ++which) {
      __nv_bfloat16* base;
      float mul;
      if (MODE == DKDV) {
        base = which == 0 ? a.out1 + (int64_t)b * a.o1b + (int64_t)hrow * a.o1h + (int64_t)row * a.o1s
                          : a.out2 + (int64_t)b * a.o2b + (int64_t)hrow * a.o2h + (int64_t)row * a.o2s;
        mul = which == 0 ? 1.f : a.scale;
      } else {
        base = a.out1 + (int64_t)b * a.o1b + (int64_t)hrow * a.o1h + (int64_t)row * a.o1s;
        mul = a.scale;
      }
#pragma unroll 1
      for (int c = hc * (D / 64); c < (hc + 1) * (D / 64); ++c) {  // this warp's half of the D columns
        uint32_t ov[32];
        if (have) {
          tmem_ld32(tmem + L::ACC + (uint32_t)(which * D + c * 32) + lane_addr, ov);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) ov[k] = 0u;
        }
        if (store) {
          float v[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(ov[k]) * mul;
#pragma unroll
          for (int k = 0; k < 32; k += 8) store8(base + c * 32 + k, v + k);
        }
      }
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, i] = sum_d dO * O: L = D / 8 lanes per row (16-byte loads), 32 / L rows per warp, so short
// rows (d 64) keep every lane busy.
__global__ void bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, int64_t ob, int64_t os, int64_t oh,
                                 const __nv_bfloat16* __restrict__ dO, int64_t db, int64_t ds, int64_t dh,
                                 float* __restrict__ delta, int B, int H, int S, int D) {
  const int L = D / 8;               // lanes per row (D = 64 -> 8, D = 128 -> 16)
  const int rows_per_warp = 32 / L;
  const int lane = threadIdx.x % 32;
  const int64_t rowid = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * rows_per_warp + lane / L;
  const int sub = lane % L;
  float acc = 0.f;
  if (rowid < (int64_t)B * H * S) {
    const int i = (int)(rowid % S);
    const int bh = (int)(rowid / S);
    const int b = bh / H, h = bh % H;
    float x[8], y[8];
    load8(o + b * ob + h * oh + (int64_t)i * os + sub * 8, x);
    load8(dO + b * db + h * dh + (int64_t)i * ds + sub * 8, y);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += x[k] * y[k];
  }
  for (int off = L / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (sub == 0 && rowid < (int64_t)B * H * S) delta[rowid] = acc;
}

bool map4(CUtensorMap* m, const void* base, int D, int S, int H, int B, int64_t ss, int64_t sh, int64_t sb,
          int box_rows) {
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)ss * 2, (uint64_t)sh * 2, (uint64_t)sb * 2};
  uint32_t box[4] = {64, (uint32_t)box_rows, 1, 1};
  return brain_host::encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D, int MODE, bool BIAS>
int launch_kernel(const CUtensorMap& a1, const CUtensorMap& a2, const CUtensorMap& b1, const CUtensorMap& b2,
                  const BwdArgs& a, cudaStream_t st) {
  using L = BwdLayout<D, MODE>;
  auto kern = fa_bwd_tc_kernel<D, MODE, BIAS>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
  const int items = MODE == DKDV ? ((a.Sk + 127) / 128) * a.B * a.Hkv : ((a.Sq + 127) / 128) * a.B * a.Hq;
  const int grid = std::min(items, brain_host::num_sms());  // persistent: CTAs loop over work items
  kern<<<grid, kThreads, L::TOTAL, st>>>(a1, a2, b1, b2, a);
  return (int)cudaGetLastError();
}

template <int D, int MODE>
int launch_mode(const CUtensorMap& a1, const CUtensorMap& a2, const CUtensorMap& b1, const CUtensorMap& b2,
                const BwdArgs& a, cudaStream_t st) {
  if (a.kmask || a.relb) return launch_kernel<D, MODE, true>(a1, a2, b1, b2, a, st);
  return launch_kernel<D, MODE, false>(a1, a2, b1, b2, a, st);
}
}  // namespace

BRAIN_STATUS_READER(attention_bwd_tc)

namespace {
int bwd_tc(const void* q, const void* k, const void* v, const int64_t* s9, const void* o, const int64_t* ostr,
           const float* lse, const void* dout, const int64_t* dostr, void* dq, const int64_t* dqstr, void* dk,
           const int64_t* dkstr, void* dv, const int64_t* dvstr, float* delta, int B, int Hq, int Hkv, int Sq, int Sk,
           int D, float scale, int causal, const uint8_t* kmask, const float* relb, cudaStream_t st) {
  if (Hkv <= 0 || Hq % Hkv) return (int)cudaErrorInvalidValue;
  if (D != 64 && D != 128) return (int)cudaErrorNotSupported;
  const int64_t* all[6] = {s9, s9 + 3, s9 + 6, dostr, ostr, dqstr};
  for (int t = 0; t < 6; ++t)
    for (int i = 0; i < 3; ++i)
      if ((all[t][i] * 2) % 16) return (int)cudaErrorNotSupported;
  for (int i = 0; i < 3; ++i)
    if (dkstr[i] % 8 || dvstr[i] % 8) return (int)cudaErrorNotSupported;
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)dout | (uintptr_t)dq | (uintptr_t)dk | (uintptr_t)dv) &
      15)
    return (int)cudaErrorNotSupported;
  if (B * Hq == 0 || Sq == 0) return 0;
  // delta = rowsum(dO * O)
  {
    const int64_t rows = (int64_t)B * Hq * Sq;
    const int64_t rows_per_block = 8 * (32 / (D / 8));
    bwd_delta_kernel<<<(unsigned)((rows + rows_per_block - 1) / rows_per_block), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(o), ostr[0], ostr[1], ostr[2],
        reinterpret_cast<const __nv_bfloat16*>(dout), dostr[0], dostr[1], dostr[2], delta, B, Hq, Sq, D);
  }
  CUtensorMap mq128, mdo128, mk64, mv64, mk128, mv128, mq64, mdo64;
  bool ok = map4(&mq128, q, D, Sq, Hq, B, s9[1], s9[2], s9[0], 128) &&
            map4(&mdo128, dout, D, Sq, Hq, B, dostr[1], dostr[2], dostr[0], 128) &&
            map4(&mk64, k, D, Sk, Hkv, B, s9[4], s9[5], s9[3], 64) &&
            map4(&mv64, v, D, Sk, Hkv, B, s9[7], s9[8], s9[6], 64) &&
            map4(&mk128, k, D, Sk, Hkv, B, s9[4], s9[5], s9[3], 128) &&
            map4(&mv128, v, D, Sk, Hkv, B, s9[7], s9[8], s9[6], 128) &&
            map4(&mq64, q, D, Sq, Hq, B, s9[1], s9[2], s9[0], 64) &&
            map4(&mdo64, dout, D, Sq, Hq, B, dostr[1], dostr[2], dostr[0], 64);
  if (!ok) return (int)cudaErrorNotSupported;
  BwdArgs a{};
  a.lse = lse;
  a.delta = delta;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.Sq = Sq; a.Sk = Sk;
  a.scale = scale;
  a.scale_log2 = scale * kLog2e;
  a.causal = causal;
  a.kmask = kmask;
  a.relb = relb;
  // dK / dV
  a.out1 = reinterpret_cast<__nv_bfloat16*>(dv);
  a.o1b = dvstr[0]; a.o1s = dvstr[1]; a.o1h = dvstr[2];
  a.out2 = reinterpret_cast<__nv_bfloat16*>(dk);
  a.o2b = dkstr[0]; a.o2s = dkstr[1]; a.o2h = dkstr[2];
  int rc = D == 64 ? launch_mode<64, DKDV>(mk128, mv128, mq64, mdo64, a, st)
                   : launch_mode<128, DKDV>(mk128, mv128, mq64, mdo64, a, st);
  if (rc) return rc;
  // dQ
  a.out1 = reinterpret_cast<__nv_bfloat16*>(dq);
  a.o1b = dqstr[0]; a.o1s = dqstr[1]; a.o1h = dqstr[2];
  a.out2 = nullptr;
  return D == 64 ? launch_mode<64, DQ>(mq128, mdo128, mk64, mv64, a, st)
                 : launch_mode<128, DQ>(mq128, mdo128, mk64, mv64, a, st);
}
}  // namespace

// Same argument contract as brain_attn_bwd (attention.cu). Returns cudaErrorNotSupported without
// launching when the layout is outside the tensor-core path (D not 64/128, unaligned strides).
BRAIN_API int brain_attn_bwd_tc(const void* q, const void* k, const void* v, const int64_t* s9, const void* o,
                                const int64_t* ostr, const float* lse, const void* dout, const int64_t* dostr,
                                void* dq, const int64_t* dqstr, void* dk, const int64_t* dkstr, void* dv,
                                const int64_t* dvstr, float* delta, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                                float scale, int causal, cudaStream_t st) {
  return bwd_tc(q, k, v, s9, o, ostr, lse, dout, dostr, dq, dqstr, dk, dkstr, dv, dvstr, delta, B, Hq, Hkv, Sq, Sk, D,
                scale, causal, nullptr, nullptr, st);
}

// Same, with the forward's key padding mask and relative bias (brain_attn_fwd_tc_masked); the bias is
// treated as a constant (no gradient).
BRAIN_API int brain_attn_bwd_tc_masked(const void* q, const void* k, const void* v, const int64_t* s9, const void* o,
                                       const int64_t* ostr, const float* lse, const void* dout, const int64_t* dostr,
                                       void* dq, const int64_t* dqstr, void* dk, const int64_t* dkstr, void* dv,
                                       const int64_t* dvstr, float* delta, int B, int Hq, int Hkv, int Sq, int Sk,
                                       int D, float scale, int causal, const uint8_t* kmask, const float* relb,
                                       cudaStream_t st) {
  return bwd_tc(q, k, v, s9, o, ostr, lse, dout, dostr, dq, dqstr, dk, dkstr, dv, dvstr, delta, B, Hq, Hkv, Sq, Sk, D,
                scale, causal, kmask, relb, st);
}
