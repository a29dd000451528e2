// Backward passes that read the materialized probabilities P instead of
// recomputing them (sm_100a). They back the reference's P-taking helpers:
//
//   kFpDV     : dV = P^T dO                        backward_stubs.py:124-181
//               (_attn_bwd_dv_from_p_kernel, triton_attn_bwd_dv_from_p)
//   kFpRowsum : rowsum_i = sum_j P_ij (dO_i . V_j)  backward_stubs.py:184-255
//               (_attn_rowsum_kernel, triton_attn_rowsum_from_p), computed as
//               dO_i . (P V)_i: one P V product per tile instead of a dO V^T
//               tile product followed by a row reduction
//   kFpDK     : dK = scale * dS^T Q                 backward_stubs.py:313-359
//   kFpDQ     : dQ = scale * dS K                   backward_stubs.py:259-311
//               with dS = P o (dO V^T - rowsum) (_attn_bwd_dk_kernel,
//               _attn_bwd_dq_kernel, triton_attn_bwd_dqdk_from_p)
//
// P is [b, h, t, t] 16-bit, row-major with a row stride that is a multiple of
// 8 elements; it is read once, tile by tile, through TMA, so these passes are
// bound by HBM bandwidth on P (2 bytes per entry read) rather than by the
// tensor core.
//
// One CTA owns 128 rows (keys for kFpDV / kFpDK, queries for kFpRowsum /
// kFpDQ) and streams W rows of the other axis per step (the P tile plus the
// streamed [W x d] tiles, through a 2..4-stage TMA ring). The P tiles are also
// prefetched into L2 a few steps ahead of their load, so the short ring does
// not wait on HBM latency.
//
// kFpDV / kFpRowsum (W = 128) are pure products: P^T dO (both operands
// MN-major) or P V accumulate in TMEM (warp 5 TMA, warp 4 MMA, warps 0..3 the
// epilogue).
//
// kFpDK / kFpDQ (W = from_p_step_rows) compute the dP^T (or dP) tile of a step into one
// of two TMEM score buffers, the elementwise warps turn it into 16-bit dS^T
// (dS) in one of two TMEM E buffers, and the accumulate product reads E as its
// A operand from TMEM. One issuing thread cannot feed the tensor pipe at its
// rate (about one tcgen05.mma per 85 cycles), so these modes use two MMA
// threads, and eight elementwise warps:
//   warps 0..7  elementwise: warp w owns TMEM lanes 32*(w%4)..+31 (one owned
//               row per thread) and columns (w/4)*W/2 ..+W/2 of each step
//   warp 8      TMA producer (kFpDK: the whole warp also stages the step's
//               query rowsums in shared memory)
//   warp 9      score products dP^T = V dO^T (kFpDK) / dP = dO V^T (kFpDQ)
//   warp 10     accumulate products dK += dS^T Q (kFpDK) / dQ += dS K (kFpDQ)
// A stage is released when both MMA threads' products that read it completed
// (l_empty counts two commits); its P tile was read by the elementwise warps
// before their E arrival, which precedes the accumulate product.
//
// Causal (kFpRowsum, kFpDK, kFpDQ): tiles that lie entirely past the diagonal
// are skipped, as the reference skips its 64 x 64 blocks past the diagonal;
// inside a visited tile P is used as given (zero above the diagonal for P
// from a causal softmax). kFpDV has no causal argument in the reference and
// reads all of P.
#include "attn_pipe.cuh"
#include "kernels.h"

namespace ttt {

template <int D, int MODE>
struct FpCfg {
  static constexpr bool KEY_MAJOR = (MODE == kFpDV || MODE == kFpDK);
  static constexpr bool ELEM = (MODE == kFpDK || MODE == kFpDQ);
  static constexpr int W = from_p_step_rows(MODE);  // streamed rows per step
  static constexpr int CW = W / 2;                  // ELEM: columns of a step per warp half
  static_assert(!ELEM || CW % 32 == 0, "column halves are processed 32 at a time");
  // P tile of a step: key-major [W queries x 128 keys], query-major [128 queries x W keys]
  static constexpr int P_ROWS = KEY_MAJOR ? W : 128;
  static constexpr int P_COLS = KEY_MAJOR ? 128 : W;
  static constexpr int TILE_P = P_ROWS * P_COLS * 2;
  static constexpr int TILE_X = W * D * 2;
  // streamed [W x d] tiles: kFpDV dO; kFpRowsum V; kFpDK dO, Q; kFpDQ V, K
  static constexpr int NX = ELEM ? 2 : 1;
  static constexpr int STAGE_TX = TILE_P + NX * TILE_X;
  static constexpr int STAGE = STAGE_TX;  // multiple of 1024 for every (D, MODE)
  // resident [128 x d] operand: kFpDK V, kFpDQ dO
  static constexpr int NR = ELEM ? 1 : 0;
  static constexpr int TILE_R = 128 * D * 2;
  static constexpr int BAR_BYTES = 24 * 8;
  static constexpr int RS_PER = (MODE == kFpDK) ? W * 4 : 0;  // rowsum slot per stage (kFpDK)
  static constexpr int BUDGET = 232448 - 1024 - BAR_BYTES - 16 - NR * TILE_R;
  static constexpr int NSTAGE = BUDGET / (STAGE + RS_PER) >= 4 ? 4 : BUDGET / (STAGE + RS_PER);
  // kFpDK: the streamed queries' rowsums of each step, staged by the producer
  // warp (W floats per stage slot, outside the 1024-aligned stages)
  static constexpr bool RS_RING = RS_PER > 0;
  // kFpDK with a two-stage ring (d = 128): a stage arrives in two parts on two
  // barriers, dO first (the score product's operand), then P, Q and the rowsums,
  // so the step's score product need not wait for the whole stage. The second
  // part uses the l_full slots that a two-stage ring leaves free.
  static constexpr bool SPLIT_STAGE = MODE == kFpDK && NSTAGE == 2;
  static constexpr int RS_BYTES = NSTAGE * RS_PER;
  static constexpr int OFF_R = 0;
  static constexpr int OFF_S = OFF_R + NR * TILE_R;
  static constexpr int OFF_RS = OFF_S + NSTAGE * STAGE;
  static constexpr int OFF_BAR = OFF_RS + RS_BYTES;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 16 + 1024;
  // ELEM: P tiles are prefetched into L2 this many steps ahead of their load
  // (their short stage ring cannot cover HBM latency alone); the product-only
  // passes measured slightly slower with it.
  static constexpr int PF = ELEM ? 4 : 0;
  // TMEM: accumulator at 0 (D columns); ELEM: score buffers (2 x W) then packed
  // E buffers (2 x W/2).
  static constexpr int C_S = D, C_E = D + 2 * W;
  static constexpr int TMEM_USED = ELEM ? D + 3 * W : D;
  static constexpr int TMEM_COLS = TMEM_USED <= 64 ? 64 : TMEM_USED <= 128 ? 128 : TMEM_USED <= 256 ? 256 : 512;
  // roles (see the file comment)
  static constexpr int NCW = ELEM ? 8 : 4;
  static constexpr int NCT = NCW * 32;
  static constexpr int WARP_LOAD = ELEM ? 8 : 5;
  static constexpr int WARP_MMA = ELEM ? 9 : 4;
  static constexpr int WARP_MMA2 = 10;  // ELEM only
  static constexpr int NTHREADS = ELEM ? 352 : 192;
  static_assert(NSTAGE >= 2, "from-P stage ring does not fit");
  static_assert(STAGE % 1024 == 0 && TILE_P % 1024 == 0 && TILE_R % 1024 == 0, "tiles must stay 1024-aligned");
  static_assert(SMEM <= 232448, "from-P tile set exceeds shared memory");
  static_assert(TMEM_USED <= 512, "TMEM overflow");
};

template <int D, bool BF16, bool CAUSAL, int MODE>
__global__ void __launch_bounds__(FpCfg<D, MODE>::NTHREADS, 1) attn_from_p_kernel(const __grid_constant__ KParams p) {
  using C = FpCfg<D, MODE>;
  constexpr int W = C::W, CW = C::CW, NP = D / 64, NSTAGE = C::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sR = smem + C::OFF_R;
  uint8_t* sS = smem + C::OFF_S;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* res_full = bars + 0;
  uint64_t* l_full = bars + 1;    // [4]
  // SPLIT_STAGE: P, Q and the rowsums of stage s arrive on l_full_b[s] (l_full[s] has dO)
  uint64_t* l_full_b = C::SPLIT_STAGE ? l_full + 2 : l_full;
  uint64_t* l_empty = bars + 5;   // [4] (ELEM: both MMA threads commit)
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_free = bars + 11;   // [2] (NCT arrivals)
  uint64_t* e_full = bars + 13;   // [2] (NCT arrivals)
  uint64_t* e_empty = bars + 15;  // [2]
  uint64_t* acc_full = bars + 17;
  uint64_t* drain = bars + 18;    // [2] one per MMA thread
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto tileP = [&](int s) { return sS + s * C::STAGE; };
  auto tileX = [&](int s, int i) { return sS + s * C::STAGE + C::TILE_P + i * C::TILE_X; };
  float* sRS = reinterpret_cast<float*>(smem + C::OFF_RS);  // RS_RING: [NSTAGE][W]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int T = p.T;
  const int r0 = blockIdx.y * 128;  // first owned row
  const int n_all = (T + W - 1) / W;
  int n_first = 0, n_end = n_all;
  if constexpr (CAUSAL && MODE != kFpDV) {
    if constexpr (C::KEY_MAJOR) {
      n_first = r0 / W;  // query tiles ending before the first key see none of it
    } else {
      n_end = min(n_all, (r0 + 127) / W + 1);  // key tiles starting past the last query
    }
  }
  const int n_tiles = n_end - n_first;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 20; ++i) mbar_init(bars + i, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_free + i, C::NCT);
      mbar_init(e_full + i, C::NCT);
    }
    if constexpr (C::ELEM)
      for (int i = 0; i < 4; ++i) mbar_init(l_empty + i, 2);
    if constexpr (C::SPLIT_STAGE) {  // dO alone; then the TMA arrival and the rowsum copy
      for (int i = 0; i < 2; ++i) {
        mbar_init(l_full + i, 1);
        mbar_init(l_full_b + i, 2);
      }
    } else if constexpr (C::RS_RING) {  // the TMA arrival and the producer warp's rowsum copy
      for (int i = 0; i < 4; ++i) mbar_init(l_full + i, 2);
    }
    *abort_flag = (p.err != nullptr && *reinterpret_cast<volatile int*>(p.err) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (*abort_flag) return;
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  Guard g{abort_flag, p.err, p.err_host};

  if (warp == C::WARP_LOAD) {
    // ------------------------------------------------------------ producer
    // Lane 0 issues the TMA loads (and the L2 prefetches PF steps ahead); with
    // RS_RING the whole warp then copies the step's W rowsums into the stage's
    // slot and lane 0 adds the second arrival.
    auto p_coords = [&](int n, int& pcol, int& prow) {
      const int j0 = (n_first + n) * W;
      prow = C::KEY_MAJOR ? j0 : r0;
      pcol = C::KEY_MAJOR ? r0 : j0;
    };
    auto prefetch_p = [&](int n) {
      int pcol, prow;
      p_coords(n, pcol, prow);
      for (int pp = 0; pp < C::P_COLS / 64; ++pp) tma_prefetch_l2_4d(&p.str[0], pcol + pp * 64, prow, hidx, bidx);
    };
    if (lane == 0) {
      tma_prefetch(&p.str[0]);
      for (int i = 0; i < C::NX; ++i) tma_prefetch(&p.str[1 + i]);
      if constexpr (C::NR > 0) {
        tma_prefetch(&p.own[0]);
        mbar_arrive_tx(res_full, C::TILE_R);
        for (int pp = 0; pp < NP; ++pp) tma_load_4d(sR + pp * 128 * 128, &p.own[0], res_full, pp * 64, r0, hidx, bidx);
      }
      for (int n = NSTAGE; n < min(n_tiles, NSTAGE + C::PF); ++n) prefetch_p(n);
    }
    const float* rs = p.delta + static_cast<int64_t>(bh) * T;
    int n = 0;
    for (; n < n_tiles; ++n) {
      const int s = n % NSTAGE;
      const int j0 = (n_first + n) * W;  // first streamed row of this step
      bool ok = true;
      if (lane == 0) {
        if (n >= NSTAGE) ok = mbar_wait(l_empty + s, ((n / NSTAGE) - 1) & 1, g, 1);
        if (ok) {
          int pcol, prow;
          p_coords(n, pcol, prow);
          if constexpr (C::SPLIT_STAGE) {
            // dO on l_full[s]; P and Q on l_full_b[s]
            mbar_arrive_tx(l_full + s, C::TILE_X);
            for (int pp = 0; pp < NP; ++pp)
              tma_load_4d(tileX(s, 0) + pp * W * 128, &p.str[1], l_full + s, pp * 64, j0, hidx, bidx);
            mbar_arrive_tx(l_full_b + s, C::TILE_P + C::TILE_X);
            for (int pp = 0; pp < C::P_COLS / 64; ++pp)
              tma_load_4d(tileP(s) + pp * C::P_ROWS * 128, &p.str[0], l_full_b + s, pcol + pp * 64, prow, hidx, bidx);
            for (int pp = 0; pp < NP; ++pp)
              tma_load_4d(tileX(s, 1) + pp * W * 128, &p.str[2], l_full_b + s, pp * 64, j0, hidx, bidx);
          } else {
            mbar_arrive_tx(l_full + s, C::STAGE_TX);
            // P tile: 64-column panels of P_ROWS rows
            for (int pp = 0; pp < C::P_COLS / 64; ++pp)
              tma_load_4d(tileP(s) + pp * C::P_ROWS * 128, &p.str[0], l_full + s, pcol + pp * 64, prow, hidx, bidx);
            for (int i = 0; i < C::NX; ++i)
              for (int pp = 0; pp < NP; ++pp)
                tma_load_4d(tileX(s, i) + pp * W * 128, &p.str[1 + i], l_full + s, pp * 64, j0, hidx, bidx);
          }
          if (C::PF > 0 && n + NSTAGE + C::PF < n_tiles) prefetch_p(n + NSTAGE + C::PF);
        }
      }
      if constexpr (C::RS_RING) {
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        float4 v;
        const int q = j0 + lane * 4;
        v.x = q < T ? __ldg(rs + q) : 0.f;
        v.y = q + 1 < T ? __ldg(rs + q + 1) : 0.f;
        v.z = q + 2 < T ? __ldg(rs + q + 2) : 0.f;
        v.w = q + 3 < T ? __ldg(rs + q + 3) : 0.f;
        if (lane * 4 < W) reinterpret_cast<float4*>(sRS + s * W)[lane] = v;
        __syncwarp();
        if (lane == 0) mbar_arrive(l_full_b + s);
      } else {
        if (!ok) break;
      }
    }
    if (lane == 0) {
      if constexpr (C::NR > 0) mbar_drain(res_full, 0);
      for (int j = max(0, n - NSTAGE); j < n; ++j) {
        mbar_drain(l_full + j % NSTAGE, (j / NSTAGE) & 1);
        if constexpr (C::SPLIT_STAGE) mbar_drain(l_full_b + j % NSTAGE, (j / NSTAGE) & 1);
      }
    }
  } else if (warp == C::WARP_MMA && !C::ELEM) {
    // ------------------------------------------------------------ MMA issuer (pure products)
    if (lane == 0) {
      bool ok = true;
      // kFpDV: acc[keys, d] += P^T dO   (A = P tile read MN-major, B = dO MN-major)
      // kFpRowsum: acc[queries, d] += P V (A = P tile K-major, B = V MN-major)
      constexpr uint32_t id = idesc_f16(128, D, BF16, MODE == kFpDV, true);
      for (int n = 0; ok && n < n_tiles; ++n) {
        const int s = n % NSTAGE;
        if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2))) break;
        tc_fence_after();
        const uint32_t aP = smem_u32(tileP(s)), bX = smem_u32(tileX(s, 0));
#pragma unroll
        for (int kk = 0; kk < W / 16; ++kk) {
          const uint64_t da = MODE == kFpDV ? desc_mnmajor(aP, W, kk) : desc_kmajor(aP, 128, kk);
          umma_ss(tmem, da, desc_mnmajor(bX, W, kk), id, (n > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(l_empty + s);
      }
      if (ok) umma_commit(acc_full);
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else if (C::ELEM && warp == C::WARP_MMA) {
    // ------------------------------------------------------------ score products (ELEM)
    // kFpDK dP^T = V dO^T, kFpDQ dP = dO V^T (A = resident, B = streamed tile 0)
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(128, W, BF16, false, false);
      const uint32_t aR = smem_u32(sR);
      bool ok = mbar_wait(res_full, 0, g, 2);
      for (int n = 0; ok && n < n_tiles; ++n) {
        const int s = n % NSTAGE, sb = n & 1;
        if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 3))) break;
        if (n >= 2 && !(ok = mbar_wait(s_free + sb, ((n >> 1) - 1) & 1, g, 4))) break;
        tc_fence_after();
        const uint32_t bX = smem_u32(tileX(s, 0));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + C::C_S + sb * W, desc_kmajor(aR, 128, kk), desc_kmajor(bX, W, kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit(s_full + sb);
        umma_commit(l_empty + s);
      }
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else if (C::ELEM && warp == C::WARP_MMA2) {
    // ------------------------------------------------------------ accumulate products (ELEM)
    // kFpDK dK += dS^T Q, kFpDQ dQ += dS K (A = E from TMEM, B = streamed tile 1 MN-major)
    if (lane == 0) {
      constexpr uint32_t id_a = idesc_f16(128, D, BF16, false, true);
      bool ok = true;
      for (int n = 0; ok && n < n_tiles; ++n) {
        const int s = n % NSTAGE, eb = n & 1;
        if (!(ok = mbar_wait(e_full + eb, (n >> 1) & 1, g, 5))) break;
        // the stage's tiles landed (already observed by the elementwise warps)
        if (!(ok = mbar_wait(l_full_b + s, (n / NSTAGE) & 1, g, 5))) break;
        tc_fence_after();
        const uint32_t bX = smem_u32(tileX(s, 1));
#pragma unroll
        for (int kk = 0; kk < W / 16; ++kk)
          umma_ts(tmem, tmem + C::C_E + eb * (W / 2) + kk * 8, desc_mnmajor(bX, W, kk), id_a,
                  (n > 0 || kk > 0) ? 1u : 0u);
        umma_commit(e_empty + eb);
        umma_commit(l_empty + s);
      }
      if (ok) umma_commit(acc_full);
      umma_commit(drain + 1);
      mbar_drain(drain + 1, 0);
    }
  } else if (warp < C::NCW) {
    // ------------------------------------------------------------ row warps
    const int quarter = warp & 3, half = warp >> 2;  // half: ELEM column half of a step
    const int r = quarter * 32 + lane;               // owned row == TMEM lane
    const int row = r0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    if constexpr (C::ELEM) {
      // kFpDQ: this row's rowsum; kFpDK: the streamed queries' rowsums, read per step
      const float* rs = p.delta + static_cast<int64_t>(bh) * T;
      const float own_rs = (MODE == kFpDQ && row < T) ? rs[row] : 0.f;
      for (int n = 0; n < n_tiles; ++n) {
        const int s = n % NSTAGE, sb = n & 1, eb = n & 1;
        if (!mbar_wait(s_full + sb, (n >> 1) & 1, g, 6)) { ok = false; break; }
        tc_fence_after();
        float dp[CW];
        tmem_ld_nw<CW>(tmem + lane_off + C::C_S + sb * W + half * CW, dp);
        tmem_wait_ld();
        reg_fence(dp);
        tc_fence_before();
        mbar_arrive(s_free + sb);
        if (!mbar_wait(l_full_b + s, (n / NSTAGE) & 1, g, 7)) { ok = false; break; }
        if (n >= 2 && !mbar_wait(e_empty + eb, ((n >> 1) - 1) & 1, g, 8)) { ok = false; break; }
        const uint8_t* tp = tileP(s);
        const uint32_t te = tmem + lane_off + C::C_E + eb * (W / 2) + half * (CW / 2);
#pragma unroll
        for (int hh = 0; hh < CW / 32; ++hh) {
          const int cb = hh * 32;  // this pass's first column within the warp's 64
          float pv[32], rv[32];
          if constexpr (MODE == kFpDK) {
            // P[c0 + cb + j, row]: column r of the [W x 128] tile (one 2-byte load per entry)
#pragma unroll
            for (int j = 0; j < 32; ++j)
              pv[j] = to_f32<BF16>(*reinterpret_cast<const uint16_t*>(tp + pl_offset(C::P_ROWS, half * CW + cb + j, r)));
            // the step's rowsums, staged by the producer warp (broadcast 16-byte loads)
            const float4* rs4 = reinterpret_cast<const float4*>(sRS + s * W + half * CW + cb);
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 f = rs4[j / 4];
              rv[j] = f.x; rv[j + 1] = f.y; rv[j + 2] = f.z; rv[j + 3] = f.w;
            }
          } else {
            // P[row, c0 + cb + j]: row r of the [128 x W] tile (16-byte swizzled chunks)
            const uint8_t* prow = tp + ((half * CW) >> 6) * 128 * 128 + r * 128;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
              const int c = (((half * CW) & 63) >> 3) + (cb >> 3) + ch;
              const uint4 w4 = *reinterpret_cast<const uint4*>(prow + ((c ^ (r & 7)) << 4));
              const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                pv[ch * 8 + 2 * i] = to_f32<BF16>(static_cast<uint16_t>(wv[i] & 0xffffu));
                pv[ch * 8 + 2 * i + 1] = to_f32<BF16>(static_cast<uint16_t>(wv[i] >> 16));
              }
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) rv[j] = own_rs;
          }
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float s0, s1;
            split(mul2(f2(pv[j], pv[j + 1]), sub2(f2(dp[cb + j], dp[cb + j + 1]), f2(rv[j], rv[j + 1]))), s0, s1);
            w[j / 2] = pack2<BF16>(s0, s1);
          }
          tmem_st16_raw(te + hh * 16, w);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(e_full + eb);
      }
    }
    if (ok && mbar_wait(acc_full, 0, g, 9)) {
      tc_fence_after();
      const bool valid = row < T;
      if constexpr (MODE == kFpRowsum) {
        // rowsum = dO_row . (P V)_row
        const uint16_t* drow = p.raw[0] + static_cast<int64_t>(bidx) * p.raw_sb[0] +
                               static_cast<int64_t>(hidx) * p.raw_sh[0] + static_cast<int64_t>(row) * p.raw_st[0];
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          tmem_ld32(tmem + lane_off + c * 32, v);
          if (valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w4 = *reinterpret_cast<const uint4*>(drow + c * 32 + q * 8);
              const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                acc = fmaf(v[q * 8 + 2 * i], to_f32<BF16>(static_cast<uint16_t>(wv[i] & 0xffffu)), acc);
                acc = fmaf(v[q * 8 + 2 * i + 1], to_f32<BF16>(static_cast<uint16_t>(wv[i] >> 16)), acc);
              }
            }
          }
        }
        if (valid) p.out_f0[static_cast<int64_t>(bh) * T + row] = acc;
      } else {
        uint16_t* orow = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                         static_cast<int64_t>(row) * p.o0_st;
        if constexpr (C::ELEM) {
          // each column half of the warps writes half of the row
          acc_cols_to_global<D / 2, BF16>(tmem + lane_off, half * (D / 2), orow, valid, p.scale);
        } else {
          acc_to_global<D, BF16>(tmem + lane_off, orow, valid, 1.f);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int D, bool BF16, bool CAUSAL, int MODE>
static cudaError_t launch_from_p_t(const KParams& p, cudaStream_t stream) {
  using C = FpCfg<D, MODE>;
  auto kern = attn_from_p_kernel<D, BF16, CAUSAL, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H, (p.T + 127) / 128);
  kern<<<grid, C::NTHREADS, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_from_p(const KParams& p, int d, bool bf16, bool causal, int mode, cudaStream_t stream) {
#define TTT_FP_MODE(D_, BF_, CA_)                                                             \
  if (d == D_ && bf16 == BF_ && causal == CA_) {                                              \
    if (mode == kFpDV) return launch_from_p_t<D_, BF_, false, kFpDV>(p, stream);              \
    if (mode == kFpRowsum) return launch_from_p_t<D_, BF_, CA_, kFpRowsum>(p, stream);        \
    if (mode == kFpDK) return launch_from_p_t<D_, BF_, CA_, kFpDK>(p, stream);                \
    if (mode == kFpDQ) return launch_from_p_t<D_, BF_, CA_, kFpDQ>(p, stream);                \
  }
#define TTT_FP_CA(D_, BF_) TTT_FP_MODE(D_, BF_, false) TTT_FP_MODE(D_, BF_, true)
  TTT_FP_CA(64, false) TTT_FP_CA(64, true) TTT_FP_CA(128, false) TTT_FP_CA(128, true)
#undef TTT_FP_CA
#undef TTT_FP_MODE
  return cudaErrorInvalidValue;
}

}  // namespace ttt
