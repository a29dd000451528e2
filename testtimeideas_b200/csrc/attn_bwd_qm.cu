// Query-major backward passes (sm_100a). One CTA owns 128 query rows of one
// head and streams BN-key tiles (BN = 64; 32 only for the 128-wide double
// backward that also returns dd_dO).
//
//   kBwdQ  : dQ = scale * dS K,  dS = P o (dP - delta),  P = 2^(S*c - lse2)
//            (replaces _attn_bwd_dq_kernel, ttt_kernels/backward_stubs.py:259-309)
//   kStats : double-backward row statistics
//              gamma_i = sum_j P_ij G_dS_ij,     G_dS = scale (u_q K^T + Q u_k^T)
//              rho_i   = sum_j P_ij G_P_ij,      G_P  = G_dS o (dP - delta) - gamma o dP + dO u_v^T
//            computed as rho = A2 - delta*gamma - gamma*A4 + A3 with
//            A2 = sum P G_dS dP, A4 = sum P dP, A3 = sum P (dO u_v^T).
//   kBwd2Q : dd_Q  = scale * (dS u_k + G_S K),     G_S  = P o (G_P - rho)
//            dd_dO = G_dP V + P u_v  (GDO only),   G_dP = P o (G_dS - gamma)
//            (with the key-major kBwd2KV pass this replaces the PyTorch matmul
//            double backward of TritonDvFn / TritonRowSumFn / TritonDqDkFn,
//            backward_stubs.py:435-514, with the complete second-order terms)
//
// Roles (352 threads): warps 0..7 elementwise, warps 8 and 10 MMA issuers
// (one thread each: one thread issues at most one tcgen05.mma per ~85 cycles,
// below the tensor pipe's rate), warp 9 TMA producer. Compute warp w owns TMEM
// lanes 32*(w%4)..+31 (one query row per thread) and columns (w/4)*BN/2 ..
// +BN/2 of every tile.
//
// Score products that share their A operand run as one N = 2*BN product: the
// streamed K and u_k tiles sit stacked in one panel ([K; u_k]), as do V and
// u_v, so Q [K; u_k]^T yields [S | Q u_k^T] and dO [V; u_v]^T yields
// [dP | dO u_v^T]; u_q K^T then accumulates into the second half of the first.
// (On B200 an M=128 UMMA with N <= 64 costs about as much as one with N=128.)
//
// Pipeline per tile n: tile n's score products are issued as soon as the
// compute warps have read the previous contents of that TMEM buffer (s_free);
// tile n-1's accumulate products once its elementwise results are in shared
// memory (e_full). Streamed tiles use a 2..4-stage TMA ring sized from the
// shared-memory budget; the two-stage ring of the d=128 statistics pass takes
// each stage in two parts ([K; u_k], then [V; u_v]) on two barriers. For the 128-wide double backward the elementwise
// results are written into the [V; u_v] part of their own stage, which only the
// score products read. Causal: key tiles past the diagonal are skipped and only
// boundary tiles are masked.
#include <type_traits>

#include "attn_pipe.cuh"
#include "kernels.h"

namespace ttt {

template <int D, int KIND, bool GDO>
struct QmCfg {
  static constexpr int BM = 128;
  static constexpr bool BWD2 = (KIND != kBwdQ);
  static constexpr int BN = KIND == kBwdQ ? 128 : ((D == 128 && KIND == kBwd2Q && GDO) ? 32 : 64);
  static constexpr int NR = BWD2 ? 3 : 2;    // resident: Q, dO, (u_q)
  static constexpr int NSC = BWD2 ? 4 : 2;   // score tiles: S, (G_dS,) dP, (dO u_v^T)
  static constexpr int NE = KIND == kBwdQ ? 1 : (KIND == kStats ? 0 : (GDO ? 4 : 2));
  static constexpr int NA = KIND == kBwdQ ? 1 : (KIND == kStats ? 0 : (GDO ? 2 : 1));
  static constexpr int NCW = 8;
  static constexpr int NCT = NCW * 32;
  // Register split: the launch gives every thread REG_LAUNCH registers (three
  // warps share one 16K-register sub-partition); the control warpgroup then
  // drops to REG_CTRL and the two elementwise warpgroups rise to REG_ELEM. Off:
  // it removes the small d=64 spills but the idle warps cost more (measured
  // 0.8-1.2% slower per step).
  static constexpr bool SPLIT_REGS = false;
  // Two MMA issuing threads: one issuing thread cannot feed the tensor pipe at
  // its rate (measured on B200: ~85 cycles per UMMA from one thread; two
  // threads reach the pipe's ~50 cycles for N=64 and ~65 for N=128). Issuer 0
  // takes the score products, issuer 1 the accumulate products; without
  // accumulate products (statistics pass) they take alternate tiles.
  static constexpr bool TWO_ISSUERS = true;
  // With two issuers, the d=128 double backward also splits its score products
  // (key side on issuer 0, value side on issuer 1): 19% faster there, 1-2%
  // slower in the other passes, which keep all score products on issuer 0.
  static constexpr bool SPLIT_SCORES = TWO_ISSUERS && KIND == kBwd2Q && D == 128;
  static constexpr int NTHREADS = NCT + (SPLIT_REGS ? 128 : 64) + (TWO_ISSUERS && !SPLIT_REGS ? 32 : 0);
  static constexpr int REG_LAUNCH = 168, REG_CTRL = 152, REG_ELEM = (3 * REG_LAUNCH - REG_CTRL) / 2;
  static_assert(REG_ELEM % 8 == 0 && 2 * REG_ELEM + REG_CTRL <= 3 * REG_LAUNCH, "register split");
  static constexpr int CPW = BN / 2;
  // streamed tiles: ST0 = [K; u_k] (or K), ST1 = [V; u_v] (or V), rows stacked per panel
  static constexpr int ST_ROWS = BWD2 ? 2 * BN : BN;
  static constexpr int ST_BYTES = ST_ROWS * D * 2;
  static constexpr int STAGE = 2 * ST_BYTES;
  static constexpr int TILE_R = BM * D * 2;
  static constexpr int TILE_E = BM * (BN > 64 ? BN : 64) * 2;  // whole 64-column panels
  // Owner-side operands that are only ever A operands of score products can sit
  // in TMEM (A-from-TMEM products), which frees shared memory for deeper
  // staging: Q and dO for the dq pass; Q and u_q for the 128-wide double backward.
  static constexpr bool RT_Q = (KIND == kBwdQ) || (KIND == kBwd2Q && D == 128 && !GDO);
  static constexpr bool RT_DO = (KIND == kBwdQ);
  static constexpr bool RT_UQ = (KIND == kBwd2Q && D == 128 && !GDO);
  static constexpr bool RES_TMEM = RT_Q || RT_DO || RT_UQ;
  static constexpr int NR_TMEM = (RT_Q ? 1 : 0) + (RT_DO ? 1 : 0) + (RT_UQ ? 1 : 0);
  static constexpr int NR_SMEM = NR - NR_TMEM;
  // elementwise results in the ST1 part of their own stage when they fit
  static constexpr bool EIS = (KIND == kBwd2Q || KIND == kBwdQ) && (NE * TILE_E <= ST_BYTES);
  static constexpr int E_BYTES = EIS ? 0 : NE * TILE_E;
  static constexpr int NBUF = (2 * NSC * BN + NA * D <= 512) ? 2 : 1;
  static constexpr int RES_COL = NBUF * NSC * BN + NA * D;  // packed Q, u_q (RES_TMEM)
  static constexpr int TMEM_USED = RES_COL + NR_TMEM * (D / 2);
  static constexpr int TMEM_COLS = TMEM_USED <= 128 ? 128 : (TMEM_USED <= 256 ? 256 : 512);
  static_assert(TMEM_USED <= 512, "TMEM overflow");
  static constexpr int FIXED = NR_SMEM * TILE_R + E_BYTES + 16 * 8 + 16 + 1024;
  static constexpr int NSTAGE = (FIXED + 4 * STAGE <= 232448) ? 4 : (FIXED + 3 * STAGE <= 232448) ? 3 : 2;
  // Statistics pass with a two-stage ring (d = 128): a stage arrives in two parts
  // on two barriers, [K; u_k] first (the key-side score products), then [V; u_v],
  // so a tile's first products need not wait for the whole stage. The second part
  // uses the l_full slots that a two-stage ring leaves free.
  static constexpr bool SPLIT_STAGE = KIND == kStats && NSTAGE == 2;
  static constexpr int OFF_R = 0;
  static constexpr int OFF_S = OFF_R + NR_SMEM * TILE_R;
  static constexpr int OFF_E = OFF_S + NSTAGE * STAGE;
  static constexpr int OFF_BAR = OFF_E + E_BYTES;
  static constexpr int NBAR = 18;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "query-major tile set exceeds shared memory");
  // TMEM column offsets of the score tiles within one buffer
  static constexpr int C_S = 0, C_GDS = BWD2 ? BN : 0, C_DP = BWD2 ? 2 * BN : BN, C_UV = 3 * BN;
};

int qm_tile_cols(int d, int kind, bool gdo) { return kind == kBwdQ ? 128 : ((d == 128 && kind == kBwd2Q && gdo) ? 32 : 64); }

template <int D, bool BF16, bool CAUSAL, int KIND, bool GDO>
__global__ void __launch_bounds__(QmCfg<D, KIND, GDO>::NTHREADS, 1) attn_qm_kernel(const __grid_constant__ KParams p) {
  using C = QmCfg<D, KIND, GDO>;
  constexpr int BM = C::BM, BN = C::BN, NP = D / 64, NBUF = C::NBUF, NSTAGE = C::NSTAGE, CPW = C::CPW;
  constexpr int SR = C::ST_ROWS;
  constexpr int WARP_MMA = C::NCW, WARP_LOAD = C::NCW + 1, WARP_MMA2 = C::NCW + 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sR = smem + C::OFF_R;
  uint8_t* sS = smem + C::OFF_S;
  uint8_t* sE = smem + C::OFF_E;
  // Row-sum scratch of the stats pass: reuses the streamed-tile stages, which
  // are idle once every compute thread has seen the last tile's scores land.
  float* red = reinterpret_cast<float*>(smem + C::OFF_S);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* res_full = bars + 0;
  uint64_t* l_full = bars + 1;   // [4] TMA -> MMA
  // SPLIT_STAGE: [V; u_v] of stage s arrives on l_full_b[s] (l_full[s] has [K; u_k])
  uint64_t* l_full_b = C::SPLIT_STAGE ? l_full + 2 : l_full;
  uint64_t* l_empty = bars + 5;  // [4] MMA -> TMA
  uint64_t* s_full = bars + 9;   // [2] MMA -> compute
  uint64_t* s_free = bars + 11;  // [2] compute -> MMA (NCT arrivals)
  // e_full[n % 2] (NCT arrivals): E of tile n written. Two barriers, because a
  // compute warp may finish tile n+1 before a slower one finishes tile n; with
  // one barrier its second arrival would complete tile n's phase early. It
  // cannot reach tile n+2 before tile n's phase completed: those scores are
  // issued only after the MMA thread has seen e_full for tile n.
  uint64_t* e_full = bars + 13;  // [2] compute -> MMA
  uint64_t* e_empty = bars + 15; // MMA -> compute
  uint64_t* acc_full = bars + 16;
  uint64_t* drain = bars + 17;  // [2] one per MMA issuer (bars + 18 for the second)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert(19 * 8 + 8 <= C::NBAR * 8 + 16, "barrier area");
  // resident tiles kept in shared memory, packed in slot order
  auto in_tmem = [&](int t) { return (t == 0 && C::RT_Q) || (t == 1 && C::RT_DO) || (t == 2 && C::RT_UQ); };
  auto tileR = [&](int t) {
    int idx = 0;
    for (int u = 0; u < t; ++u) idx += in_tmem(u) ? 0 : 1;
    return sR + idx * C::TILE_R;
  };
  auto tileS = [&](int s, int t) { return sS + s * C::STAGE + t * C::ST_BYTES; };
  auto tileE = [&](int s, int t) { return C::EIS ? tileS(s, 1) + t * C::TILE_E : sE + t * C::TILE_E; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // split mode: this CTA takes share `share` of its query block's key tiles
  const int nsplit = p.nsplit > 1 ? p.nsplit : 1;
  const GridPos gp = grid_pos();
  const int bh = gp.unit / nsplit, share = gp.unit % nsplit;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int qblk = CAUSAL ? (gridDim.y - 1 - gp.rank) : gp.rank;  // longest rows first
  const int q0 = qblk * BM;
  const int T = p.T;
  const int n_all = (T + BN - 1) / BN;
  // Causal: key tiles before the first row's band, or past the diagonal, are skipped.
  const Band band = Band::make(p, CAUSAL);
  const int n_lo = CAUSAL ? band.lo(q0) / BN : 0;  // first key tile the block visits
  const int n_hi = CAUSAL ? min(n_all, (q0 + BM - 1) / BN + 1) : n_all;
  const int n_first = n_lo + split_begin(n_hi - n_lo, share, nsplit);  // first key tile of this share
  const int n_tiles = n_lo + split_begin(n_hi - n_lo, share + 1, nsplit) - n_first;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 19; ++i) mbar_init(bars + i, 1);
    mbar_init(s_free + 0, C::NCT);
    mbar_init(s_free + 1, C::NCT);
    if (C::SPLIT_SCORES) {  // both issuers' score products
      mbar_init(s_full + 0, 2);
      mbar_init(s_full + 1, 2);
    }
    mbar_init(e_full + 0, C::NCT);
    mbar_init(e_full + 1, C::NCT);
    if (C::RES_TMEM) mbar_init(res_full, 1 + C::NCT);  // TMA + the compute warps' copies into TMEM
    // A nonzero error word means an earlier CTA or launch gave up: exit at once.
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
  const uint32_t tAcc0 = tmem + NBUF * C::NSC * BN;
  const uint32_t tAcc1 = tAcc0 + D;
  // packed resident A operands in TMEM (RES_TMEM), in slot order Q, dO, u_q
  const uint32_t tQ = tmem + C::RES_COL;
  const uint32_t tDO = tQ + (C::RT_Q ? D / 2 : 0);
  const uint32_t tUQ = tDO + (C::RT_DO ? D / 2 : 0);
  Guard g{abort_flag, p.err, p.err_host};

  if (warp >= C::NCW) {
   if constexpr (C::SPLIT_REGS) regs_release<C::REG_CTRL>();
   if (warp == WARP_LOAD) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      constexpr int NSTR = C::BWD2 ? 4 : 2;
      for (int t = 0; t < C::NR; ++t) tma_prefetch(&p.own[t]);
      for (int t = 0; t < NSTR; ++t) tma_prefetch(&p.str[t]);
      int issued[4] = {0, 0, 0, 0};
      mbar_arrive_tx(res_full, C::NR_SMEM * C::TILE_R);
      for (int t = 0; t < C::NR; ++t) {
        if (in_tmem(t)) continue;  // copied to TMEM by the compute warps
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(tileR(t) + pp * BM * 128, &p.own[t], res_full, pp * 64, q0, hidx, bidx);
      }
      for (int n = 0; n < n_tiles; ++n) {
        const int s = n % NSTAGE;
        if (n >= NSTAGE && !mbar_wait(l_empty + s, ((n / NSTAGE) - 1) & 1, g, 1)) break;
        if constexpr (C::SPLIT_STAGE) {
          // [K; u_k] on l_full[s], then [V; u_v] on l_full_b[s]
          for (int part = 0; part < 2; ++part) {
            uint64_t* bar = part ? l_full_b + s : l_full + s;
            mbar_arrive_tx(bar, 2 * BN * D * 2);
            for (int t = part; t < NSTR; t += 2) {
              uint8_t* dst = tileS(s, t & 1) + (t >> 1) * BN * 128;
              for (int pp = 0; pp < NP; ++pp)
                tma_load_4d(dst + pp * SR * 128, &p.str[t], bar, pp * 64, (n_first + n) * BN, hidx, bidx);
            }
          }
        } else {
          mbar_arrive_tx(l_full + s, NSTR * BN * D * 2);
          // str[0] = K, str[1] = V, str[2] = u_k, str[3] = u_v
          for (int t = 0; t < NSTR; ++t) {
            uint8_t* dst = tileS(s, t & 1) + (t >> 1) * BN * 128;
            for (int pp = 0; pp < NP; ++pp)
              tma_load_4d(dst + pp * SR * 128, &p.str[t], l_full + s, pp * 64, (n_first + n) * BN, hidx, bidx);
          }
        }
        issued[s] = n + 1;
      }
      mbar_drain(res_full, 0);
      for (int s = 0; s < NSTAGE; ++s)
        if (issued[s] > 0) {
          mbar_drain(l_full + s, ((issued[s] - 1) / NSTAGE) & 1);
          if constexpr (C::SPLIT_STAGE) mbar_drain(l_full_b + s, ((issued[s] - 1) / NSTAGE) & 1);
        }
    }
   } else if (warp == WARP_MMA || (C::TWO_ISSUERS && warp == WARP_MMA2)) {
    // ------------------------------------------------------------ MMA issuer(s)
    if (lane == 0) {
      constexpr uint32_t id_n1 = idesc_f16(128, BN, BF16, false, false);
      constexpr uint32_t id_n2 = idesc_f16(128, 2 * BN, BF16, false, false);
      constexpr uint32_t id_acc = idesc_f16(128, D, BF16, false, true);
      const uint32_t aQ = smem_u32(tileR(0)), aDO = smem_u32(tileR(1));
      const uint32_t aUQ = C::BWD2 ? smem_u32(tileR(2)) : 0u;
      using LS = KOff2<KOffK<BM>, KOffK<SR>>;  // score products: both operands K-major
      using LA = KOff2<KOffK<BM>, KOffMN>;     // accumulate products: E K-major, streamed tile MN-major
      // Score products of tile n; the last product's batch probes (bar0, par0) and (bar1, par1).
      // parts: bit 0 the products on the key side ([S | Q u_k^T], u_q K^T, or S),
      // bit 1 those on the value side ([dP | dO u_v^T], or dP); each part is one
      // issuer's when two issue (see TWO_ISSUERS). The probes ride on the value side.
      // With SPLIT_STAGE the value side first waits for its part of the stage; a wait that
      // gives up clears *stage_ok and returns before any value-side product or commit.
      auto issue_scores = [&](int n, const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1,
                              int parts = 3, bool* stage_ok = nullptr) -> uint32_t {
        const int sb = n % NBUF, s = n % NSTAGE;
        const uint32_t base = tmem + sb * C::NSC * BN;
        const uint32_t b0 = smem_u32(tileS(s, 0)), b1 = smem_u32(tileS(s, 1));
        uint32_t seen = 0;
        if constexpr (C::BWD2) {
          // [S | Q u_k^T] = Q [K; u_k]^T ; G_dS/scale += u_q K^T ; [dP | dO u_v^T] = dO [V; u_v]^T
          if (parts & 1) {
            if constexpr (C::RT_Q) {
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                umma_ts(base + C::C_S, tQ + kk * 8, desc_kmajor(b0, SR, kk), id_n2, kk > 0);
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                umma_ts(base + C::C_GDS, tUQ + kk * 8, desc_kmajor(b0, SR, kk), id_n1, 1u);
            } else {
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                umma_ss(base + C::C_S, desc_kmajor(aQ, BM, kk), desc_kmajor(b0, SR, kk), id_n2, kk > 0);
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                umma_ss(base + C::C_GDS, desc_kmajor(aUQ, BM, kk), desc_kmajor(b0, SR, kk), id_n1, 1u);
            }
          }
          if (parts & 2) {
            if constexpr (C::SPLIT_STAGE) {
              if (!mbar_wait(l_full_b + s, (n / NSTAGE) & 1, g, 2)) {
                *stage_ok = false;
                return 0u;
              }
              tc_fence_after();
            }
            seen = issue_ss<D / 16, LS>(base + C::C_DP, desc_kmajor(aDO, BM, 0), desc_kmajor(b1, SR, 0), id_n2, 0u,
                                        bar0, par0, bar1, par1);
          }
        } else if constexpr (C::RT_Q && C::RT_DO) {
          if (parts & 1) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              umma_ts(base + C::C_S, tQ + kk * 8, desc_kmajor(b0, SR, kk), id_n1, kk > 0);
          }
          if (parts & 2)
            seen = issue_ts<D / 16, KOff2<KOffT, KOffK<SR>>>(base + C::C_DP, tDO, desc_kmajor(b1, SR, 0), id_n1, 0u,
                                                            bar0, par0, bar1, par1);
        } else {
          if (parts & 1) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              umma_ss(base + C::C_S, desc_kmajor(aQ, BM, kk), desc_kmajor(b0, SR, kk), id_n1, kk > 0);
          }
          if (parts & 2)
            seen = issue_ss<D / 16, LS>(base + C::C_DP, desc_kmajor(aDO, BM, 0), desc_kmajor(b1, SR, 0), id_n1, 0u,
                                        bar0, par0, bar1, par1);
        }
        umma_commit(s_full + sb);
        if constexpr (C::NA == 0) umma_commit(l_empty + s);
        return seen;
      };
      // Accumulate products of tile n (its e_full already seen); probes as above.
      auto issue_acc = [&](int n, const uint64_t* bar0, uint32_t par0, const uint64_t* bar1,
                           uint32_t par1) -> uint32_t {
        const int s = n % NSTAGE;
        const uint32_t bK = smem_u32(tileS(s, 0)), bV = smem_u32(tileS(s, 1));
        const uint32_t e0 = smem_u32(tileE(s, 0));
        const uint32_t fresh = n > 0 ? 1u : 0u;
        uint32_t seen = 0;
        if constexpr (KIND == kBwdQ) {
          seen = issue_ss<BN / 16, LA>(tAcc0, desc_kmajor(e0, BM, 0), desc_mnmajor(bK, SR, 0), id_acc, fresh, bar0,
                                       par0, bar1, par1);
        } else {
          const uint32_t bUK = bK + BN * 128, bUV = bV + BN * 128;
          const uint32_t e1 = smem_u32(tileE(s, 1));
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e0, BM, kk), desc_mnmajor(bUK, SR, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
          if constexpr (!GDO) {
            seen = issue_ss<BN / 16, LA>(tAcc0, desc_kmajor(e1, BM, 0), desc_mnmajor(bK, SR, 0), id_acc, 1u, bar0,
                                         par0, bar1, par1);
          } else {
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              umma_ss(tAcc0, desc_kmajor(e1, BM, kk), desc_mnmajor(bK, SR, kk), id_acc, 1u);
            const uint32_t e2 = smem_u32(tileE(s, 2)), e3 = smem_u32(tileE(s, 3));
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              umma_ss(tAcc1, desc_kmajor(e2, BM, kk), desc_mnmajor(bV, SR, kk), id_acc,
                      (n > 0 || kk > 0) ? 1u : 0u);
            seen = issue_ss<BN / 16, LA>(tAcc1, desc_kmajor(e3, BM, 0), desc_mnmajor(bUV, SR, 0), id_acc, 1u, bar0,
                                         par0, bar1, par1);
          }
        }
        if constexpr (!C::EIS) umma_commit(e_empty);
        umma_commit(l_empty + s);
        return seen;
      };
      bool ok = mbar_wait(res_full, 0, g, 1);
      // res_full's phase 0 completed above: a probe of it always succeeds (an unused probe slot)
      const uint64_t* done = res_full;
      if constexpr (C::TWO_ISSUERS) {
        const int me = warp == WARP_MMA ? 0 : 1;
        if constexpr (C::NA == 0) {
          // statistics pass: alternate tiles, each in its own score buffer
          for (int n = me; ok && n < n_tiles; n += 2) {
            const int sb = n % NBUF, s = n % NSTAGE;
            if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2))) break;
            if (n >= NBUF && !(ok = mbar_wait(s_free + sb, ((n / NBUF) - 1) & 1, g, 3))) break;
            tc_fence_after();
            issue_scores(n, done, 0u, done, 0u, 3, &ok);
          }
        } else {
          // issuer 0: the score products of every tile (with SPLIT_SCORES the key-side
          // ones, issuer 1 the value-side ones, both committing s_full, which then counts
          // two arrivals); issuer 1: each tile's accumulate products once its elementwise
          // results are written (its score products completed before that, so its stage
          // may then be refilled).
          for (int n = 0; ok && n <= n_tiles; ++n) {
            if (n < n_tiles && (me == 0 || C::SPLIT_SCORES)) {
              const int sb = n % NBUF, s = n % NSTAGE;
              if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2))) break;
              if (n >= NBUF && !(ok = mbar_wait(s_free + sb, ((n / NBUF) - 1) & 1, g, 3))) break;
              tc_fence_after();
              issue_scores(n, done, 0u, done, 0u, C::SPLIT_SCORES ? (me == 0 ? 1 : 2) : 3);
            }
            if (me == 1 && n >= 1) {
              if (!(ok = mbar_wait(e_full + ((n - 1) & 1), ((n - 1) >> 1) & 1, g, 4))) break;
              tc_fence_after();
              issue_acc(n - 1, done, 0u, done, 0u);
            }
          }
          if (me == 1 && ok) umma_commit(acc_full);
        }
        umma_commit(drain + me);
        mbar_drain(drain + me, 0);
      } else {
        bool have_l = false, have_s = false;  // the next score step's barriers already seen complete
        for (int n = 0; ok && n < n_tiles; ++n) {
          const int sb = n % NBUF, s = n % NSTAGE;
          if (!have_l && !(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2))) break;
          if (n >= NBUF && !have_s && !(ok = mbar_wait(s_free + sb, ((n / NBUF) - 1) & 1, g, 3))) break;
          tc_fence_after();
          // barriers of tile n+1's score step
          const bool nxt = n + 1 < n_tiles;
          const uint64_t* bl = nxt ? l_full + (n + 1) % NSTAGE : done;
          const uint32_t pl = nxt ? ((n + 1) / NSTAGE) & 1 : 0u;
          const bool need_s = nxt && n + 1 >= NBUF;
          const uint64_t* bs = need_s ? s_free + (n + 1) % NBUF : done;
          const uint32_t ps = need_s ? (((n + 1) / NBUF) - 1) & 1 : 0u;
          if (C::NA > 0 && n >= 1) {
            // tile n-1's accumulate step follows: probe its e_full while issuing these scores
            uint64_t* be = e_full + ((n - 1) & 1);
            const uint32_t pe = ((n - 1) >> 1) & 1;
            const uint32_t seen = issue_scores(n, be, pe, bl, pl);
            if (!(seen & 1) && !(ok = mbar_wait(be, pe, g, 4))) break;
            tc_fence_after();
            const uint32_t seen2 = issue_acc(n - 1, bl, pl, bs, ps);
            have_l = ((seen >> 1) & 1) || (seen2 & 1);
            have_s = (seen2 >> 1) & 1;
          } else {
            const uint32_t seen = issue_scores(n, bl, pl, bs, ps);
            have_l = seen & 1;
            have_s = (seen >> 1) & 1;
          }
        }
        if constexpr (C::NA > 0) {
          if (ok && n_tiles > 0) {
            ok = mbar_wait(e_full + ((n_tiles - 1) & 1), ((n_tiles - 1) >> 1) & 1, g, 4);
            if (ok) {
              tc_fence_after();
              issue_acc(n_tiles - 1, done, 0u, done, 0u);
            }
          }
          if (ok) umma_commit(acc_full);
        }
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
   }
  } else {
    // ------------------------------------------------------------ elementwise warps 0..7
    if constexpr (C::SPLIT_REGS) regs_claim<C::REG_ELEM>();
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const int row = q0 + r;
    const int c0 = half * CPW;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t sidx = static_cast<int64_t>(bh) * p.t_pad + row;
    const int row_lo = band.lo(row);
    const int band_edge = CAUSAL ? band.lo(q0 + BM - 1) : 0;  // tiles starting before it need the band mask
    const float c = p.scale_log2, scale = p.scale;
    const float lse = p.lse2[sidx];
    const float del = p.delta[sidx];
    float gam = 0.f, rho = 0.f;
    if constexpr (KIND == kBwd2Q) {
      gam = p.gamma[sidx];
      rho = p.rho[sidx];
    }
    const F2 C2 = f2s(c), SC2 = f2s(scale), NLSE2 = f2s(-lse), DEL2 = f2s(del), GAM2 = f2s(gam), RHO2 = f2s(rho);
    F2 AG = f2s(0.f), A2 = AG, A3 = AG, A4 = AG;  // stats accumulators (column pairs)
    if constexpr (C::RES_TMEM) {
      // This thread's row, columns half*D/2 .. +D/2, of every operand kept in
      // TMEM: 16-bit pairs in memory are already the packed operand format.
#pragma unroll
      for (int slot = 0; slot < 3; ++slot) {
        if (!in_tmem(slot)) continue;
        uint32_t w[D / 4];
        if (row < T) {
          const uint4* src = reinterpret_cast<const uint4*>(
              p.raw[slot] + static_cast<int64_t>(bidx) * p.raw_sb[slot] + static_cast<int64_t>(hidx) * p.raw_sh[slot] +
              static_cast<int64_t>(row) * p.raw_st[slot] + half * (D / 2));
#pragma unroll
          for (int v = 0; v < D / 16; ++v) {
            const uint4 x = src[v];
            w[4 * v + 0] = x.x;
            w[4 * v + 1] = x.y;
            w[4 * v + 2] = x.z;
            w[4 * v + 3] = x.w;
          }
        } else {
#pragma unroll
          for (int v = 0; v < D / 4; ++v) w[v] = 0u;
        }
        const uint32_t dst = (slot == 0 ? tQ : (slot == 1 ? tDO : tUQ)) + lane_off + half * (D / 4);
#pragma unroll
        for (int c16 = 0; c16 < D / 4; c16 += 16) tmem_st16_raw(dst + c16, *reinterpret_cast<uint32_t(*)[16]>(w + c16));
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(res_full);
    }
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int sb = n % NBUF, s = n % NSTAGE;
      if (!mbar_wait(s_full + sb, (n / NBUF) & 1, g, 6)) { ok = false; break; }
      tc_fence_after();
      const uint32_t base = tmem + lane_off + sb * C::NSC * BN + c0;
      float sv[CPW], dp[CPW], gd[CPW], uv[CPW];
      tmem_ld_nw<CPW>(base + C::C_S, sv);
      tmem_ld_nw<CPW>(base + C::C_DP, dp);
      if constexpr (C::BWD2) {
        tmem_ld_nw<CPW>(base + C::C_GDS, gd);
        tmem_ld_nw<CPW>(base + C::C_UV, uv);
      }
      tmem_wait_ld();
      reg_fence(sv);
      reg_fence(dp);
      if constexpr (C::BWD2) {
        reg_fence(gd);
        reg_fence(uv);
      }
      tc_fence_before();
      mbar_arrive(s_free + sb);  // scores are in registers: the next tile's products may overwrite them

      const int kt0 = (n_first + n) * BN;  // first key of the tile
      const int j0 = kt0 + c0;
      const bool need_mask = (kt0 + BN > T) || (CAUSAL && (kt0 + BN - 1 > q0 || band_edge > kt0));
      // causal: the loop runs in a masked and an unmasked version, so that
      // interior tiles carry no per-element mask test
      auto elementwise = [&](auto masked) {
#pragma unroll
      for (int e = 0; e < CPW; e += 2) {
        float x0, x1;
        split(fma2(f2(sv[e], sv[e + 1]), C2, NLSE2), x0, x1);  // S c - lse2
        float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
        if (static_cast<bool>(masked)) {
          const int j = j0 + e;
          p0 = ((j < T) && (!CAUSAL || (j <= row && j >= row_lo))) ? p0 : 0.f;
          p1 = ((j + 1 < T) && (!CAUSAL || (j + 1 <= row && j + 1 >= row_lo))) ? p1 : 0.f;
        }
        const F2 PR = f2(p0, p1), DP = f2(dp[e], dp[e + 1]);
        if constexpr (KIND == kBwdQ) {
          split(mul2(PR, sub2(DP, DEL2)), sv[e], sv[e + 1]);
        } else if constexpr (KIND == kStats) {
          const F2 TT = mul2(PR, f2(gd[e], gd[e + 1]));  // P G_dS / scale (scaled once per row below)
          AG = add2(AG, TT);
          A2 = fma2(TT, DP, A2);
          A4 = fma2(PR, DP, A4);
          A3 = fma2(PR, f2(uv[e], uv[e + 1]), A3);
        } else {
          const F2 DPM = sub2(DP, DEL2);
          const F2 GDS = mul2(f2(gd[e], gd[e + 1]), SC2);
          const F2 GPR = fma2(GDS, DPM, sub2(f2(uv[e], uv[e + 1]), fma2(GAM2, DP, RHO2)));  // G_P - rho
          split(mul2(PR, DPM), sv[e], sv[e + 1]);                // dS
          split(mul2(PR, GPR), dp[e], dp[e + 1]);                // G_S
          split(mul2(PR, sub2(GDS, GAM2)), gd[e], gd[e + 1]);    // G_dP
          uv[e] = p0;                                            // P
          uv[e + 1] = p1;
        }
      }
      };
      if constexpr (CAUSAL) {
        if (need_mask) elementwise(std::true_type{});
        else elementwise(std::false_type{});
      } else {
        elementwise(need_mask);  // masks only a ragged last tile: one version
      }
      if constexpr (C::NE > 0) {
        // With EIS the results go into this tile's own stage (its score
        // products are complete), so no wait for the previous tile is needed.
        if constexpr (!C::EIS) {
          if (n >= 1 && !mbar_wait(e_empty, (n - 1) & 1, g, 7)) { ok = false; break; }
        }
        store_cols<BF16, CPW>(tileE(s, 0), BM, r, c0, sv);
        if constexpr (KIND == kBwd2Q) {
          store_cols<BF16, CPW>(tileE(s, 1), BM, r, c0, dp);
          if constexpr (GDO) {
            store_cols<BF16, CPW>(tileE(s, 2), BM, r, c0, gd);
            store_cols<BF16, CPW>(tileE(s, 3), BM, r, c0, uv);
          }
        }
        fence_async_smem();
        mbar_arrive(e_full + (n & 1));
      }
    }
    const bool valid = row < T;
    if constexpr (KIND == kStats) {
      float a_g, a2, a3, a4, hi_;
      split(AG, a_g, hi_);
      a_g = (a_g + hi_) * scale;
      split(A2, a2, hi_);
      a2 = (a2 + hi_) * scale;
      split(A3, a3, hi_);
      a3 += hi_;
      split(A4, a4, hi_);
      a4 += hi_;
      // the two column halves of each row combine through shared memory
      if (half == 1) {
        red[r * 4 + 0] = a_g;
        red[r * 4 + 1] = a2;
        red[r * 4 + 2] = a3;
        red[r * 4 + 3] = a4;
      }
      compute_bar<C::NCT>();
      if (half == 0 && ok && !*abort_flag && nsplit > 1) {
        // this share's four row sums; the reduction forms gamma and rho from their totals
        const float4 sums = make_float4(a_g + red[r * 4 + 0], a2 + red[r * 4 + 1], a3 + red[r * 4 + 2],
                                        a4 + red[r * 4 + 3]);
        reinterpret_cast<float4*>(p.part0)[(static_cast<int64_t>(share) * p.B * p.H + bh) * p.t_pad + row] =
            valid ? sums : make_float4(0.f, 0.f, 0.f, 0.f);
      } else if (half == 0 && ok && !*abort_flag) {
        a_g += red[r * 4 + 0];
        a2 += red[r * 4 + 1];
        a3 += red[r * 4 + 2];
        a4 += red[r * 4 + 3];
        const float rho_v = a2 - del * a_g - a_g * a4 + a3;
        p.out_f0[sidx] = valid ? a_g : 0.f;
        p.out_f1[sidx] = valid ? rho_v : 0.f;
      }
    } else {
      if (ok && mbar_wait(acc_full, 0, g, 8)) {
        tc_fence_after();
        if (nsplit > 1) {
          // unscaled fp32 partials of this share (rows up to t_pad exist in the work space)
          const int64_t prow = (static_cast<int64_t>(share) * p.B * p.H + bh) * p.t_pad + row;
          acc_cols_to_f32<D / 2>(tAcc0 + lane_off, half * (D / 2), p.part0 + prow * D, n_tiles > 0);
          if constexpr (KIND == kBwd2Q && GDO)
            acc_cols_to_f32<D / 2>(tAcc1 + lane_off, half * (D / 2), p.part1 + prow * D, n_tiles > 0);
        } else {
          uint16_t* r0 = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                         static_cast<int64_t>(row) * p.o0_st;
          acc_cols_to_global<D / 2, BF16>(tAcc0 + lane_off, half * (D / 2), r0, valid, scale);
          if constexpr (KIND == kBwd2Q && GDO) {
            uint16_t* r1 = p.out1 + static_cast<int64_t>(bidx) * p.o1_sb + static_cast<int64_t>(hidx) * p.o1_sh +
                           static_cast<int64_t>(row) * p.o1_st;
            acc_cols_to_global<D / 2, BF16>(tAcc1 + lane_off, half * (D / 2), r1, valid, 1.f);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int D, bool BF16, bool CAUSAL, int KIND, bool GDO>
static cudaError_t launch_qm_t(const KParams& p, cudaStream_t stream) {
  using C = QmCfg<D, KIND, GDO>;
  auto kern = attn_qm_kernel<D, BF16, CAUSAL, KIND, GDO>;
  // The register split may only hand out what the launch allocated; a build
  // whose register count came out lower is refused rather than launched.
  static const int launch_regs = [&] {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, kern) == cudaSuccess ? a.numRegs : 0;
  }();
  if (C::SPLIT_REGS && launch_regs < C::REG_LAUNCH) return cudaErrorLaunchOutOfResources;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H * (p.nsplit > 1 ? p.nsplit : 1), (p.T + C::BM - 1) / C::BM);
  kern<<<grid, C::NTHREADS, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_qm(const KParams& p, int d, bool bf16, bool causal, int kind, bool gdo, cudaStream_t stream) {
#define TTT_QM_KIND(D_, BF_, CA_)                                                                   \
  if (d == D_ && bf16 == BF_ && causal == CA_) {                                                  \
    if (kind == kBwdQ) return launch_qm_t<D_, BF_, CA_, kBwdQ, false>(p, stream);                 \
    if (kind == kStats) return launch_qm_t<D_, BF_, CA_, kStats, false>(p, stream);               \
    if (kind == kBwd2Q && !gdo) return launch_qm_t<D_, BF_, CA_, kBwd2Q, false>(p, stream);       \
    if (kind == kBwd2Q && gdo) return launch_qm_t<D_, BF_, CA_, kBwd2Q, true>(p, stream);         \
  }
#define TTT_QM_CA(D_, BF_) TTT_QM_KIND(D_, BF_, false) TTT_QM_KIND(D_, BF_, true)
  TTT_QM_CA(64, false) TTT_QM_CA(64, true) TTT_QM_CA(128, false) TTT_QM_CA(128, true)
#undef TTT_QM_CA
#undef TTT_QM_KIND
  return cudaErrorInvalidValue;
}

}  // namespace ttt
