// Key-major backward passes (sm_100a). One CTA owns 128 key rows of one head
// and streams 64-query tiles. Every score tile is computed transposed
// (keys x queries), so the elementwise results are already oriented as the
// A operand (M = keys) of the accumulate products.
//
//   kBwdKV  : dV = P^T dO,  dK = scale * dS^T Q
//             (replaces _attn_bwd_dv_from_p_kernel and _attn_bwd_dk_kernel,
//             ttt_kernels/backward_stubs.py:124-151 and 313-359, recomputing P
//             from lse2 instead of reading it)
//   kBwdKVQ : kBwdKV plus dQ = scale * dS K in the same pass (d = 64): the
//             elementwise warps also write dS^T to shared memory; every pair
//             of 64-query tiles gets one dS K product (M = 128 queries, both
//             operands MN-major), whose rows the elementwise warps add into an
//             fp32 dQ accumulator in global memory two tiles later. It replaces
//             the separate query-major dQ pass (kBwdQ), which recomputes S, P,
//             dP and dS for the same tiles.
//   kBwd2KV : dd_K = scale * (dS^T u_q + G_S^T Q),  dd_V = G_dP^T dO
//             (the key-side half of the complete double backward that the
//             reference approximates with torch.matmul in
//             backward_stubs.py:435-514)
//
// Roles: warps 0..7 elementwise (warp w: TMEM lanes 32*(w%4)..+31, tile
// columns (w/4)*32..+32), warp 9 TMA producer, warps 8 and 10 (and 11) MMA
// issuers: one thread issues at most one tcgen05.mma per ~85 cycles, below the
// tensor pipe's rate. The per-query statistics (lse2, delta, gamma, rho) of
// each tile arrive with it through TMA and are read with broadcast 16-byte
// loads.
//
// The elementwise results E (16-bit P^T, dS^T | dS^T, G_S^T, G_dP^T) live in
// TMEM as packed pairs and are the A operand of the accumulate products:
//   kBwdKV: over the tile's own score buffer (two buffers), each thread
//     writing only columns it read: its 16 P^T words over its half's S^T
//     columns (read by issuer 0's dV products, before issuer 0's next S^T
//     product there), its 16 dS^T words over its half's dP^T columns (issuer
//     1's dK products, then issuer 1's next dP^T);
//   kBwd2KV d=64: a dedicated region;
//   kBwd2KV d=128, where four 64-wide score tiles and two 128-wide
//     accumulators fill all 512 columns: dS^T and G_S^T over the dP^T columns,
//     G_dP^T over the (dO u_v^T)^T columns. Three issuers: issuer 0 the
//     products over S^T and G_dS^T (K [Q; u_q]^T, u_k Q^T), which no longer
//     wait for E; issuer 1 the dd_K products of tile n, then dP^T of tile n+1;
//     issuer 2 the dd_V products of tile n, then (dO u_v^T)^T of tile n+1.
// Reusing E's columns for the next score product needs no wait: tcgen05.mma
// ops issued by one thread execute in issue order, so the accumulate product
// has read E before a later product of the same thread writes there.
//
// In the double backward the streamed Q and u_q tiles are stacked in one
// panel so that K [Q; u_q]^T produces [S^T | K u_q^T] as a single N=128
// product (an M=128 UMMA with N <= 64 costs about as much as one with N=128).
// Causal: query tiles that end before the CTA's first key are skipped.
#include <type_traits>

#include "attn_pipe.cuh"
#include "kernels.h"

namespace ttt {

// Columns of K-step kk of an E tile written over score columns: queries
// 32h..32h+31 (half h of the elementwise warps) hold K-steps 2h and 2h+1.
struct KOffEHalf {
  static constexpr int at(int kk) { return 32 * (kk >> 1) + (kk & 1) * 8; }
};

template <int D, int KIND>
struct KmCfg {
  static constexpr int BK = 128;  // keys per CTA (TMEM lanes)
  static constexpr int BM = 64;   // queries per streamed tile
  static constexpr bool BWD2 = (KIND == kBwd2KV);
  static constexpr bool FUSEQ = (KIND == kBwdKVQ);
  static_assert(!FUSEQ || D == 64, "the fused dQ pass is built for d = 64 (its TMEM fits beside two score buffers)");
  // FUSEQ: a dQ accumulator of D columns for the 128 queries of a pair of tiles,
  // and the pair's dS^T tiles in shared memory (two pair buffers).
  static constexpr int DQ_COLS = FUSEQ ? D : 0;
  static constexpr int TILE_DS = BK * BM * 2;
  static constexpr int DS_BYTES = FUSEQ ? 4 * TILE_DS : 0;
  static constexpr int NR = BWD2 ? 4 : 2;   // resident: K, V, (u_k, u_v)
  static constexpr int NSC = BWD2 ? 4 : 2;  // score tiles: S^T, (G_dS^T,) dP^T, ((dO u_v^T)^T)
  static constexpr int NE = BWD2 ? 3 : 2;   // P^T, dS^T | dS^T, G_S^T, G_dP^T
  static constexpr int NA = 2;
  static constexpr int NCW = 8;
  static constexpr int NCT = NCW * 32;
  // Off: with it the share bookkeeping of split mode fits without small spills,
  // but the two idle warps cost more (measured 0.7-1.6% slower per step).
  static constexpr bool SPLIT_REGS = false;
  // Register split: the launch gives every thread REG_LAUNCH registers (three
  // warps share one 16K-register sub-partition); the control warpgroup then
  // drops to REG_CTRL and the two elementwise warpgroups rise to REG_ELEM.
  static constexpr int REG_LAUNCH = 168, REG_CTRL = 152, REG_ELEM = (3 * REG_LAUNCH - REG_CTRL) / 2;
  static_assert(REG_ELEM % 8 == 0 && 2 * REG_ELEM + REG_CTRL <= 3 * REG_LAUNCH, "register split");
  static constexpr int CPW = BM / 2;
  static constexpr int TILE_R = BK * D * 2;
  // streamed: ST0 = [Q; u_q] (or Q), ST1 = dO
  static constexpr int ST0_ROWS = BWD2 ? 2 * BM : BM;
  static constexpr int ST0_BYTES = ST0_ROWS * D * 2;
  static constexpr int ST1_BYTES = BM * D * 2;
  static constexpr int NSTAT = BWD2 ? 4 : 2;  // lse2, delta, (gamma, rho) rows per stage
  static constexpr int STAT_BYTES = BM * 4;
  static constexpr int STAGE_TX = ST0_BYTES + ST1_BYTES + NSTAT * STAT_BYTES;  // bytes TMA delivers per stage
  static constexpr int STAGE = (STAGE_TX + 1023) / 1024 * 1024;               // pitch keeps tiles 1024-aligned
  static constexpr int E_COLS = BM / 2;  // TMEM columns of one packed 16-bit E tile
  // TMEM layout
  static constexpr bool E_OWN = !BWD2;  // E over the S^T columns of its own score buffer
  static constexpr bool ETM = BWD2;     // E in a region of its own (dedicated or shared)
  static constexpr int NBUF_WANT = (2 * NSC * BM + NA * D + DQ_COLS + (ETM ? NE * E_COLS : 0) <= 512) ? 2 : 1;
  static constexpr int NBUF = NBUF_WANT;
  static constexpr int SC_COLS = NBUF * NSC * BM;
  static constexpr int ACC_COL = SC_COLS;
  static constexpr bool E_DEDICATED = ETM && (SC_COLS + NA * D + NE * E_COLS <= 512);
  // E over score columns (d=128 double backward): E tiles 0 and 1 (read by the
  // dd_K products) over the dP^T columns, E tile 2 (read by dd_V) over the
  // (dO u_v^T)^T columns, so the S^T / G_dS^T products never wait for E.
  static constexpr bool E_OVERLAP = ETM && !E_DEDICATED;
  // Two MMA issuing threads (one thread cannot feed the tensor pipe at its
  // rate): issuer 0 the score products, issuer 1 the accumulate products. With
  // E over score columns, three: issuer 0 the S^T / G_dS^T products, issuer 1
  // the dd_K products of tile n then the dP^T product of tile n+1 over the same
  // columns, issuer 2 the dd_V products then (dO u_v^T)^T; every product that
  // overwrites E follows the products that read it on the same thread.
  static constexpr bool THREE_ISSUERS = E_OVERLAP;
  static constexpr bool TWO_ISSUERS = !E_OVERLAP;
  // Split the score products too: issuer 0 those over the columns E may use
  // (S^T, G_dS^T), issuer 1 the others (dP^T, (dO u_v^T)^T) and the accumulates.
  // Measured: 8% faster for the d=128 backward, no gain or a loss for the d=64
  // double backward.
  static constexpr bool SPLIT_SCORES = TWO_ISSUERS && (D == 128 || !BWD2);
  // First order: issuer 1 would issue dP^T and both accumulates (16 UMMAs a
  // tile at d=128) against issuer 0's 8 for S^T, so issuer 0 also takes dV +=
  // P^T dO; a stage is then released by both (l_empty and acc_full count two
  // commits).
  static constexpr bool ACC_SPLIT = SPLIT_SCORES && !BWD2;
  // With ACC_SPLIT, dS^T (read by issuer 1's dK products) lies over the dP^T
  // columns that issuer 1 overwrites next, P^T (issuer 0's dV) over S^T: each
  // issuer overwrites only E that it has read itself, so no completion wait
  // (e_cons) crosses the two issuers.
  static constexpr bool E1_OVER_DP = ACC_SPLIT;
  static constexpr int NTHREADS =
      NCT + (SPLIT_REGS ? 128 : 64) + (TWO_ISSUERS && !SPLIT_REGS ? 32 : 0) + (THREE_ISSUERS ? 64 : 0);
  static constexpr int E_COL = E_DEDICATED ? SC_COLS + NA * D : (E_OVERLAP ? 2 * BM : 0);
  static_assert(!E_OVERLAP || BWD2, "E over score columns only in the double backward");
  static constexpr int DQ_COL = SC_COLS + NA * D;  // FUSEQ: the pair's dQ accumulator
  static constexpr int TMEM_USED = SC_COLS + NA * D + DQ_COLS + (E_DEDICATED ? NE * E_COLS : 0);
  static_assert(!FUSEQ || (NBUF == 2 && !E_DEDICATED), "fused dQ layout");
  static constexpr int TMEM_COLS = TMEM_USED <= 128 ? 128 : (TMEM_USED <= 256 ? 256 : 512);
  static_assert(TMEM_USED <= 512, "TMEM overflow");
  static_assert(!E_OVERLAP || NBUF == 1, "overlapping E needs a single score buffer");
  // barriers 0..20; FUSEQ adds dq_full and dq_empty; then the TMEM slot and abort flag
  static constexpr int NBAR = FUSEQ ? 25 : 21;
  static constexpr int BAR_BYTES = (NBAR + 1) * 8;
  static constexpr int FIXED = NR * TILE_R + DS_BYTES + BAR_BYTES + (STAGE_TX - STAGE);
  static constexpr int NSTAGE = (FIXED + 4 * STAGE + 1024 <= 232448) ? 4 : (FIXED + 3 * STAGE + 1024 <= 232448) ? 3 : 2;
  // Three issuers (d=128 double backward): a stage arrives in two parts on two
  // barriers, [Q; u_q] and the statistics first (issuer 0's score products and the
  // elementwise warps), then dO (issuers 1 and 2), so the next tile's first score
  // products need not wait for the whole stage. The second part uses the l_full
  // slots that a two-stage ring leaves free.
  static constexpr bool SPLIT_STAGE = THREE_ISSUERS;
  static_assert(!SPLIT_STAGE || NSTAGE <= 2, "split stages use the free l_full slots 2, 3");
  static constexpr int STAGE_TX_A = SPLIT_STAGE ? ST0_BYTES + NSTAT * STAT_BYTES : STAGE_TX;
  static constexpr int STAGE_TX_B = ST1_BYTES;
  static constexpr int OFF_R = 0;
  static constexpr int OFF_DS = OFF_R + NR * TILE_R;
  static constexpr int OFF_S = OFF_DS + DS_BYTES;
  static constexpr int OFF_BAR = OFF_S + (NSTAGE - 1) * STAGE + STAGE_TX;  // the last stage needs no padding
  static constexpr int BODY = OFF_BAR + BAR_BYTES;
  // Reserve room to realign the dynamic shared-memory base to 1024 bytes when
  // it fits; otherwise the kernel requires (and checks) an aligned base.
  static constexpr int PAD = (BODY + 1024 <= 232448) ? 1024 : 0;
  static constexpr int SMEM = BODY + PAD;
  static_assert(SMEM <= 232448, "key-major tile set exceeds shared memory");
  static_assert(ST0_BYTES % 1024 == 0 && ST1_BYTES % 1024 == 0, "streamed tiles must stay 1024-aligned");
  // score tile columns within a buffer
  static constexpr int C_S = 0, C_GDS = BWD2 ? BM : 0, C_DP = BWD2 ? 2 * BM : BM, C_UV = 3 * BM;
};

int km_tile_rows(int d, int kind) {
  (void)d;
  (void)kind;
  return 64;
}

template <int D, bool BF16, bool CAUSAL, int KIND>
__global__ void __launch_bounds__(KmCfg<D, KIND>::NTHREADS, 1) attn_km_kernel(const __grid_constant__ KParams p) {
  using C = KmCfg<D, KIND>;
  constexpr int BM = C::BM, BK = C::BK, NP = D / 64, NBUF = C::NBUF, NSTAGE = C::NSTAGE, CPW = C::CPW;
  constexpr int SR0 = C::ST0_ROWS;
  constexpr int WARP_MMA = C::NCW, WARP_LOAD = C::NCW + 1, WARP_MMA2 = C::NCW + 2, WARP_MMA3 = C::NCW + 3;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = C::PAD ? align1024(smem_raw) : smem_raw;
  if (C::PAD == 0 && (smem_u32(smem_raw) & 1023u) != 0) {
    // no room to realign: refuse to run on a misaligned base (the swizzled
    // tiles would be read wrongly) and report it through the error word
    if (threadIdx.x == 0) report_error(p.err, p.err_host, kErrMisaligned);
    return;
  }
  uint8_t* sR = smem + C::OFF_R;
  uint8_t* sS = smem + C::OFF_S;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* res_full = bars + 0;
  uint64_t* l_full = bars + 1;    // [4]
  // SPLIT_STAGE: dO of stage s arrives on l_full_b[s] (l_full[s] has the rest)
  uint64_t* l_full_b = C::SPLIT_STAGE ? l_full + 2 : l_full;
  uint64_t* l_empty = bars + 5;   // [4]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_free = bars + 11;   // [2] (NCT arrivals)
  // e_full[n % 2] (NCT arrivals): E of tile n written. Two barriers, because a
  // compute warp may finish tile n+1 before a slower one finishes tile n; with
  // one barrier its second arrival would complete tile n's phase early. It
  // cannot reach tile n+2 before tile n's phase completed: those scores are
  // issued only after the MMA thread has seen e_full for tile n.
  uint64_t* e_full = bars + 13;   // [2]
  uint64_t* e_empty = bars + 15;  // accumulate products of a tile finished (E consumed)
  uint64_t* acc_full = bars + 16;
  // one per MMA issuer: bars + 17, 18 (and 19, the e_cons slot, for a third:
  // three issuers only with E over score columns, where e_cons is unused)
  uint64_t* drain = bars + 17;
  // e_cons[b]: the accumulate products that read E in score buffer b completed
  // (two issuers, E over its own score buffer)
  uint64_t* e_cons = bars + 19;  // [2]
  // FUSEQ: dq_full (the dS K product of a pair completed: its TMEM rows are ready
  // and its dS^T tiles may be reused) and dq_empty (NCT arrivals: the compute
  // warps have read those rows, so the next pair's product may overwrite them)
  uint64_t* dq_full = bars + 21;
  uint64_t* dq_empty = bars + 22;
  // FUSEQ: stage_full (NCT arrivals: every row of a pair's dQ is staged for the TMA
  // reduce) and stage_free (one arrival: the TMA unit finished reading a staged
  // buffer, which the next pair's dS^T may then overwrite). Bounded waits, so a CTA
  // that aborts never leaves a warp parked at a hardware barrier.
  uint64_t* stage_full = bars + 23;
  uint64_t* stage_free = bars + 24;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* sDS = smem + C::OFF_DS;
  // dS^T of tile n ([BK keys x BM queries], PL layout): pair buffer (n / 2) % 2, half n % 2,
  // so a pair's two tiles form one [BK x 2 BM] MN-major operand
  auto dsT = [&](int n) { return sDS + (((n >> 1) & 1) * 2 + (n & 1)) * C::TILE_DS; };
  auto tileR = [&](int t) { return sR + t * C::TILE_R; };
  auto st0 = [&](int s) { return sS + s * C::STAGE; };
  auto st1 = [&](int s) { return sS + s * C::STAGE + C::ST0_BYTES; };
  auto statS = [&](int s, int t) {
    return reinterpret_cast<const float*>(sS + s * C::STAGE + C::ST0_BYTES + C::ST1_BYTES + t * C::STAT_BYTES);
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // split mode: this CTA takes share `share` of its key block's query tiles
  const int nsplit = p.nsplit > 1 ? p.nsplit : 1;
  const GridPos gp = grid_pos();
  const int bh = gp.unit / nsplit, share = gp.unit % nsplit;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int kblk = gp.rank;  // causal: small kblk has the most query tiles, launched first
  const int k0 = kblk * BK;
  const int T = p.T;
  const int n_q = (T + BM - 1) / BM;
  // Causal: this key block meets query tiles from its diagonal up to the last
  // query that sees its last key.
  const Band band = Band::make(p, CAUSAL);
  const int qt_first = CAUSAL ? (k0 / BM) : 0;
  const int qt_end = CAUSAL ? min(n_q, band.last_query(min(k0 + BK, T) - 1) / BM + 1) : n_q;
  const int qt0 = qt_first + split_begin(qt_end - qt_first, share, nsplit);
  const int n_tiles = qt_first + split_begin(qt_end - qt_first, share + 1, nsplit) - qt0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 21; ++i) mbar_init(bars + i, 1);
    if (C::FUSEQ) {
      mbar_init(dq_full, 1);
      mbar_init(dq_empty, C::NCT);
      mbar_init(stage_full, C::NCT);
      mbar_init(stage_free, 1);
    }
    mbar_init(s_free + 0, C::NCT);
    mbar_init(s_free + 1, C::NCT);
    if (C::SPLIT_SCORES) {  // both issuers' score products
      mbar_init(s_full + 0, 2);
      mbar_init(s_full + 1, 2);
    }
    if (C::ACC_SPLIT) {  // both issuers' accumulate products
      for (int i = 0; i < 4; ++i) mbar_init(l_empty + i, 2);
      mbar_init(acc_full, 2);
    }
    if (C::THREE_ISSUERS) {  // all three read a stage and write score columns
      mbar_init(s_full + 1, 2);  // s_full[0]: S^T, G_dS^T (issuer 0); s_full[1]: dP^T, (dO u_v^T)^T
      for (int i = 0; i < 4; ++i) mbar_init(l_empty + i, 3);
      mbar_init(acc_full, 2);  // issuers 1 and 2
    }
    mbar_init(e_full + 0, C::NCT);
    mbar_init(e_full + 1, C::NCT);
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
  const uint32_t tAcc0 = tmem + C::ACC_COL;  // dK / dd_K
  const uint32_t tAcc1 = tAcc0 + D;          // dV / dd_V
  const uint32_t tE = tmem + C::E_COL;       // packed E tiles (ETM)
  const uint32_t tDQ = tmem + C::DQ_COL;     // FUSEQ: dQ rows of the current pair
  Guard g{abort_flag, p.err, p.err_host};
  // TMEM column of K-step kk (16 queries) of E tile j of tile n. Outside a
  // dedicated region each half of the elementwise warps (queries 32h..32h+31)
  // writes E only over score columns it has read itself: 32 columns of the first
  // score tile it covers take E tiles 0 and 1 (16 words each), 32 of the second
  // take tile 2 (first order: S^T; double backward: dP^T, then (dO u_v^T)^T).
  auto e_col = [&](int j, int kk, int n) -> uint32_t {
    if constexpr (C::E_DEDICATED) return tE + j * C::E_COLS + kk * 8;
    const uint32_t off = 32 * (kk >> 1) + (kk & 1) * 8 + (C::E1_OVER_DP ? j * C::C_DP : (j == 2 ? BM : 16 * j));
    if constexpr (C::E_OWN) return tmem + (n % NBUF) * C::NSC * BM + off;
    return tE + off;
  };

  if (warp >= C::NCW) {
   if constexpr (C::SPLIT_REGS) regs_release<C::REG_CTRL>();
   if (warp == WARP_LOAD) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = 0; t < C::NR; ++t) tma_prefetch(&p.own[t]);
      for (int t = 0; t < (C::BWD2 ? 3 : 2); ++t) tma_prefetch(&p.str[t]);
      for (int t = 0; t < C::NSTAT; ++t) tma_prefetch(&p.st[t]);
      int issued[4] = {0, 0, 0, 0};
      mbar_arrive_tx(res_full, C::NR * C::TILE_R);
      for (int t = 0; t < C::NR; ++t)
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(tileR(t) + pp * BK * 128, &p.own[t], res_full, pp * 64, k0, hidx, bidx);
      for (int n = 0; n < n_tiles; ++n) {
        const int s = n % NSTAGE;
        const int qrow = (qt0 + n) * BM;
        if (n >= NSTAGE && !mbar_wait(l_empty + s, ((n / NSTAGE) - 1) & 1, g, 1)) break;
        if constexpr (C::SPLIT_STAGE) {
          // [Q; u_q] and the statistics first, then dO, each part on its own barrier
          mbar_arrive_tx(l_full + s, C::STAGE_TX_A);
          for (int pp = 0; pp < NP; ++pp) {
            tma_load_4d(st0(s) + pp * SR0 * 128, &p.str[0], l_full + s, pp * 64, qrow, hidx, bidx);
            tma_load_4d(st0(s) + pp * SR0 * 128 + BM * 128, &p.str[2], l_full + s, pp * 64, qrow, hidx, bidx);
          }
          for (int t = 0; t < C::NSTAT; ++t)
            tma_load_2d(const_cast<float*>(statS(s, t)), &p.st[t], l_full + s, qrow, bh);
          mbar_arrive_tx(l_full_b + s, C::STAGE_TX_B);
          for (int pp = 0; pp < NP; ++pp)
            tma_load_4d(st1(s) + pp * BM * 128, &p.str[1], l_full_b + s, pp * 64, qrow, hidx, bidx);
        } else {
          mbar_arrive_tx(l_full + s, C::STAGE_TX);
          // str[0] = Q, str[1] = dO, str[2] = u_q (stacked under Q)
          for (int pp = 0; pp < NP; ++pp) {
            tma_load_4d(st0(s) + pp * SR0 * 128, &p.str[0], l_full + s, pp * 64, qrow, hidx, bidx);
            tma_load_4d(st1(s) + pp * BM * 128, &p.str[1], l_full + s, pp * 64, qrow, hidx, bidx);
            if constexpr (C::BWD2)
              tma_load_4d(st0(s) + pp * SR0 * 128 + BM * 128, &p.str[2], l_full + s, pp * 64, qrow, hidx, bidx);
          }
          for (int t = 0; t < C::NSTAT; ++t)
            tma_load_2d(const_cast<float*>(statS(s, t)), &p.st[t], l_full + s, qrow, bh);
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
   } else if (warp == WARP_MMA || ((C::TWO_ISSUERS || C::THREE_ISSUERS) && warp == WARP_MMA2) ||
              (C::THREE_ISSUERS && warp == WARP_MMA3)) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_n1 = idesc_f16(128, BM, BF16, false, false);
      constexpr uint32_t id_n2 = idesc_f16(128, 2 * BM, BF16, false, false);
      constexpr uint32_t id_acc = idesc_f16(128, D, BF16, false, true);
      const uint32_t aK = smem_u32(tileR(0)), aV = smem_u32(tileR(1));
      const uint32_t aUK = C::BWD2 ? smem_u32(tileR(2)) : 0u, aUV = C::BWD2 ? smem_u32(tileR(3)) : 0u;
      using LD = KOff2<KOffK<BK>, KOffK<BM>>;   // resident A, streamed dO (rows BM)
      using LQ = KOff2<KOffK<BK>, KOffK<SR0>>;  // resident A, streamed [Q; u_q] (rows SR0)
      using LE = KOff2<std::conditional_t<C::E_DEDICATED, KOffT, KOffEHalf>, KOffMN>;  // E from TMEM, MN-major B
      // Probes pay off only with two score buffers: with one, each tile first waits for
      // the compute warps to read the previous scores, a wait no probe can skip.
      constexpr bool PR = NBUF == 2;
      // Score products whose output columns never hold E: dP^T (and (dO u_v^T)^T).
      // Each group issues its last product as one batch with two barrier probes.
      auto scores_free_cols = [&](uint32_t base, int s, const uint64_t* b0_, uint32_t p0_, const uint64_t* b1_,
                                  uint32_t p1_) -> uint32_t {
        const uint32_t b1 = smem_u32(st1(s));
        if constexpr (C::BWD2) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_DP, desc_kmajor(aV, BK, kk), desc_kmajor(b1, BM, kk), id_n1, kk > 0);
          return issue_ss<D / 16, LD, PR>(base + C::C_UV, desc_kmajor(aUV, BK, 0), desc_kmajor(b1, BM, 0), id_n1, 0u, b0_,
                                      p0_, b1_, p1_);
        } else {
          return issue_ss<D / 16, LD, PR>(base + C::C_DP, desc_kmajor(aV, BK, 0), desc_kmajor(b1, BM, 0), id_n1, 0u, b0_,
                                      p0_, b1_, p1_);
        }
      };
      // Score products into columns that E may share: S^T (and G_dS^T).
      auto scores_e_cols = [&](uint32_t base, int s, const uint64_t* b0_, uint32_t p0_, const uint64_t* b1_,
                               uint32_t p1_) -> uint32_t {
        const uint32_t b0 = smem_u32(st0(s));
        if constexpr (C::BWD2) {
          // [S^T | K u_q^T] = K [Q; u_q]^T ; G_dS^T/scale += u_k Q^T
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_S, desc_kmajor(aK, BK, kk), desc_kmajor(b0, SR0, kk), id_n2, kk > 0);
          return issue_ss<D / 16, LQ, PR>(base + C::C_GDS, desc_kmajor(aUK, BK, 0), desc_kmajor(b0, SR0, 0), id_n1, 1u,
                                      b0_, p0_, b1_, p1_);
        } else {
          return issue_ss<D / 16, LQ, PR>(base + C::C_S, desc_kmajor(aK, BK, 0), desc_kmajor(b0, SR0, 0), id_n1, 0u, b0_,
                                      p0_, b1_, p1_);
        }
      };
      // parts (first-order kernel): bit 0 dV += P^T dO, bit 1 dK += dS^T Q
      auto acc_products = [&](int n, const uint64_t* b0_, uint32_t p0_, const uint64_t* b1_, uint32_t p1_,
                              int parts = 3) -> uint32_t {
        const int s = n % NSTAGE;
        const uint32_t bQ = smem_u32(st0(s)), bDO = smem_u32(st1(s));
        const uint32_t acc_first = n > 0 ? 1u : 0u;
        if constexpr (!C::BWD2) {
          if (parts & 1) {
#pragma unroll
            for (int kk = 0; kk < BM / 16; ++kk)
              umma_ts(tAcc1, e_col(0, kk, n), desc_mnmajor(bDO, BM, kk), id_acc, (acc_first || kk > 0) ? 1u : 0u);
          }
          if (!(parts & 2)) return 0u;
          return issue_ts<BM / 16, LE, PR>(tAcc0, e_col(1, 0, n), desc_mnmajor(bQ, SR0, 0), id_acc, acc_first, b0_, p0_,
                                       b1_, p1_);
        } else {
          // dd_K += dS^T u_q + G_S^T Q ; dd_V += G_dP^T dO   (E in TMEM). The three products
          // alternate per K-step (faster than grouping them), so this step carries no probes.
          (void)b0_, (void)p0_, (void)b1_, (void)p1_;
          const uint32_t bUQ = bQ + BM * 128;
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk) {
            const uint32_t a = (acc_first || kk > 0) ? 1u : 0u;
            umma_ts(tAcc0, e_col(0, kk, n), desc_mnmajor(bUQ, SR0, kk), id_acc, a);
            umma_ts(tAcc0, e_col(1, kk, n), desc_mnmajor(bQ, SR0, kk), id_acc, 1u);
            umma_ts(tAcc1, e_col(2, kk, n), desc_mnmajor(bDO, BM, kk), id_acc, a);
          }
          return 0u;
        }
      };
      bool ok = mbar_wait(res_full, 0, g, 1);
      // res_full's phase 0 completed above: a probe of it always succeeds (an unused probe slot)
      const uint64_t* done = res_full;
      if constexpr (C::TWO_ISSUERS) {
        const int me = warp == WARP_MMA ? 0 : 1;
        // issuer 0: score products of every tile (with SPLIT_SCORES only those over the
        // columns E may use; issuer 1 the others, both committing s_full, which then
        // counts two arrivals); issuer 1: each tile's accumulate products once its E is
        // written (its score products completed before that, so its stage may be
        // refilled afterwards); with ACC_SPLIT issuer 0 takes the dV products of the tile
        for (int n = 0; ok && n <= n_tiles; ++n) {
          if (n < n_tiles && (me == 0 || C::SPLIT_SCORES)) {
            const int sb = n % NBUF, s = n % NSTAGE;
            const uint32_t base = tmem + sb * C::NSC * BM;
            if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2))) break;
            if (n >= NBUF && !(ok = mbar_wait(s_free + sb, ((n / NBUF) - 1) & 1, g, 3))) break;
            // E over its own score buffer: the accumulate products that read it completed
            if (me == 0 && C::E_OWN && !C::E1_OVER_DP && n >= NBUF &&
                !(ok = mbar_wait(e_cons + sb, ((n / NBUF) - 1) & 1, g, 5)))
              break;
            tc_fence_after();
            if (me == 0) scores_e_cols(base, s, done, 0u, done, 0u);
            if (me == 1 || !C::SPLIT_SCORES) scores_free_cols(base, s, done, 0u, done, 0u);
            umma_commit(s_full + sb);
          }
          if ((me == 1 || C::ACC_SPLIT) && n >= 1) {
            if (!(ok = mbar_wait(e_full + ((n - 1) & 1), ((n - 1) >> 1) & 1, g, 4))) break;
            tc_fence_after();
            acc_products(n - 1, done, 0u, done, 0u, C::ACC_SPLIT ? (me == 0 ? 1 : 2) : 3);
            if constexpr (C::E_DEDICATED) umma_commit(e_empty);
            // issuer 0's own score products into this buffer follow its dV products in order
            if constexpr (C::E_OWN && !C::E1_OVER_DP) {
              if (me == 1) umma_commit(e_cons + (n - 1) % NBUF);
            }
            umma_commit(l_empty + (n - 1) % NSTAGE);
            if constexpr (C::FUSEQ) {
              // after the last tile of a pair: dQ rows of its 128 queries = dS K, with
              // A = the pair's dS^T tiles read MN-major (rows = keys) and B = K (MN-major);
              // the rows of a missing second tile are never read back
              if (me == 1 && (((n - 1) & 1) || n == n_tiles)) {
                const int pr = (n - 1) >> 1;
                if (pr >= 1 && !(ok = mbar_wait(dq_empty, (pr - 1) & 1, g, 11))) break;
                tc_fence_after();
                constexpr uint32_t id_dq = idesc_f16(128, D, BF16, true, true);
                const uint32_t aDS = smem_u32(dsT(2 * pr));
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                  umma_ss(tDQ, desc_mnmajor(aDS, BK, kk), desc_mnmajor(aK, BK, kk), id_dq, kk > 0 ? 1u : 0u);
                umma_commit(dq_full);
              }
            }
          }
        }
        if ((me == 1 || C::ACC_SPLIT) && ok) umma_commit(acc_full);
        umma_commit(drain + me);
        mbar_drain(drain + me, 0);
      } else {
        // three issuers, E over the dP^T and (dO u_v^T)^T columns (single score buffer)
        const int me = warp == WARP_MMA ? 0 : (warp == WARP_MMA2 ? 1 : 2);
        for (int n = 0; ok && n <= n_tiles; ++n) {
          const int s = n % NSTAGE;
          if (me == 0) {
            // S^T | K u_q^T, then G_dS^T += u_k Q^T, once the elementwise warps read tile n-1
            if (n == n_tiles) break;
            if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2))) break;
            if (n >= 1 && !(ok = mbar_wait(s_free, (n - 1) & 1, g, 3))) break;
            tc_fence_after();
            scores_e_cols(tmem, s, done, 0u, done, 0u);
            umma_commit(s_full);
            umma_commit(l_empty + s);
            continue;
          }
          // The stage of tile n (read next by this issuer's score product) is probed in the
          // same batch as tile n-1's accumulate products, so a stage that already landed
          // costs no separate wait on this thread (it sits on the tile-to-tile chain).
          bool stage_seen = false;
          if (n >= 1) {
            // the accumulate products of tile n-1 read its E, written over this issuer's score columns
            if (!(ok = mbar_wait(e_full + ((n - 1) & 1), ((n - 1) >> 1) & 1, g, 4))) break;
            tc_fence_after();
            const int sp = (n - 1) % NSTAGE;
            const uint32_t bQ = smem_u32(st0(sp)), bDO = smem_u32(st1(sp)), bUQ = bQ + BM * 128;
            const uint32_t acc_first = n > 1 ? 1u : 0u;
            const uint64_t* pbar = n < n_tiles ? l_full_b + s : done;
            const uint32_t ppar = n < n_tiles ? static_cast<uint32_t>((n / NSTAGE) & 1) : 0u;
            static_assert(BM / 16 == 4, "the batched accumulate issue covers four K-steps");
            uint32_t seen;
            if (me == 1) {
              // dd_K += dS^T u_q + G_S^T Q (K-steps of the two products interleaved)
              seen = umma_ts_pair4_probe<LE>(tAcc0, e_col(0, 0, n - 1), desc_mnmajor(bUQ, SR0, 0), e_col(1, 0, n - 1),
                                             desc_mnmajor(bQ, SR0, 0), id_acc, acc_first, pbar, ppar, done, 0u);
            } else {
              // dd_V += G_dP^T dO
              seen = umma_ts4_tprobe<LE>(tAcc1, e_col(2, 0, n - 1), desc_mnmajor(bDO, BM, 0), id_acc, acc_first, pbar,
                                         ppar, done, 0u);
            }
            stage_seen = (seen & 1u) != 0;
            umma_commit(l_empty + sp);
          }
          if (n < n_tiles) {
            // dP^T = V dO^T (issuer 1) or (dO u_v^T)^T = u_v dO^T (issuer 2) over the E just read
            if (!stage_seen && !(ok = mbar_wait(l_full_b + s, (n / NSTAGE) & 1, g, 2))) break;
            tc_fence_after();
            const uint32_t b1 = smem_u32(st1(s)), a0 = me == 1 ? aV : aUV;
            const uint32_t dcol = tmem + (me == 1 ? C::C_DP : C::C_UV);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              umma_ss(dcol, desc_kmajor(a0, BK, kk), desc_kmajor(b1, BM, kk), id_n1, kk > 0);
            umma_commit(s_full + 1);
          }
        }
        if (me != 0 && ok) umma_commit(acc_full);
        umma_commit(drain + me);
        mbar_drain(drain + me, 0);
      }
    }
   }
  } else {
    // ------------------------------------------------------------ elementwise warps 0..7
    if constexpr (C::SPLIT_REGS) regs_claim<C::REG_ELEM>();
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const int key = k0 + r;
    const int c0 = half * CPW;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float c = p.scale_log2, scale = p.scale;
    const bool key_edge = k0 + BK > T;
    // last query that sees this thread's key: key <= qi <= key_hi (the band's dual form)
    const int key_hi = band.last_query(key);
    // query tiles ending past the last query that sees the block's first key need the band mask
    const int band_last = CAUSAL ? band.last_query(k0) : 0x3fffffff;
    const F2 C2 = f2s(c), SC2 = f2s(scale);
    // FUSEQ: add the dQ rows of pair pr into the fp32 accumulator. TMEM lane r holds
    // query 2*pr*BM + r of this share's tiles; each thread stages its half of the
    // row (fp32) into the pair's dS^T buffer, which the pair's product has finished
    // reading, as two 128-byte-swizzled [128 x 32] panels (conflict-free 16-byte
    // stores), and one thread has the TMA unit add both panels into the accumulator
    // (a reduce in L2, asynchronous to these warps). Rows of a second tile the
    // share does not have are staged as zeros; rows past t_pad are clipped by the map.
    [[maybe_unused]] auto dq_drain = [&](int pr) -> bool {
      if (!mbar_wait(dq_full, pr & 1, g, 12)) return false;
      tc_fence_after();
      float v[D / 2];
      tmem_ld_nw<D / 2>(tDQ + lane_off + half * (D / 2), v);
      tmem_wait_ld();
      reg_fence(v);
      tc_fence_before();
      mbar_arrive(dq_empty);  // the rows are in registers: the next pair's product may overwrite them
      const bool have = 2 * pr + (r >= BM ? 1 : 0) < n_tiles;
      uint8_t* row = dsT(2 * pr) + half * (BK * 128) + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 x = have ? make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3])
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(row + ((c ^ (r & 7)) << 4)) = x;
      }
      fence_async_smem();
      mbar_arrive(stage_full);
      if (threadIdx.x == 0) {
        // every row of both panels is staged
        if (!mbar_wait(stage_full, pr & 1, g, 13)) return false;
        const int q0 = (qt0 + 2 * pr) * BM;
        tma_reduce_add_3d(&p.st[2], dsT(2 * pr), 0, q0, bh);
        tma_reduce_add_3d(&p.st[2], dsT(2 * pr) + BK * 128, 32, q0, bh);
        bulk_commit();
      }
      return true;
    };
    // Before tile n (even, n >= 4) writes dS^T into the pair buffer that pair
    // n/2 - 2 staged its dQ rows in, the TMA unit must have finished reading them
    // (thread 0 issued that reduce; it is its only bulk group still reading).
    [[maybe_unused]] auto ds_reuse = [&](int n) -> bool {
      if (threadIdx.x == 0) {
        bulk_wait_read();
        mbar_arrive(stage_free);
      }
      return mbar_wait(stage_free, ((n >> 1) - 2) & 1, g, 14);
    };
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int sb = n % NBUF, s = n % NSTAGE;
      const int qt = qt0 + n;
      const int qcol0 = qt * BM + c0;
      if constexpr (C::FUSEQ) {
        // pair (n - 3) / 2, whose product was issued about two tiles ago; draining it
        // here also frees its dS^T buffer before the next pair's tiles are written
        if ((n & 1) && n >= 3 && !dq_drain((n - 3) >> 1)) { ok = false; break; }
      }
      if constexpr (C::THREE_ISSUERS) {
        // Two phases: S^T and G_dS^T come from issuer 0 well before dP^T and
        // (dO u_v^T)^T, which follow the previous tile's accumulate products;
        // P^T, G_dP^T and E tile 2 are formed while those run.
        if (!mbar_wait(s_full + 0, n & 1, g, 6)) { ok = false; break; }
        if (!mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 9)) { ok = false; break; }
        tc_fence_after();
        const uint32_t base = tmem + lane_off + c0;
        float sv[CPW], gd[CPW];
        tmem_ld_nw<CPW>(base + C::C_S, sv);
        tmem_ld_nw<CPW>(base + C::C_GDS, gd);
        tmem_wait_ld();
        reg_fence(sv);
        reg_fence(gd);
        tc_fence_before();
        mbar_arrive(s_free);  // issuer 0 may compute the next tile's S^T, G_dS^T
        const bool need_mask = key_edge || (CAUSAL && (qt * BM < k0 + BK - 1 || qt * BM + BM - 1 > band_last));
        const float4* st_lse = reinterpret_cast<const float4*>(statS(s, 0) + c0);
        const float4* st_del = reinterpret_cast<const float4*>(statS(s, 1) + c0);
        const float4* st_gam = reinterpret_cast<const float4*>(statS(s, 2) + c0);
        const float4* st_rho = reinterpret_cast<const float4*>(statS(s, 3) + c0);
        uint32_t e2[CPW / 2];  // packed G_dP^T (E tile 2)
        auto phase_a = [&](auto masked) {
#pragma unroll
          for (int q4 = 0; q4 < CPW / 4; ++q4) {
            const float4 l4 = st_lse[q4], g4 = st_gam[q4];
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int e = q4 * 4 + h2 * 2;
              float x0, x1;
              split(sub2(mul2(f2(sv[e], sv[e + 1]), C2), h2 ? f2(l4.z, l4.w) : f2(l4.x, l4.y)), x0, x1);
              float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
              if (static_cast<bool>(masked)) {
                const int qi = qcol0 + e;
                p0 = ((key < T) && (!CAUSAL || (key <= qi && qi <= key_hi))) ? p0 : 0.f;
                p1 = ((key < T) && (!CAUSAL || (key <= qi + 1 && qi + 1 <= key_hi))) ? p1 : 0.f;
              }
              const F2 PR = f2(p0, p1);
              const F2 GDS = mul2(f2(gd[e], gd[e + 1]), SC2);
              float g0, g1;
              split(mul2(PR, sub2(GDS, h2 ? f2(g4.z, g4.w) : f2(g4.x, g4.y))), g0, g1);  // G_dP^T
              e2[e >> 1] = pack2<BF16>(g0, g1);
              sv[e] = p0;
              sv[e + 1] = p1;
              split(GDS, gd[e], gd[e + 1]);
            }
          }
        };
        if constexpr (CAUSAL) {
          if (need_mask) phase_a(std::true_type{});
          else phase_a(std::false_type{});
        } else {
          phase_a(need_mask);
        }
        if (!mbar_wait(s_full + 1, n & 1, g, 10)) { ok = false; break; }
        tc_fence_after();
        float dp[CPW], uv[CPW];
        tmem_ld_nw<CPW>(base + C::C_DP, dp);
        tmem_ld_nw<CPW>(base + C::C_UV, uv);
        tmem_wait_ld();
        reg_fence(dp);
        reg_fence(uv);
#pragma unroll
        for (int q4 = 0; q4 < CPW / 4; ++q4) {
          const float4 d4 = st_del[q4], g4 = st_gam[q4], r4 = st_rho[q4];
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int e = q4 * 4 + h2 * 2;
            const F2 PR = f2(sv[e], sv[e + 1]), DP = f2(dp[e], dp[e + 1]), GDS = f2(gd[e], gd[e + 1]);
            const F2 GAM = h2 ? f2(g4.z, g4.w) : f2(g4.x, g4.y);
            const F2 RHO = h2 ? f2(r4.z, r4.w) : f2(r4.x, r4.y);
            const F2 DPM = sub2(DP, h2 ? f2(d4.z, d4.w) : f2(d4.x, d4.y));
            const F2 GPR = fma2(GDS, DPM, sub2(f2(uv[e], uv[e + 1]), fma2(GAM, DP, RHO)));  // G_P - rho
            split(mul2(PR, DPM), sv[e], sv[e + 1]);  // dS^T
            split(mul2(PR, GPR), dp[e], dp[e + 1]);  // G_S^T
          }
        }
        // E over the columns just read: dS^T, G_S^T over dP^T, G_dP^T over (dO u_v^T)^T
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = pack2<BF16>(sv[2 * j], sv[2 * j + 1]);
        tmem_st16_raw(tE + lane_off + 32 * half, w);
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = pack2<BF16>(dp[2 * j], dp[2 * j + 1]);
        tmem_st16_raw(tE + lane_off + 32 * half + 16, w);
        tmem_st16_raw(tE + lane_off + 32 * half + BM, e2);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(e_full + (n & 1));
        continue;
      }
      if (!mbar_wait(s_full + sb, (n / NBUF) & 1, g, 6)) { ok = false; break; }
      // The per-query statistics arrived by TMA on l_full[s]; that phase cannot
      // advance until this tile's elementwise step is done.
      if (!mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 9)) { ok = false; break; }
      tc_fence_after();
      const uint32_t base = tmem + lane_off + sb * C::NSC * BM + c0;
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
      mbar_arrive(s_free + sb);

      const bool need_mask = key_edge || (CAUSAL && (qt * BM < k0 + BK - 1 || qt * BM + BM - 1 > band_last));
      const float4* st_lse = reinterpret_cast<const float4*>(statS(s, 0) + c0);
      const float4* st_del = reinterpret_cast<const float4*>(statS(s, 1) + c0);
      const float4* st_gam = reinterpret_cast<const float4*>(statS(s, C::BWD2 ? 2 : 0) + c0);
      const float4* st_rho = reinterpret_cast<const float4*>(statS(s, C::BWD2 ? 3 : 0) + c0);
      // causal: the loop runs in a masked and an unmasked version, so that
      // interior tiles carry no per-element mask test
      auto elementwise = [&](auto masked) {
#pragma unroll
      for (int q4 = 0; q4 < CPW / 4; ++q4) {
        const float4 l4 = st_lse[q4], d4 = st_del[q4];
        [[maybe_unused]] float4 g4 = make_float4(0.f, 0.f, 0.f, 0.f), r4 = g4;  // double backward only
        if constexpr (C::BWD2) {
          g4 = st_gam[q4];
          r4 = st_rho[q4];
        }
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int e = q4 * 4 + h2 * 2;
          const F2 L = h2 ? f2(l4.z, l4.w) : f2(l4.x, l4.y);
          const F2 DEL = h2 ? f2(d4.z, d4.w) : f2(d4.x, d4.y);
          float x0, x1;
          split(sub2(mul2(f2(sv[e], sv[e + 1]), C2), L), x0, x1);
          float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          if (static_cast<bool>(masked)) {
            const int qi = qcol0 + e;
            p0 = ((key < T) && (!CAUSAL || (key <= qi && qi <= key_hi))) ? p0 : 0.f;
            p1 = ((key < T) && (!CAUSAL || (key <= qi + 1 && qi + 1 <= key_hi))) ? p1 : 0.f;
          }
          const F2 PR = f2(p0, p1), DP = f2(dp[e], dp[e + 1]);
          if constexpr (!C::BWD2) {
            split(mul2(PR, sub2(DP, DEL)), dp[e], dp[e + 1]);  // dS^T
            sv[e] = p0;                                       // P^T
            sv[e + 1] = p1;
          } else {
            const F2 GAM = h2 ? f2(g4.z, g4.w) : f2(g4.x, g4.y);
            const F2 RHO = h2 ? f2(r4.z, r4.w) : f2(r4.x, r4.y);
            const F2 DPM = sub2(DP, DEL);
            const F2 GDS = mul2(f2(gd[e], gd[e + 1]), SC2);
            const F2 GPR = fma2(GDS, DPM, sub2(f2(uv[e], uv[e + 1]), fma2(GAM, DP, RHO)));  // G_P - rho
            split(mul2(PR, DPM), sv[e], sv[e + 1]);              // dS^T
            split(mul2(PR, GPR), dp[e], dp[e + 1]);              // G_S^T
            split(mul2(PR, sub2(GDS, GAM)), gd[e], gd[e + 1]);   // G_dP^T
          }
        }
      }
      };
      if constexpr (CAUSAL) {
        if (need_mask) elementwise(std::true_type{});
        else elementwise(std::false_type{});
      } else {
        elementwise(need_mask);  // masks only a ragged last tile: one version
      }
      // A dedicated E region is reused every tile: wait until the previous tile's
      // accumulate products have read it. E over score columns needs no wait: the
      // products that overwrite those columns are issued after this tile's e_full.
      if (C::E_DEDICATED && n >= 1 && !mbar_wait(e_empty, (n - 1) & 1, g, 7)) { ok = false; break; }
      if constexpr (C::FUSEQ) {
        // dS^T (unscaled, 16-bit) for the pair's dS K product; the async proxy reads it
        if (!(n & 1) && n >= 4 && !ds_reuse(n)) { ok = false; break; }
        store_cols<BF16, CPW>(dsT(n), BK, r, c0, dp);
        fence_async_smem();
      }
      {
        // this thread's 16 words of E tile j (see e_col)
        auto e_put = [&](int j) -> uint32_t {
          if constexpr (C::E_DEDICATED) return tE + lane_off + (c0 >> 1) + j * C::E_COLS;
          const uint32_t off = 32 * half + (C::E1_OVER_DP ? j * C::C_DP : (j == 2 ? BM : 16 * j));
          if constexpr (C::E_OWN) return tmem + lane_off + sb * C::NSC * BM + off;
          return tE + lane_off + off;
        };
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = pack2<BF16>(sv[2 * j], sv[2 * j + 1]);
        tmem_st16_raw(e_put(0), w);
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = pack2<BF16>(dp[2 * j], dp[2 * j + 1]);
        tmem_st16_raw(e_put(1), w);
        if constexpr (C::BWD2) {
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = pack2<BF16>(gd[2 * j], gd[2 * j + 1]);
          tmem_st16_raw(e_put(2), w);
        }
        tmem_wait_st();
        tc_fence_before();
      }
      mbar_arrive(e_full + (n & 1));
    }
    if constexpr (C::FUSEQ) {
      // the pairs not drained in the loop (the last one or two); before acc_full, which
      // issuer 1 commits only after its last dS K product
      if (ok) {
        const int drained = n_tiles >= 3 ? (n_tiles - 2) >> 1 : 0;
        for (int pr = drained; pr < ((n_tiles + 1) >> 1); ++pr)
          if (!dq_drain(pr)) {
            ok = false;
            break;
          }
      }
      // the accumulator additions complete (and stop reading shared memory) before the CTA ends
      if (threadIdx.x == 0) bulk_wait_all();
    }
    if (ok && mbar_wait(acc_full, 0, g, 8)) {
      tc_fence_after();
      if (nsplit > 1) {
        // unscaled fp32 partials of this share (rows up to t_pad exist in the work space)
        const int64_t row = (static_cast<int64_t>(share) * p.B * p.H + bh) * p.t_pad + key;
        acc_cols_to_f32<D / 2>(tAcc0 + lane_off, half * (D / 2), p.part0 + row * D, n_tiles > 0);
        acc_cols_to_f32<D / 2>(tAcc1 + lane_off, half * (D / 2), p.part1 + row * D, n_tiles > 0);
      } else {
        const bool valid = key < T;
        uint16_t* r0 = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                       static_cast<int64_t>(key) * p.o0_st;
        uint16_t* r1 = p.out1 + static_cast<int64_t>(bidx) * p.o1_sb + static_cast<int64_t>(hidx) * p.o1_sh +
                       static_cast<int64_t>(key) * p.o1_st;
        acc_cols_to_global<D / 2, BF16>(tAcc0 + lane_off, half * (D / 2), r0, valid, scale);
        acc_cols_to_global<D / 2, BF16>(tAcc1 + lane_off, half * (D / 2), r1, valid, 1.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int D, bool BF16, bool CAUSAL, int KIND>
static cudaError_t launch_km_t(const KParams& p, cudaStream_t stream) {
  using C = KmCfg<D, KIND>;
  auto kern = attn_km_kernel<D, BF16, CAUSAL, KIND>;
  // The register split may only hand out what the launch allocated; a build
  // whose register count came out lower is refused rather than launched.
  static const int launch_regs = [&] {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, kern) == cudaSuccess ? a.numRegs : 0;
  }();
  if (C::SPLIT_REGS && launch_regs < C::REG_LAUNCH) return cudaErrorLaunchOutOfResources;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H * (p.nsplit > 1 ? p.nsplit : 1), (p.T + C::BK - 1) / C::BK);
  kern<<<grid, C::NTHREADS, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_km(const KParams& p, int d, bool bf16, bool causal, int kind, cudaStream_t stream) {
#define TTT_KM_KIND(D_, BF_, CA_)                                                  \
  if (d == D_ && bf16 == BF_ && causal == CA_) {                                   \
    if (kind == kBwdKV) return launch_km_t<D_, BF_, CA_, kBwdKV>(p, stream);       \
    if constexpr (D_ == 64) {                                                      \
      if (kind == kBwdKVQ) return launch_km_t<D_, BF_, CA_, kBwdKVQ>(p, stream);   \
    }                                                                              \
    if (kind == kBwd2KV) return launch_km_t<D_, BF_, CA_, kBwd2KV>(p, stream);     \
  }
#define TTT_KM_CA(D_, BF_) TTT_KM_KIND(D_, BF_, false) TTT_KM_KIND(D_, BF_, true)
  TTT_KM_CA(64, false) TTT_KM_CA(64, true) TTT_KM_CA(128, false) TTT_KM_CA(128, true)
#undef TTT_KM_CA
#undef TTT_KM_KIND
  return cudaErrorInvalidValue;
}

}  // namespace ttt
