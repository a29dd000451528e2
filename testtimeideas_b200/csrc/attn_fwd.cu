// Forward attention kernel (sm_100a): O = softmax(scale * Q K^T) V, plus the
// base-2 row log-sum-exp that the backward passes recompute P from.
//
// Replaces the Triton forward kernels of the reference
// (ttt_kernels/triton_attention.py:86-256: _attn_fwd_kernel,
// _attn_fwd_kernel_stats, _attn_probs_kernel) and the PyTorch math forward of
// the save_p modes (triton_attention.py:51-59, 270-273).
//
// Two kernels: attn_fwd2_kernel (below, two query tiles per CTA, P kept in
// tensor memory) computes O and lse2; attn_fwd_kernel (this one) is used only
// when the normalized P is also materialized and T % 8 != 0 (for other T the
// row-LSE forward is followed by attn_pwrite_kernel, attn_pwrite.cu, which
// stores P by TMA).
//
// attn_fwd_kernel: one CTA owns 128 query rows of one head and streams 128-key tiles:
//   warp 5      TMA producer: Q once, then K/V tiles into a 2-stage ring.
//   warp 4      MMA issuer:   S_n = Q K_n^T into TMEM (double buffered), then
//                             O += P_n V_n into a TMEM accumulator.
//   warps 0..3  softmax:      thread r owns query row r (TMEM lane r): reads
//                             S_n, keeps the running max / sum, writes the
//                             16-bit P_n tile into shared memory, and rescales
//                             its O row in TMEM only when the running max grew
//                             by more than 2^8 (so P stays <= 256).
// Causal: key tiles past the diagonal are never loaded or multiplied; the
// diagonal tile is masked elementwise.
// save_p: after the main loop the CTA recomputes S for each visible tile and
// writes the normalized P (16-bit, row-major [T, T] per head) to HBM.
#include "attn_common.cuh"
#include "attn_pipe.cuh"
#include "kernels.h"

namespace ttt {

template <int D, bool SAVE_P>
struct FwdCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int TILE_Q = BM * D * 2;
  static constexpr int TILE_KV = BN * D * 2;
  static constexpr int TILE_P = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + TILE_Q;
  static constexpr int OFF_V = OFF_K + 2 * TILE_KV;
  static constexpr int OFF_P = OFF_V + 2 * TILE_KV;
  static constexpr int OFF_BAR = OFF_P + 2 * TILE_P;
  static constexpr int NBAR = 16;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "forward tile set exceeds shared memory");
};

template <int D, bool BF16, bool CAUSAL, bool SAVE_P>
__global__ void __launch_bounds__(192, 1) attn_fwd_kernel(const __grid_constant__ KParams p) {
  using C = FwdCfg<D, SAVE_P>;
  constexpr int BM = C::BM, BN = C::BN, NP = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sK0 = smem + C::OFF_K;
  uint8_t* sV0 = smem + C::OFF_V;
  uint8_t* sP0 = smem + C::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* p_full = bars + 7;    // [2]
  uint64_t* pv_done = bars + 9;   // [2]
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int qblk = CAUSAL ? (gridDim.y - 1 - blockIdx.y) : blockIdx.y;  // longest rows first
  const int q0 = qblk * BM;
  const int T = p.T;
  const int n_all = (T + BN - 1) / BN;
  const int n_tiles = CAUSAL ? min(n_all, (q0 + BM - 1) / BN + 1) : n_all;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(bars + i, 1);
    mbar_init(p_full + 0, 128);
    mbar_init(p_full + 1, 128);
    // A nonzero error word means an earlier CTA or launch gave up: exit at once.
    *abort_flag = (p.err != nullptr && *reinterpret_cast<volatile int*>(p.err) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (*abort_flag) return;
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;        // S buffers at columns 0 and 128
  const uint32_t tO = tmem + 256;  // O accumulator, D columns
  Guard g{abort_flag, p.err, p.err_host};

  if (warp == 5) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch(&p.own[0]);
      tma_prefetch(&p.str[0]);
      tma_prefetch(&p.str[1]);
      int issued[2] = {0, 0};
      mbar_arrive_tx(q_full, C::TILE_Q);
      for (int pp = 0; pp < NP; ++pp) tma_load_4d(sQ + pp * BM * 128, &p.own[0], q_full, pp * 64, q0, hidx, bidx);
      const int passes = SAVE_P ? 2 : 1;
      int n_glob = 0;
      for (int pass = 0; pass < passes; ++pass) {
        for (int n = 0; n < n_tiles; ++n, ++n_glob) {
          const int s = n_glob & 1;
          if (n_glob >= 2 && !mbar_wait(kv_empty + s, ((n_glob - 2) >> 1) & 1, g, 1)) goto prod_done;
          const bool need_v = (pass == 0);
          mbar_arrive_tx(kv_full + s, need_v ? 2 * C::TILE_KV : C::TILE_KV);
          for (int pp = 0; pp < NP; ++pp)
            tma_load_4d(sK0 + s * C::TILE_KV + pp * BN * 128, &p.str[0], kv_full + s, pp * 64, n * BN, hidx, bidx);
          if (need_v)
            for (int pp = 0; pp < NP; ++pp)
              tma_load_4d(sV0 + s * C::TILE_KV + pp * BN * 128, &p.str[1], kv_full + s, pp * 64, n * BN, hidx,
                          bidx);
          issued[s] = n_glob + 1;
        }
      }
    prod_done:
      // Wait for every load this thread issued before the CTA may exit.
      mbar_drain(q_full, 0);
      for (int s = 0; s < 2; ++s)
        if (issued[s] > 0) mbar_drain(kv_full + s, ((issued[s] - 1) >> 1) & 1);
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(128, BN, BF16, false, false);
      constexpr uint32_t id_o = idesc_f16(128, D, BF16, false, true);
      bool ok = mbar_wait(q_full, 0, g, 2);
      auto issue_s = [&](int n_glob, int buf) -> bool {
        const int s = n_glob & 1;
        if (!mbar_wait(kv_full + s, (n_glob >> 1) & 1, g, 3)) return false;
        tc_fence_after();
        const uint32_t aq = smem_u32(sQ), bk = smem_u32(sK0 + s * C::TILE_KV);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tS + buf * 128, desc_kmajor(aq, BM, kk), desc_kmajor(bk, BN, kk), id_s, kk > 0);
        umma_commit(s_full + buf);
        return true;
      };
      if (ok) ok = issue_s(0, 0);
      for (int n = 0; ok && n < n_tiles; ++n) {
        if (n + 1 < n_tiles && !issue_s(n + 1, (n + 1) & 1)) { ok = false; break; }
        const int b = n & 1;
        if (!mbar_wait(p_full + b, (n >> 1) & 1, g, 4)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ap = smem_u32(sP0 + b * C::TILE_P), bv = smem_u32(sV0 + b * C::TILE_KV);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_ss(tO, desc_kmajor(ap, BM, kk), desc_mnmajor(bv, BN, kk), id_o, (n > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pv_done + b);
        umma_commit(kv_empty + b);
      }
      if (SAVE_P && ok) {
        // Second pass: S tiles again (K only), buffers keep alternating.
        for (int n = 0; ok && n < n_tiles; ++n) {
          const int n_glob = n_tiles + n;
          const int buf = n_glob & 1;
          // buffer `buf` was last read by the softmax warps for tile n_glob-2
          if (n_glob >= 2 && !mbar_wait(p_full + buf, ((n_glob - 2) >> 1) & 1, g, 5)) { ok = false; break; }
          if (!issue_s(n_glob, buf)) { ok = false; break; }
          umma_commit(kv_empty + (n_glob & 1));
        }
      }
      // Drain: every tcgen05 op issued above must finish before TMEM is freed.
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..3
    const int r = threadIdx.x;  // query row within the block == TMEM lane
    const int row = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float c = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int b = n & 1;
      if (!mbar_wait(s_full + b, (n >> 1) & 1, g, 6)) { ok = false; break; }
      tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int q = 0; q < BN / 32; ++q)
        tmem_ld32(tS + lane_off + b * 128 + q * 32, *reinterpret_cast<float(*)[32]>(sv + q * 32));
      const int k0 = n * BN;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < BN; ++j) {
        const int col = k0 + j;
        const bool keep = (col < T) && (!CAUSAL || col <= row);
        const float x = keep ? sv[j] * c : -INFINITY;
        sv[j] = x;
        mx = fmaxf(mx, x);
      }
      if (n == 0) {
        m_used = mx;
      } else {
        const float m_new = fmaxf(m_used, mx);
        const bool need = m_new > m_used + 8.f;
        if (__any_sync(0xffffffffu, need)) {
          // O may only be touched once the previous P V product has landed.
          if (!mbar_wait(pv_done + ((n - 1) & 1), ((n - 1) >> 1) & 1, g, 7)) { ok = false; break; }
          tc_fence_after();
          const float alpha = need ? fast_exp2(m_used - m_new) : 1.f;
          if (need) {
            l *= alpha;
            m_used = m_new;
          }
#pragma unroll
          for (int q = 0; q < D / 16; ++q) {
            float o[16];
            tmem_ld16(tO + lane_off + q * 16, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= alpha;
            tmem_st16(tO + lane_off + q * 16, o);
          }
        }
      }
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < BN; ++j) {
        sv[j] = fast_exp2(sv[j] - m_used);
        rs += sv[j];
      }
      l += rs;
      // P buffer b was read by the P V product of tile n-2.
      if (n >= 2 && !mbar_wait(pv_done + b, ((n - 2) >> 1) & 1, g, 8)) { ok = false; break; }
      uint8_t* tileP = sP0 + b * C::TILE_P;
      store_row64<BF16>(tileP, BM, r, 0, sv);
      store_row64<BF16>(tileP, BM, r, 64, sv + 64);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full + b);
    }
    if (ok && mbar_wait(pv_done + ((n_tiles - 1) & 1), ((n_tiles - 1) >> 1) & 1, g, 9)) {
      tc_fence_after();
      const bool valid = row < T;
      const float inv_l = 1.f / l;
      uint16_t* orow = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                       static_cast<int64_t>(row) * p.o0_st;
      acc_to_global<D, BF16>(tO + lane_off, orow, valid, inv_l);
      const float lse2 = m_used + __log2f(l);
      p.out_f0[static_cast<int64_t>(bh) * p.t_pad + row] = valid ? lse2 : INFINITY;
      if (SAVE_P) {
        // Normalized P for every visible tile: P = 2^(S*c - lse2).
        uint16_t* prow = reinterpret_cast<uint16_t*>(p.out1) + static_cast<int64_t>(bh) * T * T +
                         static_cast<int64_t>(row) * T;
        for (int n = 0; n < n_tiles; ++n) {
          const int n_glob = n_tiles + n;
          const int b = n_glob & 1;
          if (!mbar_wait(s_full + b, (n_glob >> 1) & 1, g, 10)) break;
          tc_fence_after();
          const int k0 = n * BN;
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            float v[32];
            tmem_ld32(tS + lane_off + b * 128 + q * 32, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = k0 + q * 32 + j;
              const bool keep = (col < T) && (!CAUSAL || col <= row);
              v[j] = keep ? fast_exp2(v[j] * c - lse2) : 0.f;
            }
            if (valid) {
              const int cbase = k0 + q * 32;
              if (cbase + 32 <= T && (T & 7) == 0) {
                store_global32<BF16>(prow + cbase, v, 1.f);
              } else {
                for (int j = 0; j < 32; ++j)
                  if (cbase + j < T) {
                    const uint32_t w = pack2<BF16>(v[j], 0.f);
                    prow[cbase + j] = static_cast<uint16_t>(w & 0xffffu);
                  }
              }
            }
          }
          tc_fence_before();
          mbar_arrive(p_full + b);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- two-tile forward
// The kernel used when P is not materialized. One CTA owns 256 query rows of
// one head as two 128-row query tiles, each with its own softmax warpgroup, and
// streams 128-key tiles through a TMA ring:
//   warp 9      TMA producer: Q0, Q1 once, then K_n and V_n (separate barriers,
//                             so S can start before V lands).
//   warp 8      MMA issuer:   S0_0, S1_0, then per key tile n:
//                             O0 += P0_n V_n, S0_{n+1}, O1 += P1_n V_n, S1_{n+1}.
//                             While one warpgroup exponentiates tile n the
//                             tensor core works on the other query tile.
//   warps 10,11 idle (they complete the control warpgroup for the register split).
//   warps 0..3  softmax of Q0, warps 4..7 softmax of Q1 (thread = query row =
//                             TMEM lane): reads S_n, keeps the running max and
//                             sum, writes 16-bit P_n back over the first 64
//                             columns of S_n (packed pairs), and rescales its O
//                             row only when the running max grew by more than
//                             2^8.
// P_n is the A operand of its P V product straight from tensor memory; the
// next S product of the same query tile overwrites those columns, which is
// safe because one thread issues both and tcgen05.mma executes in issue order.
// By the time S_{n+1} is complete, O += P_n V_n has completed as well, so a
// warpgroup that has seen S_{n+1} may rescale O without a further wait.
// TMEM: S0 at columns 0..127, S1 at 128..255, O0 at 256, O1 at 256 + D.
template <int D>
struct Fwd2Cfg {
  static constexpr int BM = 128, BN = 128, NQ = 2;
  static constexpr int TILE_Q = BM * D * 2;
  static constexpr int TILE_KV = BN * D * 2;
  static constexpr int NSTAGE = D == 64 ? 4 : 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NQ * TILE_Q;
  static constexpr int OFF_V = OFF_K + NSTAGE * TILE_KV;
  static constexpr int OFF_BAR = OFF_V + NSTAGE * TILE_KV;
  // barrier slots: q_full, k_full[NSTAGE], v_full[NSTAGE], kv_empty[NSTAGE],
  // s_full[2], p_full[2], pv_done[2], drain
  static constexpr int B_Q = 0, B_K = 1, B_V = 1 + NSTAGE, B_E = 1 + 2 * NSTAGE, B_S = 1 + 3 * NSTAGE;
  static constexpr int B_P = B_S + 2, B_O = B_P + 2, B_DR = B_O + 2, NBAR = B_DR + 1;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  // Three warpgroups: two softmax warpgroups and a control warpgroup (MMA
  // issuer, TMA producer, two idle warps). The launch gives every thread
  // REG_LAUNCH registers (three warps share one 16K-register sub-partition);
  // the control warpgroup then drops to REG_CTRL and the softmax warpgroups,
  // which hold a full 128-column score row each, rise to REG_SOFTMAX.
  static constexpr int NTHREADS = 384;
  static constexpr int REG_LAUNCH = 168;
  static constexpr int REG_CTRL = D == 64 ? 56 : 72;  // the d=128 MMA loop needs more than 56
  static constexpr int REG_SOFTMAX = (3 * REG_LAUNCH - REG_CTRL) / 2;
  static_assert(2 * REG_SOFTMAX + REG_CTRL <= 3 * REG_LAUNCH, "register split exceeds the launch allocation");
  static_assert(SMEM <= 232448, "two-tile forward exceeds shared memory");
};

template <int D, bool BF16, bool CAUSAL>
__global__ void __launch_bounds__(384, 1) attn_fwd2_kernel(const __grid_constant__ KParams p) {
  using C = Fwd2Cfg<D>;
  constexpr int BM = C::BM, BN = C::BN, NP = D / 64, NS = C::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + C::B_Q;
  uint64_t* k_full = bars + C::B_K;
  uint64_t* v_full = bars + C::B_V;
  uint64_t* kv_empty = bars + C::B_E;
  uint64_t* s_full = bars + C::B_S;
  uint64_t* p_full = bars + C::B_P;
  uint64_t* pv_done = bars + C::B_O;
  uint64_t* drain = bars + C::B_DR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // split mode: this CTA takes share `share` of its key-tile stream
  const int nsplit = p.nsplit > 1 ? p.nsplit : 1;
  const GridPos gp = grid_pos();
  const int bh = gp.unit / nsplit, share = gp.unit % nsplit;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int blk = CAUSAL ? (gridDim.y - 1 - gp.rank) : gp.rank;  // longest rows first
  const int q0 = blk * 2 * BM;
  const int T = p.T;
  const int n_all = (T + BN - 1) / BN;
  // Key tiles [lo_w, hi_w) visited by query tile w (none when the tile starts
  // past the sequence). Causal: tiles before the band of the tile's first row
  // and past its diagonal are skipped.
  const Band band = Band::make(p, CAUSAL);
  const int qs0 = q0, qs1 = q0 + BM;
  const int hi0_all = qs0 >= T ? 0 : (CAUSAL ? min(n_all, qs0 / BN + 1) : n_all);
  const int hi1_all = qs1 >= T ? 0 : (CAUSAL ? min(n_all, qs1 / BN + 1) : n_all);
  const int lo0_all = CAUSAL ? band.lo(qs0) / BN : 0;
  const int lo1_all = CAUSAL ? band.lo(min(qs1, T - 1)) / BN : 0;
  // the whole block streams key tiles [s_lo, s_hi); split mode gives this CTA
  // a contiguous share of them (the two ranges overlap there: the split runs
  // only without a band), and each query tile keeps its part of the share
  const int s_lo = lo0_all;
  const int s_hi = max(hi0_all, hi1_all > lo1_all ? hi1_all : 0);
  const int a0 = s_lo + split_begin(s_hi - s_lo, share, nsplit), a1 = s_lo + split_begin(s_hi - s_lo, share + 1, nsplit);
  const int lo0 = max(lo0_all, a0), hi0 = min(hi0_all, a1);
  const int lo1 = max(lo1_all, a0), hi1 = min(hi1_all, a1);
  const int nt0 = max(0, hi0 - lo0), nt1 = max(0, hi1 - lo1);
  // the CTA streams key tiles n_lo .. n_lo + n_kv - 1 (relative index r = n - n_lo)
  const int n_lo = nsplit > 1 ? a0 : lo0;
  const int n_kv = nsplit > 1 ? a1 - a0 : max(hi0, nt1 > 0 ? hi1 : 0) - n_lo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NBAR; ++i) mbar_init(bars + i, 1);
    mbar_init(p_full + 0, 128);
    mbar_init(p_full + 1, 128);
    *abort_flag = (p.err != nullptr && *reinterpret_cast<volatile int*>(p.err) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (*abort_flag) return;
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  Guard g{abort_flag, p.err, p.err_host};

  if (warp >= 8) {
   regs_release<C::REG_CTRL>();
   if (warp == 9) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch(&p.own[0]);
      tma_prefetch(&p.str[0]);
      tma_prefetch(&p.str[1]);
      mbar_arrive_tx(q_full, (nt1 > 0 ? 2 : 1) * C::TILE_Q);
      for (int pp = 0; pp < NP; ++pp) tma_load_4d(sQ + pp * BM * 128, &p.own[0], q_full, pp * 64, qs0, hidx, bidx);
      if (nt1 > 0)
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(sQ + C::TILE_Q + pp * BM * 128, &p.own[0], q_full, pp * 64, qs1, hidx, bidx);
      int n = 0;
      for (; n < n_kv; ++n) {
        const int s = n % NS;
        const int key0 = (n_lo + n) * BN;
        if (n >= NS && !mbar_wait(kv_empty + s, ((n / NS) - 1) & 1, g, 1)) break;
        mbar_arrive_tx(k_full + s, C::TILE_KV);
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(sK + s * C::TILE_KV + pp * BN * 128, &p.str[0], k_full + s, pp * 64, key0, hidx, bidx);
        mbar_arrive_tx(v_full + s, C::TILE_KV);
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(sV + s * C::TILE_KV + pp * BN * 128, &p.str[1], v_full + s, pp * 64, key0, hidx, bidx);
      }
      // Wait for every load this thread issued before the CTA may exit.
      mbar_drain(q_full, 0);
      for (int j = max(0, n - NS); j < n; ++j) {
        mbar_drain(k_full + j % NS, (j / NS) & 1);
        mbar_drain(v_full + j % NS, (j / NS) & 1);
      }
    }
   } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(128, BN, BF16, false, false);
      constexpr uint32_t id_o = idesc_f16(128, D, BF16, false, true);
      // query tile w takes part in relative steps [first[w], first[w] + nt[w])
      const int first[2] = {lo0 - n_lo, lo1 - n_lo}, nt[2] = {nt0, nt1};
      int k_seen = 0;  // key tiles whose K load this thread has waited for
      bool ok = mbar_wait(q_full, 0, g, 2);
      auto wait_k = [&](int n) -> bool {
        if (n < k_seen) return true;
        if (!mbar_wait(k_full + n % NS, (n / NS) & 1, g, 3)) return false;
        k_seen = n + 1;
        tc_fence_after();
        return true;
      };
      auto issue_s = [&](int w, int n) {
        const uint32_t aq = smem_u32(sQ + w * C::TILE_Q), bk = smem_u32(sK + (n % NS) * C::TILE_KV);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + w * 128, desc_kmajor(aq, BM, kk), desc_kmajor(bk, BN, kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit(s_full + w);
      };
      if (ok && n_kv > 0 && (ok = wait_k(0))) {
        for (int w = 0; w < 2; ++w)
          if (first[w] == 0 && nt[w] > 0) issue_s(w, 0);
      }
      for (int n = 0; ok && n < n_kv; ++n) {
        const int s = n % NS;
        if (!(ok = mbar_wait(v_full + s, (n / NS) & 1, g, 4))) break;
        const uint32_t bv = smem_u32(sV + s * C::TILE_KV);
        for (int w = 0; w < 2 && ok; ++w) {
          const int i = n - first[w];  // this query tile's own step index
          if (i >= 0 && i < nt[w]) {
            if (!(ok = mbar_wait(p_full + w, i & 1, g, 5))) break;
            tc_fence_after();
            const uint32_t tP = tmem + w * 128, tO = tmem + 256 + w * D;
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              umma_ts(tO, tP + kk * 8, desc_mnmajor(bv, BN, kk), id_o, (i > 0 || kk > 0) ? 1u : 0u);
            umma_commit(pv_done + w);
          }
          if (i + 1 >= 0 && i + 1 < nt[w]) {
            if (!(ok = wait_k(n + 1))) break;
            issue_s(w, n + 1);
          }
        }
        if (!ok) break;
        umma_commit(kv_empty + s);
      }
      // Drain: every tcgen05 op issued above must finish before TMEM is freed.
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
   }
  } else {
    // ------------------------------------------------------------ softmax warps 0..7
    regs_claim<C::REG_SOFTMAX>();
    const int w = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int row = q0 + w * BM + r;
    const int ntw = w ? nt1 : nt0;
    const int low = w ? lo1 : lo0;  // first key tile of this query tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + w * 128;
    const uint32_t tO = tmem + lane_off + 256 + w * D;
    const float c = p.scale_log2;
    const int qw0 = q0 + w * BM;
    const int row_lo = band.lo(row);
    // key tiles from this one on are fully visible to the whole query tile (below the diagonal)
    const int band_edge = CAUSAL ? band.lo(qw0 + BM - 1) : 0;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int n = 0; n < ntw; ++n) {
      if (!mbar_wait(s_full + w, n & 1, g, 6)) { ok = false; break; }
      tc_fence_after();
      float sv[BN];
      tmem_ld_nw<64>(tS, *reinterpret_cast<float(*)[64]>(sv));
      tmem_ld_nw<64>(tS + 64, *reinterpret_cast<float(*)[64]>(sv + 64));
      tmem_wait_ld();
      reg_fence(sv);
      const int k0 = (low + n) * BN;
      if ((k0 + BN > T) || (CAUSAL && (k0 + BN - 1 > qw0 || band_edge > k0))) {
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int col = k0 + j;
          sv[j] = ((col < T) && (!CAUSAL || (col <= row && col >= row_lo))) ? sv[j] : -INFINITY;
        }
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int j = 8; j < BN; ++j) mx8[j & 7] = fmaxf(mx8[j & 7], sv[j]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_new = fmaxf(m_used, mx * c);
      if (n == 0) {
        m_used = m_new;
      } else {
        const bool need = m_new > m_used + 8.f;
        if (__any_sync(0xffffffffu, need)) {
          // O += P_{n-1} V_{n-1} completed before S_n did (issue order), so O is settled.
          const float alpha = need ? fast_exp2(m_used - m_new) : 1.f;
          if (need) {
            l *= alpha;
            m_used = m_new;
          }
#pragma unroll
          for (int q = 0; q < D / 16; ++q) {
            float o[16];
            tmem_ld16(tO + q * 16, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= alpha;
            tmem_st16(tO + q * 16, o);
          }
        }
      }
      // A row whose window has not started yet has no visible key so far (m_used = -inf):
      // its P is 0, and the exponent offset must stay finite.
      const F2 C2 = f2s(c), NM = f2s(m_used == -INFINITY ? 0.f : -m_used);
      F2 acc[4] = {f2s(0.f), f2s(0.f), f2s(0.f), f2s(0.f)};
#pragma unroll
      for (int q = 0; q < BN / 32; ++q) {
        uint32_t pw[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int e = q * 32 + 2 * j;
          float x0, x1;
          split(fma2(f2(sv[e], sv[e + 1]), C2, NM), x0, x1);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          acc[j & 3] = add2(acc[j & 3], f2(p0, p1));
          pw[j] = pack2<BF16>(p0, p1);
        }
        tmem_st16_raw(tS + q * 16, pw);
      }
      float a0, a1;
      split(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])), a0, a1);
      l += a0 + a1;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full + w);
    }
    if (nsplit > 1) {
      // unnormalized O row, running max (log2 domain) and sum of this share; a
      // share without tiles for this query tile leaves (0, -inf, 0)
      if (ok && (ntw == 0 || mbar_wait(pv_done + w, (ntw - 1) & 1, g, 9)) && row < p.t_pad) {
        tc_fence_after();
        const int64_t prow = (static_cast<int64_t>(share) * p.B * p.H + bh) * p.t_pad + row;
        acc_cols_to_f32<D>(tO, 0, p.part0 + prow * D, ntw > 0);
        reinterpret_cast<float2*>(p.part1)[prow] = ntw > 0 ? make_float2(m_used, l) : make_float2(-INFINITY, 0.f);
      }
    } else if (ok && ntw > 0) {
      if (mbar_wait(pv_done + w, (ntw - 1) & 1, g, 9)) {
        tc_fence_after();
        const bool valid = row < T;
        uint16_t* orow = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                         static_cast<int64_t>(row) * p.o0_st;
        acc_to_global<D, BF16>(tO, orow, valid, 1.f / l);
        if (row < p.t_pad) p.out_f0[static_cast<int64_t>(bh) * p.t_pad + row] = valid ? m_used + __log2f(l) : INFINITY;
      }
    } else if (ok && row < p.t_pad) {
      p.out_f0[static_cast<int64_t>(bh) * p.t_pad + row] = INFINITY;  // pad rows of a tile past the sequence
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <int D, bool BF16, bool CAUSAL>
static cudaError_t launch_fwd2_t(const KParams& p, cudaStream_t stream) {
  using C = Fwd2Cfg<D>;
  auto kern = attn_fwd2_kernel<D, BF16, CAUSAL>;
  // The register split may only hand out what the launch allocated; a build
  // whose register count came out lower is refused rather than launched.
  static const int launch_regs = [&] {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, kern) == cudaSuccess ? a.numRegs : 0;
  }();
  if (launch_regs < C::REG_LAUNCH) return cudaErrorLaunchOutOfResources;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H * (p.nsplit > 1 ? p.nsplit : 1), (p.T + 2 * C::BM - 1) / (2 * C::BM));
  kern<<<grid, C::NTHREADS, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

template <int D, bool BF16, bool CAUSAL, bool SAVE_P>
static cudaError_t launch_fwd_t(const KParams& p, cudaStream_t stream) {
  if constexpr (!SAVE_P) return launch_fwd2_t<D, BF16, CAUSAL>(p, stream);
  using C = FwdCfg<D, SAVE_P>;
  auto kern = attn_fwd_kernel<D, BF16, CAUSAL, SAVE_P>;
  static bool configured = false;  // per-instantiation; attribute is per-device but idempotent
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  configured = true;
  (void)configured;
  dim3 grid(p.B * p.H, (p.T + C::BM - 1) / C::BM);
  kern<<<grid, 192, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_fwd(const KParams& p, int d, bool bf16, bool causal, bool save_p, cudaStream_t stream) {
#define TTT_FWD_CASE(D_, BF_, CA_, SP_) \
  if (d == D_ && bf16 == BF_ && causal == CA_ && save_p == SP_) return launch_fwd_t<D_, BF_, CA_, SP_>(p, stream);
#define TTT_FWD_SP(D_, BF_, CA_) TTT_FWD_CASE(D_, BF_, CA_, false) TTT_FWD_CASE(D_, BF_, CA_, true)
#define TTT_FWD_CA(D_, BF_) TTT_FWD_SP(D_, BF_, false) TTT_FWD_SP(D_, BF_, true)
  TTT_FWD_CA(64, false) TTT_FWD_CA(64, true) TTT_FWD_CA(128, false) TTT_FWD_CA(128, true)
#undef TTT_FWD_CA
#undef TTT_FWD_SP
#undef TTT_FWD_CASE
  return cudaErrorInvalidValue;
}

}  // namespace ttt
