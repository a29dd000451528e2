// Key-major backward passes (sm_100a). One CTA owns 128 key rows of one head
// and streams BM-query tiles (BM = 64, or 32 for the 128-wide double backward,
// whose four resident key-side tiles leave room for two 32-row stages only).
// Every score tile is computed transposed (keys x queries); the per-query
// statistics (lse2, delta, gamma, rho) arrive with each streamed tile via TMA.
//
//   kBwdKV  : dV = P^T dO,  dK = scale * dS^T Q
//             (replaces _attn_bwd_dv_from_p_kernel and _attn_bwd_dk_kernel,
//             ttt_kernels/backward_stubs.py:124-151 and 313-359, recomputing P
//             from lse2 instead of reading it)
//   kBwd2KV : dd_K = scale * (dS^T u_q + G_S^T Q),  dd_V = G_dP^T dO
//             (the key-side half of the complete double backward that the
//             reference approximates with torch.matmul in
//             backward_stubs.py:435-514)
//
// Roles and pipeline as in attn_bwd_qm.cu: warps 0..7 elementwise (warp w:
// TMEM lanes 32*(w%4)..+31, tile columns (w/4)*BM/2..+BM/2), warp 8 MMA issuer,
// warp 9 TMA producer. In the double backward the streamed Q and u_q tiles are
// stacked in one panel so that K [Q; u_q]^T produces [S^T | K u_q^T] as a
// single N = 2*BM product.
// Causal: query tiles that end before the CTA's first key are skipped.
#include "attn_pipe.cuh"
#include "kernels.h"

namespace ttt {

template <int D, int KIND>
struct KmCfg {
  static constexpr int BK = 128;  // keys per CTA (TMEM lanes)
  static constexpr bool BWD2 = (KIND == kBwd2KV);
  static constexpr int BM = (D == 128 && BWD2) ? 32 : 64;  // queries per streamed tile
  static constexpr int NR = BWD2 ? 4 : 2;     // resident: K, V, (u_k, u_v)
  static constexpr int NSTAT = BWD2 ? 4 : 2;  // streamed stats: lse2, delta, (gamma, rho)
  static constexpr int NSC = BWD2 ? 4 : 2;    // score tiles: S^T, (G_dS^T,) dP^T, ((dO u_v^T)^T)
  static constexpr int NE = BWD2 ? 3 : 2;     // P^T, dS^T | dS^T, G_S^T, G_dP^T
  static constexpr int NA = 2;
  static constexpr int NCW = 8;
  static constexpr int NCT = NCW * 32;
  static constexpr int NTHREADS = NCT + 64;
  static constexpr int CPW = BM / 2;
  static constexpr int TILE_R = BK * D * 2;
  // streamed: ST0 = [Q; u_q] (or Q), ST1 = dO, then the statistics rows
  static constexpr int ST0_ROWS = BWD2 ? 2 * BM : BM;
  static constexpr int ST0_BYTES = ST0_ROWS * D * 2;
  static constexpr int ST1_BYTES = BM * D * 2;
  static constexpr int STAT_BYTES = BM * 4;
  static constexpr int STAGE_TX = ST0_BYTES + ST1_BYTES + NSTAT * STAT_BYTES;  // bytes TMA delivers per stage
  static constexpr int STAGE = (STAGE_TX + 1023) / 1024 * 1024;               // stage pitch keeps tiles 1024-aligned
  static constexpr int TILE_E = BK * 64 * 2;                                    // one 64-column panel
  static constexpr int NBUF = (2 * NSC * BM + NA * D <= 512) ? 2 : 1;
  static constexpr int TMEM_USED = NBUF * NSC * BM + NA * D;
  static constexpr int TMEM_COLS = TMEM_USED <= 128 ? 128 : (TMEM_USED <= 256 ? 256 : 512);
  static_assert(TMEM_USED <= 512, "TMEM overflow");
  static constexpr int FIXED = NR * TILE_R + NE * TILE_E + 16 * 8 + 16 + 1024 + STAGE_TX;
  static constexpr int NSTAGE = (FIXED + 3 * STAGE <= 232448) ? 4 : (FIXED + 2 * STAGE <= 232448) ? 3 : 2;
  static constexpr int OFF_R = 0;
  static constexpr int OFF_E = OFF_R + NR * TILE_R;
  static constexpr int OFF_S = OFF_E + NE * TILE_E;  // stages last; the last one needs no padding
  static constexpr int OFF_BAR = OFF_S + (NSTAGE - 1) * STAGE + STAGE_TX;
  static constexpr int NBAR = 16;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "key-major tile set exceeds shared memory");
  static_assert(ST0_BYTES % 1024 == 0 && ST1_BYTES % 1024 == 0, "streamed tiles must stay 1024-aligned");
  static constexpr int C_S = 0, C_GDS = BWD2 ? BM : 0, C_DP = BWD2 ? 2 * BM : BM, C_UV = 3 * BM;
};

int km_tile_rows(int d, int kind) { return (d == 128 && kind == kBwd2KV) ? 32 : 64; }

template <int D, bool BF16, bool CAUSAL, int KIND>
__global__ void __launch_bounds__(KmCfg<D, KIND>::NTHREADS, 1) attn_km_kernel(const __grid_constant__ KParams p) {
  using C = KmCfg<D, KIND>;
  constexpr int BM = C::BM, BK = C::BK, NP = D / 64, NBUF = C::NBUF, NSTAGE = C::NSTAGE, CPW = C::CPW;
  constexpr int SR0 = C::ST0_ROWS;
  constexpr int WARP_MMA = C::NCW, WARP_LOAD = C::NCW + 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sR = smem + C::OFF_R;
  uint8_t* sS = smem + C::OFF_S;
  uint8_t* sE = smem + C::OFF_E;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* res_full = bars + 0;
  uint64_t* l_full = bars + 1;   // [4]
  uint64_t* l_empty = bars + 5;  // [4]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_free = bars + 11;  // [2] (NCT arrivals)
  uint64_t* e_full = bars + 13;  // NCT arrivals
  uint64_t* e_empty = bars + 14;
  uint64_t* acc_full = bars + 15;
  uint64_t* drain = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto tileR = [&](int t) { return sR + t * C::TILE_R; };
  auto st0 = [&](int s) { return sS + s * C::STAGE; };
  auto st1 = [&](int s) { return sS + s * C::STAGE + C::ST0_BYTES; };
  auto statS = [&](int s, int t) {
    return reinterpret_cast<float*>(sS + s * C::STAGE + C::ST0_BYTES + C::ST1_BYTES + t * C::STAT_BYTES);
  };
  auto tileE = [&](int t) { return sE + t * C::TILE_E; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int kblk = blockIdx.y;  // causal: small kblk has the most query tiles, launched first
  const int k0 = kblk * BK;
  const int T = p.T;
  const int n_q = (T + BM - 1) / BM;
  const int qt0 = CAUSAL ? (k0 / BM) : 0;
  const int n_tiles = n_q - qt0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 17; ++i) mbar_init(bars + i, 1);
    mbar_init(s_free + 0, C::NCT);
    mbar_init(s_free + 1, C::NCT);
    mbar_init(e_full, C::NCT);
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
  const uint32_t tAcc0 = tmem + NBUF * C::NSC * BM;  // dK / dd_K
  const uint32_t tAcc1 = tAcc0 + D;                  // dV / dd_V
  Guard g{abort_flag, p.err};

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
        mbar_arrive_tx(l_full + s, C::STAGE_TX);
        // str[0] = Q, str[1] = dO, str[2] = u_q (stacked under Q)
        for (int pp = 0; pp < NP; ++pp) {
          tma_load_4d(st0(s) + pp * SR0 * 128, &p.str[0], l_full + s, pp * 64, qrow, hidx, bidx);
          tma_load_4d(st1(s) + pp * BM * 128, &p.str[1], l_full + s, pp * 64, qrow, hidx, bidx);
          if constexpr (C::BWD2)
            tma_load_4d(st0(s) + pp * SR0 * 128 + BM * 128, &p.str[2], l_full + s, pp * 64, qrow, hidx, bidx);
        }
        for (int t = 0; t < C::NSTAT; ++t) tma_load_2d(statS(s, t), &p.st[t], l_full + s, qrow, bh);
        issued[s] = n + 1;
      }
      mbar_drain(res_full, 0);
      for (int s = 0; s < NSTAGE; ++s)
        if (issued[s] > 0) mbar_drain(l_full + s, ((issued[s] - 1) / NSTAGE) & 1);
    }
  } else if (warp == WARP_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_n1 = idesc_f16(128, BM, BF16, false, false);
      constexpr uint32_t id_n2 = idesc_f16(128, 2 * BM, BF16, false, false);
      constexpr uint32_t id_acc = idesc_f16(128, D, BF16, false, true);
      const uint32_t aK = smem_u32(tileR(0)), aV = smem_u32(tileR(1));
      const uint32_t aUK = C::BWD2 ? smem_u32(tileR(2)) : 0u, aUV = C::BWD2 ? smem_u32(tileR(3)) : 0u;
      auto issue_scores = [&](int n) -> bool {
        const int sb = n % NBUF, s = n % NSTAGE;
        if (!mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2)) return false;
        if (n >= NBUF && !mbar_wait(s_free + sb, ((n / NBUF) - 1) & 1, g, 3)) return false;
        tc_fence_after();
        const uint32_t base = tmem + sb * C::NSC * BM;
        const uint32_t b0 = smem_u32(st0(s)), b1 = smem_u32(st1(s));
        if constexpr (C::BWD2) {
          // [S^T | K u_q^T] = K [Q; u_q]^T ; G_dS^T/scale += u_k Q^T ; dP^T = V dO^T ; (dO u_v^T)^T = u_v dO^T
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_S, desc_kmajor(aK, BK, kk), desc_kmajor(b0, SR0, kk), id_n2, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_GDS, desc_kmajor(aUK, BK, kk), desc_kmajor(b0, SR0, kk), id_n1, 1u);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_DP, desc_kmajor(aV, BK, kk), desc_kmajor(b1, BM, kk), id_n1, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_UV, desc_kmajor(aUV, BK, kk), desc_kmajor(b1, BM, kk), id_n1, kk > 0);
        } else {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_S, desc_kmajor(aK, BK, kk), desc_kmajor(b0, SR0, kk), id_n1, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + C::C_DP, desc_kmajor(aV, BK, kk), desc_kmajor(b1, BM, kk), id_n1, kk > 0);
        }
        umma_commit(s_full + sb);
        return true;
      };
      auto issue_acc = [&](int n) -> bool {
        const int s = n % NSTAGE;
        if (!mbar_wait(e_full, n & 1, g, 4)) return false;
        tc_fence_after();
        const uint32_t bQ = smem_u32(st0(s)), bDO = smem_u32(st1(s));
        const uint32_t e0 = smem_u32(tileE(0)), e1 = smem_u32(tileE(1));
        if constexpr (!C::BWD2) {
          // dV += P^T dO ; dK += dS^T Q
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc1, desc_kmajor(e0, BK, kk), desc_mnmajor(bDO, BM, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e1, BK, kk), desc_mnmajor(bQ, SR0, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
        } else {
          // dd_K += dS^T u_q + G_S^T Q ; dd_V += G_dP^T dO
          const uint32_t bUQ = bQ + BM * 128, e2 = smem_u32(tileE(2));
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e0, BK, kk), desc_mnmajor(bUQ, SR0, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e1, BK, kk), desc_mnmajor(bQ, SR0, kk), id_acc, 1u);
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc1, desc_kmajor(e2, BK, kk), desc_mnmajor(bDO, BM, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(e_empty);
        umma_commit(l_empty + s);
        return true;
      };
      bool ok = mbar_wait(res_full, 0, g, 1);
      for (int n = 0; ok && n < n_tiles; ++n) {
        ok = issue_scores(n);
        if (ok && n >= 1) ok = issue_acc(n - 1);
      }
      if (ok) ok = issue_acc(n_tiles - 1);
      if (ok) umma_commit(acc_full);
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ elementwise warps 0..7
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const int key = k0 + r;
    const int c0 = half * CPW;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float c = p.scale_log2, scale = p.scale;
    const bool key_edge = k0 + BK > T;
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int sb = n % NBUF, s = n % NSTAGE;
      if (!mbar_wait(s_full + sb, (n / NBUF) & 1, g, 6)) { ok = false; break; }
      // The per-query statistics were delivered by TMA on l_full[s]; that
      // phase cannot advance until this tile's elementwise step is done.
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

      const int qt = qt0 + n;
      const int qcol0 = qt * BM + c0;
      const bool need_mask = key_edge || (CAUSAL && qt * BM < k0 + BK - 1);
      const float4* st_lse = reinterpret_cast<const float4*>(statS(s, 0) + c0);
      const float4* st_del = reinterpret_cast<const float4*>(statS(s, 1) + c0);
      const float4* st_gam = reinterpret_cast<const float4*>(statS(s, C::BWD2 ? 2 : 0) + c0);
      const float4* st_rho = reinterpret_cast<const float4*>(statS(s, C::BWD2 ? 3 : 0) + c0);
#pragma unroll
      for (int q4 = 0; q4 < CPW / 4; ++q4) {
        const float4 l4 = st_lse[q4];
        const float4 d4 = st_del[q4];
        float4 g4 = make_float4(0.f, 0.f, 0.f, 0.f), r4 = g4;
        if constexpr (C::BWD2) {
          g4 = st_gam[q4];
          r4 = st_rho[q4];
        }
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
        const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
        const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = q4 * 4 + u;
          float pr = fast_exp2(fmaf(sv[e], c, -lv[u]));
          if (need_mask) {
            const int qi = qcol0 + e;
            pr = ((key < T) && (!CAUSAL || key <= qi)) ? pr : 0.f;
          }
          if constexpr (!C::BWD2) {
            dp[e] = pr * (dp[e] - dv[u]);  // dS^T
            sv[e] = pr;                    // P^T
          } else {
            const float dpm = dp[e] - dv[u];
            const float gds = gd[e] * scale;
            const float gP = fmaf(gds, dpm, fmaf(-gv[u], dp[e], uv[e]));
            sv[e] = pr * dpm;             // dS^T
            dp[e] = pr * (gP - rv[u]);    // G_S^T
            gd[e] = pr * (gds - gv[u]);   // G_dP^T
          }
        }
      }
      if (n >= 1 && !mbar_wait(e_empty, (n - 1) & 1, g, 7)) { ok = false; break; }
      store_cols<BF16, CPW>(tileE(0), BK, r, c0, sv);
      store_cols<BF16, CPW>(tileE(1), BK, r, c0, dp);
      if constexpr (C::BWD2) store_cols<BF16, CPW>(tileE(2), BK, r, c0, gd);
      fence_async_smem();
      mbar_arrive(e_full);
    }
    if (ok && mbar_wait(acc_full, 0, g, 8)) {
      tc_fence_after();
      const bool valid = key < T;
      uint16_t* r0 = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                     static_cast<int64_t>(key) * p.o0_st;
      uint16_t* r1 = p.out1 + static_cast<int64_t>(bidx) * p.o1_sb + static_cast<int64_t>(hidx) * p.o1_sh +
                     static_cast<int64_t>(key) * p.o1_st;
      acc_cols_to_global<D / 2, BF16>(tAcc0 + lane_off, half * (D / 2), r0, valid, scale);
      acc_cols_to_global<D / 2, BF16>(tAcc1 + lane_off, half * (D / 2), r1, valid, 1.f);
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
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H, (p.T + C::BK - 1) / C::BK);
  kern<<<grid, C::NTHREADS, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_km(const KParams& p, int d, bool bf16, bool causal, int kind, cudaStream_t stream) {
#define TTT_KM_KIND(D_, BF_, CA_)                                                  \
  if (d == D_ && bf16 == BF_ && causal == CA_) {                                   \
    if (kind == kBwdKV) return launch_km_t<D_, BF_, CA_, kBwdKV>(p, stream);       \
    if (kind == kBwd2KV) return launch_km_t<D_, BF_, CA_, kBwd2KV>(p, stream);     \
  }
#define TTT_KM_CA(D_, BF_) TTT_KM_KIND(D_, BF_, false) TTT_KM_KIND(D_, BF_, true)
  TTT_KM_CA(64, false) TTT_KM_CA(64, true) TTT_KM_CA(128, false) TTT_KM_CA(128, true)
#undef TTT_KM_CA
#undef TTT_KM_KIND
  return cudaErrorInvalidValue;
}

}  // namespace ttt
