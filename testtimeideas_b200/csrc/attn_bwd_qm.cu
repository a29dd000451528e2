// Query-major backward passes (sm_100a). One CTA owns 128 query rows of one
// head and streams 64-key tiles; thread r of the four compute warps owns
// query row r (TMEM lane r).
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
//            (together with the key-major kBwd2KV pass this replaces the
//            PyTorch matmul double backward of TritonDvFn / TritonRowSumFn /
//            TritonDqDkFn, backward_stubs.py:435-514, with the complete
//            second-order terms)
//
// Roles: warp 5 = TMA producer, warp 4 = MMA issuer (one thread), warps 0..3 =
// elementwise. Score tiles (S, dP, G_dS, dO u_v^T) land in TMEM; the
// elementwise results that feed the second GEMM (dS, G_S, G_dP, P) go to
// shared memory in the 128-byte-swizzled K-major layout; accumulators stay in
// TMEM until the epilogue. Causal: key tiles past the diagonal are skipped.
#include "attn_common.cuh"
#include "kernels.h"

namespace ttt {

template <int D, int KIND, bool GDO>
struct QmCfg {
  static constexpr int BM = 128, BN = 64;
  static constexpr bool BWD2 = (KIND != kBwdQ);
  static constexpr int NR = BWD2 ? 3 : 2;    // resident: Q, dO, (u_q)
  static constexpr int NSTR = BWD2 ? 4 : 2;  // streamed: K, V, (u_k, u_v)
  static constexpr int NSC = BWD2 ? 4 : 2;   // score tiles: S, dP, (G_dS, dO u_v^T)
  static constexpr int NE = KIND == kBwdQ ? 1 : (KIND == kStats ? 0 : (GDO ? 4 : 2));
  static constexpr int NA = KIND == kBwdQ ? 1 : (KIND == kStats ? 0 : (GDO ? 2 : 1));
  static constexpr int TILE_R = BM * D * 2;
  static constexpr int TILE_S = BN * D * 2;
  static constexpr int TILE_E = BM * BN * 2;
  static constexpr int NBUF = (2 * NSC * BN + NA * D <= 512) ? 2 : 1;
  static constexpr int TMEM_USED = NBUF * NSC * BN + NA * D;
  static constexpr int TMEM_COLS = TMEM_USED <= 128 ? 128 : (TMEM_USED <= 256 ? 256 : 512);
  static_assert(TMEM_USED <= 512, "TMEM overflow");
  static constexpr int FIXED = NR * TILE_R + NBUF * NE * TILE_E;
  static constexpr int NSTAGE = (FIXED + 2 * NSTR * TILE_S + 2048 <= 232448) ? 2 : 1;
  static constexpr int OFF_R = 0;
  static constexpr int OFF_S = OFF_R + NR * TILE_R;
  static constexpr int OFF_E = OFF_S + NSTAGE * NSTR * TILE_S;
  static constexpr int OFF_BAR = OFF_E + NBUF * NE * TILE_E;
  static constexpr int NBAR = 16;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "query-major tile set exceeds shared memory");
};

template <int D, bool BF16, bool CAUSAL, int KIND, bool GDO>
__global__ void __launch_bounds__(192, 1) attn_qm_kernel(const __grid_constant__ KParams p) {
  using C = QmCfg<D, KIND, GDO>;
  constexpr int BM = C::BM, BN = C::BN, NP = D / 64, NBUF = C::NBUF, NSTAGE = C::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sR = smem + C::OFF_R;
  uint8_t* sS = smem + C::OFF_S;
  uint8_t* sE = smem + C::OFF_E;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* res_full = bars + 0;
  uint64_t* l_full = bars + 1;   // [2]
  uint64_t* l_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;   // [2]
  uint64_t* e_full = bars + 7;   // [2] (128 arrivals)
  uint64_t* e_empty = bars + 9;  // [2]
  uint64_t* acc_full = bars + 11;
  uint64_t* drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto tileR = [&](int t) { return sR + t * C::TILE_R; };
  auto tileS = [&](int s, int t) { return sS + (s * C::NSTR + t) * C::TILE_S; };
  auto tileE = [&](int b, int t) { return sE + (b * C::NE + t) * C::TILE_E; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int qblk = CAUSAL ? (gridDim.y - 1 - blockIdx.y) : blockIdx.y;
  const int q0 = qblk * BM;
  const int T = p.T;
  const int n_all = (T + BN - 1) / BN;
  const int n_tiles = CAUSAL ? min(n_all, (q0 + BM - 1) / BN + 1) : n_all;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 13; ++i) mbar_init(bars + i, 1);
    mbar_init(e_full + 0, 128);
    mbar_init(e_full + 1, 128);
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
  Guard g{abort_flag, p.err};

  if (warp == 5) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = 0; t < C::NR; ++t) tma_prefetch(&p.own[t]);
      for (int t = 0; t < C::NSTR; ++t) tma_prefetch(&p.str[t]);
      int issued[2] = {0, 0};
      mbar_arrive_tx(res_full, C::NR * C::TILE_R);
      for (int t = 0; t < C::NR; ++t)
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(tileR(t) + pp * BM * 128, &p.own[t], res_full, pp * 64, q0, hidx, bidx);
      for (int n = 0; n < n_tiles; ++n) {
        const int s = n % NSTAGE;
        if (n >= NSTAGE && !mbar_wait(l_empty + s, ((n / NSTAGE) - 1) & 1, g, 1)) break;
        mbar_arrive_tx(l_full + s, C::NSTR * C::TILE_S);
        for (int t = 0; t < C::NSTR; ++t)
          for (int pp = 0; pp < NP; ++pp)
            tma_load_4d(tileS(s, t) + pp * BN * 128, &p.str[t], l_full + s, pp * 64, n * BN, hidx, bidx);
        issued[s] = n + 1;
      }
      mbar_drain(res_full, 0);
      for (int s = 0; s < NSTAGE; ++s)
        if (issued[s] > 0) mbar_drain(l_full + s, ((issued[s] - 1) / NSTAGE) & 1);
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_sc = idesc_f16(128, BN, BF16, false, false);
      constexpr uint32_t id_acc = idesc_f16(128, D, BF16, false, true);
      const uint32_t aQ = smem_u32(tileR(0)), aDO = smem_u32(tileR(1));
      const uint32_t aUQ = C::BWD2 ? smem_u32(tileR(2)) : 0u;
      auto issue_scores = [&](int n) -> bool {
        const int sb = n % NBUF, s = n % NSTAGE;
        if (!mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2)) return false;
        tc_fence_after();
        const uint32_t base = tmem + sb * C::NSC * BN;
        const uint32_t bK = smem_u32(tileS(s, 0)), bV = smem_u32(tileS(s, 1));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(base, desc_kmajor(aQ, BM, kk), desc_kmajor(bK, BN, kk), id_sc, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(base + BN, desc_kmajor(aDO, BM, kk), desc_kmajor(bV, BN, kk), id_sc, kk > 0);
        if constexpr (C::BWD2) {
          const uint32_t bUK = smem_u32(tileS(s, 2)), bUV = smem_u32(tileS(s, 3));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + 2 * BN, desc_kmajor(aUQ, BM, kk), desc_kmajor(bK, BN, kk), id_sc, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + 2 * BN, desc_kmajor(aQ, BM, kk), desc_kmajor(bUK, BN, kk), id_sc, 1u);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + 3 * BN, desc_kmajor(aDO, BM, kk), desc_kmajor(bUV, BN, kk), id_sc, kk > 0);
        }
        umma_commit(s_full + sb);
        if constexpr (C::NA == 0) umma_commit(l_empty + s);
        return true;
      };
      auto issue_acc = [&](int n) -> bool {
        const int sb = n % NBUF, s = n % NSTAGE;
        if (!mbar_wait(e_full + sb, (n / NBUF) & 1, g, 3)) return false;
        tc_fence_after();
        const uint32_t bK = smem_u32(tileS(s, 0)), bV = smem_u32(tileS(s, 1));
        const uint32_t e0 = smem_u32(tileE(sb, 0));
        if constexpr (KIND == kBwdQ) {
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e0, BM, kk), desc_mnmajor(bK, BN, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
        } else {
          const uint32_t bUK = smem_u32(tileS(s, 2)), bUV = smem_u32(tileS(s, 3));
          const uint32_t e1 = smem_u32(tileE(sb, 1));
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e0, BM, kk), desc_mnmajor(bUK, BN, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e1, BM, kk), desc_mnmajor(bK, BN, kk), id_acc, 1u);
          if constexpr (GDO) {
            const uint32_t e2 = smem_u32(tileE(sb, 2)), e3 = smem_u32(tileE(sb, 3));
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              umma_ss(tAcc1, desc_kmajor(e2, BM, kk), desc_mnmajor(bV, BN, kk), id_acc,
                      (n > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              umma_ss(tAcc1, desc_kmajor(e3, BM, kk), desc_mnmajor(bUV, BN, kk), id_acc, 1u);
          }
        }
        umma_commit(e_empty + sb);
        umma_commit(l_empty + s);
        return true;
      };
      constexpr int LA = NBUF - 1;
      bool ok = mbar_wait(res_full, 0, g, 4);
      for (int n = 0; ok && n < LA && n < n_tiles; ++n) ok = issue_scores(n);
      for (int n = 0; ok && n < n_tiles; ++n) {
        const int m = n + LA;
        if (m < n_tiles) {
          if constexpr (C::NA == 0) {
            if (m >= NBUF && !mbar_wait(e_full + (m % NBUF), ((m / NBUF) - 1) & 1, g, 5)) { ok = false; break; }
          }
          if (!issue_scores(m)) { ok = false; break; }
        }
        if constexpr (C::NA > 0) {
          if (!issue_acc(n)) { ok = false; break; }
        }
      }
      if constexpr (C::NA > 0) {
        if (ok) umma_commit(acc_full);
      }
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ elementwise warps 0..3
    const int r = threadIdx.x;
    const int row = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const int64_t sidx = static_cast<int64_t>(bh) * p.t_pad + row;
    const float c = p.scale_log2, scale = p.scale;
    const float lse = p.lse2[sidx];
    const float del = p.delta[sidx];
    float gam = 0.f, rho = 0.f;
    if constexpr (KIND == kBwd2Q) {
      gam = p.gamma[sidx];
      rho = p.rho[sidx];
    }
    float a_g = 0.f, a2 = 0.f, a3 = 0.f, a4 = 0.f;
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int sb = n % NBUF;
      if (!mbar_wait(s_full + sb, (n / NBUF) & 1, g, 6)) { ok = false; break; }
      tc_fence_after();
      if constexpr (C::NE > 0) {
        if (n >= NBUF && !mbar_wait(e_empty + sb, ((n / NBUF) - 1) & 1, g, 7)) { ok = false; break; }
      }
      const uint32_t base = tmem + lane_off + sb * C::NSC * BN;
#pragma unroll
      for (int half = 0; half < BN / 32; ++half) {
        const int cc = half * 32;
        float sv[32], dp[32], gd[32], uv[32];
        tmem_ld32(base + cc, sv);
        tmem_ld32(base + BN + cc, dp);
        if constexpr (C::BWD2) {
          tmem_ld32(base + 2 * BN + cc, gd);
          tmem_ld32(base + 3 * BN + cc, uv);
        }
        const int j0 = n * BN + cc;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = j0 + e;
          const bool valid = (j < T) && (!CAUSAL || j <= row);
          const float pr = valid ? fast_exp2(sv[e] * c - lse) : 0.f;
          if constexpr (KIND == kBwdQ) {
            sv[e] = pr * (dp[e] - del);
          } else if constexpr (KIND == kStats) {
            const float t = pr * (gd[e] * scale);
            a_g += t;
            a2 += t * dp[e];
            a4 += pr * dp[e];
            a3 += pr * uv[e];
          } else {
            const float dpm = dp[e] - del;
            const float gds = gd[e] * scale;
            const float gP = gds * dpm - gam * dp[e] + uv[e];
            sv[e] = pr * dpm;          // dS
            dp[e] = pr * (gP - rho);   // G_S
            gd[e] = pr * (gds - gam);  // G_dP
            uv[e] = pr;                // P
          }
        }
        if constexpr (KIND == kBwdQ) {
          store_row32<BF16>(tileE(sb, 0), BM, r, cc, sv);
        } else if constexpr (KIND == kBwd2Q) {
          store_row32<BF16>(tileE(sb, 0), BM, r, cc, sv);
          store_row32<BF16>(tileE(sb, 1), BM, r, cc, dp);
          if constexpr (GDO) {
            store_row32<BF16>(tileE(sb, 2), BM, r, cc, gd);
            store_row32<BF16>(tileE(sb, 3), BM, r, cc, uv);
          }
        }
      }
      if constexpr (C::NE > 0) fence_async_smem();
      tc_fence_before();
      mbar_arrive(e_full + sb);
    }
    const bool valid = row < T;
    if constexpr (KIND == kStats) {
      if (ok) {
        const float rho_v = a2 - del * a_g - a_g * a4 + a3;
        p.out_f0[sidx] = valid ? a_g : 0.f;
        p.out_f1[sidx] = valid ? rho_v : 0.f;
      }
    } else {
      if (ok && mbar_wait(acc_full, 0, g, 8)) {
        tc_fence_after();
        uint16_t* r0 = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                       static_cast<int64_t>(row) * p.o0_st;
        acc_to_global<D, BF16>(tAcc0 + lane_off, r0, valid, scale);
        if constexpr (KIND == kBwd2Q && GDO) {
          uint16_t* r1 = p.out1 + static_cast<int64_t>(bidx) * p.o1_sb + static_cast<int64_t>(hidx) * p.o1_sh +
                         static_cast<int64_t>(row) * p.o1_st;
          acc_to_global<D, BF16>(tAcc1 + lane_off, r1, valid, 1.f);
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
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H, (p.T + C::BM - 1) / C::BM);
  kern<<<grid, 192, C::SMEM, stream>>>(p);
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
