// Key-major backward passes (sm_100a). One CTA owns 128 key rows of one head
// and streams 64-query tiles; thread r of the four compute warps owns key row
// r (TMEM lane r), so every score tile is computed transposed (keys x queries)
// and the per-query statistics (lse2, delta, gamma, rho) arrive with each
// streamed tile through TMA.
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
// Causal: query tiles that end before the CTA's first key are skipped.
#include "attn_common.cuh"
#include "kernels.h"

namespace ttt {

template <int D, int KIND>
struct KmCfg {
  static constexpr int BM = 64, BK = 128;     // BM queries per streamed tile, BK keys per CTA
  static constexpr bool BWD2 = (KIND == kBwd2KV);
  static constexpr int NR = BWD2 ? 4 : 2;     // resident: K, V, (u_k, u_v)
  static constexpr int NSTR = BWD2 ? 3 : 2;   // streamed: Q, dO, (u_q)
  static constexpr int NSTAT = BWD2 ? 4 : 2;  // streamed stats: lse2, delta, (gamma, rho)
  static constexpr int NSC = BWD2 ? 4 : 2;    // score tiles: S^T, dP^T, (G_dS^T, (dO u_v^T)^T)
  static constexpr int NE = BWD2 ? 3 : 2;     // P^T, dS^T | dS^T, G_S^T, G_dP^T
  static constexpr int NA = 2;
  static constexpr int TILE_R = BK * D * 2;
  static constexpr int TILE_S = BM * D * 2;
  static constexpr int STAT_BYTES = BM * 4;
  static constexpr int STAGE_TX = NSTR * TILE_S + NSTAT * STAT_BYTES;  // bytes TMA delivers per stage
  static constexpr int STAGE = (STAGE_TX + 1023) / 1024 * 1024;       // stage pitch keeps tiles 1024-aligned
  static constexpr int TILE_E = BK * BM * 2;
  static constexpr int NBUF = (2 * NSC * BM + NA * D <= 512) ? 2 : 1;
  static constexpr int TMEM_USED = NBUF * NSC * BM + NA * D;
  static constexpr int TMEM_COLS = TMEM_USED <= 128 ? 128 : (TMEM_USED <= 256 ? 256 : 512);
  static_assert(TMEM_USED <= 512, "TMEM overflow");
  static constexpr int FIXED = NR * TILE_R + NBUF * NE * TILE_E;
  static constexpr int NSTAGE = (FIXED + STAGE + STAGE_TX + 2048 <= 232448) ? 2 : 1;
  static constexpr int OFF_R = 0;
  static constexpr int OFF_E = OFF_R + NR * TILE_R;
  static constexpr int OFF_S = OFF_E + NBUF * NE * TILE_E;  // stages last: stats need only 16B alignment
  static constexpr int OFF_BAR = OFF_S + (NSTAGE - 1) * STAGE + STAGE_TX;
  static constexpr int NBAR = 16;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "key-major tile set exceeds shared memory");
};

template <int D, bool BF16, bool CAUSAL, int KIND>
__global__ void __launch_bounds__(192, 1) attn_km_kernel(const __grid_constant__ KParams p) {
  using C = KmCfg<D, KIND>;
  constexpr int BM = C::BM, BK = C::BK, NP = D / 64, NBUF = C::NBUF, NSTAGE = C::NSTAGE;
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
  // Stage layout: NSTR 16-bit tiles (each 1024-aligned because TILE_S is a
  // multiple of 1024 and the stage starts 1024-aligned), then NSTAT fp32 rows.
  static_assert(C::TILE_S % 1024 == 0, "");
  auto tileR = [&](int t) { return sR + t * C::TILE_R; };
  auto tileS = [&](int s, int t) { return sS + s * C::STAGE + t * C::TILE_S; };
  auto statS = [&](int s, int t) {
    return reinterpret_cast<float*>(sS + s * C::STAGE + C::NSTR * C::TILE_S + t * C::STAT_BYTES);
  };
  auto tileE = [&](int b, int t) { return sE + (b * C::NE + t) * C::TILE_E; };

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
  const uint32_t tAcc0 = tmem + NBUF * C::NSC * BM;  // dK / dd_K
  const uint32_t tAcc1 = tAcc0 + D;                  // dV / dd_V
  Guard g{abort_flag, p.err};

  if (warp == 5) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = 0; t < C::NR; ++t) tma_prefetch(&p.own[t]);
      for (int t = 0; t < C::NSTR; ++t) tma_prefetch(&p.str[t]);
      for (int t = 0; t < C::NSTAT; ++t) tma_prefetch(&p.st[t]);
      int issued[2] = {0, 0};
      mbar_arrive_tx(res_full, C::NR * C::TILE_R);
      for (int t = 0; t < C::NR; ++t)
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(tileR(t) + pp * BK * 128, &p.own[t], res_full, pp * 64, k0, hidx, bidx);
      for (int n = 0; n < n_tiles; ++n) {
        const int s = n % NSTAGE;
        const int qrow = (qt0 + n) * BM;
        if (n >= NSTAGE && !mbar_wait(l_empty + s, ((n / NSTAGE) - 1) & 1, g, 1)) break;
        mbar_arrive_tx(l_full + s, C::STAGE_TX);
        for (int t = 0; t < C::NSTR; ++t)
          for (int pp = 0; pp < NP; ++pp)
            tma_load_4d(tileS(s, t) + pp * BM * 128, &p.str[t], l_full + s, pp * 64, qrow, hidx, bidx);
        for (int t = 0; t < C::NSTAT; ++t) tma_load_2d(statS(s, t), &p.st[t], l_full + s, qrow, bh);
        issued[s] = n + 1;
      }
      mbar_drain(res_full, 0);
      for (int s = 0; s < NSTAGE; ++s)
        if (issued[s] > 0) mbar_drain(l_full + s, ((issued[s] - 1) / NSTAGE) & 1);
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_sc = idesc_f16(128, BM, BF16, false, false);
      constexpr uint32_t id_acc = idesc_f16(128, D, BF16, false, true);
      const uint32_t aK = smem_u32(tileR(0)), aV = smem_u32(tileR(1));
      const uint32_t aUK = C::BWD2 ? smem_u32(tileR(2)) : 0u, aUV = C::BWD2 ? smem_u32(tileR(3)) : 0u;
      auto issue_scores = [&](int n) -> bool {
        const int sb = n % NBUF, s = n % NSTAGE;
        if (!mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 2)) return false;
        tc_fence_after();
        const uint32_t base = tmem + sb * C::NSC * BM;
        const uint32_t bQ = smem_u32(tileS(s, 0)), bDO = smem_u32(tileS(s, 1));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(base, desc_kmajor(aK, BK, kk), desc_kmajor(bQ, BM, kk), id_sc, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(base + BM, desc_kmajor(aV, BK, kk), desc_kmajor(bDO, BM, kk), id_sc, kk > 0);
        if constexpr (C::BWD2) {
          const uint32_t bUQ = smem_u32(tileS(s, 2));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + 2 * BM, desc_kmajor(aK, BK, kk), desc_kmajor(bUQ, BM, kk), id_sc, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + 2 * BM, desc_kmajor(aUK, BK, kk), desc_kmajor(bQ, BM, kk), id_sc, 1u);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(base + 3 * BM, desc_kmajor(aUV, BK, kk), desc_kmajor(bDO, BM, kk), id_sc, kk > 0);
        }
        umma_commit(s_full + sb);
        return true;
      };
      auto issue_acc = [&](int n) -> bool {
        const int sb = n % NBUF, s = n % NSTAGE;
        if (!mbar_wait(e_full + sb, (n / NBUF) & 1, g, 3)) return false;
        tc_fence_after();
        const uint32_t bQ = smem_u32(tileS(s, 0)), bDO = smem_u32(tileS(s, 1));
        const uint32_t e0 = smem_u32(tileE(sb, 0)), e1 = smem_u32(tileE(sb, 1));
        if constexpr (!C::BWD2) {
          // dV += P^T dO ; dK += dS^T Q
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc1, desc_kmajor(e0, BK, kk), desc_mnmajor(bDO, BM, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e1, BK, kk), desc_mnmajor(bQ, BM, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
        } else {
          // dd_K += dS^T u_q + G_S^T Q ; dd_V += G_dP^T dO
          const uint32_t bUQ = smem_u32(tileS(s, 2)), e2 = smem_u32(tileE(sb, 2));
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e0, BK, kk), desc_mnmajor(bUQ, BM, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc0, desc_kmajor(e1, BK, kk), desc_mnmajor(bQ, BM, kk), id_acc, 1u);
#pragma unroll
          for (int kk = 0; kk < BM / 16; ++kk)
            umma_ss(tAcc1, desc_kmajor(e2, BK, kk), desc_mnmajor(bDO, BM, kk), id_acc, (n > 0 || kk > 0) ? 1u : 0u);
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
        if (m < n_tiles && !issue_scores(m)) { ok = false; break; }
        if (!issue_acc(n)) { ok = false; break; }
      }
      if (ok) umma_commit(acc_full);
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ elementwise warps 0..3
    const int r = threadIdx.x;
    const int key = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float c = p.scale_log2, scale = p.scale;
    bool ok = true;
    for (int n = 0; n < n_tiles; ++n) {
      const int sb = n % NBUF, s = n % NSTAGE;
      if (!mbar_wait(s_full + sb, (n / NBUF) & 1, g, 6)) { ok = false; break; }
      // The per-query statistics were delivered by TMA on l_full[s]; that
      // phase cannot advance until this tile's elementwise step is done.
      if (!mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 9)) { ok = false; break; }
      tc_fence_after();
      if (n >= NBUF && !mbar_wait(e_empty + sb, ((n / NBUF) - 1) & 1, g, 7)) { ok = false; break; }
      const float* st_lse = statS(s, 0);
      const float* st_del = statS(s, 1);
      const float* st_gam = statS(s, C::BWD2 ? 2 : 0);
      const float* st_rho = statS(s, C::BWD2 ? 3 : 0);
      const uint32_t base = tmem + lane_off + sb * C::NSC * BM;
      const int qrow0 = (qt0 + n) * BM;
#pragma unroll
      for (int half = 0; half < BM / 32; ++half) {
        const int cc = half * 32;
        float sv[32], dp[32], gd[32], uv[32];
        tmem_ld32(base + cc, sv);
        tmem_ld32(base + BM + cc, dp);
        if constexpr (C::BWD2) {
          tmem_ld32(base + 2 * BM + cc, gd);
          tmem_ld32(base + 3 * BM + cc, uv);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int qi = qrow0 + cc + e;
          const bool valid = (qi < T) && (key < T) && (!CAUSAL || key <= qi);
          const float pr = valid ? fast_exp2(sv[e] * c - st_lse[cc + e]) : 0.f;
          const float del = st_del[cc + e];
          if constexpr (!C::BWD2) {
            sv[e] = pr;               // P^T
            dp[e] = pr * (dp[e] - del);  // dS^T
          } else {
            const float gam = st_gam[cc + e], rho = st_rho[cc + e];
            const float dpm = dp[e] - del;
            const float gds = gd[e] * scale;
            const float gP = gds * dpm - gam * dp[e] + uv[e];
            sv[e] = pr * dpm;          // dS^T
            dp[e] = pr * (gP - rho);   // G_S^T
            gd[e] = pr * (gds - gam);  // G_dP^T
          }
        }
        store_row32<BF16>(tileE(sb, 0), BK, r, cc, sv);
        store_row32<BF16>(tileE(sb, 1), BK, r, cc, dp);
        if constexpr (C::BWD2) store_row32<BF16>(tileE(sb, 2), BK, r, cc, gd);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(e_full + sb);
    }
    if (ok && mbar_wait(acc_full, 0, g, 8)) {
      tc_fence_after();
      const bool valid = key < T;
      uint16_t* r0 = p.out0 + static_cast<int64_t>(bidx) * p.o0_sb + static_cast<int64_t>(hidx) * p.o0_sh +
                     static_cast<int64_t>(key) * p.o0_st;
      uint16_t* r1 = p.out1 + static_cast<int64_t>(bidx) * p.o1_sb + static_cast<int64_t>(hidx) * p.o1_sh +
                     static_cast<int64_t>(key) * p.o1_st;
      acc_to_global<D, BF16>(tAcc0 + lane_off, r0, valid, scale);
      acc_to_global<D, BF16>(tAcc1 + lane_off, r1, valid, 1.f);
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
  kern<<<grid, 192, C::SMEM, stream>>>(p);
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
