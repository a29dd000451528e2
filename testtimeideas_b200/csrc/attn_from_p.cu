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
// kFpDQ) and streams W rows of the other axis per step:
//   warp 5      TMA producer (P tile + the streamed [W x d] tiles, ring of stages)
//   warp 4      MMA issuer
//   warps 0..3  one owned row per thread: the elementwise dS step (kFpDK,
//               kFpDQ) and the epilogue.
// kFpDV / kFpRowsum are pure products: P^T dO (both operands MN-major) or P V
// accumulate in TMEM. kFpDK / kFpDQ compute the dP^T (or dP) tile of a step
// into one of two TMEM score buffers, the elementwise warps turn it into
// 16-bit dS^T (dS) in one of two TMEM E buffers, and the accumulate product
// reads E as its A operand from TMEM.
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
  static constexpr int W = ELEM ? 64 : 128;  // streamed rows per step
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
  static constexpr int BUDGET = 232448 - 1024 - BAR_BYTES - NR * TILE_R;
  static constexpr int NSTAGE = BUDGET / STAGE >= 4 ? 4 : BUDGET / STAGE;
  static constexpr int OFF_R = 0;
  static constexpr int OFF_S = OFF_R + NR * TILE_R;
  static constexpr int OFF_BAR = OFF_S + NSTAGE * STAGE;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 16 + 1024;
  // TMEM: accumulator at 0 (D columns); ELEM: score buffers (2 x W) then packed
  // E buffers (2 x W/2).
  static constexpr int C_S = D, C_E = D + 2 * W;
  static constexpr int TMEM_USED = ELEM ? D + 3 * W : D;
  static constexpr int TMEM_COLS = TMEM_USED <= 64 ? 64 : TMEM_USED <= 128 ? 128 : TMEM_USED <= 256 ? 256 : 512;
  static constexpr int NTHREADS = 192;
  static_assert(NSTAGE >= 2, "from-P stage ring does not fit");
  static_assert(STAGE % 1024 == 0 && TILE_P % 1024 == 0 && TILE_R % 1024 == 0, "tiles must stay 1024-aligned");
  static_assert(SMEM <= 232448, "from-P tile set exceeds shared memory");
};

template <int D, bool BF16, bool CAUSAL, int MODE>
__global__ void __launch_bounds__(192, 1) attn_from_p_kernel(const __grid_constant__ KParams p) {
  using C = FpCfg<D, MODE>;
  constexpr int W = C::W, NP = D / 64, NSTAGE = C::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sR = smem + C::OFF_R;
  uint8_t* sS = smem + C::OFF_S;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* res_full = bars + 0;
  uint64_t* l_full = bars + 1;    // [4]
  uint64_t* l_empty = bars + 5;   // [4]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_free = bars + 11;   // [2] (128 arrivals)
  uint64_t* e_full = bars + 13;   // [2] (128 arrivals)
  uint64_t* e_empty = bars + 15;  // [2]
  uint64_t* acc_full = bars + 17;
  uint64_t* drain = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto tileP = [&](int s) { return sS + s * C::STAGE; };
  auto tileX = [&](int s, int i) { return sS + s * C::STAGE + C::TILE_P + i * C::TILE_X; };

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
    for (int i = 0; i < 19; ++i) mbar_init(bars + i, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_free + i, 128);
      mbar_init(e_full + i, 128);
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

  if (warp == 5) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch(&p.str[0]);
      for (int i = 0; i < C::NX; ++i) tma_prefetch(&p.str[1 + i]);
      if constexpr (C::NR > 0) {
        tma_prefetch(&p.own[0]);
        mbar_arrive_tx(res_full, C::TILE_R);
        for (int pp = 0; pp < NP; ++pp) tma_load_4d(sR + pp * 128 * 128, &p.own[0], res_full, pp * 64, r0, hidx, bidx);
      }
      int n = 0;
      for (; n < n_tiles; ++n) {
        const int s = n % NSTAGE;
        const int j0 = (n_first + n) * W;  // first streamed row of this step
        if (n >= NSTAGE && !mbar_wait(l_empty + s, ((n / NSTAGE) - 1) & 1, g, 1)) break;
        mbar_arrive_tx(l_full + s, C::STAGE_TX);
        // P tile: 64-column panels of P_ROWS rows
        const int prow = C::KEY_MAJOR ? j0 : r0;
        const int pcol = C::KEY_MAJOR ? r0 : j0;
        for (int pp = 0; pp < C::P_COLS / 64; ++pp)
          tma_load_4d(tileP(s) + pp * C::P_ROWS * 128, &p.str[0], l_full + s, pcol + pp * 64, prow, hidx, bidx);
        for (int i = 0; i < C::NX; ++i)
          for (int pp = 0; pp < NP; ++pp)
            tma_load_4d(tileX(s, i) + pp * W * 128, &p.str[1 + i], l_full + s, pp * 64, j0, hidx, bidx);
      }
      if constexpr (C::NR > 0) mbar_drain(res_full, 0);
      for (int j = max(0, n - NSTAGE); j < n; ++j) mbar_drain(l_full + j % NSTAGE, (j / NSTAGE) & 1);
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      if constexpr (!C::ELEM) {
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
      } else {
        // score: kFpDK dP^T = V dO^T, kFpDQ dP = dO V^T (A = resident, B = streamed tile 0)
        // accumulate: kFpDK dK += dS^T Q, kFpDQ dQ += dS K (A = E from TMEM, B = tile 1 MN-major)
        constexpr uint32_t id_s = idesc_f16(128, W, BF16, false, false);
        constexpr uint32_t id_a = idesc_f16(128, D, BF16, false, true);
        const uint32_t aR = smem_u32(sR);
        ok = mbar_wait(res_full, 0, g, 2);
        auto acc_step = [&](int n) -> bool {
          const int s = n % NSTAGE, eb = n & 1;
          if (!mbar_wait(e_full + eb, (n >> 1) & 1, g, 5)) return false;
          tc_fence_after();
          const uint32_t bX = smem_u32(tileX(s, 1));
#pragma unroll
          for (int kk = 0; kk < W / 16; ++kk)
            umma_ts(tmem, tmem + C::C_E + eb * (W / 2) + kk * 8, desc_mnmajor(bX, W, kk), id_a,
                    (n > 0 || kk > 0) ? 1u : 0u);
          umma_commit(e_empty + eb);
          umma_commit(l_empty + s);
          return true;
        };
        for (int n = 0; ok && n < n_tiles; ++n) {
          const int s = n % NSTAGE, sb = n & 1;
          if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 3))) break;
          if (n >= 2 && !(ok = mbar_wait(s_free + sb, ((n >> 1) - 1) & 1, g, 4))) break;
          tc_fence_after();
          const uint32_t bX = smem_u32(tileX(s, 0));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_ss(tmem + C::C_S + sb * W, desc_kmajor(aR, 128, kk), desc_kmajor(bX, W, kk), id_s,
                    kk > 0 ? 1u : 0u);
          umma_commit(s_full + sb);
          if (n >= 1 && !(ok = acc_step(n - 1))) break;
        }
        if (ok && n_tiles > 0) ok = acc_step(n_tiles - 1);
      }
      if (ok) umma_commit(acc_full);
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ row warps 0..3
    const int r = threadIdx.x;  // owned row == TMEM lane
    const int row = r0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    bool ok = true;
    if constexpr (C::ELEM) {
      // kFpDQ: this row's rowsum; kFpDK: the streamed queries' rowsums, read per step
      const float* rs = p.delta + static_cast<int64_t>(bh) * T;
      const float own_rs = (MODE == kFpDQ && row < T) ? rs[row] : 0.f;
      for (int n = 0; n < n_tiles; ++n) {
        const int s = n % NSTAGE, sb = n & 1;
        const int j0 = (n_first + n) * W;
        if (!mbar_wait(s_full + sb, (n >> 1) & 1, g, 6)) { ok = false; break; }
        tc_fence_after();
        float dp[W];
        tmem_ld_nw<W>(tmem + lane_off + C::C_S + sb * W, dp);
        tmem_wait_ld();
        reg_fence(dp);
        tc_fence_before();
        mbar_arrive(s_free + sb);
        if (!mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 7)) { ok = false; break; }
        const uint8_t* tp = tileP(s);
        float pv[W];
        if constexpr (MODE == kFpDK) {
          // P[j0 + j, row]: column r of the [W x 128] tile (one 2-byte load per entry)
#pragma unroll
          for (int j = 0; j < W; ++j)
            pv[j] = to_f32<BF16>(*reinterpret_cast<const uint16_t*>(tp + pl_offset(W, j, r)));
        } else {
          // P[row, j0 + j]: row r of the [128 x W] tile (16-byte swizzled chunks)
#pragma unroll
          for (int ch = 0; ch < W / 8; ++ch) {
            const uint4 w4 = *reinterpret_cast<const uint4*>(tp + r * 128 + ((ch ^ (r & 7)) << 4));
            const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              pv[ch * 8 + 2 * i] = to_f32<BF16>(static_cast<uint16_t>(wv[i] & 0xffffu));
              pv[ch * 8 + 2 * i + 1] = to_f32<BF16>(static_cast<uint16_t>(wv[i] >> 16));
            }
          }
        }
        uint32_t w[W / 2];
#pragma unroll
        for (int j = 0; j < W; j += 2) {
          float d0 = own_rs, d1 = own_rs;
          if constexpr (MODE == kFpDK) {
            d0 = (j0 + j < T) ? __ldg(rs + j0 + j) : 0.f;
            d1 = (j0 + j + 1 < T) ? __ldg(rs + j0 + j + 1) : 0.f;
          }
          float s0, s1;
          split(mul2(f2(pv[j], pv[j + 1]), sub2(f2(dp[j], dp[j + 1]), f2(d0, d1))), s0, s1);
          w[j / 2] = pack2<BF16>(s0, s1);
        }
        const int eb = n & 1;
        if (n >= 2 && !mbar_wait(e_empty + eb, ((n >> 1) - 1) & 1, g, 8)) { ok = false; break; }
        const uint32_t te = tmem + lane_off + C::C_E + eb * (W / 2);
        tmem_st16_raw(te, *reinterpret_cast<uint32_t(*)[16]>(w));
        tmem_st16_raw(te + 16, *reinterpret_cast<uint32_t(*)[16]>(w + 16));
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
        acc_to_global<D, BF16>(tmem + lane_off, orow, valid, MODE == kFpDV ? 1.f : p.scale);
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
