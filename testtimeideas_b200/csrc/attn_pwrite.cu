// The normalized probabilities P of the save_p forward (sm_100a):
// P[b, h, i, j] = 2^(S_ij * c - lse2_i), S = Q K^T, c = scale * log2(e), for the
// key tiles a query block sees (zero elsewhere is the caller's), after the
// row-LSE forward (attn_fwd2_kernel) has written lse2. This is the materialized
// P of the reference's save_p modes (ttt_kernels/triton_attention.py:51-59,
// 270-273) and of its _attn_probs_kernel (:227-256), which backward_stubs.py's
// from-P helpers read.
//
// The pass is bound by the HBM write of P (2 bytes per entry against 2*d
// flops of the recomputed score): one CTA owns 128 query rows of one head,
// keeps Q resident, and streams 128-key tiles of K:
//   warps 0..7  elementwise: warp w owns TMEM lanes 32*(w%4)..+31 (one query
//               row per thread) and columns 64*(w/4)..+63 of each tile; each
//               thread turns its 64 scores into 16-bit P and writes them as
//               eight 16-byte chunks of one row of a 128-byte-swizzled
//               shared-memory tile (two [128 x 64] panels per key tile)
//   warp 8      TMA producer: Q once, then K tiles into a 4-stage ring
//   warp 9      MMA issuer: S_n = Q K_n^T into one of two TMEM score buffers
//   warp 10     store thread: stores each finished P tile with TMA (two
//               [128 x 64] boxes; rows and columns past T are clipped by the
//               tensor map), keeping one store in flight while the next tile
//               is formed in the other staging buffer
// Requires T % 8 == 0 (the row stride of P, 2T bytes, must be a multiple of 16
// for the tensor map); the C ABI keeps the single-kernel forward for other T.
#include "attn_pipe.cuh"
#include "kernels.h"

namespace ttt {

// 4-D tiled store of a shared-memory box into global memory, tracked by this
// thread's bulk async-group. Coordinates are never negative here.
TTT_DEV void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
      : "memory");
}
// Wait until at most one of this thread's bulk groups is still reading shared memory.
TTT_DEV void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

template <int D>
struct PwCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int TILE_Q = BM * D * 2;
  static constexpr int TILE_K = BN * D * 2;
  static constexpr int TILE_P = BM * BN * 2;  // one staging buffer: two [128 x 64] panels
  static constexpr int NBAR = 20;
  static constexpr int BAR_BYTES = NBAR * 8 + 16;
  static constexpr int BUDGET = 232448 - 1024 - BAR_BYTES - TILE_Q - 2 * TILE_P;
  static constexpr int NSTAGE = BUDGET / TILE_K >= 4 ? 4 : BUDGET / TILE_K;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + TILE_Q;
  static constexpr int OFF_P = OFF_K + NSTAGE * TILE_K;
  static constexpr int OFF_BAR = OFF_P + 2 * TILE_P;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;
  static constexpr int NCW = 8, NCT = NCW * 32;
  static constexpr int WARP_LOAD = 8, WARP_MMA = 9, WARP_STORE = 10;
  static constexpr int NTHREADS = 352;
  static constexpr int TMEM_COLS = 2 * BN;
  static_assert(NSTAGE >= 2, "P-writer stage ring does not fit");
  static_assert(SMEM <= 232448, "P-writer tile set exceeds shared memory");
};

template <int D, bool BF16, bool CAUSAL>
__global__ void __launch_bounds__(PwCfg<D>::NTHREADS, 1) attn_pwrite_kernel(const __grid_constant__ KParams p) {
  using C = PwCfg<D>;
  constexpr int BM = C::BM, BN = C::BN, NP = D / 64, NSTAGE = C::NSTAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem + C::OFF_Q;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* res_full = bars + 0;
  uint64_t* l_full = bars + 1;    // [4] TMA -> MMA
  uint64_t* l_empty = bars + 5;   // [4] MMA -> TMA
  uint64_t* s_full = bars + 9;    // [2] MMA -> elementwise
  uint64_t* s_free = bars + 11;   // [2] elementwise (NCT arrivals) -> MMA
  uint64_t* st_full = bars + 13;  // [2] elementwise (NCT arrivals) -> store thread
  uint64_t* st_free = bars + 15;  // [2] store thread -> elementwise (staging buffer read by TMA)
  uint64_t* drain = bars + 17;    // MMA issuer's final commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto tileK = [&](int s) { return smem + C::OFF_K + s * C::TILE_K; };
  auto tileP = [&](int b) { return smem + C::OFF_P + b * C::TILE_P; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const GridPos gp = grid_pos();
  const int bh = gp.unit;
  const int bidx = bh / p.H, hidx = bh % p.H;
  const int qblk = CAUSAL ? (gridDim.y - 1 - gp.rank) : gp.rank;  // longest rows first
  const int q0 = qblk * BM;
  const int T = p.T;
  const int n_all = (T + BN - 1) / BN;
  const int n_tiles = CAUSAL ? min(n_all, (q0 + BM - 1) / BN + 1) : n_all;  // key tiles up to the diagonal

  if (threadIdx.x == 0) {
    for (int i = 0; i < 19; ++i) mbar_init(bars + i, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_free + i, C::NCT);
      mbar_init(st_full + i, C::NCT);
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
    if (lane == 0) {
      tma_prefetch(&p.own[0]);
      tma_prefetch(&p.str[0]);
      mbar_arrive_tx(res_full, C::TILE_Q);
      for (int pp = 0; pp < NP; ++pp) tma_load_4d(sQ + pp * BM * 128, &p.own[0], res_full, pp * 64, q0, hidx, bidx);
      int n = 0;
      for (; n < n_tiles; ++n) {
        const int s = n % NSTAGE;
        if (n >= NSTAGE && !mbar_wait(l_empty + s, ((n / NSTAGE) - 1) & 1, g, 1)) break;
        mbar_arrive_tx(l_full + s, C::TILE_K);
        for (int pp = 0; pp < NP; ++pp)
          tma_load_4d(tileK(s) + pp * BN * 128, &p.str[0], l_full + s, pp * 64, n * BN, hidx, bidx);
      }
      mbar_drain(res_full, 0);
      for (int j = max(0, n - NSTAGE); j < n; ++j) mbar_drain(l_full + j % NSTAGE, (j / NSTAGE) & 1);
    }
  } else if (warp == C::WARP_MMA) {
    // ------------------------------------------------------------ MMA issuer: S_n = Q K_n^T
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(BM, BN, BF16, false, false);
      const uint32_t aQ = smem_u32(sQ);
      bool ok = mbar_wait(res_full, 0, g, 2);
      for (int n = 0; ok && n < n_tiles; ++n) {
        const int s = n % NSTAGE, sb = n & 1;
        if (!(ok = mbar_wait(l_full + s, (n / NSTAGE) & 1, g, 3))) break;
        if (n >= 2 && !(ok = mbar_wait(s_free + sb, ((n >> 1) - 1) & 1, g, 4))) break;
        tc_fence_after();
        const uint32_t bK = smem_u32(tileK(s));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss(tmem + sb * BN, desc_kmajor(aQ, BM, kk), desc_kmajor(bK, BN, kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit(s_full + sb);
        umma_commit(l_empty + s);
      }
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else if (warp == C::WARP_STORE) {
    // ------------------------------------------------------------ store thread
    // One TMA store (two [128 x 64] boxes) per tile; the staging buffer of tile n-1
    // is released once its store has been read out of shared memory, so one store
    // stays in flight while tile n+1 is formed in that buffer.
    if (lane == 0) {
      tma_prefetch(&p.str[1]);
      int n = 0;
      for (; n < n_tiles; ++n) {
        const int sb = n & 1;
        if (!mbar_wait(st_full + sb, (n >> 1) & 1, g, 5)) break;
        for (int pp = 0; pp < 2; ++pp)
          tma_store_4d(&p.str[1], tileP(sb) + pp * BM * 128, n * BN + pp * 64, q0, hidx, bidx);
        bulk_commit();
        if (n >= 1) {
          bulk_wait_read_1();
          mbar_arrive(st_free + ((n - 1) & 1));
        }
      }
      bulk_wait_all();  // every store of this CTA has completed
      if (n >= 1) mbar_arrive(st_free + ((n - 1) & 1));
    }
  } else if (warp < C::NCW) {
    // ------------------------------------------------------------ elementwise warps
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;  // query row within the block == TMEM lane
    const int row = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float c = p.scale_log2;
    const float lse2 = row < T ? p.lse2[static_cast<int64_t>(bh) * p.t_pad + row] : INFINITY;
    for (int n = 0; n < n_tiles; ++n) {
      const int sb = n & 1;
      if (!mbar_wait(s_full + sb, (n >> 1) & 1, g, 6)) break;
      tc_fence_after();
      float v[64];
      tmem_ld_nw<64>(tmem + lane_off + sb * BN + half * 64, v);
      tmem_wait_ld();
      reg_fence(v);
      tc_fence_before();
      mbar_arrive(s_free + sb);
      const int col0 = n * BN + half * 64;
      // only the diagonal tile (causal) and a tile reaching past T need the mask
      const bool masked = (CAUSAL && col0 + 63 > q0) || col0 + 64 > T;
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 64; j += 2) {
        float p0 = fast_exp2(fmaf(v[j], c, -lse2)), p1 = fast_exp2(fmaf(v[j + 1], c, -lse2));
        if (masked) {
          const int cj = col0 + j;
          p0 = (cj < T && (!CAUSAL || cj <= row)) ? p0 : 0.f;
          p1 = (cj + 1 < T && (!CAUSAL || cj + 1 <= row)) ? p1 : 0.f;
        }
        w[j >> 1] = pack2<BF16>(p0, p1);
      }
      // the staging buffer's previous store (tile n-2) has been read by the TMA unit
      if (n >= 2 && !mbar_wait(st_free + sb, ((n >> 1) - 1) & 1, g, 7)) break;
      uint8_t* rowp = tileP(sb) + half * BM * 128 + r * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<uint4*>(rowp + ((ch ^ (r & 7)) << 4)) =
            make_uint4(w[4 * ch], w[4 * ch + 1], w[4 * ch + 2], w[4 * ch + 3]);
      fence_async_smem();  // the TMA store reads these bytes through the async proxy
      mbar_arrive(st_full + sb);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int D, bool BF16, bool CAUSAL>
static cudaError_t launch_pwrite_t(const KParams& p, cudaStream_t stream) {
  using C = PwCfg<D>;
  auto kern = attn_pwrite_kernel<D, BF16, CAUSAL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B * p.H, (p.T + C::BM - 1) / C::BM);
  kern<<<grid, C::NTHREADS, C::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_pwrite(const KParams& p, int d, bool bf16, bool causal, cudaStream_t stream) {
#define TTT_PW(D_, BF_, CA_) \
  if (d == D_ && bf16 == BF_ && causal == CA_) return launch_pwrite_t<D_, BF_, CA_>(p, stream);
  TTT_PW(64, false, false) TTT_PW(64, false, true) TTT_PW(64, true, false) TTT_PW(64, true, true)
  TTT_PW(128, false, false) TTT_PW(128, false, true) TTT_PW(128, true, false) TTT_PW(128, true, true)
#undef TTT_PW
  return cudaErrorInvalidValue;
}

}  // namespace ttt
