// Small kernels: the delta = rowsum(dO o O) preprocessing pass and a tcgen05
// GEMM self-test that exercises the two operand layouts every attention
// kernel uses.
//
// delta replaces _attn_rowsum_kernel (ttt_kernels/backward_stubs.py:184-221):
// the reference computes sum_j P_ij (dO_i . V_j), a T x T pass with a
// T x T x d product; since P V = O that equals dO_i . O_i, an O(T d) read.
#include "attn_common.cuh"
#include "kernels.h"

namespace ttt {

// D/8 threads per row, each reading 16 bytes of O and of dO (rows start
// 16-byte aligned: the views' base pointers are 16-byte aligned and their
// strides are multiples of 8 elements). A warp covers 32/(D/8) rows per
// iteration and issues the loads of UNROLL iterations before using any, so
// each SM keeps enough bytes in flight to stream at HBM rate; the grid is a
// few CTAs per SM striding over all rows.
template <int D, bool BF16>
__global__ void __launch_bounds__(256) attn_delta_kernel(DeltaArgs a) {
  constexpr int TPR = D / 8;            // threads per row
  constexpr int RPW = 32 / TPR;         // rows per warp per iteration
  constexpr int UNROLL = 4;
  constexpr int RPB = 8 * RPW * UNROLL; // rows per CTA per pass
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / TPR, c8 = (lane % TPR) * 8;
  const int64_t total = static_cast<int64_t>(a.B) * a.H * a.t_pad;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * RPB; base < total;
       base += static_cast<int64_t>(gridDim.x) * RPB) {
    uint4 ov[UNROLL], dv[UNROLL];
    int64_t rows[UNROLL];
    bool live[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t row = base + (static_cast<int64_t>(u) * 8 + warp) * RPW + sub;
      rows[u] = row;
      const int bh = static_cast<int>(row / a.t_pad);
      const int t = static_cast<int>(row % a.t_pad);
      live[u] = row < total && t < a.T;
      ov[u] = make_uint4(0u, 0u, 0u, 0u);
      dv[u] = make_uint4(0u, 0u, 0u, 0u);
      if (live[u]) {
        const int b = bh / a.H, h = bh % a.H;
        ov[u] = __ldg(reinterpret_cast<const uint4*>(a.o + b * a.o_sb + h * a.o_sh + static_cast<int64_t>(t) * a.o_st + c8));
        dv[u] = __ldg(reinterpret_cast<const uint4*>(a.dout + b * a.d_sb + h * a.d_sh + static_cast<int64_t>(t) * a.d_st + c8));
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const uint32_t* ow = reinterpret_cast<const uint32_t*>(&ov[u]);
      const uint32_t* dw = reinterpret_cast<const uint32_t*>(&dv[u]);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc = fmaf(to_f32<BF16>(static_cast<uint16_t>(ow[i] & 0xffffu)), to_f32<BF16>(static_cast<uint16_t>(dw[i] & 0xffffu)), acc);
        acc = fmaf(to_f32<BF16>(static_cast<uint16_t>(ow[i] >> 16)), to_f32<BF16>(static_cast<uint16_t>(dw[i] >> 16)), acc);
      }
#pragma unroll
      for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane % TPR == 0 && rows[u] < total) a.delta[rows[u]] = live[u] ? acc : 0.f;
    }
  }
}

cudaError_t launch_delta(const DeltaArgs& a, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(a.B) * a.H * a.t_pad;
  // SM count per device ordinal, looked up once (a stale entry only resizes the grid)
  static int sm_of[64] = {0};
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) sms = sm_of[dev];
  if (sms <= 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    if (dev >= 0 && dev < 64) sm_of[dev] = sms;
  }
  const int rpb = 8 * (32 / (a.D / 8)) * 4;
  const int64_t need = (rows + rpb - 1) / rpb;
  const dim3 grid(static_cast<unsigned>(need < 8LL * sms ? need : 8LL * sms));
  if (a.D == 64 && !a.bf16) attn_delta_kernel<64, false><<<grid, 256, 0, stream>>>(a);
  else if (a.D == 64 && a.bf16) attn_delta_kernel<64, true><<<grid, 256, 0, stream>>>(a);
  else if (a.D == 128 && !a.bf16) attn_delta_kernel<128, false><<<grid, 256, 0, stream>>>(a);
  else if (a.D == 128 && a.bf16) attn_delta_kernel<128, true><<<grid, 256, 0, stream>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// ---------------------------------------------------------------- split reduction
// One thread per 8 consecutive columns of one output row: reads the row's 8
// fp32 partials of every share (two 16-byte loads each, shares in order),
// scales the sum and stores eight 16-bit values with one 16-byte store.
template <bool BF16>
__global__ void __launch_bounds__(256) split_reduce_kernel(SplitReduceArgs a) {
  const int o = blockIdx.y;
  const int per_row = a.D / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t bh_count = static_cast<int64_t>(a.B) * a.H;
  if (idx >= bh_count * a.T * per_row) return;
  const int c8 = static_cast<int>(idx % per_row);
  const int64_t row = idx / per_row;
  const int t = static_cast<int>(row % a.T);
  const int bh = static_cast<int>(row / a.T);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < a.nsplit; ++s) {
    const float4* src = reinterpret_cast<const float4*>(
        a.part[o] + ((static_cast<int64_t>(s) * bh_count + bh) * a.t_pad + t) * a.D + c8 * 8);
    const float4 x = src[0], y = src[1];
    acc[0] += x.x; acc[1] += x.y; acc[2] += x.z; acc[3] += x.w;
    acc[4] += y.x; acc[5] += y.y; acc[6] += y.z; acc[7] += y.w;
  }
  const float m = a.scale[o];
  uint4 w;
  w.x = pack2<BF16>(acc[0] * m, acc[1] * m);
  w.y = pack2<BF16>(acc[2] * m, acc[3] * m);
  w.z = pack2<BF16>(acc[4] * m, acc[5] * m);
  w.w = pack2<BF16>(acc[6] * m, acc[7] * m);
  const int b = bh / a.H, h = bh % a.H;
  *reinterpret_cast<uint4*>(a.out[o] + b * a.sb[o] + h * a.sh[o] + static_cast<int64_t>(t) * a.st[o] + c8 * 8) = w;
}

cudaError_t launch_split_reduce(const SplitReduceArgs& a, cudaStream_t stream) {
  if (a.n_out < 1 || a.n_out > 2 || a.nsplit < 1 || (a.D % 8) != 0) return cudaErrorInvalidValue;
  const int64_t n = static_cast<int64_t>(a.B) * a.H * a.T * (a.D / 8);
  const dim3 grid(static_cast<unsigned>((n + 255) / 256), a.n_out);
  if (a.bf16) split_reduce_kernel<true><<<grid, 256, 0, stream>>>(a);
  else split_reduce_kernel<false><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

// gamma = sum of the shares' sum P G_dS; rho = A2 - delta gamma - gamma A4 + A3
// from the summed A2 = sum P G_dS dP, A3 = sum P (dO u_v^T), A4 = sum P dP (the
// identity the stats pass uses unsplit). One thread per row.
__global__ void __launch_bounds__(256) stats_reduce_kernel(StatsReduceArgs a) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t rows = static_cast<int64_t>(a.BH) * a.t_pad;
  if (row >= rows) return;
  float g = 0.f, a2 = 0.f, a3 = 0.f, a4 = 0.f;
  for (int s = 0; s < a.nsplit; ++s) {
    const float4 v = a.part[static_cast<int64_t>(s) * rows + row];
    g += v.x;
    a2 += v.y;
    a3 += v.z;
    a4 += v.w;
  }
  const bool valid = static_cast<int>(row % a.t_pad) < a.T;
  a.gamma[row] = valid ? g : 0.f;
  a.rho[row] = valid ? a2 - a.delta[row] * g - g * a4 + a3 : 0.f;
}

cudaError_t launch_stats_reduce(const StatsReduceArgs& a, cudaStream_t stream) {
  if (a.nsplit < 1) return cudaErrorInvalidValue;
  const int64_t rows = static_cast<int64_t>(a.BH) * a.t_pad;
  stats_reduce_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

// One thread per 8 columns of a row (the thread of column group 0 also writes lse2).
template <bool BF16>
__global__ void __launch_bounds__(256) fwd_combine_kernel(FwdCombineArgs a) {
  const int per_row = a.D / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t rows = static_cast<int64_t>(a.B) * a.H * a.t_pad;
  if (idx >= rows * per_row) return;
  const int c8 = static_cast<int>(idx % per_row);
  const int64_t row = idx / per_row;  // bh * t_pad + t
  const int t = static_cast<int>(row % a.t_pad);
  if (t >= a.T) {
    if (c8 == 0) a.lse2[row] = INFINITY;
    return;
  }
  float M = -INFINITY;
  for (int s = 0; s < a.nsplit; ++s) M = fmaxf(M, a.part_ml[static_cast<int64_t>(s) * rows + row].x);
  float L = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < a.nsplit; ++s) {
    const float2 ml = a.part_ml[static_cast<int64_t>(s) * rows + row];
    if (ml.y == 0.f) continue;  // a share without keys for this row
    const float w = exp2f(ml.x - M);
    L += w * ml.y;
    const float4* src = reinterpret_cast<const float4*>(a.part_o + (static_cast<int64_t>(s) * rows + row) * a.D + c8 * 8);
    const float4 x = src[0], y = src[1];
    o[0] += w * x.x; o[1] += w * x.y; o[2] += w * x.z; o[3] += w * x.w;
    o[4] += w * y.x; o[5] += w * y.y; o[6] += w * y.z; o[7] += w * y.w;
  }
  const float inv = 1.f / L;
  uint4 v;
  v.x = pack2<BF16>(o[0] * inv, o[1] * inv);
  v.y = pack2<BF16>(o[2] * inv, o[3] * inv);
  v.z = pack2<BF16>(o[4] * inv, o[5] * inv);
  v.w = pack2<BF16>(o[6] * inv, o[7] * inv);
  const int bh = static_cast<int>(row / a.t_pad);
  const int b = bh / a.H, h = bh % a.H;
  *reinterpret_cast<uint4*>(a.out + b * a.sb + h * a.sh + static_cast<int64_t>(t) * a.st + c8 * 8) = v;
  if (c8 == 0) a.lse2[row] = M + log2f(L);
}

cudaError_t launch_fwd_combine(const FwdCombineArgs& a, cudaStream_t stream) {
  if (a.nsplit < 1 || (a.D % 8) != 0) return cudaErrorInvalidValue;
  const int64_t n = static_cast<int64_t>(a.B) * a.H * a.t_pad * (a.D / 8);
  const dim3 grid(static_cast<unsigned>((n + 255) / 256));
  if (a.bf16) fwd_combine_kernel<true><<<grid, 256, 0, stream>>>(a);
  else fwd_combine_kernel<false><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- self-test
// C[128 x N] = A[128 x K] * B, B K-major ([N x K] rows) or MN-major ([K x N] rows).
struct SelftestParams {
  CUtensorMap ta, tb;
  const uint16_t* a;  // row-major A, read directly when A sits in TMEM
  float* c;
  int n, k;
  int* err;
};

template <bool BF16, bool B_MN, bool A_TMEM>
__global__ void __launch_bounds__(128, 1) selftest_umma_kernel(const __grid_constant__ SelftestParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;                 // PL(128, K)
  uint8_t* sB = smem + 128 * 128 * 2;  // PL(N, K) or PL(K, N), at most 256 x 128
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 128 * 128 * 2 + 256 * 128 * 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5;
  const int N = p.n, K = p.k;
  if (threadIdx.x == 0) {
    mbar_init(bars + 0, 1);
    mbar_init(bars + 1, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  Guard g{abort_flag, p.err, nullptr};
  if constexpr (A_TMEM) {
    // Row r of A (this thread's lane) into TMEM columns 256 .. 256+K/2, two
    // 16-bit elements per 32-bit column, low half first.
    const int r = threadIdx.x;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t* arow = reinterpret_cast<const uint32_t*>(p.a) + r * (K / 2);
    for (int c0 = 0; c0 < K / 2; c0 += 16) {
      uint32_t w[16];
      for (int j = 0; j < 16; ++j) w[j] = arow[c0 + j];
      tmem_st16_raw(tmem + lane_off + 256 + c0, w);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (threadIdx.x == 0) {
    const int bytes = (A_TMEM ? 0 : 128 * K * 2) + N * K * 2;
    mbar_arrive_tx(bars + 0, bytes);
    if (!A_TMEM)
      for (int pp = 0; pp < K / 64; ++pp) tma_load_4d(sA + pp * 128 * 128, &p.ta, bars + 0, pp * 64, 0, 0, 0);
    if (B_MN) {
      for (int pp = 0; pp < N / 64; ++pp) tma_load_4d(sB + pp * K * 128, &p.tb, bars + 0, pp * 64, 0, 0, 0);
    } else {
      for (int pp = 0; pp < K / 64; ++pp) tma_load_4d(sB + pp * N * 128, &p.tb, bars + 0, pp * 64, 0, 0, 0);
    }
    if (mbar_wait(bars + 0, 0, g, 1)) {
      tc_fence_after();
      const uint32_t idesc = idesc_f16(128, N, BF16, false, B_MN);
      for (int kk = 0; kk < K / 16; ++kk) {
        const uint64_t db = B_MN ? desc_mnmajor(smem_u32(sB), K, kk) : desc_kmajor(smem_u32(sB), N, kk);
        if constexpr (A_TMEM) {
          umma_ts(tmem, tmem + 256 + kk * 8, db, idesc, kk > 0 ? 1u : 0u);
        } else {
          umma_ss(tmem, desc_kmajor(smem_u32(sA), 128, kk), db, idesc, kk > 0 ? 1u : 0u);
        }
      }
      umma_commit(bars + 1);
    } else {
      mbar_drain(bars + 0, 0);
      umma_commit(bars + 1);
    }
  }
  __syncwarp();
  if (mbar_wait(bars + 1, 0, g, 2)) {
    tc_fence_after();
    const int r = threadIdx.x;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    for (int c0 = 0; c0 < N; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + lane_off + c0, v);
      for (int j = 0; j < 32; ++j) p.c[r * N + c0 + j] = v[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

cudaError_t launch_selftest_umma(const CUtensorMap& ta, const CUtensorMap& tb, const void* a, float* c, int n, int k,
                                 bool bf16, bool b_mn_major, bool a_tmem, int* err, cudaStream_t stream) {
  SelftestParams p;
  p.ta = ta;
  p.tb = tb;
  p.a = static_cast<const uint16_t*>(a);
  p.c = c;
  p.n = n;
  p.k = k;
  p.err = err;
  const int smem = 128 * 128 * 2 + 256 * 128 * 2 + 64 + 1024;
  auto launch = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<1, 128, smem, stream>>>(p);
    return cudaGetLastError();
  };
  if (a_tmem) {
    if (!bf16 && !b_mn_major) return launch(selftest_umma_kernel<false, false, true>);
    if (!bf16 && b_mn_major) return launch(selftest_umma_kernel<false, true, true>);
    if (bf16 && !b_mn_major) return launch(selftest_umma_kernel<true, false, true>);
    return launch(selftest_umma_kernel<true, true, true>);
  }
  if (!bf16 && !b_mn_major) return launch(selftest_umma_kernel<false, false, false>);
  if (!bf16 && b_mn_major) return launch(selftest_umma_kernel<false, true, false>);
  if (bf16 && !b_mn_major) return launch(selftest_umma_kernel<true, false, false>);
  return launch(selftest_umma_kernel<true, true, false>);
}

// Failure-path self-test of the bounded waits: one thread initializes an
// mbarrier that expects one arrival and waits on its first phase with the same
// mbar_wait every kernel uses, but with the caller's limit. Nothing arrives
// and no TMA or UMMA work is in flight, so the wait runs out after limit_ns,
// records kErrTimeout | (kSelftestWaitSite << 8) in the error word (and its
// host-mapped mirror) and returns: the kernel ends normally, the context stays
// usable.
constexpr int kSelftestWaitSite = 0xfe;
__global__ void __launch_bounds__(32, 1) selftest_wait_kernel(unsigned long long limit_ns, int* err, int* err_host) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  abort_flag = 0;
  fence_mbar_init();
  Guard g{&abort_flag, err, err_host};
  if (mbar_wait(&bar, 0, g, kSelftestWaitSite, limit_ns)) {
    // cannot happen (nothing arrives); reported so that a test would notice
    report_error(err, err_host, kErrMisaligned);
  }
}

cudaError_t launch_selftest_wait(unsigned long long limit_ns, int* err, int* err_host, cudaStream_t stream) {
  selftest_wait_kernel<<<1, 32, 0, stream>>>(limit_ns, err, err_host);
  return cudaGetLastError();
}

}  // namespace ttt
