// Internal launch interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>

#include "attn_common.cuh"

namespace ttt {

cudaError_t launch_fwd(const KParams& p, int d, bool bf16, bool causal, bool save_p, cudaStream_t stream);
// The normalized P of the save_p forward after the row-LSE forward: own[0] = Q,
// str[0] = K, str[1] = P (map of encode_p, box 64 x 128), lse2 = the forward's
// rows; requires T % 8 == 0.
cudaError_t launch_pwrite(const KParams& p, int d, bool bf16, bool causal, cudaStream_t stream);
// Query-major passes: kind in {kBwdQ, kStats, kBwd2Q}; gdo selects dd_dO output (kBwd2Q only).
cudaError_t launch_qm(const KParams& p, int d, bool bf16, bool causal, int kind, bool gdo, cudaStream_t stream);
// Key-major passes: kind in {kBwdKV, kBwd2KV}.
cudaError_t launch_km(const KParams& p, int d, bool bf16, bool causal, int kind, cudaStream_t stream);
// Rows of the streamed tiles (and of the per-query statistics boxes) each pass
// expects in its tensor maps.
int qm_tile_cols(int d, int kind, bool gdo);
int km_tile_rows(int d, int kind);

// Passes that read the materialized probabilities P ([b, h, t, t], map in
// str[0]) instead of recomputing them.
enum FpMode : int {
  kFpDV = 0,      // dV = P^T dO                    (str[1] = dO)
  kFpRowsum = 1,  // rowsum = rowsum(dO o (P V))    (str[1] = V, raw[0] = dO, out_f0 = rowsum [b*h, t])
  kFpDK = 2,      // dK = scale dS^T Q              (own[0] = V, str[1] = dO, str[2] = Q, delta = rowsum [b*h, t])
  kFpDQ = 3,      // dQ = scale dS K                (own[0] = dO, str[1] = V, str[2] = K, delta = rowsum [b*h, t])
};
// Streamed rows per step of each from-P pass (measured best: 128 for the
// product-only passes and for kFpDK, 64 for kFpDQ).
constexpr int from_p_step_rows(int mode) { return mode == kFpDQ ? 64 : 128; }
// Rows of the P box and of the streamed [rows x d] tiles each mode expects.
inline int from_p_box_rows(int mode) { return mode == kFpDK ? from_p_step_rows(mode) : 128; }
inline int from_p_stream_rows(int mode) { return from_p_step_rows(mode); }
cudaError_t launch_from_p(const KParams& p, int d, bool bf16, bool causal, int mode, cudaStream_t stream);

// delta[bh, t] = sum_d dO[b,h,t,d] * O[b,h,t,d] for t < T, 0 for T <= t < t_pad.
struct DeltaArgs {
  const uint16_t* o;
  int64_t o_sb, o_sh, o_st;
  const uint16_t* dout;
  int64_t d_sb, d_sh, d_st;
  float* delta;
  int B, H, T, t_pad, D;
  bool bf16;
};
cudaError_t launch_delta(const DeltaArgs& a, cudaStream_t stream);

// Split-mode reduction: out[b, h, t, :] = scale * sum over s (in order) of
// part[s][b*h][t][:] for t < T, for up to two outputs (blockIdx.y).
struct SplitReduceArgs {
  const float* part[2];
  uint16_t* out[2];
  int64_t sb[2], sh[2], st[2];
  float scale[2];
  int n_out, nsplit;
  int B, H, T, t_pad, D;
  bool bf16;
};
cudaError_t launch_split_reduce(const SplitReduceArgs& a, cudaStream_t stream);

// Split-mode reduction of the row statistics: part holds per share the four row
// sums (sum P G_dS, sum P G_dS dP, sum P (dO u_v^T), sum P dP) as a float4 per
// row, [nsplit][b*h][t_pad]; writes gamma and rho for rows t < T, 0 beyond.
struct StatsReduceArgs {
  const float4* part;
  const float* delta;
  float* gamma;
  float* rho;
  int nsplit, BH, T, t_pad;
};
cudaError_t launch_stats_reduce(const StatsReduceArgs& a, cudaStream_t stream);

// Split-mode combination of the forward: per row and share, an unnormalized O
// row (part_o, [nsplit][b*h][t_pad][d]) with its running max m (base-2 log
// domain) and sum l (part_ml). Writes O = sum_s 2^(m_s - M) O_s / L and
// lse2 = M + log2 L, M = max_s m_s, L = sum_s 2^(m_s - M) l_s; rows t >= T get
// lse2 = +inf.
struct FwdCombineArgs {
  const float* part_o;
  const float2* part_ml;
  uint16_t* out;
  int64_t sb, sh, st;
  float* lse2;
  int nsplit, B, H, T, t_pad, D;
  bool bf16;
};
cudaError_t launch_fwd_combine(const FwdCombineArgs& a, cudaStream_t stream);

// Self-test GEMM used to validate descriptor conventions: C = A B with A a
// 128 x K tile (K-major) and B either N x K (K-major, "score" form) or K x N
// (MN-major, "accumulate" form); inputs through the same 4-D tensor maps.
// With a_tmem the A tile is copied into TMEM and the product is issued with A
// from TMEM (the TS form).
// Runs one bounded mbarrier wait that nothing completes (limit_ns, then the
// error word and its mirror receive kErrTimeout | (0xfe << 8)); see misc.cu.
cudaError_t launch_selftest_wait(unsigned long long limit_ns, int* err, int* err_host, cudaStream_t stream);

cudaError_t launch_selftest_umma(const CUtensorMap& ta, const CUtensorMap& tb, const void* a, float* c, int n, int k,
                                 bool bf16, bool b_mn_major, bool a_tmem, int* err, cudaStream_t stream);

}  // namespace ttt
