// Kernel-side parameter block and helpers shared by the forward, backward and
// double-backward attention kernels.
//
// Data layout in HBM (per head bh = b*H + h):
//   Q, K, V, dO, u_q, u_k, u_v : [b, h, T, d] 16-bit, arbitrary b/h/t strides
//                                (multiples of 8 elements), unit d stride;
//                                read only through TMA tensor maps.
//   lse2, delta, gamma, rho    : fp32 [b*h, t_pad], t_pad = roundup(T, 128).
//                                lse2 is the row log-sum-exp in base 2 of
//                                scale*log2(e)*Q K^T; rows in [T, t_pad) hold
//                                +inf (lse2) or 0 (the others).
//   outputs (O, dq, dk, dv, ...): [b, h, T, d] 16-bit with given strides.
#pragma once

#include "tc100.cuh"

namespace ttt {

// Which pass a generic backward kernel instance runs.
enum Kind : int {
  kBwdQ = 0,     // dQ (query-major)
  kStats = 1,    // gamma, rho row statistics of the double backward (query-major)
  kBwd2Q = 2,    // dd_q (+ dd_dO) of the double backward (query-major)
  kBwdKV = 3,    // dK, dV (key-major)
  kBwd2KV = 4,   // dd_k, dd_v of the double backward (key-major)
  kBwdKVQ = 5,   // dK, dV and dQ in one key-major pass (dQ added into an fp32 accumulator)
};

struct KParams {
  // Owner-side tiles (128 rows, resident for the whole CTA) and streamed tiles
  // (BN rows per step). Which tensor sits in which slot depends on the pass.
  CUtensorMap own[4];
  CUtensorMap str[4];
  // fp32 [b*h, t_pad] row statistics streamed per column tile (key-major).
  CUtensorMap st[4];
  // Raw views of the owner-side inputs (same slots as own[]), for kernels that
  // stage them in tensor memory with plain loads.
  const uint16_t* raw[4];
  int64_t raw_sb[4], raw_sh[4], raw_st[4];
  // Raw row statistics (query-major kernels read their own rows directly).
  const float* lse2;
  const float* delta;
  const float* gamma;
  const float* rho;
  // fp32 outputs (forward: lse2; stats pass: gamma, rho).
  float* out_f0;
  float* out_f1;
  // 16-bit outputs.
  uint16_t* out0;
  int64_t o0_sb, o0_sh, o0_st;
  uint16_t* out1;
  int64_t o1_sb, o1_sh, o1_st;
  int B, H, T, t_pad;
  int window;        // causal only, 0 = none: see Band
  int window_kind;   // 0 sliding window, 1 chunk-local (see Band)
  float scale;       // softmax scale applied to Q K^T
  float scale_log2;  // scale * log2(e)
  int* err;          // device error word (0 = ok), may be null
  int* err_host;     // host-mapped mirror of the error word, may be null
  // Split mode (nsplit > 1; passes that support it): grid column x works on head
  // x / nsplit and on share x % nsplit of its block's tile stream, and writes
  // unscaled fp32 partial results part0 / part1, [nsplit][b*h][t_pad][d], in place
  // of out0 / out1; a reduction kernel sums the shares in order afterwards.
  int nsplit;
  float* part0;
  float* part1;
  // kBwdKVQ: fp32 dQ accumulator [b*h][t_pad][d], zero before the pass; every
  // key block adds its dS K rows into it (unscaled), through the tensor map
  // st[2] (dims d, t_pad, b*h; box 32 x 128 x 1, 128-byte swizzle).
  float* acc_q;
};

// Launch order of a pass's CTAs, a grid of (units, blocks) with units = heads
// (times split shares): units are taken kUnitGroup at a time and, within a
// group, block rank by block rank, so that the CTAs running together share the
// streamed tiles of a few heads in L2. (Taking every head's first block first
// streams all heads' tiles at once, from DRAM, when there are many heads.)
// Returns this CTA's unit and its block rank (rank 0 is launched first).
constexpr int kUnitGroup = 4;
struct GridPos {
  int unit, rank;
};
TTT_DEV GridPos grid_pos() {
  const int units = static_cast<int>(gridDim.x), nblk = static_cast<int>(gridDim.y);
  const int64_t lin = blockIdx.x + static_cast<int64_t>(blockIdx.y) * gridDim.x;
  const int64_t per_group = static_cast<int64_t>(kUnitGroup) * nblk;
  const int group = static_cast<int>(lin / per_group);
  const int base = group * kUnitGroup;
  const int gs = min(kUnitGroup, units - base);
  const int idx = static_cast<int>(lin - group * per_group);
  return {base + idx % gs, idx / gs};
}

// Contiguous share `split` of `n` items cut into `nsplit` nearly equal parts.
TTT_DEV int split_begin(int n, int split, int nsplit) {
  return static_cast<int>((static_cast<int64_t>(n) * split) / nsplit);
}

// Causal attention with a lower bound on each row's visible keys: key j is
// visible to query i iff lo(i) <= j <= i. Kinds:
//   none          lo(i) = 0
//   sliding       lo(i) = max(0, i - W + 1)   (an additive mask from
//                 make_window_mask, cloud_ttt_e2e/ttt_e2e/utils.py:40-54)
//   chunk-local   queries in full chunks [cW, cW + W) see keys from cW; the
//                 queries of a last partial chunk see the last W keys: the
//                 chunk loop of WindowedSelfAttention for T > W
//                 (cloud_ttt_e2e/ttt_e2e/attention.py:112-127)
// lo is non-decreasing in i and last_query (the last query seeing key j) in j.
struct Band {
  int kind;  // 0 none, 1 sliding, 2 chunk-local
  int W, T, tf;  // tf = start of a partial last chunk (= T when there is none)
  TTT_DEV static Band make(const KParams& p, bool causal) {
    Band b;
    b.kind = (causal && p.window > 0) ? 1 + p.window_kind : 0;
    b.W = p.window > 0 ? p.window : 1;
    b.T = p.T;
    b.tf = (p.T / b.W) * b.W;
    return b;
  }
  TTT_DEV int lo(int i) const {
    if (kind == 1) return max(0, i - W + 1);
    if (kind == 2) return i < tf ? (i / W) * W : max(0, T - W);
    return 0;
  }
  TTT_DEV int last_query(int j) const {
    if (kind == 1) return j + W - 1;
    if (kind == 2) return (tf < T && j >= T - W) ? T - 1 : (j / W + 1) * W - 1;
    return 0x3fffffff;
  }
};

// Dynamic shared memory is only guaranteed 16-byte aligned; the 128-byte
// swizzle atoms need 1024-byte alignment.
TTT_DEV uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// Time-bounded wait used only while draining after an abort: it ignores the
// abort flag (the CTA is already aborting) but still gives up after the limit.
TTT_DEV void mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_test(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) return;
  }
}

// Store 32 fp32 values (a row segment) as 16-bit to global memory, 16-byte stores.
template <bool BF16>
TTT_DEV void store_global32(uint16_t* dst, const float* v, float mul) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack2<BF16>(v[q * 8 + 0] * mul, v[q * 8 + 1] * mul);
    w.y = pack2<BF16>(v[q * 8 + 2] * mul, v[q * 8 + 3] * mul);
    w.z = pack2<BF16>(v[q * 8 + 4] * mul, v[q * 8 + 5] * mul);
    w.w = pack2<BF16>(v[q * 8 + 6] * mul, v[q * 8 + 7] * mul);
    reinterpret_cast<uint4*>(dst)[q] = w;
  }
}

// Copy a [128 x D] fp32 accumulator from TMEM (columns col0..col0+D-1, lane =
// row) to a 16-bit global row, scaled by `mul`. All 32 lanes of the warp must
// call this (tcgen05.ld is warp-collective); only rows with `valid` store.
template <int D, bool BF16>
TTT_DEV void acc_to_global(uint32_t taddr_row, uint16_t* dst_row, bool valid, float mul) {
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    float v[32];
    tmem_ld32(taddr_row + c * 32, v);
    if (valid) store_global32<BF16>(dst_row + c * 32, v, mul);
  }
}

}  // namespace ttt
