// Helpers shared by the pipelined backward kernels: batched TMEM loads with a
// single wait, column-slice stores into the swizzled shared-memory tiles, and
// the named barrier of the compute warps.
#pragma once

#include "attn_common.cuh"

namespace ttt {

// Issue a 16- or 32-column TMEM load without waiting; call tmem_wait_ld()
// and reg_fence() before reading the registers.
TTT_DEV void tmem_ld16_nw(uint32_t taddr, float (&v)[16]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

TTT_DEV void tmem_ld32_nw(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

template <int W>
TTT_DEV void tmem_ld_nw(uint32_t taddr, float (&v)[W]) {
  static_assert(W == 16 || W == 32 || W == 64, "");
  if constexpr (W == 16) {
    tmem_ld16_nw(taddr, v);
  } else if constexpr (W == 32) {
    tmem_ld32_nw(taddr, v);
  } else {
    tmem_ld32_nw(taddr, *reinterpret_cast<float(*)[32]>(v));
    tmem_ld32_nw(taddr + 32, *reinterpret_cast<float(*)[32]>(v + 32));
  }
}

TTT_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Orders the reads of registers filled by an asynchronous TMEM load after the
// preceding tcgen05.wait::ld (volatile asm statements keep their order).
template <int N>
TTT_DEV void reg_fence(float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+f"(v[i]));
}

// Write W (16, 32 or 64) consecutive values of row r, columns c0 .. c0+W-1
// (c0 a multiple of W inside one 64-column panel), into a PL(R, C) tile.
template <bool BF16, int W>
TTT_DEV void store_cols(uint8_t* tile, int R, int r, int c0, const float* v) {
  uint8_t* rowp = tile + (c0 >> 6) * R * 128 + r * 128;
  const int ch0 = (c0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < W / 8; ++q) {
    uint4 w;
    w.x = pack2<BF16>(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = pack2<BF16>(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = pack2<BF16>(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = pack2<BF16>(v[q * 8 + 6], v[q * 8 + 7]);
    *reinterpret_cast<uint4*>(rowp + (((ch0 + q) ^ (r & 7)) << 4)) = w;
  }
}

// ---------------------------------------------------------------- packed fp32x2
// Two independent fp32 lanes in one 64-bit register pair (sm_100a packed ops):
// the elementwise steps work on column pairs with half the instructions.
struct F2 {
  unsigned long long v;
};
TTT_DEV F2 f2(float lo, float hi) {
  F2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(lo), "f"(hi));
  return r;
}
TTT_DEV F2 f2s(float x) { return f2(x, x); }
TTT_DEV void split(F2 x, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(x.v)); }
TTT_DEV F2 add2(F2 a, F2 b) {
  F2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
TTT_DEV F2 sub2(F2 a, F2 b) {
  F2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
TTT_DEV F2 mul2(F2 a, F2 b) {
  F2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
TTT_DEV F2 fma2(F2 a, F2 b, F2 c) {
  F2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}

// The K-steps of one product, issued as one batch that also probes two barrier
// phases (see umma_ss8_probe). With PROBE false, or a K-step count without a
// probe helper, the K-steps are issued plainly and nothing is reported as seen
// (0): a probe costs ~44 cycles of issue, a loss where the waits it could
// replace are rarely satisfied in time.
template <int KS, class L, bool PROBE = true>
TTT_DEV uint32_t issue_ss(uint32_t d, uint64_t a0, uint64_t b0, uint32_t idesc, uint32_t acc_first,
                          const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1) {
  if constexpr (PROBE && KS == 8) {
    return umma_ss8_probe<L>(d, a0, b0, idesc, acc_first, bar0, par0, bar1, par1);
  } else if constexpr (PROBE && KS == 4) {
    return umma_ss4_probe<L>(d, a0, b0, idesc, acc_first, bar0, par0, bar1, par1);
  } else {
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
      umma_ss(d, a0 + L::a(kk), b0 + L::b(kk), idesc, kk > 0 ? 1u : acc_first);
    return 0u;
  }
}
template <int KS, class L, bool PROBE = true>
TTT_DEV uint32_t issue_ts(uint32_t d, uint32_t a0, uint64_t b0, uint32_t idesc, uint32_t acc_first,
                          const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1) {
  if constexpr (PROBE && KS == 8) {
    return umma_ts8_probe<L>(d, a0, b0, idesc, acc_first, bar0, par0, bar1, par1);
  } else if constexpr (PROBE && KS == 4) {
    return umma_ts4_probe<L>(d, a0, b0, idesc, acc_first, bar0, par0, bar1, par1);
  } else {
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) umma_ts(d, a0 + L::a(kk), b0 + L::b(kk), idesc, kk > 0 ? 1u : acc_first);
    return 0u;
  }
}

// Fire-and-forget vector add of four floats into global memory (the
// reduction happens in L2); dst must be 16-byte aligned.
TTT_DEV void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Named barrier 1 over the compute warps only (the producer and MMA warps
// never take part).
template <int NTHREADS>
TTT_DEV void compute_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(NTHREADS) : "memory");
}

// Copy `ncols` accumulator columns starting at col0 (a multiple of 32) of a
// TMEM row to a 16-bit global row, scaled by `mul`; warp-collective.
template <int NCOLS, bool BF16>
TTT_DEV void acc_cols_to_global(uint32_t taddr_row, int col0, uint16_t* dst_row, bool valid, float mul) {
#pragma unroll
  for (int c = 0; c < NCOLS / 32; ++c) {
    float v[32];
    tmem_ld32(taddr_row + col0 + c * 32, v);
    if (valid) store_global32<BF16>(dst_row + col0 + c * 32, v, mul);
  }
}

// Split mode: copy NCOLS fp32 accumulator columns col0.. of this thread's TMEM
// lane to an fp32 partial row (zeros when `have` is false: a share without
// tiles never wrote its accumulator). Warp-collective like the loads.
template <int NCOLS>
TTT_DEV void acc_cols_to_f32(uint32_t taddr_row, int col0, float* dst_row, bool have) {
#pragma unroll
  for (int c = 0; c < NCOLS / 32; ++c) {
    float v[32];
    if (have) {
      tmem_ld32(taddr_row + col0 + c * 32, v);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    float4* d4 = reinterpret_cast<float4*>(dst_row + col0 + c * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
}

}  // namespace ttt
