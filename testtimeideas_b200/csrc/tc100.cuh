// sm_100a building blocks for the attention kernels: mbarriers with bounded
// waits, TMA tile loads, tcgen05 tensor-memory allocation, UMMA issue/commit,
// TMEM <-> register moves and the shared-memory / instruction descriptors.
//
// Every wait in this file is bounded: a wait that does not complete within
// kWaitLimitNs sets the CTA's abort flag and the global error word, and
// returns false so the caller can drain and exit instead of hanging the GPU.
//
// No load in this file (or anywhere in the library) uses cluster-wide
// delivery: every CTA issues its own TMA loads into its own shared memory.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#define TTT_DEV __device__ __forceinline__

namespace ttt {

// ---------------------------------------------------------------- errors
// Error word layout written by kernels into the caller's err_flag (int32):
// 0 = ok; otherwise kErrTimeout | (site << 8) | (blockIdx-derived low bits).
constexpr int kErrTimeout = 0x40000000;
constexpr int kErrMisaligned = 0x20000000;  // dynamic shared memory base not 1024-aligned
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

TTT_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

TTT_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
TTT_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
TTT_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// One arrival that also announces `bytes` of TMA transactions.
TTT_DEV void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
TTT_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
TTT_DEV uint32_t mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done;
}

// Shared abort/error context of one CTA.
struct Guard {
  volatile int* abort;  // shared memory flag, set by the first wait that times out
  int* err;             // global error word (may be null)
  int* err_host;        // host-mapped mirror of the error word (may be null)
};

// Record an error: the first code wins in the device word; the host-mapped
// mirror (pinned host memory the binding registered) receives it too, so the
// host sees it without synchronizing. Only error paths call this.
TTT_DEV void report_error(int* err, int* err_host, int code) {
  if (err) atomicCAS(err, 0, code);
  if (err_host) {
    *reinterpret_cast<volatile int*>(err_host) = code;
    __threadfence_system();
  }
}

// Bounded parity wait. Returns true when the phase with `parity` completed,
// false if this CTA is aborting (timeout here or elsewhere in the CTA).
TTT_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, const Guard& g, int site,
                       unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_test(bar, parity)) return true;
    if ((it & 15u) == 0) {
      if (*g.abort) return false;
      // another CTA of this grid (or an earlier launch) already gave up
      if ((it & 255u) == 0 && g.err && *reinterpret_cast<volatile int*>(g.err) != 0) {
        *g.abort = 1;
        return false;
      }
      if (global_ns() - t0 > limit_ns) {
        *g.abort = 1;
        report_error(g.err, g.err_host, kErrTimeout | ((site & 0xff) << 8) | (blockIdx.x & 0xff));
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
TTT_DEV void tma_prefetch(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled load (coordinates innermost first) into this CTA's shared memory.
TTT_DEV void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Bring a 4-D tile into L2 ahead of its load (no shared memory, no barrier):
// a later tma_load_4d of the same box then reads it from L2.
TTT_DEV void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// 2-D tiled load (coordinates innermost first).
TTT_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled reduce-add of a shared-memory box into global memory (fp32 add in
// L2 by the TMA unit), tracked by this thread's bulk async-group. The
// coordinates are never negative here.
TTT_DEV void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
      : "memory");
}
TTT_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's bulk groups have finished reading shared memory /
// have completed entirely.
TTT_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
TTT_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor core / TMA) before signalling the consumer.
TTT_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05
// Warp-collective TMEM allocation; the base address is written to *dst.
TTT_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
TTT_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
TTT_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
TTT_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TTT_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]   (kind::f16: fp16 or bf16 operands, fp32 accumulate)
TTT_DEV void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]: A is M x K 16-bit, row m in TMEM lane m,
// elements (m, 2j) and (m, 2j+1) packed low/high in 32-bit column j.
TTT_DEV void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05 op previously issued by this
// thread has completed.
TTT_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Load 32 consecutive 32-bit TMEM columns of this thread's lane and wait for
// them (lane = warp's quarter * 32 + laneid, set in `taddr` by the caller).
TTT_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Same for 16 columns.
TTT_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive 32-bit TMEM columns of this thread's lane and wait.
TTT_DEV void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n\t"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

// Store 16 consecutive 32-bit TMEM columns of this thread's lane from raw
// words (no wait; pair with tmem_wait_st()).
TTT_DEV void tmem_st16_raw(uint32_t taddr, const uint32_t (&w)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n" ::"r"(taddr),
      "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]),
      "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15])
      : "memory");
}
TTT_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- register split
// Per-warpgroup register budget (setmaxnreg). Every warp of a warpgroup must
// execute the same one. The increases draw on registers released by the
// decreases out of the block's launch allocation (threads x registers at
// launch), so the new budgets, summed over the block's warpgroups, must not
// exceed that allocation; the host checks the sum against the kernel's
// register count before launching.
template <int N>
TTT_DEV void regs_release() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg takes a multiple of 8 in [24, 256]");
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(N));
}
template <int N>
TTT_DEV void regs_claim() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg takes a multiple of 8 in [24, 256]");
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(N));
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor, 128-byte swizzle (the layout TMA writes for
// a box whose inner extent is 128 bytes). Fields: start address >> 4 [0,14),
// leading byte offset >> 4 [16,30), stride byte offset >> 4 [32,46),
// descriptor version 1 at bit 46, swizzle mode 2 (128B) at [61,64).
TTT_DEV uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation:
// D format [4,6)=1 (f32), A format [7,10), B format [10,13) (0 f16, 1 bf16),
// A major bit 15, B major bit 16 (0 = K-major, 1 = MN-major),
// N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------- tile layout
// "Panel" layout PL(R, C) of a 16-bit [R x C] tile in shared memory, C a
// multiple of 64: C/64 column panels, each R rows x 128 bytes, panel p at byte
// p*R*128; within a panel row r sits at r*128 and its 16-byte chunk c is stored
// at chunk position (c ^ (r & 7)). A TMA load of a [R x 64] box with 128-byte
// swizzle into a 1024-aligned buffer produces exactly one such panel.
//
// K-major operand view (rows = M or N, columns = K): UMMA K-step kk (16
// elements) starts at panel kk/4, byte (kk%4)*32; stride byte offset 1024
// (8-row groups), leading byte offset unused (16).
TTT_DEV uint64_t desc_kmajor(uint32_t tile_saddr, int rows, int kk) {
  const uint32_t a = tile_saddr + static_cast<uint32_t>((kk >> 2) * rows * 128 + (kk & 3) * 32);
  return sdesc_sw128(a, 16, 1024);
}
// MN-major operand view (rows = K, columns = M or N): K-step kk covers rows
// 16*kk .. 16*kk+15 (two 8-row groups 1024 bytes apart); consecutive 64-wide
// MN panels are rows*128 bytes apart (leading byte offset).
TTT_DEV uint64_t desc_mnmajor(uint32_t tile_saddr, int rows, int kk) {
  const uint32_t a = tile_saddr + static_cast<uint32_t>(kk * 2048);
  return sdesc_sw128(a, static_cast<uint32_t>(rows * 128), 1024);
}

// ---------------------------------------------------------------- batched issue with barrier probes
// A satisfied mbarrier.try_wait takes ~160 cycles on the issuing thread, and the
// tensor core's instruction queue covers only ~40 cycles of issue gaps, so
// every wait between UMMA batches idles the tensor pipe. These helpers issue
// the K-steps of one product (4 or 8 UMMAs, kind::f16) in a single asm
// statement that starts with try_wait probes of two barrier phases and reads
// their results only after the UMMAs are queued: the probes' latency overlaps
// the issue. The returned bits (bit0: bar0's phase par0 complete, bit1: bar1's)
// let the caller skip waits that are already satisfied; a clear bit means
// "not yet", and the caller falls back to a bounded mbar_wait.
//
// L describes the per-K-step offsets of the A and B operands relative to
// K-step 0, as compile-time constants L::a(kk), L::b(kk): descriptor units (16
// bytes) for shared-memory operands, columns for an A operand in TMEM.
template <int ROWS>
struct KOffK {  // K-major PL tile with ROWS rows: K-step kk at panel kk/4, byte (kk%4)*32
  static constexpr int at(int kk) { return ((kk >> 2) * ROWS * 128 + (kk & 3) * 32) >> 4; }
};
struct KOffMN {  // MN-major PL tile: K-step kk at row 16*kk
  static constexpr int at(int kk) { return (kk * 2048) >> 4; }
};
struct KOffT {  // A operand in TMEM, K-steps packed contiguously: 8 columns per K-step
  static constexpr int at(int kk) { return kk * 8; }
};
template <class A, class B>
struct KOff2 {
  static constexpr int a(int kk) { return A::at(kk); }
  static constexpr int b(int kk) { return B::at(kk); }
};

template <class L>
TTT_DEV uint32_t umma_ss4_probe(uint32_t d, uint64_t a0, uint64_t b0, uint32_t idesc, uint32_t acc_first,
                                 const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1) {
  uint32_t r0, r1;
  asm volatile(
      "{\n\t.reg .pred p0, p1, q, t;\n\t.reg .b64 da, db;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p0, [%2], %3;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p1, [%4], %5;\n\t"
      "setp.ne.b32 q, %9, 0;\n\tsetp.eq.b32 t, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%6], %7, %8, %10, q;\n\t"
      "add.s64 da, %7, %11; add.s64 db, %8, %14; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %12; add.s64 db, %8, %15; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %13; add.s64 db, %8, %16; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "selp.u32 %0, 1, 0, p0;\n\tselp.u32 %1, 1, 0, p1;\n\t}\n"
      : "=r"(r0), "=r"(r1)
      : "r"(smem_u32(bar0)), "r"(par0), "r"(smem_u32(bar1)), "r"(par1), "r"(d), "l"(a0), "l"(b0), "r"(acc_first),
        "r"(idesc), "n"(L::a(1)), "n"(L::a(2)), "n"(L::a(3)), "n"(L::b(1)), "n"(L::b(2)), "n"(L::b(3))
      : "memory");
  return r0 | (r1 << 1);
}

template <class L>
TTT_DEV uint32_t umma_ts4_probe(uint32_t d, uint32_t a0, uint64_t b0, uint32_t idesc, uint32_t acc_first,
                                 const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1) {
  uint32_t r0, r1;
  asm volatile(
      "{\n\t.reg .pred p0, p1, q, t;\n\t.reg .b32 ta;\n\t.reg .b64 db;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p0, [%2], %3;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p1, [%4], %5;\n\t"
      "setp.ne.b32 q, %9, 0;\n\tsetp.eq.b32 t, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%6], [%7], %8, %10, q;\n\t"
      "add.u32 ta, %7, %11; add.s64 db, %8, %14; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %12; add.s64 db, %8, %15; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %13; add.s64 db, %8, %16; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "selp.u32 %0, 1, 0, p0;\n\tselp.u32 %1, 1, 0, p1;\n\t}\n"
      : "=r"(r0), "=r"(r1)
      : "r"(smem_u32(bar0)), "r"(par0), "r"(smem_u32(bar1)), "r"(par1), "r"(d), "r"(a0), "l"(b0), "r"(acc_first),
        "r"(idesc), "n"(L::a(1)), "n"(L::a(2)), "n"(L::a(3)), "n"(L::b(1)), "n"(L::b(2)), "n"(L::b(3))
      : "memory");
  return r0 | (r1 << 1);
}

template <class L>
TTT_DEV uint32_t umma_ss8_probe(uint32_t d, uint64_t a0, uint64_t b0, uint32_t idesc, uint32_t acc_first,
                                 const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1) {
  uint32_t r0, r1;
  asm volatile(
      "{\n\t.reg .pred p0, p1, q, t;\n\t.reg .b64 da, db;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p0, [%2], %3;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p1, [%4], %5;\n\t"
      "setp.ne.b32 q, %9, 0;\n\tsetp.eq.b32 t, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%6], %7, %8, %10, q;\n\t"
      "add.s64 da, %7, %11; add.s64 db, %8, %18; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %12; add.s64 db, %8, %19; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %13; add.s64 db, %8, %20; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %14; add.s64 db, %8, %21; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %15; add.s64 db, %8, %22; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %16; add.s64 db, %8, %23; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "add.s64 da, %7, %17; add.s64 db, %8, %24; tcgen05.mma.cta_group::1.kind::f16 [%6], da, db, %10, t;\n\t"
      "selp.u32 %0, 1, 0, p0;\n\tselp.u32 %1, 1, 0, p1;\n\t}\n"
      : "=r"(r0), "=r"(r1)
      : "r"(smem_u32(bar0)), "r"(par0), "r"(smem_u32(bar1)), "r"(par1), "r"(d), "l"(a0), "l"(b0), "r"(acc_first),
        "r"(idesc), "n"(L::a(1)), "n"(L::a(2)), "n"(L::a(3)), "n"(L::a(4)), "n"(L::a(5)), "n"(L::a(6)), "n"(L::a(7)), "n"(L::b(1)), "n"(L::b(2)), "n"(L::b(3)), "n"(L::b(4)), "n"(L::b(5)), "n"(L::b(6)), "n"(L::b(7))
      : "memory");
  return r0 | (r1 << 1);
}

template <class L>
TTT_DEV uint32_t umma_ts8_probe(uint32_t d, uint32_t a0, uint64_t b0, uint32_t idesc, uint32_t acc_first,
                                 const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1) {
  uint32_t r0, r1;
  asm volatile(
      "{\n\t.reg .pred p0, p1, q, t;\n\t.reg .b32 ta;\n\t.reg .b64 db;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p0, [%2], %3;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p1, [%4], %5;\n\t"
      "setp.ne.b32 q, %9, 0;\n\tsetp.eq.b32 t, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%6], [%7], %8, %10, q;\n\t"
      "add.u32 ta, %7, %11; add.s64 db, %8, %18; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %12; add.s64 db, %8, %19; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %13; add.s64 db, %8, %20; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %14; add.s64 db, %8, %21; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %15; add.s64 db, %8, %22; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %16; add.s64 db, %8, %23; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %17; add.s64 db, %8, %24; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "selp.u32 %0, 1, 0, p0;\n\tselp.u32 %1, 1, 0, p1;\n\t}\n"
      : "=r"(r0), "=r"(r1)
      : "r"(smem_u32(bar0)), "r"(par0), "r"(smem_u32(bar1)), "r"(par1), "r"(d), "r"(a0), "l"(b0), "r"(acc_first),
        "r"(idesc), "n"(L::a(1)), "n"(L::a(2)), "n"(L::a(3)), "n"(L::a(4)), "n"(L::a(5)), "n"(L::a(6)), "n"(L::a(7)), "n"(L::b(1)), "n"(L::b(2)), "n"(L::b(3)), "n"(L::b(4)), "n"(L::b(5)), "n"(L::b(6)), "n"(L::b(7))
      : "memory");
  return r0 | (r1 << 1);
}

// umma_ts4_probe with non-suspending probes (mbarrier.test_wait): for a barrier
// that may still be incomplete when the batch is issued, where a suspending
// try_wait would hold back the UMMAs behind it.
template <class L>
TTT_DEV uint32_t umma_ts4_tprobe(uint32_t d, uint32_t a0, uint64_t b0, uint32_t idesc, uint32_t acc_first,
                                 const uint64_t* bar0, uint32_t par0, const uint64_t* bar1, uint32_t par1) {
  uint32_t r0, r1;
  asm volatile(
      "{\n\t.reg .pred p0, p1, q, t;\n\t.reg .b32 ta;\n\t.reg .b64 db;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p0, [%2], %3;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p1, [%4], %5;\n\t"
      "setp.ne.b32 q, %9, 0;\n\tsetp.eq.b32 t, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%6], [%7], %8, %10, q;\n\t"
      "add.u32 ta, %7, %11; add.s64 db, %8, %14; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %12; add.s64 db, %8, %15; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "add.u32 ta, %7, %13; add.s64 db, %8, %16; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %10, t;\n\t"
      "selp.u32 %0, 1, 0, p0;\n\tselp.u32 %1, 1, 0, p1;\n\t}\n"
      : "=r"(r0), "=r"(r1)
      : "r"(smem_u32(bar0)), "r"(par0), "r"(smem_u32(bar1)), "r"(par1), "r"(d), "r"(a0), "l"(b0), "r"(acc_first),
        "r"(idesc), "n"(L::a(1)), "n"(L::a(2)), "n"(L::a(3)), "n"(L::b(1)), "n"(L::b(2)), "n"(L::b(3))
      : "memory");
  return r0 | (r1 << 1);
}

// Two products into one accumulator, A from TMEM, their four K-steps
// interleaved (A0 B0, A1 B1 for each K-step), issued as one batch behind two
// barrier probes. Unlike umma_ss8_probe the probes use the non-suspending
// mbarrier.test_wait, so an incomplete phase never delays the UMMAs. Only the
// very first UMMA takes acc_first; every later one accumulates.
template <class L>
TTT_DEV uint32_t umma_ts_pair4_probe(uint32_t d, uint32_t a0, uint64_t b0, uint32_t a1, uint64_t b1, uint32_t idesc,
                                      uint32_t acc_first, const uint64_t* bar0, uint32_t par0, const uint64_t* bar1,
                                      uint32_t par1) {
  uint32_t r0, r1;
  asm volatile(
      "{\n\t.reg .pred p0, p1, q, t;\n\t.reg .b32 ta;\n\t.reg .b64 db;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p0, [%2], %3;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p1, [%4], %5;\n\t"
      "setp.ne.b32 q, %11, 0;\n\tsetp.eq.b32 t, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%6], [%7], %8, %12, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%6], [%9], %10, %12, t;\n\t"
      "add.u32 ta, %7, %13; add.s64 db, %8, %16; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %12, t;\n\t"
      "add.u32 ta, %9, %13; add.s64 db, %10, %16; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %12, t;\n\t"
      "add.u32 ta, %7, %14; add.s64 db, %8, %17; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %12, t;\n\t"
      "add.u32 ta, %9, %14; add.s64 db, %10, %17; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %12, t;\n\t"
      "add.u32 ta, %7, %15; add.s64 db, %8, %18; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %12, t;\n\t"
      "add.u32 ta, %9, %15; add.s64 db, %10, %18; tcgen05.mma.cta_group::1.kind::f16 [%6], [ta], db, %12, t;\n\t"
      "selp.u32 %0, 1, 0, p0;\n\tselp.u32 %1, 1, 0, p1;\n\t}\n"
      : "=r"(r0), "=r"(r1)
      : "r"(smem_u32(bar0)), "r"(par0), "r"(smem_u32(bar1)), "r"(par1), "r"(d), "r"(a0), "l"(b0), "r"(a1), "l"(b1),
        "r"(acc_first), "r"(idesc), "n"(L::a(1)), "n"(L::a(2)), "n"(L::a(3)), "n"(L::b(1)), "n"(L::b(2)),
        "n"(L::b(3))
      : "memory");
  return r0 | (r1 << 1);
}

// Byte offset of element (r, c) in PL(R, C) (16-bit elements).
TTT_DEV uint32_t pl_offset(int R, int r, int c) {
  const int panel = c >> 6;
  const int chunk = (c >> 3) & 7;
  const int within = c & 7;
  return static_cast<uint32_t>(panel * R * 128 + r * 128 + ((chunk ^ (r & 7)) << 4) + within * 2);
}

// ---------------------------------------------------------------- math
TTT_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BF16>
TTT_DEV uint32_t pack2(float lo, float hi);
template <>
TTT_DEV uint32_t pack2<false>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
TTT_DEV uint32_t pack2<true>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <bool BF16>
TTT_DEV float to_f32(uint16_t bits);
template <>
TTT_DEV float to_f32<false>(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}
template <>
TTT_DEV float to_f32<true>(uint16_t bits) {
  return __bfloat162float(__ushort_as_bfloat16(bits));
}

// Write 64 consecutive values (columns c0..c0+63, c0 % 64 == 0) of row r into
// a PL(R, C) tile: eight 16-byte stores, conflict-free across a warp of rows.
template <bool BF16>
TTT_DEV void store_row64(uint8_t* tile, int R, int r, int c0, const float* v) {
  uint8_t* rowp = tile + (c0 >> 6) * R * 128 + r * 128;
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    uint4 w;
    w.x = pack2<BF16>(v[ch * 8 + 0], v[ch * 8 + 1]);
    w.y = pack2<BF16>(v[ch * 8 + 2], v[ch * 8 + 3]);
    w.z = pack2<BF16>(v[ch * 8 + 4], v[ch * 8 + 5]);
    w.w = pack2<BF16>(v[ch * 8 + 6], v[ch * 8 + 7]);
    *reinterpret_cast<uint4*>(rowp + ((ch ^ (r & 7)) << 4)) = w;
  }
}

// Write 32 consecutive values (columns c0..c0+31, c0 % 32 == 0) of row r.
template <bool BF16>
TTT_DEV void store_row32(uint8_t* tile, int R, int r, int c0, const float* v) {
  uint8_t* rowp = tile + (c0 >> 6) * R * 128 + r * 128;
  const int ch0 = (c0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack2<BF16>(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = pack2<BF16>(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = pack2<BF16>(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = pack2<BF16>(v[q * 8 + 6], v[q * 8 + 7]);
    *reinterpret_cast<uint4*>(rowp + (((ch0 + q) ^ (r & 7)) << 4)) = w;
  }
}

}  // namespace ttt
