/*
 * ttt_attn.h - C ABI of libttt_attn.so, the sm_100a (B200) grad-grad-safe
 * attention library.
 *
 * The library computes, per head, O = softmax(scale * Q K^T [causal mask]) V,
 * the first-order gradients (dQ, dK, dV) for an upstream dO, and the complete
 * second-order terms (the gradients of <dQ,u_q> + <dK,u_k> + <dV,u_v> with
 * respect to Q, K, V and, optionally, dO).
 *
 * Conventions shared by every entry point:
 *  - Tensors are [b, h, t, d] views in 16-bit floating point (fp16 or bf16),
 *    given as a device pointer plus element strides of the b, h and t
 *    dimensions; the d stride is 1. Strides must be positive multiples of 8
 *    elements (16 bytes) and pointers 16-byte aligned.
 *  - d must be 64 or 128.
 *  - Row statistics (lse2, delta, gamma, rho) are fp32 arrays [b*h, t_pad]
 *    with t_pad = ttt_attn_t_pad(t) = roundup(t, 128), owned by the caller.
 *  - Nothing here allocates device memory; all buffers come from the caller.
 *  - Optional work space (`work`, `work_bytes` in the pass arguments): a
 *    caller-owned device buffer of at least ttt_attn_work_bytes(pb) bytes,
 *    256-byte aligned, lets a pass whose grid is too small to fill the GPU
 *    (few heads, causal) split each CTA's stream of tiles over several CTAs
 *    and sum their fp32 partial results in a fixed order afterwards, and lets
 *    the d = 64 first-order backward compute dQ inside its key-major pass.
 *    With work == NULL or too small a buffer the passes run unsplit and dQ
 *    gets its own pass. The forms compute the same quantities; their fp32
 *    summation orders differ, so the 16-bit results may differ in the last
 *    bit.
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *    stream); no entry point synchronizes the host.
 *  - Return value: TTT_OK or a ttt_status code. Argument errors are detected
 *    on the host before anything is enqueued. `err` (optional, device int32)
 *    receives a nonzero code if a kernel gave up on a bounded wait
 *    (TTT_ERR_WORD_TIMEOUT | site << 8 | block bits); the caller reads it
 *    after synchronizing, or polls a registered host mirror
 *    (ttt_attn_error_mirror). While it is nonzero, kernels given that word
 *    exit at once: the caller clears it (in stream order) to go on.
 *
 * Reference interface each entry point replaces (paths inside
 * ry2009/TestTimeIdeas) is cited on the declaration.
 */
#ifndef TTT_ATTN_H_
#define TTT_ATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTT_ATTN_ABI_VERSION 3

enum ttt_status {
  TTT_OK = 0,
  TTT_ERR_NULL = 1,        /* a required pointer is NULL */
  TTT_ERR_DTYPE = 2,       /* dtype is not TTT_F16 or TTT_BF16 */
  TTT_ERR_HEAD_DIM = 3,    /* d is not 64 or 128 */
  TTT_ERR_SHAPE = 4,       /* b, h or t out of range */
  TTT_ERR_STRIDE = 5,      /* a stride is not a positive multiple of 8 elements */
  TTT_ERR_ALIGN = 6,       /* a pointer is not 16-byte aligned */
  TTT_ERR_TENSOR_MAP = 7,  /* the driver rejected a TMA tensor map */
  TTT_ERR_LAUNCH = 8,      /* a kernel launch failed */
  TTT_ERR_DRIVER = 9,      /* the driver entry point for tensor maps is unavailable */
  TTT_ERR_UNSUPPORTED = 10, /* valid request this build does not implement */
  TTT_ERR_SCRATCH = 11,     /* b*h*t_pad exceeds TTT_ATTN_NOALLOC_MAX_ROWS (ttt_attn_bwd2_noalloc) */
  TTT_ERR_SCRATCH_SETUP = 12, /* the built-in scratch array's device address could not be obtained */
  TTT_ERR_MIRROR = 13         /* ttt_attn_error_mirror: not pinned host memory mapped at the same address */
};

enum ttt_dtype { TTT_F16 = 0, TTT_BF16 = 1 };

typedef struct {
  void* ptr;          /* device address of element [0, 0, 0, 0] */
  int64_t sb, sh, st; /* element strides of the b, h and t dimensions */
} ttt_view;

typedef struct {
  int32_t b, h, t, d;
  int32_t dtype;  /* enum ttt_dtype */
  int32_t causal; /* nonzero: key j is visible to query i only if j <= i */
  float scale;    /* softmax scale; callers map scale=None to 1/sqrt(d) */
  int32_t window;      /* 0, or (with causal != 0) a band of `window` keys, W: */
  int32_t window_kind; /* 0 sliding: key j visible to query i iff i - W < j <= i, the
                          additive mask of cloud_ttt_e2e/ttt_e2e/utils.py:40-54;
                          1 chunk-local: queries of the full chunk [cW, cW + W) see
                          keys cW .. i, those of a partial last chunk the last W keys,
                          the chunk loop of cloud_ttt_e2e/ttt_e2e/attention.py:112-127.
                          window > 0 without causal returns TTT_ERR_UNSUPPORTED, as do
                          the P-materializing forward and the from-P passes. */
} ttt_problem;

/* Forward. Writes o and lse2 (base-2 log-sum-exp of scale*log2(e)*q k^T per
 * row; rows t..t_pad-1 get +inf). If p != NULL also writes the normalized
 * probabilities P as [b*h, t, t] 16-bit row-major (entries of causal key tiles
 * past the diagonal tile are left unwritten): for t % 8 == 0 by a second pass
 * after the row-LSE forward (which then may run split, as without P), for
 * other t by a single forward kernel.
 * Replaces: ttt_kernels/triton_attention.py:278-337 (_attn_fwd_kernel,
 * _attn_fwd_kernel_stats, _attn_probs_kernel launches) and the probability
 * forward of the save_p modes, triton_attention.py:51-59 and 270-273. */
typedef struct {
  ttt_problem pb;
  ttt_view q, k, v;
  ttt_view o;
  float* lse2;
  void* p;
  int32_t* err;
  void* work; /* optional work space (see the conventions above) */
  int64_t work_bytes;
} ttt_fwd_args;
int ttt_attn_fwd(const ttt_fwd_args* a, void* stream);

/* First-order backward for upstream gradient dout. Writes delta =
 * rowsum(dout o o) (fp32 [b*h, t_pad], consumed by ttt_attn_bwd2) and dq, dk,
 * dv. P is recomputed from lse2.
 * Replaces: backward_stubs.py:154-181 (triton_attn_bwd_dv_from_p),
 * :224-255 (triton_attn_rowsum_from_p), :362-425 (triton_attn_bwd_dqdk_from_p)
 * and the recompute backward of triton_attention.py:416-420. */
typedef struct {
  ttt_problem pb;
  ttt_view q, k, v, o, dout;
  const float* lse2;
  float* delta;
  ttt_view dq, dk, dv;
  int32_t* err;
  void* work; /* optional work space (see the conventions above) */
  int64_t work_bytes;
} ttt_bwd_args;
int ttt_attn_bwd(const ttt_bwd_args* a, void* stream);

/* Double backward. Given the probes uq, uk, uv (upstream gradients of dq, dk,
 * dv), writes gq, gk, gv = d<dq,uq>+<dk,uk>+<dv,uv> / d(q, k, v) and, if
 * gdout.ptr != NULL, the gradient with respect to dout. gamma and rho are
 * caller-owned fp32 [b*h, t_pad] scratch rows.
 * Replaces: backward_stubs.py:435-439 (TritonDvFn.backward), :450-459
 * (TritonRowSumFn.backward), :471-514 (TritonDqDkFn.backward) and the stubs
 * triton_attn_bwd2_dq / _dk / _dv, backward_stubs.py:539-548. Unlike those,
 * the terms through P's dependence on q and k are included. */
typedef struct {
  ttt_problem pb;
  ttt_view q, k, v, dout;
  const float* lse2;
  const float* delta;
  ttt_view uq, uk, uv;
  float* gamma;
  float* rho;
  ttt_view gq, gk, gv;
  ttt_view gdout;
  int32_t* err;
  void* work; /* optional work space (see the conventions above) */
  int64_t work_bytes;
} ttt_bwd2_args;
int ttt_attn_bwd2(const ttt_bwd2_args* a, void* stream);

/* Passes over materialized probabilities. p is P = softmax(scale * q k^T
 * [causal mask]) as a [b, h, t, t] 16-bit view (same dtype as the other
 * tensors): p.sb, p.sh are the head strides and p.st the row stride, all
 * positive multiples of 8 elements with p.st >= t; entries are read as
 * given. rowsum arrays are fp32 [b*h, t], contiguous. pb.d, pb.dtype as
 * elsewhere; pb.causal: tiles entirely past the diagonal are skipped (the
 * entries there are taken to be zero); pb.scale as in the forward. */
typedef struct {
  ttt_problem pb;
  ttt_view p;
  ttt_view q, k, v, dout;
  const float* rowsum; /* input of ttt_attn_dqdk_from_p */
  float* rowsum_out;   /* output of ttt_attn_rowsum_from_p */
  ttt_view dq, dk, dv;
  int32_t* err;
} ttt_from_p_args;
/* dv = P^T dout (reads all of P; pb.causal and pb.scale are ignored).
 * Replaces: backward_stubs.py:124-181 (_attn_bwd_dv_from_p_kernel,
 * triton_attn_bwd_dv_from_p). */
int ttt_attn_dv_from_p(const ttt_from_p_args* a, void* stream);
/* rowsum_out[bh, i] = sum_j P_ij (dout_i . v_j).
 * Replaces: backward_stubs.py:184-255 (_attn_rowsum_kernel,
 * triton_attn_rowsum_from_p). */
int ttt_attn_rowsum_from_p(const ttt_from_p_args* a, void* stream);
/* dq = scale * dS k, dk = scale * dS^T q with dS = P o (dout v^T - rowsum).
 * Replaces: backward_stubs.py:259-425 (_attn_bwd_dq_kernel,
 * _attn_bwd_dk_kernel, triton_attn_bwd_dqdk_from_p). */
int ttt_attn_dqdk_from_p(const ttt_from_p_args* a, void* stream);

/* Kernel kinds reported by the profiling hook. */
enum ttt_kernel_kind {
  TTT_K_FWD = 0,         /* forward (O, lse2 [, P]) */
  TTT_K_DELTA = 1,       /* delta = rowsum(dout o o) */
  TTT_K_BWD_KV = 2,      /* dk, dv (key-major) */
  TTT_K_BWD_Q = 3,       /* dq (query-major) */
  TTT_K_BWD2_STATS = 4,  /* gamma, rho row statistics */
  TTT_K_BWD2_Q = 5,      /* dd_q (+ dd_dout) */
  TTT_K_BWD2_KV = 6,     /* dd_k, dd_v */
  TTT_K_FROM_P = 7,      /* passes over materialized P */
  TTT_K_COUNT = 8
};

/* Profiling hook (no reference counterpart; the reference times whole steps
 * with time.time(), tests/bench_gradgrad_sweep.py:31-39). While enabled, each
 * kernel launch is bracketed by two CUDA events recorded on its stream.
 * ttt_attn_profile_enable returns the previous setting. */
int ttt_attn_profile_enable(int on);
/* Waits for the recorded events, adds per-kind launch counts and elapsed
 * milliseconds into counts[k] / total_ms[k] for k < n_kinds, and clears the
 * record. */
int ttt_attn_profile_collect(int32_t* counts, double* total_ms, int n_kinds);

/* Allocation-free double backward (no counterpart in the reference). Same
 * arguments and results as ttt_attn_bwd2, except that a->gamma, a->rho and
 * a->work are ignored (the passes run unsplit): the two scratch rows come from
 * a fixed array built into the library
 * (2 * TTT_ATTN_NOALLOC_MAX_ROWS floats, 8 MiB, held by every GPU that loads
 * the library until the process exits), so callers that may not allocate
 * device memory during execution supply only inputs and outputs. Requires
 * b*h*t_pad <= TTT_ATTN_NOALLOC_MAX_ROWS, else returns TTT_ERR_SCRATCH before
 * enqueuing anything. All calls on a device share the array: calls that
 * overlap on the GPU race. The first call on a device looks up the array's
 * device address (with that device current; cached per CUDA context, so a
 * device reset or another context gets its own lookup) and should come before
 * any stream capture. Under lazy module loading (CUDA's default since 12.2)
 * that first call is also when the driver loads the module holding the array
 * and allocates it: callers that may not allocate during execution make one
 * warm-up call per device during set-up, or run with CUDA_MODULE_LOADING=EAGER. */
#define TTT_ATTN_NOALLOC_MAX_ROWS (1 << 20)
int ttt_attn_bwd2_noalloc(const ttt_bwd2_args* a, void* stream);

/* Failure reporting without a host synchronization (no reference counterpart:
 * the reference's Triton kernels have no bounded waits). host_word must be
 * pinned host memory (cudaHostAlloc / cudaMallocHost) that the device sees at
 * the same address (unified addressing), 4-byte aligned; it is registered for
 * the CUDA context current on the calling thread (NULL unregisters). From then
 * on, a kernel of that context that reports an error into a pass's `err` word
 * also stores the same code into host_word, on the error path only, so the
 * host can poll it, e.g. at the entry of its next call. The library never
 * clears it; the caller does. */
int ttt_attn_error_mirror(int32_t* host_word);
/* The code in the mirror registered for the current context (0 when none is
 * registered or no kernel has reported an error since the last take), which
 * it clears. No synchronization: a report still in flight shows up at a later
 * take. The caller also clears the device error word it passes to the passes
 * (in stream order), or later launches that get it exit at once. */
int ttt_attn_error_take(void);

/* Test hook for the failure path (no reference counterpart): one kernel runs the
 * library's bounded mbarrier wait on a barrier that nothing completes, with a
 * limit of limit_ns (1 .. 1e10). No TMA or tensor-core work is in flight; when
 * the limit passes, the kernel records TTT_ERR_WORD_TIMEOUT | (0xfe << 8) in *err
 * (device int32) and in the registered mirror, and returns. */
#define TTT_ERR_WORD_TIMEOUT 0x40000000
int ttt_attn_selftest_wait(int64_t limit_ns, int32_t* err, void* stream);

/* roundup(t, 128): the row count of every statistics array. */
int ttt_attn_t_pad(int t);
/* Bytes of work space with which every pass of problem *pb (forward,
 * backward, double backward with or without the dout gradient) runs in its
 * fastest form: the split slices of a causal problem over few heads (see
 * ttt_attn_split_count), and, for d = 64, the fp32 dQ accumulator
 * ([b*h][t_pad][d]) with which ttt_attn_bwd computes dQ inside its key-major
 * pass instead of a second, query-major pass (whose dQ rows it adds in an
 * unspecified order, so dq may differ from run to run in the last bit). 0 when
 * neither applies. Depends on the current device's SM count. No reference
 * counterpart (the reference's Triton launches pick their grid per call). */
int64_t ttt_attn_work_bytes(const ttt_problem* pb);
/* Number of shares each CTA's tile stream of the backward passes of *pb is
 * split into when the work space is given (1: unsplit). */
int ttt_attn_split_count(const ttt_problem* pb);
/* Static description of a status code. */
const char* ttt_attn_status_string(int status);
/* TTT_ATTN_ABI_VERSION of the loaded library. */
int ttt_attn_abi_version(void);

/* Test hook (no reference counterpart): one 128 x n x k tcgen05 GEMM,
 * c[128 x n] (fp32, row-major) = a[128 x k] * b, all row-major and contiguous.
 * mode bit 0: b is [k x n] (MN-major operand) instead of [n x k] (K-major);
 * mode bit 1: a is staged in tensor memory (A-from-TMEM product form).
 * n in {64, 128, 256}, k in {64, 128}. */
int ttt_attn_selftest_umma(const void* a, const void* b, float* c, int n, int k, int dtype, int mode, int32_t* err,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TTT_ATTN_H_ */
