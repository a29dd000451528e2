// Allocation-free variant of the double backward: ttt_attn_bwd2_noalloc.
//
// Some callers cannot allocate device memory while this op runs: host
// frameworks that hand a plugin only its input and output buffers and forbid
// allocation during execution (runtimes that plan all memory ahead of time),
// and latency-critical paths that must never reach an allocator. The regular
// ttt_attn_bwd2 needs two caller-provided fp32 scratch rows (gamma and rho,
// each [b*h, t_pad]); this variant takes them from a fixed array compiled into
// the library instead, so the caller provides nothing beyond the inputs and
// outputs, and nothing here calls cudaMalloc, cudaFree or any other
// allocating routine.
//
// The array is a file-scope __device__ object of 2 * TTT_ATTN_NOALLOC_MAX_ROWS
// floats (8 MiB): every GPU that loads the library holds it until the process
// exits. Problems with b*h*t_pad above TTT_ATTN_NOALLOC_MAX_ROWS are rejected
// with TTT_ERR_SCRATCH before anything is enqueued.
//
// All calls on a device share the array and it keeps the last call's contents.
// Nothing needs clearing: the statistics pass writes every gamma/rho row it
// later reads (pad rows included) before any kernel reads them. Calls that
// overlap on the GPU (streams without ordering between them) race on it.
//
// In host code the array's name is a host-side stand-in, not a device address,
// so it is never handed to a kernel directly: the first call on each device
// (with that device current) obtains the device address with
// cudaGetSymbolAddress, checks the result, and caches it for the device's
// context (a device reset or another context gets its own lookup). That first
// call should come before any stream capture. Under lazy module loading (the
// CUDA default since 12.2) it is also the moment the driver loads this file's
// module and so allocates the array: a caller that may not allocate while it
// runs makes one warm-up call per device during its set-up, or sets
// CUDA_MODULE_LOADING=EAGER so that the array exists once the library's
// module is loaded.
#include <cuda_runtime.h>

#include <map>
#include <mutex>

#include "host_ctx.h"
#include "ttt_attn.h"

namespace {

constexpr long long kMaxRows = TTT_ATTN_NOALLOC_MAX_ROWS;
__device__ __align__(256) float g_bwd2_scratch[2 * kMaxRows];

std::mutex g_mu;
std::map<unsigned long long, float*> g_scratch;  // context id -> device address of the array

// Device address of the scratch array in the current context (looked up once).
int scratch_for_current_context(float** out) {
  unsigned long long ctx = 0;
  if (!ttt::current_context_id(&ctx)) return TTT_ERR_SCRATCH_SETUP;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_scratch.find(ctx);
  if (it == g_scratch.end()) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_bwd2_scratch);
    if (e != cudaSuccess || addr == nullptr) return TTT_ERR_SCRATCH_SETUP;
    it = g_scratch.emplace(ctx, static_cast<float*>(addr)).first;
  }
  *out = it->second;
  return TTT_OK;
}

}  // namespace

extern "C" int ttt_attn_bwd2_noalloc(const ttt_bwd2_args* a, void* stream) {
  if (a == nullptr) return TTT_ERR_NULL;
  const ttt_problem& pb = a->pb;
  if (pb.b < 1 || pb.h < 1 || pb.t < 1 || pb.t > (1 << 22)) return TTT_ERR_SHAPE;
  // b*h is bounded first (as every entry point bounds it), so the row count
  // below cannot overflow: at most 2^31 * 2^22.
  const long long bh = static_cast<long long>(pb.b) * pb.h;
  if (bh > 0x7fffffffLL) return TTT_ERR_SHAPE;
  const long long rows = bh * ttt_attn_t_pad(pb.t);
  if (rows > kMaxRows) return TTT_ERR_SCRATCH;
  float* scratch = nullptr;
  const int s = scratch_for_current_context(&scratch);
  if (s != TTT_OK) return s;
  ttt_bwd2_args args = *a;
  args.gamma = scratch;
  args.rho = scratch + kMaxRows;
  args.work = nullptr;  // unsplit passes: no work space beyond the built-in rows
  args.work_bytes = 0;
  return ttt_attn_bwd2(&args, stream);
}
