// extern "C" entry points of libttt_attn.so: argument validation, TMA tensor
// map encoding and the launch sequence of each pass. Declarations and the
// contract live in include/ttt_attn.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "ttt_attn.h"
#include "host_ctx.h"
#include "kernels.h"

namespace {

using ttt::KParams;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int check_problem(const ttt_problem& pb) {
  if (pb.dtype != TTT_F16 && pb.dtype != TTT_BF16) return TTT_ERR_DTYPE;
  if (pb.d != 64 && pb.d != 128) return TTT_ERR_HEAD_DIM;
  if (pb.b < 1 || pb.h < 1 || pb.t < 1) return TTT_ERR_SHAPE;
  if (pb.t > (1 << 22)) return TTT_ERR_SHAPE;
  if (static_cast<int64_t>(pb.b) * pb.h > 0x7fffffff) return TTT_ERR_SHAPE;
  if (pb.window < 0) return TTT_ERR_SHAPE;
  if (pb.window > 0 && pb.causal == 0) return TTT_ERR_UNSUPPORTED;
  if (pb.window_kind != 0 && pb.window_kind != 1) return TTT_ERR_UNSUPPORTED;
  return TTT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_view(const ttt_view& v, const ttt_problem& pb) {
  if (v.ptr == nullptr) return TTT_ERR_NULL;
  if (!aligned16(v.ptr)) return TTT_ERR_ALIGN;
  const int64_t s[3] = {v.sb, v.sh, v.st};
  const int64_t n[3] = {pb.b, pb.h, pb.t};
  for (int i = 0; i < 3; ++i) {
    if (n[i] == 1) continue;  // stride of a size-1 dimension is never used
    if (s[i] <= 0 || (s[i] % 8) != 0) return TTT_ERR_STRIDE;
  }
  if (pb.t > 1 && v.st < pb.d) return TTT_ERR_STRIDE;
  return TTT_OK;
}

int check_stats(const float* p) {
  if (p == nullptr) return TTT_ERR_NULL;
  if (!aligned16(p)) return TTT_ERR_ALIGN;
  return TTT_OK;
}

// 4-D map over a [b, h, t, d] view: dims (d, t, h, b), box (64, rows, 1, 1),
// 128-byte swizzle, out-of-bounds rows read as zero.
int encode_view(CUtensorMap* m, const ttt_view& v, const ttt_problem& pb, int rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return TTT_ERR_DRIVER;
  // Size-1 dimensions get the contiguous stride so the driver sees a valid map.
  int64_t st = pb.t > 1 ? v.st : pb.d;
  int64_t sh = pb.h > 1 ? v.sh : st * pb.t;
  int64_t sb = pb.b > 1 ? v.sb : sh * pb.h;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(pb.d), static_cast<cuuint64_t>(pb.t),
                        static_cast<cuuint64_t>(pb.h), static_cast<cuuint64_t>(pb.b)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(st * 2), static_cast<cuuint64_t>(sh * 2),
                           static_cast<cuuint64_t>(sb * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      pb.dtype == TTT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(m, dt, 4, v.ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TTT_OK : TTT_ERR_TENSOR_MAP;
}

// 2-D map over fp32 statistics [bh, t_pad], box (cols, 1).
int encode_stats(CUtensorMap* m, const float* p, int bh, int t_pad, int cols) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return TTT_ERR_DRIVER;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(t_pad), static_cast<cuuint64_t>(bh)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(t_pad) * 4};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(cols), 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TTT_OK : TTT_ERR_TENSOR_MAP;
}

// 3-D map over the fp32 dQ accumulator [bh][t_pad][d] of the fused backward:
// dims (d, t_pad, bh), box (32, 128, 1), 128-byte swizzle; the kernel adds
// [128 x 32] boxes into it (TMA reduce), rows past t_pad clipped.
int encode_acc_q(CUtensorMap* m, float* acc, int bh, int t_pad, int d) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return TTT_ERR_DRIVER;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(t_pad), static_cast<cuuint64_t>(bh)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 4, static_cast<cuuint64_t>(t_pad) * d * 4};
  cuuint32_t box[3] = {32, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, acc, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TTT_OK : TTT_ERR_TENSOR_MAP;
}

// P view [b, h, t, t]: row stride p.st >= t, head strides; all multiples of 8.
int check_p_view(const ttt_view& v, const ttt_problem& pb) {
  if (v.ptr == nullptr) return TTT_ERR_NULL;
  if (!aligned16(v.ptr)) return TTT_ERR_ALIGN;
  const int64_t s[3] = {v.sb, v.sh, v.st};
  const int64_t n[3] = {pb.b, pb.h, pb.t};
  for (int i = 0; i < 3; ++i) {
    if (n[i] == 1 && i < 2) continue;
    if (s[i] <= 0 || (s[i] % 8) != 0) return TTT_ERR_STRIDE;
  }
  if (v.st < pb.t) return TTT_ERR_STRIDE;
  return TTT_OK;
}

// 4-D map over a [b, h, t, t] probability view: dims (t, t, h, b), box (64, rows, 1, 1).
int encode_p(CUtensorMap* m, const ttt_view& v, const ttt_problem& pb, int rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return TTT_ERR_DRIVER;
  const int64_t st = v.st;
  const int64_t sh = pb.h > 1 ? v.sh : st * pb.t;
  const int64_t sb = pb.b > 1 ? v.sb : sh * pb.h;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(pb.t), static_cast<cuuint64_t>(pb.t),
                        static_cast<cuuint64_t>(pb.h), static_cast<cuuint64_t>(pb.b)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(st * 2), static_cast<cuuint64_t>(sh * 2),
                           static_cast<cuuint64_t>(sb * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      pb.dtype == TTT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(m, dt, 4, v.ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TTT_OK : TTT_ERR_TENSOR_MAP;
}

// Host-mapped mirrors of the device error word, one per context, registered by
// ttt_attn_error_mirror. Kernels write a mirror only when they report an error.
std::mutex g_mirror_mu;
std::map<unsigned long long, int32_t*> g_mirror;
bool g_any_mirror = false;  // read under g_mirror_mu; skips the context lookup while none is registered

int32_t* error_mirror() {
  {
    std::lock_guard<std::mutex> lk(g_mirror_mu);
    if (!g_any_mirror) return nullptr;
  }
  unsigned long long ctx = 0;
  if (!ttt::current_context_id(&ctx)) return nullptr;
  std::lock_guard<std::mutex> lk(g_mirror_mu);
  auto it = g_mirror.find(ctx);
  return it == g_mirror.end() ? nullptr : it->second;
}

void fill_common(KParams& k, const ttt_problem& pb, int32_t* err) {
  k.B = pb.b;
  k.H = pb.h;
  k.T = pb.t;
  k.t_pad = ttt_attn_t_pad(pb.t);
  k.scale = pb.scale;
  k.window = pb.causal != 0 ? pb.window : 0;
  k.window_kind = pb.window_kind;
  k.scale_log2 = pb.scale * 1.4426950408889634f;
  k.err = err;
  k.err_host = err != nullptr ? error_mirror() : nullptr;
}

void set_raw(KParams& k, int slot, const ttt_view& v) {
  k.raw[slot] = static_cast<const uint16_t*>(v.ptr);
  k.raw_sb[slot] = v.sb;
  k.raw_sh[slot] = v.sh;
  k.raw_st[slot] = v.st;
}

void set_out0(KParams& k, const ttt_view& v) {
  k.out0 = static_cast<uint16_t*>(v.ptr);
  k.o0_sb = v.sb;
  k.o0_sh = v.sh;
  k.o0_st = v.st;
}
void set_out1(KParams& k, const ttt_view& v) {
  k.out1 = static_cast<uint16_t*>(v.ptr);
  k.o1_sb = v.sb;
  k.o1_sh = v.sh;
  k.o1_st = v.st;
}

#define TTT_TRY(expr)          \
  do {                         \
    const int _s = (expr);     \
    if (_s != TTT_OK) return _s; \
  } while (0)

int launched(cudaError_t e) { return e == cudaSuccess ? TTT_OK : TTT_ERR_LAUNCH; }

// ---------------------------------------------------------------- profiling hook
struct ProfRecord {
  int kind;
  int device;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof;
std::map<int, std::vector<cudaEvent_t>> g_event_pool;  // per device

cudaEvent_t take_event(int device) {
  auto& pool = g_event_pool[device];
  if (!pool.empty()) {
    cudaEvent_t e = pool.back();
    pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Brackets one launch with events when profiling is on.
class ProfScope {
 public:
  ProfScope(int kind, cudaStream_t s) : kind_(kind), s_(s) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on) return;
    cudaGetDevice(&dev_);
    start_ = take_event(dev_);
    if (start_) cudaEventRecord(start_, s_);
  }
  ~ProfScope() {
    if (!start_) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    cudaEvent_t stop = take_event(dev_);
    if (!stop) return;
    cudaEventRecord(stop, s_);
    g_prof.push_back({kind_, dev_, start_, stop});
  }

 private:
  int kind_;
  cudaStream_t s_;
  int dev_ = 0;
  cudaEvent_t start_ = nullptr;
};

// ---------------------------------------------------------------- side stream
// The two passes that follow each other's inputs but not each other's outputs
// (dK/dV and dQ of the backward; dd_q and dd_k/dd_v of the double backward)
// run on the caller's stream and on a library-owned side stream that forks
// from it and joins back (event record / wait only, no host synchronization),
// so that one pass's last CTAs overlap the other's first, when the passes
// are small (overlap_pays). While profiling is on, everything stays on the
// caller's stream so that each launch's events time that kernel alone.
struct Side {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mu;
// One side stream per context (keyed by its id, so a device reset or a
// non-primary context never receives a stream created in another context).
std::map<unsigned long long, Side> g_side;

// Overlap pays when a pass has too few CTAs to fill the GPU for long (under two
// waves of one CTA per SM); with more, the passes' tails are short and running
// them side by side only mixes their working sets in L2.
int sm_count() {
  static int sms = [] {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return 0;
    return n;
  }();
  return sms;
}

bool overlap_pays(const ttt_problem& pb) {
  const int sms = sm_count();
  const int64_t ctas = static_cast<int64_t>(pb.b) * pb.h * ((pb.t + 127) / 128);
  return sms > 0 && ctas < 2 * static_cast<int64_t>(sms);
}

// ---------------------------------------------------------------- split planning
// A causal pass over few heads has few CTAs of very unequal length (the first
// key block of a head meets every query tile, the last one a single tile), so
// the longest CTA sets the pass's time while most SMs idle. Such a pass splits
// each CTA's tile stream into `nsplit` nearly equal shares, one CTA each, so
// that the grid holds about 1.5 CTAs per SM; the shares' fp32 partials are
// summed in order by a reduction kernel. Non-causal and banded problems have
// CTAs of equal length and stay unsplit.
// rows: the query rows (or keys) one unsplit CTA owns (128 in the backward
// passes, 256 in the forward).
int split_count(const ttt_problem& pb, int rows = 128) {
  const int sms = sm_count();
  if (pb.causal == 0 || pb.window > 0 || sms <= 0) return 1;
  const int64_t base = static_cast<int64_t>(pb.b) * pb.h * ((pb.t + rows - 1) / rows);
  if (2 * base >= 3 * static_cast<int64_t>(sms)) return 1;
  const int64_t n = (3 * static_cast<int64_t>(sms) + 2 * base - 1) / (2 * base);
  return static_cast<int>(n < 2 ? 2 : (n > 4 ? 4 : n));
}

// The work space of a split problem: four slices of [nsplit][b*h][t_pad][d]
// fp32. The key-major passes write their two partial arrays into slices 0 and
// 1, the query-major passes (which may run at the same time on the side
// stream) into 2 and 3; the row-statistics pass (float4 per row) uses slice 0
// before the key-major pass runs.
constexpr int kWorkSlices = 4;
int64_t slice_floats(const ttt_problem& pb, int nsplit) {
  return static_cast<int64_t>(nsplit) * pb.b * pb.h * ttt_attn_t_pad(pb.t) * pb.d;
}
// The forward's split uses [nsplit][b*h][t_pad][d] fp32 O rows followed by
// [nsplit][b*h][t_pad] (max, sum) pairs.
int64_t fwd_work_need(const ttt_problem& pb) {
  const int n = split_count(pb, 256);
  return n > 1 ? static_cast<int64_t>(n) * pb.b * pb.h * ttt_attn_t_pad(pb.t) * (pb.d + 2) * 4 : 0;
}
// Split slices of the backward passes, in bytes (0 when no pass splits).
int64_t bwd_split_bytes(const ttt_problem& pb) {
  const int n = split_count(pb);
  return n > 1 ? kWorkSlices * slice_floats(pb, n) * 4 : 0;
}
// The fp32 dQ accumulator [b*h][t_pad][d] of the fused first-order backward
// (d = 64: dQ inside the key-major pass), placed after the split slices.
int64_t acc_q_bytes(const ttt_problem& pb) {
  return pb.d == 64 ? static_cast<int64_t>(pb.b) * pb.h * ttt_attn_t_pad(pb.t) * pb.d * 4 : 0;
}
int64_t work_need(const ttt_problem& pb) {
  const int64_t bwd = bwd_split_bytes(pb) + acc_q_bytes(pb);
  const int64_t fwd = fwd_work_need(pb);
  return bwd > fwd ? bwd : fwd;
}

struct Work {
  int nsplit = 1;  // 1: run unsplit
  float* base = nullptr;
  int64_t slice = 0;
  float* acc_q = nullptr;  // the fused first-order backward's dQ accumulator (null: two passes)
  float* at(int i) const { return base + i * slice; }
};
// Each use of the work space needs its own part to fit: a buffer sized for the
// split slices alone still splits the passes.
Work plan_work(const ttt_problem& pb, void* work, int64_t work_bytes) {
  Work w;
  if (work == nullptr || (reinterpret_cast<uintptr_t>(work) & 255u) != 0) return w;
  const int n = split_count(pb);
  const int64_t split_b = bwd_split_bytes(pb);
  if (n > 1 && work_bytes >= split_b) {
    w.nsplit = n;
    w.base = static_cast<float*>(work);
    w.slice = slice_floats(pb, n);
  }
  const int64_t acc_b = acc_q_bytes(pb);
  if (acc_b > 0 && work_bytes >= split_b + acc_b)
    w.acc_q = reinterpret_cast<float*>(static_cast<char*>(work) + split_b);
  return w;
}
void use_work(KParams& k, const Work& w, int first_slice) {
  k.nsplit = w.nsplit;
  if (w.nsplit > 1) {
    k.part0 = w.at(first_slice);
    k.part1 = w.at(first_slice + 1);
  }
}

// Sums the shares of n_out (1 or 2) partial arrays starting at slice
// first_slice into out0 (times scale0) and out1 (times scale1).
int reduce_splits(const Work& w, int first_slice, const ttt_problem& pb, int n_out, const ttt_view& out0,
                  float scale0, const ttt_view* out1, float scale1, cudaStream_t s) {
  ttt::SplitReduceArgs r;
  std::memset(&r, 0, sizeof(r));
  const ttt_view* outs[2] = {&out0, out1};
  const float scales[2] = {scale0, scale1};
  for (int i = 0; i < n_out; ++i) {
    r.part[i] = w.at(first_slice + i);
    r.out[i] = static_cast<uint16_t*>(outs[i]->ptr);
    r.sb[i] = outs[i]->sb, r.sh[i] = outs[i]->sh, r.st[i] = outs[i]->st;
    r.scale[i] = scales[i];
  }
  r.n_out = n_out;
  r.nsplit = w.nsplit;
  r.B = pb.b, r.H = pb.h, r.T = pb.t, r.t_pad = ttt_attn_t_pad(pb.t), r.D = pb.d;
  r.bf16 = pb.dtype == TTT_BF16;
  return launched(ttt::launch_split_reduce(r, s));
}

class Fork {
 public:
  Fork(cudaStream_t main, bool enable) : main_(main), side_(main) {
    if (!enable) return;
    {
      std::lock_guard<std::mutex> lk(g_prof_mu);
      if (g_prof_on) return;
    }
    unsigned long long ctx = 0;
    if (!ttt::current_context_id(&ctx)) return;
    std::lock_guard<std::mutex> lk(g_side_mu);
    Side& sd = g_side[ctx];
    if (sd.stream == nullptr) {
      if (cudaStreamCreateWithFlags(&sd.stream, cudaStreamNonBlocking) != cudaSuccess) {
        sd.stream = nullptr;
        return;
      }
      if (cudaEventCreateWithFlags(&sd.fork, cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&sd.join, cudaEventDisableTiming) != cudaSuccess)
        return;
    }
    if (sd.fork == nullptr || sd.join == nullptr) return;
    if (cudaEventRecord(sd.fork, main_) != cudaSuccess || cudaStreamWaitEvent(sd.stream, sd.fork, 0) != cudaSuccess)
      return;
    side_ = sd.stream;
    join_ = sd.join;
  }
  // The stream for the second pass (the caller's stream when not forked).
  cudaStream_t side() const { return side_; }
  ~Fork() {
    if (side_ == main_ || join_ == nullptr) return;
    std::lock_guard<std::mutex> lk(g_side_mu);
    cudaEventRecord(join_, side_);
    cudaStreamWaitEvent(main_, join_, 0);
  }

 private:
  cudaStream_t main_, side_;
  cudaEvent_t join_ = nullptr;
};

}  // namespace

extern "C" {

int ttt_attn_t_pad(int t) { return (t + 127) / 128 * 128; }

int ttt_attn_abi_version(void) { return TTT_ATTN_ABI_VERSION; }

int64_t ttt_attn_work_bytes(const ttt_problem* pb) {
  if (pb == nullptr || check_problem(*pb) != TTT_OK) return 0;
  return work_need(*pb);
}

int ttt_attn_split_count(const ttt_problem* pb) {
  if (pb == nullptr || check_problem(*pb) != TTT_OK) return 1;
  return split_count(*pb);
}

const char* ttt_attn_status_string(int s) {
  switch (s) {
    case TTT_OK: return "ok";
    case TTT_ERR_NULL: return "a required pointer is NULL";
    case TTT_ERR_DTYPE: return "dtype must be fp16 or bf16";
    case TTT_ERR_HEAD_DIM: return "head dim d must be 64 or 128";
    case TTT_ERR_SHAPE: return "b, h or t out of range";
    case TTT_ERR_STRIDE: return "strides must be positive multiples of 8 elements with unit d stride";
    case TTT_ERR_ALIGN: return "pointers must be 16-byte aligned";
    case TTT_ERR_TENSOR_MAP: return "the driver rejected a TMA tensor map";
    case TTT_ERR_LAUNCH: return "kernel launch failed";
    case TTT_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable";
    case TTT_ERR_UNSUPPORTED: return "unsupported request";
    case TTT_ERR_SCRATCH: return "b*h*t_pad exceeds the fixed scratch of the allocation-free entry point";
    case TTT_ERR_SCRATCH_SETUP: return "could not obtain the device address of the built-in scratch array";
    case TTT_ERR_MIRROR: return "the error mirror must be pinned host memory mapped at the same device address";
    default: return "unknown status";
  }
}

int ttt_attn_fwd(const ttt_fwd_args* a, void* stream) {
  if (a == nullptr) return TTT_ERR_NULL;
  const ttt_problem& pb = a->pb;
  TTT_TRY(check_problem(pb));
  TTT_TRY(check_view(a->q, pb));
  TTT_TRY(check_view(a->k, pb));
  TTT_TRY(check_view(a->v, pb));
  TTT_TRY(check_view(a->o, pb));
  TTT_TRY(check_stats(a->lse2));
  if (a->p != nullptr && !aligned16(a->p)) return TTT_ERR_ALIGN;
  if (a->p != nullptr && pb.window > 0) return TTT_ERR_UNSUPPORTED;
  KParams k;
  std::memset(&k, 0, sizeof(k));
  fill_common(k, pb, a->err);
  TTT_TRY(encode_view(&k.own[0], a->q, pb, 128));
  TTT_TRY(encode_view(&k.str[0], a->k, pb, 128));
  TTT_TRY(encode_view(&k.str[1], a->v, pb, 128));
  set_out0(k, a->o);
  k.out_f0 = a->lse2;
  k.out1 = static_cast<uint16_t*>(a->p);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // P with T % 8 == 0: the row-LSE forward (split like the forward without P),
  // then a pass that recomputes S and stores P by TMA; other T keep the
  // single-kernel forward that writes P itself
  const bool pwrite = a->p != nullptr && (pb.t % 8) == 0;
  // split mode (the forward without a P epilogue only): shares of each CTA's key stream
  const int nf = (a->p == nullptr || pwrite) ? split_count(pb, 256) : 1;
  const bool split = nf > 1 && a->work != nullptr && a->work_bytes >= fwd_work_need(pb) &&
                     (reinterpret_cast<uintptr_t>(a->work) & 255u) == 0;
  const int64_t o_floats = static_cast<int64_t>(nf) * pb.b * pb.h * ttt_attn_t_pad(pb.t) * pb.d;
  if (split) {
    k.nsplit = nf;
    k.part0 = static_cast<float*>(a->work);
    k.part1 = k.part0 + o_floats;
  }
  ProfScope prof(TTT_K_FWD, s);
  TTT_TRY(launched(ttt::launch_fwd(k, pb.d, pb.dtype == TTT_BF16, pb.causal != 0, a->p != nullptr && !pwrite, s)));
  if (split) {
    ttt::FwdCombineArgs c;
    c.part_o = k.part0;
    c.part_ml = reinterpret_cast<const float2*>(k.part1);
    c.out = static_cast<uint16_t*>(a->o.ptr);
    c.sb = a->o.sb, c.sh = a->o.sh, c.st = a->o.st;
    c.lse2 = a->lse2;
    c.nsplit = nf, c.B = pb.b, c.H = pb.h, c.T = pb.t, c.t_pad = ttt_attn_t_pad(pb.t), c.D = pb.d;
    c.bf16 = pb.dtype == TTT_BF16;
    TTT_TRY(launched(ttt::launch_fwd_combine(c, s)));
  }
  if (!pwrite) return TTT_OK;
  KParams kp;
  std::memset(&kp, 0, sizeof(kp));
  fill_common(kp, pb, a->err);
  TTT_TRY(encode_view(&kp.own[0], a->q, pb, 128));
  TTT_TRY(encode_view(&kp.str[0], a->k, pb, 128));
  // P is contiguous [b, h, t, t]
  const ttt_view pv{a->p, static_cast<int64_t>(pb.h) * pb.t * pb.t, static_cast<int64_t>(pb.t) * pb.t, pb.t};
  TTT_TRY(encode_p(&kp.str[1], pv, pb, 128));
  kp.lse2 = a->lse2;
  return launched(ttt::launch_pwrite(kp, pb.d, pb.dtype == TTT_BF16, pb.causal != 0, s));
}

int ttt_attn_bwd(const ttt_bwd_args* a, void* stream) {
  if (a == nullptr) return TTT_ERR_NULL;
  const ttt_problem& pb = a->pb;
  TTT_TRY(check_problem(pb));
  const ttt_view* views[] = {&a->q, &a->k, &a->v, &a->o, &a->dout, &a->dq, &a->dk, &a->dv};
  for (const ttt_view* v : views) TTT_TRY(check_view(*v, pb));
  TTT_TRY(check_stats(a->lse2));
  TTT_TRY(check_stats(a->delta));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = pb.dtype == TTT_BF16, causal = pb.causal != 0;
  const int t_pad = ttt_attn_t_pad(pb.t), bh = pb.b * pb.h;

  ttt::DeltaArgs da;
  da.o = static_cast<const uint16_t*>(a->o.ptr);
  da.o_sb = a->o.sb;
  da.o_sh = a->o.sh;
  da.o_st = a->o.st;
  da.dout = static_cast<const uint16_t*>(a->dout.ptr);
  da.d_sb = a->dout.sb;
  da.d_sh = a->dout.sh;
  da.d_st = a->dout.st;
  da.delta = a->delta;
  da.B = pb.b;
  da.H = pb.h;
  da.T = pb.t;
  da.t_pad = t_pad;
  da.D = pb.d;
  da.bf16 = bf16;
  {
    ProfScope prof(TTT_K_DELTA, s);
    TTT_TRY(launched(ttt::launch_delta(da, s)));
  }

  const Work w = plan_work(pb, a->work, a->work_bytes);
  if (w.acc_q != nullptr) {
    // One key-major pass for dK, dV and dQ: dQ rows are added into the zeroed fp32
    // accumulator, then scaled and converted (the split reduction with one share).
    const size_t acc_bytes = static_cast<size_t>(acc_q_bytes(pb));
    if (cudaMemsetAsync(w.acc_q, 0, acc_bytes, s) != cudaSuccess) return TTT_ERR_LAUNCH;
    KParams k;
    std::memset(&k, 0, sizeof(k));
    fill_common(k, pb, a->err);
    TTT_TRY(encode_view(&k.own[0], a->k, pb, 128));
    TTT_TRY(encode_view(&k.own[1], a->v, pb, 128));
    const int rows = ttt::km_tile_rows(pb.d, ttt::kBwdKVQ);
    TTT_TRY(encode_view(&k.str[0], a->q, pb, rows));
    TTT_TRY(encode_view(&k.str[1], a->dout, pb, rows));
    TTT_TRY(encode_stats(&k.st[0], a->lse2, bh, t_pad, rows));
    TTT_TRY(encode_stats(&k.st[1], a->delta, bh, t_pad, rows));
    set_out0(k, a->dk);
    set_out1(k, a->dv);
    use_work(k, w, 0);
    k.acc_q = w.acc_q;
    TTT_TRY(encode_acc_q(&k.st[2], w.acc_q, bh, t_pad, pb.d));
    ProfScope prof(TTT_K_BWD_KV, s);
    TTT_TRY(launched(ttt::launch_km(k, pb.d, bf16, causal, ttt::kBwdKVQ, s)));
    if (w.nsplit > 1) TTT_TRY(reduce_splits(w, 0, pb, 2, a->dk, pb.scale, &a->dv, 1.f, s));
    Work acc;
    acc.nsplit = 1;
    acc.base = w.acc_q;
    acc.slice = 0;
    return reduce_splits(acc, 0, pb, 1, a->dq, pb.scale, nullptr, 0.f, s);
  }
  Fork fork(s, overlap_pays(pb));
  // dK, dV: key-major.
  {
    KParams k;
    std::memset(&k, 0, sizeof(k));
    fill_common(k, pb, a->err);
    TTT_TRY(encode_view(&k.own[0], a->k, pb, 128));
    TTT_TRY(encode_view(&k.own[1], a->v, pb, 128));
    const int rows = ttt::km_tile_rows(pb.d, ttt::kBwdKV);
    TTT_TRY(encode_view(&k.str[0], a->q, pb, rows));
    TTT_TRY(encode_view(&k.str[1], a->dout, pb, rows));
    TTT_TRY(encode_stats(&k.st[0], a->lse2, bh, t_pad, rows));
    TTT_TRY(encode_stats(&k.st[1], a->delta, bh, t_pad, rows));
    set_out0(k, a->dk);
    set_out1(k, a->dv);
    use_work(k, w, 0);
    ProfScope prof(TTT_K_BWD_KV, s);
    TTT_TRY(launched(ttt::launch_km(k, pb.d, bf16, causal, ttt::kBwdKV, s)));
    if (w.nsplit > 1) TTT_TRY(reduce_splits(w, 0, pb, 2, a->dk, pb.scale, &a->dv, 1.f, s));
  }
  // dQ: query-major.
  {
    KParams k;
    std::memset(&k, 0, sizeof(k));
    fill_common(k, pb, a->err);
    TTT_TRY(encode_view(&k.own[0], a->q, pb, 128));
    TTT_TRY(encode_view(&k.own[1], a->dout, pb, 128));
    const int cols = ttt::qm_tile_cols(pb.d, ttt::kBwdQ, false);
    TTT_TRY(encode_view(&k.str[0], a->k, pb, cols));
    TTT_TRY(encode_view(&k.str[1], a->v, pb, cols));
    set_raw(k, 0, a->q);
    set_raw(k, 1, a->dout);
    k.lse2 = a->lse2;
    k.delta = a->delta;
    set_out0(k, a->dq);
    use_work(k, w, 2);
    cudaStream_t s2 = fork.side();
    ProfScope prof(TTT_K_BWD_Q, s2);
    TTT_TRY(launched(ttt::launch_qm(k, pb.d, bf16, causal, ttt::kBwdQ, false, s2)));
    if (w.nsplit > 1) TTT_TRY(reduce_splits(w, 2, pb, 1, a->dq, pb.scale, nullptr, 0.f, s2));
  }
  return TTT_OK;
}

int ttt_attn_bwd2(const ttt_bwd2_args* a, void* stream) {
  if (a == nullptr) return TTT_ERR_NULL;
  const ttt_problem& pb = a->pb;
  TTT_TRY(check_problem(pb));
  const ttt_view* views[] = {&a->q, &a->k, &a->v, &a->dout, &a->uq, &a->uk, &a->uv, &a->gq, &a->gk, &a->gv};
  for (const ttt_view* v : views) TTT_TRY(check_view(*v, pb));
  const bool gdo = a->gdout.ptr != nullptr;
  if (gdo) TTT_TRY(check_view(a->gdout, pb));
  TTT_TRY(check_stats(a->lse2));
  TTT_TRY(check_stats(a->delta));
  TTT_TRY(check_stats(a->gamma));
  TTT_TRY(check_stats(a->rho));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = pb.dtype == TTT_BF16, causal = pb.causal != 0;
  const int t_pad = ttt_attn_t_pad(pb.t), bh = pb.b * pb.h;

  // Query-major: row statistics, then dd_q (+ dd_dout).
  KParams kq;
  std::memset(&kq, 0, sizeof(kq));
  fill_common(kq, pb, a->err);
  TTT_TRY(encode_view(&kq.own[0], a->q, pb, 128));
  TTT_TRY(encode_view(&kq.own[1], a->dout, pb, 128));
  TTT_TRY(encode_view(&kq.own[2], a->uq, pb, 128));
  set_raw(kq, 0, a->q);
  set_raw(kq, 1, a->dout);
  set_raw(kq, 2, a->uq);
  auto encode_stream_q = [&](int cols) -> int {
    TTT_TRY(encode_view(&kq.str[0], a->k, pb, cols));
    TTT_TRY(encode_view(&kq.str[1], a->v, pb, cols));
    TTT_TRY(encode_view(&kq.str[2], a->uk, pb, cols));
    TTT_TRY(encode_view(&kq.str[3], a->uv, pb, cols));
    return TTT_OK;
  };
  TTT_TRY(encode_stream_q(ttt::qm_tile_cols(pb.d, ttt::kStats, false)));
  kq.lse2 = a->lse2;
  kq.delta = a->delta;
  kq.out_f0 = a->gamma;
  kq.out_f1 = a->rho;
  const Work w = plan_work(pb, a->work, a->work_bytes);
  {
    use_work(kq, w, 0);
    ProfScope prof(TTT_K_BWD2_STATS, s);
    TTT_TRY(launched(ttt::launch_qm(kq, pb.d, bf16, causal, ttt::kStats, false, s)));
    if (w.nsplit > 1) {
      ttt::StatsReduceArgs r;
      r.part = reinterpret_cast<const float4*>(w.at(0));
      r.delta = a->delta;
      r.gamma = a->gamma;
      r.rho = a->rho;
      r.nsplit = w.nsplit;
      r.BH = bh;
      r.T = pb.t;
      r.t_pad = t_pad;
      TTT_TRY(launched(ttt::launch_stats_reduce(r, s)));
    }
  }
  if (ttt::qm_tile_cols(pb.d, ttt::kBwd2Q, gdo) != ttt::qm_tile_cols(pb.d, ttt::kStats, false))
    TTT_TRY(encode_stream_q(ttt::qm_tile_cols(pb.d, ttt::kBwd2Q, gdo)));
  kq.gamma = a->gamma;
  kq.rho = a->rho;
  kq.out_f0 = nullptr;
  kq.out_f1 = nullptr;
  set_out0(kq, a->gq);
  if (gdo) set_out1(kq, a->gdout);
  use_work(kq, w, 2);
  Fork fork(s, overlap_pays(pb));
  {
    cudaStream_t s2 = fork.side();
    ProfScope prof(TTT_K_BWD2_Q, s2);
    TTT_TRY(launched(ttt::launch_qm(kq, pb.d, bf16, causal, ttt::kBwd2Q, gdo, s2)));
    if (w.nsplit > 1) TTT_TRY(reduce_splits(w, 2, pb, gdo ? 2 : 1, a->gq, pb.scale, &a->gdout, 1.f, s2));
  }

  // Key-major: dd_k, dd_v.
  KParams kk;
  std::memset(&kk, 0, sizeof(kk));
  fill_common(kk, pb, a->err);
  TTT_TRY(encode_view(&kk.own[0], a->k, pb, 128));
  TTT_TRY(encode_view(&kk.own[1], a->v, pb, 128));
  TTT_TRY(encode_view(&kk.own[2], a->uk, pb, 128));
  TTT_TRY(encode_view(&kk.own[3], a->uv, pb, 128));
  const int rows = ttt::km_tile_rows(pb.d, ttt::kBwd2KV);
  TTT_TRY(encode_view(&kk.str[0], a->q, pb, rows));
  TTT_TRY(encode_view(&kk.str[1], a->dout, pb, rows));
  TTT_TRY(encode_view(&kk.str[2], a->uq, pb, rows));
  TTT_TRY(encode_stats(&kk.st[0], a->lse2, bh, t_pad, rows));
  TTT_TRY(encode_stats(&kk.st[1], a->delta, bh, t_pad, rows));
  TTT_TRY(encode_stats(&kk.st[2], a->gamma, bh, t_pad, rows));
  TTT_TRY(encode_stats(&kk.st[3], a->rho, bh, t_pad, rows));
  set_out0(kk, a->gk);
  set_out1(kk, a->gv);
  {
    use_work(kk, w, 0);
    ProfScope prof(TTT_K_BWD2_KV, s);
    TTT_TRY(launched(ttt::launch_km(kk, pb.d, bf16, causal, ttt::kBwd2KV, s)));
    if (w.nsplit > 1) TTT_TRY(reduce_splits(w, 0, pb, 2, a->gk, pb.scale, &a->gv, 1.f, s));
  }
  return TTT_OK;
}

int ttt_attn_dv_from_p(const ttt_from_p_args* a, void* stream) {
  if (a == nullptr) return TTT_ERR_NULL;
  const ttt_problem& pb = a->pb;
  TTT_TRY(check_problem(pb));
  if (pb.window > 0) return TTT_ERR_UNSUPPORTED;
  TTT_TRY(check_p_view(a->p, pb));
  TTT_TRY(check_view(a->dout, pb));
  TTT_TRY(check_view(a->dv, pb));
  KParams k;
  std::memset(&k, 0, sizeof(k));
  fill_common(k, pb, a->err);
  TTT_TRY(encode_p(&k.str[0], a->p, pb, ttt::from_p_box_rows(ttt::kFpDV)));
  TTT_TRY(encode_view(&k.str[1], a->dout, pb, ttt::from_p_stream_rows(ttt::kFpDV)));
  set_out0(k, a->dv);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope prof(TTT_K_FROM_P, s);
  return launched(ttt::launch_from_p(k, pb.d, pb.dtype == TTT_BF16, false, ttt::kFpDV, s));
}

int ttt_attn_rowsum_from_p(const ttt_from_p_args* a, void* stream) {
  if (a == nullptr) return TTT_ERR_NULL;
  const ttt_problem& pb = a->pb;
  TTT_TRY(check_problem(pb));
  if (pb.window > 0) return TTT_ERR_UNSUPPORTED;
  TTT_TRY(check_p_view(a->p, pb));
  TTT_TRY(check_view(a->dout, pb));
  TTT_TRY(check_view(a->v, pb));
  if (a->rowsum_out == nullptr) return TTT_ERR_NULL;
  KParams k;
  std::memset(&k, 0, sizeof(k));
  fill_common(k, pb, a->err);
  TTT_TRY(encode_p(&k.str[0], a->p, pb, ttt::from_p_box_rows(ttt::kFpRowsum)));
  TTT_TRY(encode_view(&k.str[1], a->v, pb, ttt::from_p_stream_rows(ttt::kFpRowsum)));
  set_raw(k, 0, a->dout);
  k.out_f0 = a->rowsum_out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope prof(TTT_K_FROM_P, s);
  return launched(ttt::launch_from_p(k, pb.d, pb.dtype == TTT_BF16, pb.causal != 0, ttt::kFpRowsum, s));
}

int ttt_attn_dqdk_from_p(const ttt_from_p_args* a, void* stream) {
  if (a == nullptr) return TTT_ERR_NULL;
  const ttt_problem& pb = a->pb;
  TTT_TRY(check_problem(pb));
  if (pb.window > 0) return TTT_ERR_UNSUPPORTED;
  TTT_TRY(check_p_view(a->p, pb));
  const ttt_view* views[] = {&a->q, &a->k, &a->v, &a->dout, &a->dq, &a->dk};
  for (const ttt_view* v : views) TTT_TRY(check_view(*v, pb));
  if (a->rowsum == nullptr) return TTT_ERR_NULL;
  const bool bf16 = pb.dtype == TTT_BF16, causal = pb.causal != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    // dK: key-major, V resident, P / dO / Q streamed per 128 queries
    KParams k;
    std::memset(&k, 0, sizeof(k));
    fill_common(k, pb, a->err);
    TTT_TRY(encode_view(&k.own[0], a->v, pb, 128));
    TTT_TRY(encode_p(&k.str[0], a->p, pb, ttt::from_p_box_rows(ttt::kFpDK)));
    TTT_TRY(encode_view(&k.str[1], a->dout, pb, ttt::from_p_stream_rows(ttt::kFpDK)));
    TTT_TRY(encode_view(&k.str[2], a->q, pb, ttt::from_p_stream_rows(ttt::kFpDK)));
    k.delta = a->rowsum;
    set_out0(k, a->dk);
    ProfScope prof(TTT_K_FROM_P, s);
    TTT_TRY(launched(ttt::launch_from_p(k, pb.d, bf16, causal, ttt::kFpDK, s)));
  }
  {
    // dQ: query-major, dO resident, P / V / K streamed per 128 keys
    KParams k;
    std::memset(&k, 0, sizeof(k));
    fill_common(k, pb, a->err);
    TTT_TRY(encode_view(&k.own[0], a->dout, pb, 128));
    TTT_TRY(encode_p(&k.str[0], a->p, pb, ttt::from_p_box_rows(ttt::kFpDQ)));
    TTT_TRY(encode_view(&k.str[1], a->v, pb, ttt::from_p_stream_rows(ttt::kFpDQ)));
    TTT_TRY(encode_view(&k.str[2], a->k, pb, ttt::from_p_stream_rows(ttt::kFpDQ)));
    k.delta = a->rowsum;
    set_out0(k, a->dq);
    ProfScope prof(TTT_K_FROM_P, s);
    TTT_TRY(launched(ttt::launch_from_p(k, pb.d, bf16, causal, ttt::kFpDQ, s)));
  }
  return TTT_OK;
}

int ttt_attn_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  const int prev = g_prof_on ? 1 : 0;
  g_prof_on = on != 0;
  return prev;
}

int ttt_attn_profile_collect(int32_t* counts, double* total_ms, int n_kinds) {
  std::vector<ProfRecord> recs;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    recs.swap(g_prof);
  }
  int status = TTT_OK;
  for (const ProfRecord& r : recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.stop) != cudaSuccess || cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess)
      status = TTT_ERR_LAUNCH;
    if (r.kind >= 0 && r.kind < n_kinds) {
      if (counts) counts[r.kind] += 1;
      if (total_ms) total_ms[r.kind] += ms;
    }
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_event_pool[r.device].push_back(r.start);
    g_event_pool[r.device].push_back(r.stop);
  }
  return status;
}

int ttt_attn_error_mirror(int32_t* host_word) {
  unsigned long long ctx = 0;
  if (!ttt::current_context_id(&ctx)) return TTT_ERR_LAUNCH;
  if (host_word != nullptr) {
    if ((reinterpret_cast<uintptr_t>(host_word) & 3u) != 0) return TTT_ERR_ALIGN;
    // kernels write it through the same address: pinned host memory mapped into
    // the device's address space at that address (unified addressing)
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, host_word) != cudaSuccess || at.type != cudaMemoryTypeHost ||
        at.devicePointer != static_cast<void*>(host_word))
      return TTT_ERR_MIRROR;
  }
  std::lock_guard<std::mutex> lk(g_mirror_mu);
  if (host_word != nullptr) {
    g_mirror[ctx] = host_word;
  } else {
    g_mirror.erase(ctx);
  }
  g_any_mirror = !g_mirror.empty();
  return TTT_OK;
}

int ttt_attn_error_take(void) {
  unsigned long long ctx = 0;
  {
    std::lock_guard<std::mutex> lk(g_mirror_mu);
    if (!g_any_mirror) return 0;
  }
  if (!ttt::current_context_id(&ctx)) return 0;
  std::lock_guard<std::mutex> lk(g_mirror_mu);
  auto it = g_mirror.find(ctx);
  if (it == g_mirror.end()) return 0;
  volatile int32_t* w = it->second;
  const int32_t code = *w;
  if (code != 0) *w = 0;
  return code;
}

int ttt_attn_selftest_wait(int64_t limit_ns, int32_t* err, void* stream) {
  if (err == nullptr) return TTT_ERR_NULL;
  if (limit_ns <= 0 || limit_ns > 10000000000LL) return TTT_ERR_SHAPE;
  return launched(ttt::launch_selftest_wait(static_cast<unsigned long long>(limit_ns), err, error_mirror(),
                                            static_cast<cudaStream_t>(stream)));
}

int ttt_attn_selftest_umma(const void* a, const void* b, float* c, int n, int k, int dtype, int mode, int32_t* err,
                           void* stream) {
  const int b_mn_major = mode & 1;
  const bool a_tmem = (mode & 2) != 0;
  if (!a || !b || !c) return TTT_ERR_NULL;
  if (dtype != TTT_F16 && dtype != TTT_BF16) return TTT_ERR_DTYPE;
  if (!(n == 64 || n == 128 || n == 256) || !(k == 64 || k == 128)) return TTT_ERR_SHAPE;
  if (!aligned16(a) || !aligned16(b) || !aligned16(c)) return TTT_ERR_ALIGN;
  CUtensorMap ta, tb;
  ttt_problem pa{1, 1, 128, k, dtype, 0, 1.f};
  ttt_view va{const_cast<void*>(a), 128 * k, 128 * k, k};
  TTT_TRY(encode_view(&ta, va, pa, 128));
  if (b_mn_major) {
    // b is [k x n]: rows = k, row length n (encoded as "d" = n, box 64 columns x k rows)
    EncodeTiledFn fn = encode_fn();
    if (!fn) return TTT_ERR_DRIVER;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(k), 1, 1};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(n) * 2, static_cast<cuuint64_t>(n) * k * 2,
                             static_cast<cuuint64_t>(n) * k * 2};
    cuuint32_t box[4] = {64, static_cast<cuuint32_t>(k), 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(&tb, dtype == TTT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                    const_cast<void*>(b), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return TTT_ERR_TENSOR_MAP;
  } else {
    ttt_problem pbk{1, 1, n, k, dtype, 0, 1.f};
    ttt_view vb{const_cast<void*>(b), n * k, n * k, k};
    TTT_TRY(encode_view(&tb, vb, pbk, n));
  }
  return launched(ttt::launch_selftest_umma(ta, tb, a, c, n, k, dtype == TTT_BF16, b_mn_major != 0, a_tmem, err,
                                            static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
