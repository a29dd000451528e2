// PyTorch operators over the C ABI of libttt_attn.so: ttt::fwd, ttt::bwd and
// ttt::bwd2 (TORCH_LIBRARY), the launch wrappers the reference writes inline
// in Python (ttt_kernels/triton_attention.py:278-337 for the forward,
// :340-420 for the backward; backward_stubs.py:124-514 for the terms of the
// double backward). Dispatch, argument checks, output allocation (PyTorch's
// caching allocator, on the current device and stream) and the call into the
// C ABI happen here in C++; the autograd Functions in attention.py call these
// operators, and their shape functions (fake implementations) are registered
// in Python so that torch.compile can trace through them.
//
// Failure reporting: this file owns one int32 error word per device (device
// memory) and a pinned host mirror of it, registered with
// ttt_attn_error_mirror for the device's context. Kernels that give up on a
// bounded wait write both; every operator checks the mirror at entry (no
// synchronization) and raises, after clearing both words in stream order, so a
// timeout surfaces at the first call made after the failing kernel reported it.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "ttt_attn.h"

namespace {

struct DeviceWords {
  at::Tensor word;    // int32 [1] on the device
  at::Tensor mirror;  // int32 [1], pinned host memory (undefined if registration failed)
};

std::mutex g_mu;
// Never destroyed: tensors held past interpreter shutdown must not be freed
// after the CUDA runtime has gone.
std::map<int, DeviceWords>* g_words = new std::map<int, DeviceWords>();

// The device's error word, created (and its mirror registered) on first use;
// the device must be current.
at::Tensor error_word_for(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_words->find(dev);
  if (it != g_words->end()) return it->second.word;
  DeviceWords w;
  w.word = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
  at::Tensor m = at::zeros({1}, at::TensorOptions().dtype(at::kInt).pinned_memory(true));
  if (ttt_attn_error_mirror(m.data_ptr<int32_t>()) == TTT_OK) w.mirror = m;
  g_words->emplace(dev, w);
  return w.word;
}

void raise_if_pending(int dev, at::Tensor& word) {
  const int code = ttt_attn_error_take();
  if (code == 0) return;
  word.zero_();
  char hex[16];
  std::snprintf(hex, sizeof(hex), "0x%08x", static_cast<unsigned>(code));
  TORCH_CHECK(false, "libttt_attn kernel gave up on a bounded wait on cuda:", dev, " (error word ", hex,
              "); results of the calls since then are invalid");
}

void check(int status, const char* op) {
  TORCH_CHECK(status == TTT_OK, "libttt_attn: ", ttt_attn_status_string(status), " (status ", status, ") in ", op);
}

// x, or a contiguous copy when its layout cannot feed a TMA tensor map (d
// stride != 1, a b/h/t stride not a positive multiple of 8 elements, or a base
// address that is not 16-byte aligned).
at::Tensor prep(const at::Tensor& x) {
  TORCH_CHECK(x.dim() == 4, "expected a [b, h, t, d] tensor, got ", x.sizes());
  bool ok = x.stride(3) == 1 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15u) == 0;
  for (int i = 0; i < 3 && ok; ++i)
    if (x.size(i) > 1 && (x.stride(i) <= 0 || x.stride(i) % 8 != 0)) ok = false;
  return ok ? x : x.contiguous();
}

ttt_view view(const at::Tensor& x) {
  ttt_view v;
  v.ptr = x.data_ptr();
  v.sb = x.stride(0);
  v.sh = x.stride(1);
  v.st = x.stride(2);
  return v;
}

void validate(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "ttt attention kernels need CUDA tensors");
  TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(),
              "q, k, v must share one [b, h, t, d] shape, got ", q.sizes(), ", ", k.sizes(), ", ", v.sizes());
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(), "q, k, v must share one dtype");
  TORCH_CHECK(q.scalar_type() == at::kHalf || q.scalar_type() == at::kBFloat16,
              "ttt attention kernels take fp16 or bf16 tensors, got ", q.scalar_type());
  TORCH_CHECK(q.dim() == 4 && (q.size(3) == 64 || q.size(3) == 128), "head dim must be 64 or 128, got ", q.sizes());
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device(), "q, k, v must be on one device");
}

ttt_problem problem(const at::Tensor& q, bool causal, double scale, int64_t window, int64_t window_kind) {
  ttt_problem pb;
  pb.b = static_cast<int32_t>(q.size(0));
  pb.h = static_cast<int32_t>(q.size(1));
  pb.t = static_cast<int32_t>(q.size(2));
  pb.d = static_cast<int32_t>(q.size(3));
  pb.dtype = q.scalar_type() == at::kBFloat16 ? TTT_BF16 : TTT_F16;
  pb.causal = causal ? 1 : 0;
  pb.scale = static_cast<float>(scale);
  pb.window = static_cast<int32_t>(window);
  pb.window_kind = static_cast<int32_t>(window_kind);
  return pb;
}

// Work space with which small causal problems split their passes over more
// CTAs (undefined tensor when none would split, or with split == false).
at::Tensor work_space(const ttt_problem& pb, const at::Tensor& like, bool split) {
  const int64_t n = split ? ttt_attn_work_bytes(&pb) : 0;
  return n > 0 ? at::empty({n}, like.options().dtype(at::kByte)) : at::Tensor();
}

int64_t t_pad(int64_t t) { return ttt_attn_t_pad(static_cast<int>(t)); }

std::tuple<at::Tensor, at::Tensor> op_fwd(const at::Tensor& q_, const at::Tensor& k_, const at::Tensor& v_, bool causal,
                                          double scale, int64_t window, int64_t window_kind, bool split) {
  validate(q_, k_, v_);
  c10::cuda::CUDAGuard guard(q_.device());
  const int dev = q_.get_device();
  at::Tensor word = error_word_for(dev);
  raise_if_pending(dev, word);
  const at::Tensor q = prep(q_), k = prep(k_), v = prep(v_);
  const int64_t b = q.size(0), h = q.size(1), t = q.size(2), d = q.size(3);
  at::Tensor o = at::empty({b, h, t, d}, q.options());
  at::Tensor lse2 = at::empty({b * h, t_pad(t)}, q.options().dtype(at::kFloat));
  ttt_fwd_args a{};
  a.pb = problem(q, causal, scale, window, window_kind);
  a.q = view(q), a.k = view(k), a.v = view(v), a.o = view(o);
  a.lse2 = lse2.data_ptr<float>();
  a.p = nullptr;
  a.err = word.data_ptr<int32_t>();
  at::Tensor work = work_space(a.pb, q, split);
  a.work = work.defined() ? work.data_ptr() : nullptr;
  a.work_bytes = work.defined() ? work.numel() : 0;
  check(ttt_attn_fwd(&a, c10::cuda::getCurrentCUDAStream().stream()), "ttt::fwd");
  return {o, lse2};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> op_bwd(const at::Tensor& q_, const at::Tensor& k_,
                                                                  const at::Tensor& v_, const at::Tensor& o_,
                                                                  const at::Tensor& dout_, const at::Tensor& lse2,
                                                                  bool causal, double scale, int64_t window,
                                                                  int64_t window_kind, bool split) {
  validate(q_, k_, v_);
  TORCH_CHECK(o_.sizes() == q_.sizes() && dout_.sizes() == q_.sizes(), "o and dout must have q's shape");
  c10::cuda::CUDAGuard guard(q_.device());
  const int dev = q_.get_device();
  at::Tensor word = error_word_for(dev);
  raise_if_pending(dev, word);
  const at::Tensor q = prep(q_), k = prep(k_), v = prep(v_), o = prep(o_.to(q_.scalar_type()));
  const at::Tensor dout = prep(dout_.to(q_.scalar_type()));
  const at::Tensor l2 = lse2.contiguous();
  const int64_t b = q.size(0), h = q.size(1), t = q.size(2);
  TORCH_CHECK(l2.scalar_type() == at::kFloat && l2.numel() == b * h * t_pad(t), "lse2 must be fp32 [b*h, t_pad]");
  at::Tensor dq = at::empty(q.sizes(), q.options()), dk = at::empty(q.sizes(), q.options());
  at::Tensor dv = at::empty(q.sizes(), q.options());
  at::Tensor delta = at::empty({b * h, t_pad(t)}, q.options().dtype(at::kFloat));
  ttt_bwd_args a{};
  a.pb = problem(q, causal, scale, window, window_kind);
  a.q = view(q), a.k = view(k), a.v = view(v), a.o = view(o), a.dout = view(dout);
  a.lse2 = l2.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dq = view(dq), a.dk = view(dk), a.dv = view(dv);
  a.err = word.data_ptr<int32_t>();
  at::Tensor work = work_space(a.pb, q, split);
  a.work = work.defined() ? work.data_ptr() : nullptr;
  a.work_bytes = work.defined() ? work.numel() : 0;
  check(ttt_attn_bwd(&a, c10::cuda::getCurrentCUDAStream().stream()), "ttt::bwd");
  return {dq, dk, dv, delta};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> op_bwd2(
    const at::Tensor& q_, const at::Tensor& k_, const at::Tensor& v_, const at::Tensor& dout_,
    const at::Tensor& lse2, const at::Tensor& delta, const at::Tensor& uq_, const at::Tensor& uk_,
    const at::Tensor& uv_, bool causal, double scale, bool need_gdout, int64_t window, int64_t window_kind,
    bool split) {
  validate(q_, k_, v_);
  for (const at::Tensor* x : {&dout_, &uq_, &uk_, &uv_})
    TORCH_CHECK(x->sizes() == q_.sizes(), "dout and the probes must have q's shape");
  c10::cuda::CUDAGuard guard(q_.device());
  const int dev = q_.get_device();
  at::Tensor word = error_word_for(dev);
  raise_if_pending(dev, word);
  const auto st = q_.scalar_type();
  const at::Tensor q = prep(q_), k = prep(k_), v = prep(v_), dout = prep(dout_.to(st));
  const at::Tensor uq = prep(uq_.to(st)), uk = prep(uk_.to(st)), uv = prep(uv_.to(st));
  const at::Tensor l2 = lse2.contiguous(), dl = delta.contiguous();
  const int64_t b = q.size(0), h = q.size(1), t = q.size(2);
  TORCH_CHECK(l2.scalar_type() == at::kFloat && l2.numel() == b * h * t_pad(t), "lse2 must be fp32 [b*h, t_pad]");
  TORCH_CHECK(dl.scalar_type() == at::kFloat && dl.numel() == b * h * t_pad(t), "delta must be fp32 [b*h, t_pad]");
  at::Tensor gq = at::empty(q.sizes(), q.options()), gk = at::empty(q.sizes(), q.options());
  at::Tensor gv = at::empty(q.sizes(), q.options());
  at::Tensor gdout = need_gdout ? at::empty(q.sizes(), q.options()) : at::empty({0}, q.options());
  at::Tensor rows = at::empty({2, b * h, t_pad(t)}, q.options().dtype(at::kFloat));  // gamma, rho
  ttt_bwd2_args a{};
  a.pb = problem(q, causal, scale, window, window_kind);
  a.q = view(q), a.k = view(k), a.v = view(v), a.dout = view(dout);
  a.lse2 = l2.data_ptr<float>();
  a.delta = dl.data_ptr<float>();
  a.uq = view(uq), a.uk = view(uk), a.uv = view(uv);
  a.gamma = rows.data_ptr<float>();
  a.rho = a.gamma + b * h * t_pad(t);
  a.gq = view(gq), a.gk = view(gk), a.gv = view(gv);
  a.gdout = need_gdout ? view(gdout) : ttt_view{nullptr, 0, 0, 0};
  a.err = word.data_ptr<int32_t>();
  at::Tensor work = work_space(a.pb, q, split);
  a.work = work.defined() ? work.data_ptr() : nullptr;
  a.work_bytes = work.defined() ? work.numel() : 0;
  check(ttt_attn_bwd2(&a, c10::cuda::getCurrentCUDAStream().stream()), "ttt::bwd2");
  return {gq, gk, gv, gdout};
}

at::Tensor op_error_word(c10::Device device) {
  TORCH_CHECK(device.is_cuda(), "ttt::error_word takes a CUDA device");
  const int dev = device.has_index() ? device.index() : c10::cuda::current_device();
  c10::cuda::CUDAGuard guard(dev);
  return error_word_for(dev);
}

}  // namespace

TORCH_LIBRARY(ttt, m) {
  // window / window_kind: the band of ttt_problem; split=false keeps every pass unsplit
  // (no work space), which the tests use to compare the two forms.
  m.def("fwd(Tensor q, Tensor k, Tensor v, bool causal, float scale, int window=0, int window_kind=0, "
        "bool split=True) -> (Tensor o, Tensor lse2)");
  m.def("bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor dout, Tensor lse2, bool causal, float scale, "
        "int window=0, int window_kind=0, bool split=True) -> (Tensor dq, Tensor dk, Tensor dv, Tensor delta)");
  m.def("bwd2(Tensor q, Tensor k, Tensor v, Tensor dout, Tensor lse2, Tensor delta, Tensor uq, Tensor uk, "
        "Tensor uv, bool causal, float scale, bool need_gdout, int window=0, int window_kind=0, bool split=True) "
        "-> (Tensor gq, Tensor gk, Tensor gv, Tensor gdout)");
  // The device's error word (int32 [1]; the same storage on every call).
  m.def("error_word(Device device) -> Tensor");
}

TORCH_LIBRARY_IMPL(ttt, CUDA, m) {
  m.impl("fwd", &op_fwd);
  m.impl("bwd", &op_bwd);
  m.impl("bwd2", &op_bwd2);
}

TORCH_LIBRARY_IMPL(ttt, CompositeExplicitAutograd, m) { m.impl("error_word", &op_error_word); }
