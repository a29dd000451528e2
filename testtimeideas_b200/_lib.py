"""Bindings of libttt_attn.so (include/ttt_attn.h) and the tensor-level ops.

The forward, backward and double backward run through the PyTorch operators
ttt::fwd, ttt::bwd and ttt::bwd2 of libttt_torch.so (C++ over the C ABI; their
shape functions are registered here, so torch.compile traces through them).
The remaining entry points (P-materializing forward, passes over a given P,
the allocation-free double backward, test hooks) are called through ctypes.

Every op here runs the sm_100a kernels; there is no CPU or PyTorch fallback:
if a library is missing or the tensors are not CUDA fp16/bf16 with
d in {64, 128}, the op raises.
"""

from __future__ import annotations

import ctypes
import math
import os
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_lib" / "libttt_attn.so"
TORCH_OPS_PATH = _PKG / "_lib" / "libttt_torch.so"

TTT_F16, TTT_BF16 = 0, 1
_STATUS = {
    0: "ok", 1: "null pointer", 2: "dtype", 3: "head dim", 4: "shape", 5: "stride", 6: "alignment",
    7: "tensor map", 8: "launch", 9: "driver entry point", 10: "unsupported", 11: "scratch", 12: "scratch setup",
    13: "error mirror",
}


class View(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("sb", ctypes.c_int64), ("sh", ctypes.c_int64), ("st", ctypes.c_int64)]


class Problem(ctypes.Structure):
    _fields_ = [("b", ctypes.c_int32), ("h", ctypes.c_int32), ("t", ctypes.c_int32), ("d", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("causal", ctypes.c_int32), ("scale", ctypes.c_float),
                ("window", ctypes.c_int32), ("window_kind", ctypes.c_int32)]


class FwdArgs(ctypes.Structure):
    _fields_ = [("pb", Problem), ("q", View), ("k", View), ("v", View), ("o", View),
                ("lse2", ctypes.c_void_p), ("p", ctypes.c_void_p), ("err", ctypes.c_void_p),
                ("work", ctypes.c_void_p), ("work_bytes", ctypes.c_int64)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("pb", Problem), ("q", View), ("k", View), ("v", View), ("o", View), ("dout", View),
                ("lse2", ctypes.c_void_p), ("delta", ctypes.c_void_p),
                ("dq", View), ("dk", View), ("dv", View), ("err", ctypes.c_void_p),
                ("work", ctypes.c_void_p), ("work_bytes", ctypes.c_int64)]


class Bwd2Args(ctypes.Structure):
    _fields_ = [("pb", Problem), ("q", View), ("k", View), ("v", View), ("dout", View),
                ("lse2", ctypes.c_void_p), ("delta", ctypes.c_void_p),
                ("uq", View), ("uk", View), ("uv", View),
                ("gamma", ctypes.c_void_p), ("rho", ctypes.c_void_p),
                ("gq", View), ("gk", View), ("gv", View), ("gdout", View), ("err", ctypes.c_void_p),
                ("work", ctypes.c_void_p), ("work_bytes", ctypes.c_int64)]


class FromPArgs(ctypes.Structure):
    _fields_ = [("pb", Problem), ("p", View), ("q", View), ("k", View), ("v", View), ("dout", View),
                ("rowsum", ctypes.c_void_p), ("rowsum_out", ctypes.c_void_p),
                ("dq", View), ("dk", View), ("dv", View), ("err", ctypes.c_void_p)]


# Every symbol include/ttt_attn.h declares.
EXPORTED = ("ttt_attn_fwd", "ttt_attn_bwd", "ttt_attn_bwd2", "ttt_attn_t_pad", "ttt_attn_status_string",
            "ttt_attn_abi_version", "ttt_attn_selftest_umma", "ttt_attn_profile_enable", "ttt_attn_profile_collect",
            "ttt_attn_bwd2_noalloc", "ttt_attn_dv_from_p", "ttt_attn_rowsum_from_p", "ttt_attn_dqdk_from_p",
            "ttt_attn_work_bytes", "ttt_attn_split_count", "ttt_attn_error_mirror", "ttt_attn_error_take",
            "ttt_attn_selftest_wait")
ERR_WORD_TIMEOUT = 0x40000000  # TTT_ERR_WORD_TIMEOUT
SELFTEST_WAIT_SITE = 0xFE
NOALLOC_MAX_ROWS = 1 << 20  # TTT_ATTN_NOALLOC_MAX_ROWS
KERNEL_KINDS = ("fwd", "delta", "bwd_kv", "bwd_q", "bwd2_stats", "bwd2_q", "bwd2_kv", "from_p")

_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load libttt_attn.so (once). Raises if it has not been built."""
    global _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} not found: build the CUDA library first (python -m testtimeideas_b200.build)")
        lib = ctypes.CDLL(str(p))
        for name in ("ttt_attn_fwd", "ttt_attn_bwd", "ttt_attn_bwd2", "ttt_attn_bwd2_noalloc", "ttt_attn_dv_from_p",
                     "ttt_attn_rowsum_from_p", "ttt_attn_dqdk_from_p"):
            getattr(lib, name).restype = ctypes.c_int
            getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.ttt_attn_t_pad.restype = ctypes.c_int
        lib.ttt_attn_t_pad.argtypes = [ctypes.c_int]
        lib.ttt_attn_status_string.restype = ctypes.c_char_p
        lib.ttt_attn_status_string.argtypes = [ctypes.c_int]
        lib.ttt_attn_abi_version.restype = ctypes.c_int
        lib.ttt_attn_work_bytes.restype = ctypes.c_int64
        lib.ttt_attn_work_bytes.argtypes = [ctypes.c_void_p]
        lib.ttt_attn_split_count.restype = ctypes.c_int
        lib.ttt_attn_split_count.argtypes = [ctypes.c_void_p]
        lib.ttt_attn_selftest_umma.restype = ctypes.c_int
        lib.ttt_attn_selftest_umma.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p]
        lib.ttt_attn_error_mirror.restype = ctypes.c_int
        lib.ttt_attn_error_mirror.argtypes = [ctypes.c_void_p]
        lib.ttt_attn_error_take.restype = ctypes.c_int
        lib.ttt_attn_error_take.argtypes = []
        lib.ttt_attn_selftest_wait.restype = ctypes.c_int
        lib.ttt_attn_selftest_wait.argtypes = [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        lib.ttt_attn_profile_enable.restype = ctypes.c_int
        lib.ttt_attn_profile_enable.argtypes = [ctypes.c_int]
        lib.ttt_attn_profile_collect.restype = ctypes.c_int
        lib.ttt_attn_profile_collect.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        if path is None:
            _lib = lib
        return lib


class KernelError(RuntimeError):
    pass


_ops_loaded = False


def load_torch_ops() -> None:
    """Load libttt_torch.so (once): registers ttt::fwd, ttt::bwd, ttt::bwd2 and
    ttt::error_word, and their shape functions. Raises if it has not been built."""
    global _ops_loaded
    if _ops_loaded:
        return
    with _lib_lock:
        if _ops_loaded:
            return
        if not TORCH_OPS_PATH.exists():
            raise RuntimeError(
                f"{TORCH_OPS_PATH} not found: build the libraries first (python -m testtimeideas_b200.build)")
        torch.ops.load_library(str(TORCH_OPS_PATH))
        _register_fakes()
        _ops_loaded = True


def _register_fakes() -> None:
    """Output shapes of the operators for tracing (FakeTensor / torch.compile)."""

    @torch.library.register_fake("ttt::fwd")
    def _fwd(q, k, v, causal, scale, window=0, window_kind=0, split=True):
        b, h, t, d = q.shape
        return q.new_empty((b, h, t, d)), q.new_empty((b * h, t_pad(t)), dtype=torch.float32)

    @torch.library.register_fake("ttt::bwd")
    def _bwd(q, k, v, o, dout, lse2, causal, scale, window=0, window_kind=0, split=True):
        b, h, t, d = q.shape
        return (q.new_empty((b, h, t, d)), q.new_empty((b, h, t, d)), q.new_empty((b, h, t, d)),
                q.new_empty((b * h, t_pad(t)), dtype=torch.float32))

    @torch.library.register_fake("ttt::bwd2")
    def _bwd2(q, k, v, dout, lse2, delta, uq, uk, uv, causal, scale, need_gdout, window=0, window_kind=0,
              split=True):
        b, h, t, d = q.shape
        return (q.new_empty((b, h, t, d)), q.new_empty((b, h, t, d)), q.new_empty((b, h, t, d)),
                q.new_empty((b, h, t, d)) if need_gdout else q.new_empty((0,)))

    @torch.library.register_fake("ttt::error_word")
    def _err(device):
        return torch.empty((1,), dtype=torch.int32, device=device)


def _op(fn, *args):
    """Call an operator; a failure it reports from the library becomes KernelError."""
    if torch.compiler.is_compiling():
        return fn(*args)
    try:
        return fn(*args)
    except RuntimeError as e:
        msg = str(e)
        if "libttt_attn" in msg:
            raise KernelError(msg.splitlines()[0]) from None
        raise


def _check(status: int) -> None:
    if status != 0:
        msg = load_library().ttt_attn_status_string(status).decode()
        raise KernelError(f"libttt_attn: {msg} (status {status})")


def t_pad(t: int) -> int:
    return (t + 127) // 128 * 128


# ---------------------------------------------------------------- device error word
# Per device, libttt_torch.so owns the int32 error word the kernels report into
# (device memory) and a pinned host mirror of it, registered with the library
# for the device's context (ttt_attn_error_mirror). A kernel that gives up on a
# bounded wait writes the mirror too, so every op checks it at entry without
# synchronizing: a timeout surfaces as KernelError at the first op the host
# issues after the failing kernel reported it (check_device_errors also
# synchronizes and reads the word itself).
_err_words: dict[int, torch.Tensor] = {}


def _dev_index(device: torch.device | None) -> int:
    if device is None or device.index is None:
        return torch.cuda.current_device()
    return device.index


def error_word(device: torch.device) -> torch.Tensor:
    idx = _dev_index(device)
    w = _err_words.get(idx)
    if w is None:
        load_torch_ops()
        w = torch.ops.ttt.error_word(torch.device("cuda", idx))
        _err_words[idx] = w
    return w


def raise_pending(device: torch.device | None = None) -> None:
    """Raise KernelError if a kernel on `device` has reported a failed bounded wait
    to the host mirror; no synchronization. Clears both words (the device word in
    stream order), so that later launches run again."""
    idx = _dev_index(device)
    if idx not in _err_words:
        return  # no op has run on this device yet
    with _on(torch.device("cuda", idx)):
        code = load_library().ttt_attn_error_take()
        if code == 0:
            return
        _err_words[idx].zero_()
    raise KernelError(f"libttt_attn kernel gave up on a bounded wait on cuda:{idx} (error word 0x{code:08x}); "
                      "results of the calls since then are invalid")


def check_device_errors(device: torch.device | None = None) -> None:
    """Synchronize and raise if any kernel on `device` gave up on a bounded wait."""
    dev = torch.device("cuda", _dev_index(device))
    w = error_word(dev)
    torch.cuda.synchronize(dev)
    with _on(dev):
        code = int(w.item())
        pending = load_library().ttt_attn_error_take()
        if code == 0:
            code = pending
        if code != 0:
            w.zero_()
            torch.cuda.synchronize(dev)
    if code != 0:
        raise KernelError(f"libttt_attn kernel timeout on {dev} (error word 0x{code:08x})")


def selftest_wait(limit_ns: int, device: torch.device | None = None) -> None:
    """Run the library's bounded mbarrier wait on a barrier nothing completes, with a
    limit of `limit_ns` (test hook of the failure path). Asynchronous: the error word
    and the host mirror receive the timeout code once the limit has passed."""
    dev = torch.device("cuda", _dev_index(device))
    with _on(dev):
        w = error_word(dev)
        _check(load_library().ttt_attn_selftest_wait(int(limit_ns), w.data_ptr(), _stream()))


_SYNC_CHECK = os.environ.get("TTT_ATTN_SYNC_CHECK", "0") == "1"


# ---------------------------------------------------------------- argument plumbing
def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return TTT_F16
    if t.dtype == torch.bfloat16:
        return TTT_BF16
    raise TypeError(f"ttt attention kernels take fp16 or bf16 tensors, got {t.dtype}")


def prep(x: torch.Tensor) -> torch.Tensor:
    """Return x, or a contiguous copy when its layout cannot feed a TMA tensor map
    (d stride != 1, a stride not a multiple of 8 elements, or a misaligned base)."""
    if x.dim() != 4:
        raise ValueError(f"expected a [b, h, t, d] tensor, got shape {tuple(x.shape)}")
    shape, st = x.shape, x.stride()
    ok = st[3] == 1 and x.data_ptr() % 16 == 0
    if ok:
        for i in range(3):
            if shape[i] > 1 and (st[i] <= 0 or st[i] % 8 != 0):
                ok = False
    return x if ok else x.contiguous()


def view(x: torch.Tensor | None) -> View:
    if x is None:
        return View(None, 0, 0, 0)
    st = x.stride()
    return View(x.data_ptr(), st[0], st[1], st[2])


WINDOW_KINDS = {"sliding": 0, "chunk": 1}


def window_args(window=0) -> tuple[int, int]:
    """window: 0, an int W (sliding: key j visible to query i iff i - W < j <= i) or
    a (W, kind) pair with kind "sliding" or "chunk" (chunk-local, see include/ttt_attn.h);
    returns (W, kind code)."""
    w, kind = (window, "sliding") if isinstance(window, int) else window
    return int(w), WINDOW_KINDS[kind]


def problem(q: torch.Tensor, causal: bool, scale: float, window=0) -> Problem:
    b, h, t, d = q.shape
    w, kind = window_args(window)
    return Problem(b, h, t, d, _dtype_code(q), 1 if causal else 0, float(scale), w, kind)


def validate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("ttt attention kernels need CUDA tensors")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"q, k, v must share one [b, h, t, d] shape, got {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("q, k, v must share one dtype")
    _dtype_code(q)
    if q.shape[-1] not in (64, 128):
        raise ValueError(f"head dim must be 64 or 128, got {q.shape[-1]}")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k, v must be on one device")


def work_space(pb: Problem, device: torch.device):
    """(buffer, pointer, bytes) of the work space with which the passes of `pb`
    split their tiles over more CTAs (include/ttt_attn.h); (None, None, 0) when
    no pass would split. The caching allocator's blocks are 512-byte aligned."""
    n = int(load_library().ttt_attn_work_bytes(ctypes.byref(pb)))
    if n <= 0:
        return None, None, 0
    buf = torch.empty(n, dtype=torch.uint8, device=device)
    return buf, buf.data_ptr(), n


class _on:
    """Make `device` current for the block; a no-op when it already is (the common
    case, cheaper than torch.cuda.device)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.prev != self.idx:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev != self.idx:
            torch.cuda.set_device(self.prev)


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def default_scale(d: int) -> float:
    return 1.0 / math.sqrt(d)


# ---------------------------------------------------------------- ops
def attn_fwd(q, k, v, causal: bool, scale: float, save_p: bool = False, window: int = 0, split: bool = True):
    """O, lse2 (fp32 [b*h, t_pad]) and, with save_p, P ([b, h, t, t]; else None).
    split=False keeps small causal problems unsplit (see include/ttt_attn.h)."""
    if save_p:
        return _attn_fwd_with_p(q, k, v, causal, scale, window)
    validate(q, k, v)
    load_torch_ops()
    w, kind = window_args(window)
    o, lse2 = _op(torch.ops.ttt.fwd, q, k, v, bool(causal), float(scale), w, kind, bool(split))
    if _SYNC_CHECK:
        check_device_errors(q.device)
    return o, lse2, None


def _attn_fwd_with_p(q, k, v, causal: bool, scale: float, window: int = 0):
    """The forward that also writes P (for the from-P helpers), through the C ABI."""
    validate(q, k, v)
    raise_pending(q.device)
    lib = load_library()
    q, k, v = prep(q), prep(k), prep(v)
    b, h, t, d = q.shape
    with _on(q.device):
        o = torch.empty((b, h, t, d), dtype=q.dtype, device=q.device)
        lse2 = torch.empty((b * h, t_pad(t)), dtype=torch.float32, device=q.device)
        # causal: the kernel writes only key tiles up to the diagonal; the rest stays zero
        p = (torch.zeros if causal else torch.empty)((b, h, t, t), dtype=q.dtype, device=q.device)
        pb = problem(q, causal, scale, window)
        work, wptr, wbytes = work_space(pb, q.device)
        args = FwdArgs(pb, view(q), view(k), view(v), view(o), lse2.data_ptr(), p.data_ptr(),
                       error_word(q.device).data_ptr(), wptr, wbytes)
        _check(lib.ttt_attn_fwd(ctypes.byref(args), _stream()))
        if _SYNC_CHECK:
            check_device_errors(q.device)
    return o, lse2, p


def attn_bwd(q, k, v, o, dout, lse2, causal: bool, scale: float, window: int = 0, split: bool = True):
    """dq, dk, dv and delta = rowsum(dout o o) (fp32 [b*h, t_pad])."""
    validate(q, k, v)
    load_torch_ops()
    w, kind = window_args(window)
    dq, dk, dv, delta = _op(torch.ops.ttt.bwd, q, k, v, o, dout, lse2, bool(causal), float(scale), w, kind,
                            bool(split))
    if _SYNC_CHECK:
        check_device_errors(q.device)
    return dq, dk, dv, delta


def attn_bwd2(q, k, v, dout, lse2, delta, uq, uk, uv, causal: bool, scale: float, need_gdout: bool,
              window: int = 0, split: bool = True):
    """Second-order gradients gq, gk, gv (and gdout when requested, else None).
    A probe given as None is zero."""
    validate(q, k, v)
    load_torch_ops()
    zeros = None
    if uq is None or uk is None or uv is None:
        zeros = torch.zeros_like(q, memory_format=torch.contiguous_format)
    uq, uk, uv = (zeros if u is None else u for u in (uq, uk, uv))
    w, kind = window_args(window)
    gq, gk, gv, gdout = _op(torch.ops.ttt.bwd2, q, k, v, dout, lse2, delta, uq, uk, uv, bool(causal), float(scale),
                            bool(need_gdout), w, kind, bool(split))
    if _SYNC_CHECK:
        check_device_errors(q.device)
    return gq, gk, gv, (gdout if need_gdout else None)


def selftest_umma(a: torch.Tensor, b: torch.Tensor, b_mn_major: bool, a_tmem: bool = False) -> torch.Tensor:
    """c = a @ (b if b_mn_major else b.T) on one tcgen05 tile (test hook); with a_tmem the
    A operand is staged in tensor memory."""
    lib = load_library()
    a, b = a.contiguous(), b.contiguous()
    k = a.shape[1]
    n = b.shape[1] if b_mn_major else b.shape[0]
    c = torch.empty((128, n), dtype=torch.float32, device=a.device)
    _check(lib.ttt_attn_selftest_umma(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, k, _dtype_code(a),
                                      (1 if b_mn_major else 0) | (2 if a_tmem else 0),
                                      error_word(a.device).data_ptr(), _stream()))
    return c


# ---------------------------------------------------------------- profiling hook
def profile_enable(on: bool = True) -> bool:
    """Bracket every kernel launch with CUDA events (on its stream). Returns the previous setting."""
    return bool(load_library().ttt_attn_profile_enable(1 if on else 0))


def profile_collect() -> dict:
    """{kind: (launches, total_ms)} since the last collect; waits for the recorded events."""
    n = len(KERNEL_KINDS)
    counts = (ctypes.c_int32 * n)()
    ms = (ctypes.c_double * n)()
    _check(load_library().ttt_attn_profile_collect(counts, ms, n))
    return {k: (int(counts[i]), float(ms[i])) for i, k in enumerate(KERNEL_KINDS)}


def attn_bwd2_noalloc(q, k, v, dout, lse2, delta, uq, uk, uv, causal: bool, scale: float, need_gdout: bool):
    """attn_bwd2 through ttt_attn_bwd2_noalloc: the gamma/rho scratch comes from the
    library's built-in array (b*h*t_pad <= NOALLOC_MAX_ROWS), for callers that may
    not allocate device memory while the op runs; only outputs are allocated here."""
    validate(q, k, v)
    raise_pending(q.device)
    lib = load_library()
    q, k, v, dout = prep(q), prep(k), prep(v), prep(dout.to(q.dtype))
    uq, uk, uv = (prep(u.to(q.dtype)) for u in (uq, uk, uv))
    with _on(q.device):
        gq, gk, gv = (torch.empty_like(q, memory_format=torch.contiguous_format) for _ in range(3))
        gdout = torch.empty_like(q, memory_format=torch.contiguous_format) if need_gdout else None
        args = Bwd2Args(problem(q, causal, scale), view(q), view(k), view(v), view(dout), lse2.data_ptr(),
                        delta.data_ptr(), view(uq), view(uk), view(uv), None, None,
                        view(gq), view(gk), view(gv), view(gdout), error_word(q.device).data_ptr())
        _check(lib.ttt_attn_bwd2_noalloc(ctypes.byref(args), _stream()))
        if _SYNC_CHECK:
            check_device_errors(q.device)
    return gq, gk, gv, gdout


# ---------------------------------------------------------------- passes over materialized P
def prep_p(p: torch.Tensor) -> torch.Tensor:
    """P as a [b, h, t, t] view TMA can read: unit column stride, 16-byte aligned
    base, row and head strides multiples of 8 elements. Otherwise copied into a
    zero-padded buffer whose rows are rounded up to 8 elements."""
    if p.dim() != 4 or p.shape[-1] != p.shape[-2]:
        raise ValueError(f"expected P as [b, h, t, t], got shape {tuple(p.shape)}")
    b, h, t, _ = p.shape
    ok = p.stride(3) == 1 and p.data_ptr() % 16 == 0 and p.stride(2) >= t and p.stride(2) % 8 == 0
    for size, stride in ((b, p.stride(0)), (h, p.stride(1))):
        if size > 1 and (stride <= 0 or stride % 8 != 0):
            ok = False
    if ok:
        return p
    tp = (t + 7) // 8 * 8
    buf = torch.zeros((b, h, t, tp), dtype=p.dtype, device=p.device)
    buf[..., :t].copy_(p)
    return buf[..., :t]


def _from_p_check(p: torch.Tensor, *xs: torch.Tensor) -> None:
    if not p.is_cuda or any(not x.is_cuda for x in xs):
        raise ValueError("ttt attention kernels need CUDA tensors")
    ref = xs[0]
    _dtype_code(ref)
    if ref.shape[-1] not in (64, 128):
        raise ValueError(f"head dim must be 64 or 128, got {ref.shape[-1]}")
    for x in xs:
        if x.shape != ref.shape or x.dtype != ref.dtype:
            raise ValueError("the [b, h, t, d] operands must share one shape and dtype")
    b, h, t, _ = ref.shape
    if tuple(p.shape) != (b, h, t, t):
        raise ValueError(f"P must be [b, h, t, t] = {(b, h, t, t)}, got {tuple(p.shape)}")


def _from_p_args(p, ref, causal: bool, scale: float, **views) -> FromPArgs:
    a = FromPArgs()
    a.pb = problem(ref, causal, scale)
    a.p = view(p)
    for name, x in views.items():
        if isinstance(x, torch.Tensor) and x.dtype == torch.float32 and x.dim() == 2:
            setattr(a, name, x.data_ptr())
        else:
            setattr(a, name, view(x))
    a.err = error_word(ref.device).data_ptr()
    return a


def dv_from_p(p: torch.Tensor, dout: torch.Tensor) -> torch.Tensor:
    """dV = P^T dout for P [b, h, t, t] and dout [b, h, t, d] (every entry of P is read)."""
    _from_p_check(p, dout)
    raise_pending(dout.device)
    lib = load_library()
    p, dout = prep_p(p.to(dout.dtype)), prep(dout)
    with torch.cuda.device(dout.device):
        dv = torch.empty_like(dout, memory_format=torch.contiguous_format)
        args = _from_p_args(p, dout, False, 1.0, dout=dout, dv=dv)
        _check(lib.ttt_attn_dv_from_p(ctypes.byref(args), _stream()))
        if _SYNC_CHECK:
            check_device_errors(dout.device)
    return dv


def rowsum_from_p(p: torch.Tensor, dout: torch.Tensor, v: torch.Tensor, causal: bool) -> torch.Tensor:
    """rowsum[b, h, i] = sum_j P_ij (dout_i . v_j), fp32 [b, h, t]."""
    _from_p_check(p, dout, v)
    raise_pending(dout.device)
    lib = load_library()
    p, dout, v = prep_p(p.to(dout.dtype)), prep(dout), prep(v)
    b, h, t, _ = dout.shape
    with torch.cuda.device(dout.device):
        rs = torch.empty((b * h, t), dtype=torch.float32, device=dout.device)
        args = _from_p_args(p, dout, causal, 1.0, dout=dout, v=v, rowsum_out=rs)
        _check(lib.ttt_attn_rowsum_from_p(ctypes.byref(args), _stream()))
        if _SYNC_CHECK:
            check_device_errors(dout.device)
    return rs.view(b, h, t)


def dqdk_from_p(q, k, v, dout, p, rowsum, causal: bool, scale: float):
    """dq = scale dS k, dk = scale dS^T q with dS = P o (dout v^T - rowsum)."""
    _from_p_check(p, q, k, v, dout)
    raise_pending(q.device)
    lib = load_library()
    q, k, v, dout = prep(q), prep(k), prep(v), prep(dout)
    p = prep_p(p.to(q.dtype))
    b, h, t, _ = q.shape
    rs = rowsum.reshape(b * h, t).to(torch.float32).contiguous()
    with _on(q.device):
        dq, dk = (torch.empty_like(q, memory_format=torch.contiguous_format) for _ in range(2))
        args = _from_p_args(p, q, causal, scale, q=q, k=k, v=v, dout=dout, rowsum=rs, dq=dq, dk=dk)
        _check(lib.ttt_attn_dqdk_from_p(ctypes.byref(args), _stream()))
        if _SYNC_CHECK:
            check_device_errors(q.device)
    return dq, dk
