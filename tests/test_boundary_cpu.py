"""Host-side tests that need no GPU: the C-ABI library loads and exports every
declared symbol, host argument validation, and the autograd wiring of the
Python surface (checked on CPU by substituting oracle-backed ops for the
kernels behind the same seam)."""

import ctypes
import math
import re
from pathlib import Path

import pytest
import torch

import testtimeideas_b200 as tb
from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib, attention

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "ttt_attn.h"


def _declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int64_t|int|const char\*)\s+(ttt_attn_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from testtimeideas_b200 import build
        build.build()
    return _lib.load_library()


def test_header_declares_entry_points():
    names = _declared_functions()
    for n in ("ttt_attn_fwd", "ttt_attn_bwd", "ttt_attn_bwd2"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert set(_lib.EXPORTED) >= set(_declared_functions())


def test_host_helpers(lib):
    assert lib.ttt_attn_abi_version() == 3
    assert lib.ttt_attn_t_pad(1) == 128 and lib.ttt_attn_t_pad(128) == 128 and lib.ttt_attn_t_pad(129) == 256
    assert lib.ttt_attn_status_string(0) == b"ok"
    assert b"64 or 128" in lib.ttt_attn_status_string(3)


def test_work_bytes_query(lib):
    # invalid problems need no work space
    bad = _lib.Problem(1, 1, 128, 96, 0, 1, 0.125)
    assert lib.ttt_attn_work_bytes(ctypes.byref(bad)) == 0
    assert lib.ttt_attn_work_bytes(None) == 0
    assert lib.ttt_attn_split_count(None) == 1
    # d = 128, non-causal: nothing splits and dQ keeps its own pass
    wide = _lib.Problem(1, 1, 16384, 128, 0, 0, 0.125)
    assert lib.ttt_attn_work_bytes(ctypes.byref(wide)) == 0
    # d = 64: the fused backward's fp32 dQ accumulator [b*h][t_pad][d]
    noncausal = _lib.Problem(2, 3, 1000, 64, 0, 0, 0.125)
    assert lib.ttt_attn_split_count(ctypes.byref(noncausal)) == 1
    assert lib.ttt_attn_work_bytes(ctypes.byref(noncausal)) == 2 * 3 * 1024 * 64 * 4
    if not torch.cuda.is_available():
        # without a GPU the SM count is unknown, so nothing splits
        causal = _lib.Problem(1, 1, 16384, 64, 0, 1, 0.125)
        assert lib.ttt_attn_split_count(ctypes.byref(causal)) == 1
        assert lib.ttt_attn_work_bytes(ctypes.byref(causal)) == 16384 * 64 * 4


def _fwd_args(**over):
    pb = _lib.Problem(1, 1, 128, 64, 0, 0, 0.125)
    for k, v in over.items():
        setattr(pb, k, v)
    dummy = 4096  # never dereferenced: validation fails or the test stops before a launch
    vw = _lib.View(dummy, 128 * 64, 128 * 64, 64)
    return _lib.FwdArgs(pb, vw, vw, vw, vw, dummy, None, None)


@pytest.mark.parametrize("field,value,status", [
    ("dtype", 7, 2), ("d", 96, 3), ("d", 256, 3), ("t", 0, 4), ("b", 0, 4), ("h", -1, 4),
])
def test_host_validation_rejects_bad_problems(lib, field, value, status):
    args = _fwd_args(**{field: value})
    assert lib.ttt_attn_fwd(ctypes.byref(args), None) == status


def test_host_validation_rejects_bad_views(lib):
    args = _fwd_args()
    args.q = _lib.View(None, 0, 0, 64)
    assert lib.ttt_attn_fwd(ctypes.byref(args), None) == 1
    args = _fwd_args()
    args.k = _lib.View(4096 + 8, 128 * 64, 128 * 64, 64)
    assert lib.ttt_attn_fwd(ctypes.byref(args), None) == 6
    args = _fwd_args()
    args.v = _lib.View(4096, 128 * 64, 128 * 64, 63)
    assert lib.ttt_attn_fwd(ctypes.byref(args), None) == 5
    args = _fwd_args()
    args.lse2 = None
    assert lib.ttt_attn_fwd(ctypes.byref(args), None) == 1
    assert lib.ttt_attn_fwd(None, None) == 1


def test_prep_makes_unsupported_layouts_contiguous():
    x = torch.randn(2, 3, 16, 64)
    assert _lib.prep(x) is x
    xt = torch.randn(2, 16, 3, 64).transpose(1, 2)  # [b, t, h, d] memory: strides stay multiples of 8
    assert _lib.prep(xt) is xt
    xs = torch.randn(2, 3, 16, 128)[..., ::2]
    assert _lib.prep(xs).is_contiguous()
    xe = torch.randn(1, 1, 1, 64).expand(2, 3, 16, 64)
    assert _lib.prep(xe).is_contiguous()


def test_kernel_path_rejects_cpu_and_bad_dtypes():
    q = torch.randn(1, 1, 8, 64)
    with pytest.raises(ValueError):
        _lib.validate(q, q, q)


# ---------------------------------------------------------------- autograd wiring on CPU
def _fake_ops(monkeypatch, calls):
    """Replace the kernel ops by oracle-backed CPU functions with the same contract."""

    def band(window):
        w, kind = (window, "sliding") if isinstance(window, int) else window
        return {"window": w, "window_kind": {"sliding": "sliding", "chunk": "chunk"}[kind]}

    def fwd(q, k, v, causal, scale, save_p=False, window=0):
        calls.append("fwd")
        out = orc.closed_form_gradgrad(q, k, v, q, q, q, q, causal=causal, scale=scale, **band(window))
        b, h, t, d = q.shape
        lse2 = torch.full((b * h, _lib.t_pad(t)), math.inf, dtype=torch.float32)
        lse2[:, :t] = torch.from_numpy(out["lse"]).reshape(b * h, t).float() / math.log(2.0)
        return torch.from_numpy(out["o"]).to(q.dtype), lse2, None

    def bwd(q, k, v, o, dout, lse2, causal, scale, window=0):
        calls.append("bwd")
        out = orc.closed_form_gradgrad(q.detach(), k.detach(), v.detach(), dout.detach(), q.detach(), q.detach(),
                                       q.detach(), causal=causal, scale=scale, **band(window))
        b, h, t, d = q.shape
        delta = torch.zeros((b * h, _lib.t_pad(t)))
        delta[:, :t] = torch.from_numpy(out["delta"]).reshape(b * h, t).float()
        cast = lambda a: torch.from_numpy(a).to(q.dtype)  # noqa: E731
        return cast(out["dq"]), cast(out["dk"]), cast(out["dv"]), delta

    def bwd2(q, k, v, dout, lse2, delta, uq, uk, uv, causal, scale, need_gdout, window=0):
        calls.append("bwd2" + ("+gdo" if need_gdout else ""))
        z = torch.zeros_like(q)
        uq, uk, uv = (z if u is None else u for u in (uq, uk, uv))
        out = orc.closed_form_gradgrad(q.detach(), k.detach(), v.detach(), dout.detach(), uq, uk, uv,
                                       causal=causal, scale=scale, **band(window))
        cast = lambda a: torch.from_numpy(a).to(q.dtype)  # noqa: E731
        return cast(out["gq"]), cast(out["gk"]), cast(out["gv"]), cast(out["gdo"]) if need_gdout else None

    monkeypatch.setattr(_lib, "attn_fwd", fwd)
    monkeypatch.setattr(_lib, "attn_bwd", bwd)
    monkeypatch.setattr(_lib, "attn_bwd2", bwd2)
    monkeypatch.setattr(attention, "_kernel_path", lambda q: True)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("mode", ["recompute", "save_p_triton_full", "custom"])
def test_autograd_wiring_matches_oracle(monkeypatch, causal, mode):
    calls = []
    _fake_ops(monkeypatch, calls)
    inp = orc.seeded_inputs(1, 2, 24, 64, seed=5, dtype=torch.float64)
    q, k, v = (inp[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    o = tb.triton_attention(q, k, v, causal=causal, bwd_mode=mode)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), inp["do"], create_graph=True)
    gq, gk, gv = torch.autograd.grad((dq, dk, dv), (q, k, v), (inp["uq"], inp["uk"], inp["uv"]))
    ref = orc.math_gradgrad(*(inp[n] for n in ("q", "k", "v", "do", "uq", "uk", "uv")), causal=causal)
    for name, x in zip(("o", "dq", "dk", "dv", "gq", "gk", "gv"), (o, dq, dk, dv, gq, gk, gv)):
        assert orc.normalized_err(x.detach(), ref[name]) < 1e-9, name
    assert calls == ["fwd", "bwd", "bwd2"]


def test_autograd_wiring_dout_requires_grad(monkeypatch):
    """When dO itself depends on the parameters (meta-learning), the double
    backward also returns d/d dO."""
    calls = []
    _fake_ops(monkeypatch, calls)
    inp = orc.seeded_inputs(1, 1, 16, 64, seed=6, dtype=torch.float64)
    q, k, v = (inp[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    w = inp["do"].clone().requires_grad_(True)
    o = tb.triton_attention(q, k, v, causal=True)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), w, create_graph=True)
    gq, gk, gv, gw = torch.autograd.grad((dq, dk, dv), (q, k, v, w), (inp["uq"], inp["uk"], inp["uv"]))
    ref = orc.math_gradgrad(*(inp[n] for n in ("q", "k", "v", "do", "uq", "uk", "uv")), causal=True, need_gdo=True)
    assert orc.normalized_err(gw, ref["gdo"]) < 1e-9
    assert calls == ["fwd", "bwd", "bwd2+gdo"]


def test_no_grad_backward_uses_plain_bwd(monkeypatch):
    calls = []
    _fake_ops(monkeypatch, calls)
    inp = orc.seeded_inputs(1, 1, 16, 64, seed=8, dtype=torch.float64)
    q = inp["q"].clone().requires_grad_(True)
    o = tb.triton_attention(q, inp["k"], inp["v"])
    o.backward(inp["do"])
    assert calls == ["fwd", "bwd"]
    with pytest.raises(RuntimeError):
        # the double backward is once-differentiable: a third order is refused
        q2 = inp["q"].clone().requires_grad_(True)
        o2 = tb.triton_attention(q2, inp["k"], inp["v"])
        (dq,) = torch.autograd.grad(o2, (q2,), inp["do"], create_graph=True)
        (g,) = torch.autograd.grad(dq, (q2,), inp["uq"], create_graph=True)
        torch.autograd.grad(g.sum(), (q2,))


@pytest.mark.parametrize("mode", ["recompute", "save_p", "save_p_triton_full", "dv_only"])
def test_cpu_math_path_matches_oracle(mode):
    """CPU tensors run the reference's math path, create_graph included."""
    import ttt_kernels
    inp = orc.seeded_inputs(1, 1, 20, 16, seed=9, dtype=torch.float64)
    q, k, v = (inp[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    o = ttt_kernels.triton_attention(q, k, v, causal=True, bwd_mode=mode)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), inp["do"], create_graph=True)
    gq, gk, gv = torch.autograd.grad((dq, dk, dv), (q, k, v), (inp["uq"], inp["uk"], inp["uv"]))
    ref = orc.math_gradgrad(*(inp[n] for n in ("q", "k", "v", "do", "uq", "uk", "uv")), causal=True)
    for name, x in zip(("gq", "gk", "gv"), (gq, gk, gv)):
        assert orc.normalized_err(x, ref[name]) < 1e-10, name


def test_dropin_surface_names():
    import ttt_kernels
    from ttt_kernels import backward_stubs, triton_attention as ta_mod  # noqa: F401
    assert ttt_kernels.__all__ == ["triton_attention"]
    import inspect
    sig = inspect.signature(ttt_kernels.triton_attention)
    assert list(sig.parameters) == ["q", "k", "v", "causal", "scale", "bwd_mode"]
    assert sig.parameters["bwd_mode"].default == "recompute"
    for name in ("triton_attn_bwd_dv", "triton_attn_bwd_dq", "triton_attn_bwd_dk", "triton_attn_bwd2_dq",
                 "triton_attn_bwd2_dk", "triton_attn_bwd2_dv"):
        assert callable(getattr(backward_stubs, name))


@pytest.mark.parametrize("kind", ["sliding", "chunk"])
def test_band_attention_wiring_matches_oracle(monkeypatch, kind):
    """ttt_e2e.BandAttentionFn's autograd wiring (forward, differentiable
    backward, double backward incl. the upstream gradient) on CPU through the
    same fake kernel ops, against the oracle with the same band."""
    from testtimeideas_b200 import ttt_e2e
    calls = []
    _fake_ops(monkeypatch, calls)
    inp = orc.seeded_inputs(1, 2, 40, 16, seed=4, scale_in=0.5)
    q, k, v, do = (inp[n].double().requires_grad_(True) for n in ("q", "k", "v", "do"))
    out = ttt_e2e.BandAttentionFn.apply(q, k, v, 12, kind)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), do, create_graph=True)
    l2 = (dq * inp["uq"]).sum() + (dk * inp["uk"]).sum() + (dv * inp["uv"]).sum()
    gq, gk, gv, gdo = torch.autograd.grad(l2, (q, k, v, do))
    ref = orc.math_gradgrad(*(inp[n] for n in ("q", "k", "v", "do", "uq", "uk", "uv")), causal=True, need_gdo=True,
                            window=12, window_kind=kind)
    for name, val in (("o", out), ("dq", dq), ("gq", gq), ("gk", gk), ("gv", gv), ("gdo", gdo)):
        assert orc.normalized_err(val.detach(), ref[name]) < 1e-10, name
    assert calls == ["fwd", "bwd", "bwd2+gdo"]


def test_failure_hooks_validate_on_the_host(lib):
    # argument errors are caught before anything is enqueued (no GPU needed)
    assert lib.ttt_attn_selftest_wait(1000, None, None) == 1  # TTT_ERR_NULL
    word = ctypes.c_int32(0)
    assert lib.ttt_attn_selftest_wait(0, ctypes.addressof(word), None) == 4  # TTT_ERR_SHAPE: limit out of range
    assert lib.ttt_attn_selftest_wait(20_000_000_000, ctypes.addressof(word), None) == 4
    assert b"pinned host memory" in lib.ttt_attn_status_string(13)


def test_torch_operators_register_with_shape_functions():
    """libttt_torch.so loads without a GPU and registers ttt::fwd / bwd / bwd2, whose
    shape functions let FakeTensor tracing (torch.compile) run without the kernels."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    if not _lib.TORCH_OPS_PATH.exists():
        from testtimeideas_b200 import build
        build.build_all()
    _lib.load_torch_ops()
    for name in ("fwd", "bwd", "bwd2", "error_word"):
        assert hasattr(torch.ops.ttt, name), name
    with FakeTensorMode():
        q = torch.empty(2, 3, 200, 64, dtype=torch.bfloat16, device="cuda")
        o, lse2 = torch.ops.ttt.fwd(q, q, q, True, 0.125)
        assert o.shape == q.shape and o.dtype == q.dtype
        assert lse2.shape == (6, 256) and lse2.dtype == torch.float32
        dq, dk, dv, delta = torch.ops.ttt.bwd(q, q, q, o, q, lse2, True, 0.125)
        assert dq.shape == dk.shape == dv.shape == q.shape and delta.shape == (6, 256)
        gq, gk, gv, gdo = torch.ops.ttt.bwd2(q, q, q, q, lse2, delta, q, q, q, True, 0.125, True)
        assert gq.shape == gk.shape == gv.shape == gdo.shape == q.shape
        assert torch.ops.ttt.bwd2(q, q, q, q, lse2, delta, q, q, q, True, 0.125, False)[3].numel() == 0
