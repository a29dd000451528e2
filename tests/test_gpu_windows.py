"""Banded causal masks on the sm_100a kernels: the sliding window of
make_window_mask and the chunk-local band of WindowedSelfAttention's chunk loop
(both pinned to the reference by tests/test_ttt_e2e_cpu.py), through the C ABI
and through the TTT-E2E drop-in. Tolerance as elsewhere: max|x - ref| /
max(1, max|ref|) <= 2e-3 (fp16), 1e-2 (bf16) against float64."""

import math

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib, ttt_e2e

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
NAMES = ("q", "k", "v", "do", "uq", "uk", "uv")
CASES = [(200, 64, "sliding"), (257, 100, "sliding"), (129, 1, "sliding"), (384, 300, "sliding"),
         (512, 128, "chunk"), (300, 64, "chunk"), (200, 96, "chunk"), (260, 130, "chunk")]


def _err(x, ref):
    return orc.normalized_err(x.float().cpu(), torch.as_tensor(ref))


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("t,w,kind", CASES, ids=[f"t{t}w{w}{k}" for t, w, k in CASES])
def test_band_kernels_match_oracle(d, dtype, t, w, kind):
    b, h = 1, 2
    inp = orc.seeded_inputs(b, h, t, d, seed=t + w + d, scale_in=0.5)
    ref = orc.closed_form_gradgrad(*(inp[n].numpy() for n in NAMES), causal=True, window=w, window_kind=kind)
    x = {n: inp[n].to(dtype).cuda() for n in NAMES}
    scale, band = 1.0 / math.sqrt(d), (w, kind)
    o, lse2, _ = _lib.attn_fwd(x["q"], x["k"], x["v"], True, scale, window=band)
    assert _err(o, ref["o"]) <= TOL[dtype]
    dq, dk, dv, delta = _lib.attn_bwd(x["q"], x["k"], x["v"], o, x["do"], lse2, True, scale, window=band)
    for name, val in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert _err(val, ref[name]) <= TOL[dtype], name
    gq, gk, gv, gdo = _lib.attn_bwd2(x["q"], x["k"], x["v"], x["do"], lse2, delta, x["uq"], x["uk"], x["uv"], True,
                                     scale, True, window=band)
    for name, val in (("gq", gq), ("gk", gk), ("gv", gv), ("gdo", gdo)):
        assert _err(val, ref[name]) <= TOL[dtype], name
    _lib.check_device_errors()


def test_band_needs_causal_and_no_p():
    x = torch.zeros(1, 1, 128, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.KernelError):
        _lib.attn_fwd(x, x, x, False, 0.125, window=16)
    with pytest.raises(_lib.KernelError):
        _lib.attn_fwd(x, x, x, True, 0.125, save_p=True, window=16)


def test_gradgrad_attention_fn_with_window_mask():
    b, h, t, d, w, dtype = 2, 3, 300, 64, 70, torch.bfloat16
    inp = orc.seeded_inputs(b, h, t, d, seed=3, scale_in=0.5)
    ref = orc.math_gradgrad(*(inp[n] for n in NAMES), causal=True, need_gdo=True, window=w, window_kind="sliding")
    q, k, v, do = (inp[n].to(dtype).cuda().requires_grad_(True) for n in ("q", "k", "v", "do"))
    mask = ttt_e2e.make_window_mask(t, w, q.device, dtype).view(1, 1, t, t)
    out = ttt_e2e.GradGradAttentionFn.apply(q, k, v, mask)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), do, create_graph=True)
    u = {n: inp[n].to(dtype).cuda() for n in ("uq", "uk", "uv")}
    l2 = (dq * u["uq"]).float().sum() + (dk * u["uk"]).float().sum() + (dv * u["uv"]).float().sum()
    gq, gk, gv, gdo = torch.autograd.grad(l2, (q, k, v, do))
    for name, val in (("o", out), ("dq", dq), ("dk", dk), ("dv", dv), ("gq", gq), ("gk", gk), ("gv", gv),
                      ("gdo", gdo)):
        assert _err(val.detach(), ref[name]) <= TOL[dtype], name
    with pytest.raises(ValueError):
        ttt_e2e.GradGradAttentionFn.apply(q, k, v, torch.zeros(t, t, device="cuda", dtype=dtype))


@pytest.mark.parametrize("t,window", [(200, 64), (256, 128), (100, 128), (100, None)])
def test_windowed_self_attention_cuda_matches_cpu(t, window):
    """The module on CUDA (bf16, one kernel call over the band) against the
    reference formulation on CPU (float64, chunk loop) with the same weights:
    output, input gradient with create_graph, and the second-order input gradient."""
    d_model, n_heads = 128, 2
    torch.manual_seed(7)
    cpu = ttt_e2e.WindowedSelfAttention(d_model, n_heads, window).double()
    gpu = ttt_e2e.WindowedSelfAttention(d_model, n_heads, window).to("cuda", torch.bfloat16)
    gpu.load_state_dict({n: p.to(torch.bfloat16) for n, p in cpu.state_dict().items()})
    gen = torch.Generator().manual_seed(t)
    x, g, u = (torch.randn(2, t, d_model, generator=gen, dtype=torch.float64) for _ in range(3))

    def run(mod, dev, dtype):
        xx = x.to(dev, dtype).requires_grad_(True)
        y = mod(xx)
        (gx,) = torch.autograd.grad(y, xx, g.to(dev, dtype), create_graph=True)
        (ggx,) = torch.autograd.grad((gx.float() * u.to(dev, torch.float32)).sum(), xx)
        return y.detach(), gx.detach(), ggx

    ref = run(cpu, "cpu", torch.float64)
    got = run(gpu, "cuda", torch.bfloat16)
    # bf16 weights and activations through four projections: a looser bound than the kernel tests
    for a, r in zip(got, ref):
        assert orc.normalized_err(a.float().cpu(), r) <= 5e-2
    _lib.check_device_errors()
