"""GPU tests of the PyTorch operators ttt::fwd, ttt::bwd and ttt::bwd2
(libttt_torch.so over the C ABI): torch.library's operator checks (schema,
shape functions against the real kernels, dispatch), and torch.compile
tracing through the reference-compatible entry point."""

import math

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(b, h, t, d, dtype, seed=3):
    inp = orc.seeded_inputs(b, h, t, d, seed=seed, scale_in=0.5)
    return {n: x.to(dtype).cuda() for n, x in inp.items()}


@pytest.mark.parametrize("causal", [False, True])
def test_opcheck(causal):
    _lib.load_torch_ops()
    x = _inputs(1, 2, 192, 64, torch.float16)
    scale = 1.0 / math.sqrt(64)
    o, lse2 = torch.ops.ttt.fwd(x["q"], x["k"], x["v"], causal, scale)
    _, _, _, delta = torch.ops.ttt.bwd(x["q"], x["k"], x["v"], o, x["do"], lse2, causal, scale)
    torch.library.opcheck(torch.ops.ttt.fwd.default, (x["q"], x["k"], x["v"], causal, scale))
    torch.library.opcheck(torch.ops.ttt.bwd.default, (x["q"], x["k"], x["v"], o, x["do"], lse2, causal, scale))
    torch.library.opcheck(torch.ops.ttt.bwd2.default, (x["q"], x["k"], x["v"], x["do"], lse2, delta, x["uq"], x["uk"],
                                                       x["uv"], causal, scale, True))
    _lib.check_device_errors()


def test_compiled_forward_matches_eager():
    import ttt_kernels
    x = _inputs(2, 2, 256, 128, torch.bfloat16)
    f = torch.compile(lambda q, k, v: ttt_kernels.triton_attention(q, k, v, causal=True), fullgraph=True)
    with torch.no_grad():
        got = f(x["q"], x["k"], x["v"])
        ref = ttt_kernels.triton_attention(x["q"], x["k"], x["v"], causal=True)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    _lib.check_device_errors()


def test_compiled_forward_and_backward_match_eager():
    import ttt_kernels
    x = _inputs(1, 2, 192, 64, torch.float16, seed=9)

    def step(q, k, v):
        return ttt_kernels.triton_attention(q, k, v, causal=True)

    f = torch.compile(step)
    outs = []
    for fn in (f, step):
        q, k, v = (x[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
        o = fn(q, k, v)
        g = torch.autograd.grad(o, (q, k, v), x["do"])
        outs.append((o.detach(), *g))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    _lib.check_device_errors()
