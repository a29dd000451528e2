"""GPU parity at ragged and tiny sequence lengths: T = 1, 2, a few below and above
the 64-row streamed tile and the 128-row CTA block, for both head dims, causal and
non-causal. Every kernel of the step (forward, delta, first-order backward, the
statistics pass and both halves of the double backward, with the dout gradient)
runs with its partial tiles masked at the sequence end; the results must match
the float64 oracle to the path's tolerance, and pad rows of the statistics must
hold their pad values.
"""

import math

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
NAMES = ("q", "k", "v", "do", "uq", "uk", "uv")
LENGTHS = (1, 2, 17, 63, 65, 127, 129)


@pytest.fixture(scope="module", autouse=True)
def _library():
    lib = _lib.load_library()  # raises if the extension was not built: no fallback
    yield lib
    _lib.check_device_errors()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("t", LENGTHS)
def test_ragged_lengths_gradgrad(t, causal, d):
    dtype = torch.float16 if d == 64 else torch.bfloat16
    b, h = 1, 2
    inp = {n: x.to(dtype).cuda() for n, x in orc.seeded_inputs(b, h, t, d, seed=1000 + t + d, scale_in=0.5).items()}
    scale = 1.0 / math.sqrt(d)
    q, k, v = inp["q"], inp["k"], inp["v"]
    o, lse2, _ = _lib.attn_fwd(q, k, v, causal, scale)
    dq, dk, dv, delta = _lib.attn_bwd(q, k, v, o, inp["do"], lse2, causal, scale)
    gq, gk, gv, gdo = _lib.attn_bwd2(q, k, v, inp["do"], lse2, delta, inp["uq"], inp["uk"], inp["uv"], causal, scale,
                                     need_gdout=True)
    torch.cuda.synchronize()
    ref = orc.math_gradgrad(*(inp[n].detach().cpu().double() for n in NAMES), causal=causal, need_gdo=True)
    got = {"o": o, "dq": dq, "dk": dk, "dv": dv, "gq": gq, "gk": gk, "gv": gv, "gdo": gdo}
    for name, x in got.items():
        err = orc.normalized_err(x.detach().float().cpu(), ref[name])
        assert err <= TOL[dtype], f"T={t} {name}: normalized max-abs error {err:.3e} > {TOL[dtype]:.0e}"
    # statistics rows past the sequence keep their pad values
    assert torch.isinf(lse2[:, t:]).all() and (lse2[:, t:] > 0).all()
    assert (delta[:, t:] == 0).all()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("t", (1, 8, 24, 127, 136))
def test_ragged_lengths_probabilities(t, causal, d):
    """The P output of the forward at short and ragged lengths: T % 8 == 0 takes the row-LSE
    forward and the TMA-store P pass (a partial box at the sequence end), other T the
    single-kernel forward. Entries above the diagonal stay exactly zero."""
    dtype = torch.float16 if d == 64 else torch.bfloat16
    b, h = 1, 2
    inp = {n: x.to(dtype).cuda() for n, x in orc.seeded_inputs(b, h, t, d, seed=2000 + t + d, scale_in=0.5).items()}
    scale = 1.0 / math.sqrt(d)
    o, lse2, p = _lib.attn_fwd(inp["q"], inp["k"], inp["v"], causal, scale, save_p=True)
    torch.cuda.synchronize()
    s = (inp["q"].double() @ inp["k"].double().transpose(-1, -2)) * scale
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(t, t, dtype=torch.bool, device=s.device), 1), float("-inf"))
    pr = torch.softmax(s, -1)
    assert tuple(p.shape) == (b, h, t, t)
    assert (p.double() - pr).abs().max().item() <= TOL[dtype]
    if causal:
        upper = torch.triu(torch.ones(t, t, dtype=torch.bool, device=p.device), 1)
        assert int((p[..., upper] != 0).sum()) == 0
    ref = orc.math_gradgrad(*(inp[n].detach().cpu().double() for n in NAMES), causal=causal)
    assert orc.normalized_err(o.float().cpu(), ref["o"]) <= TOL[dtype]


@pytest.mark.parametrize("d,dtype,shape", [
    (64, torch.float16, (1, 2, 384)),
    (128, torch.bfloat16, (1, 2, 384)),
    (64, torch.float16, (1, 1, 2048)),   # causal: split forward, shares with very different row maxima
])
@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
def test_growing_row_max(d, dtype, shape, causal):
    """Keys whose norm grows along the sequence, so that a row's running max rises by far
    more than 2^8 (log2 domain) after its first key tiles: the forward's conditional O
    rescale runs, several times per row, and split shares carry maxima far apart."""
    b, h, t = shape
    inp = orc.seeded_inputs(b, h, t, d, seed=77 + t + d, scale_in=0.5)
    ramp = torch.linspace(0.25, 16.0, t, dtype=inp["k"].dtype).view(1, 1, t, 1)
    inp["k"] = inp["k"] * ramp
    inp = {n: x.to(dtype).cuda() for n, x in inp.items()}
    scale = 1.0 / math.sqrt(d)
    s2 = (inp["q"].float() @ inp["k"].float().transpose(-1, -2)) * scale * math.log2(math.e)
    assert (s2[..., -1].abs().max() - s2[..., 0].abs().max()).item() > 8  # past the rescale threshold (2^8)
    q, k, v = inp["q"], inp["k"], inp["v"]
    o, lse2, _ = _lib.attn_fwd(q, k, v, causal, scale)
    dq, dk, dv, delta = _lib.attn_bwd(q, k, v, o, inp["do"], lse2, causal, scale)
    gq, gk, gv, gdo = _lib.attn_bwd2(q, k, v, inp["do"], lse2, delta, inp["uq"], inp["uk"], inp["uv"], causal, scale,
                                     need_gdout=True)
    torch.cuda.synchronize()
    ref = orc.math_gradgrad(*(inp[n].detach().cpu().double() for n in NAMES), causal=causal, need_gdo=True)
    got = {"o": o, "dq": dq, "dk": dk, "dv": dv, "gq": gq, "gk": gk, "gv": gv, "gdo": gdo}
    for name, x in got.items():
        err = orc.normalized_err(x.detach().float().cpu(), ref[name])
        assert err <= TOL[dtype], f"{name}: normalized max-abs error {err:.3e} > {TOL[dtype]:.0e}"
