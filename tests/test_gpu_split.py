"""GPU tests of split mode: a causal pass over few heads spreads each CTA's tile
stream over several CTAs when the caller supplies work space
(ttt_attn_work_bytes), and a reduction kernel sums their fp32 partials in
order. The split results must match the oracle to the same tolerance as the
unsplit ones, and match the unsplit kernels (same math, other summation order).
"""

import ctypes
import math

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


def _inputs(b, h, t, d, dtype, seed):
    return {n: x.to(dtype).cuda() for n, x in orc.seeded_inputs(b, h, t, d, seed=seed, scale_in=0.5).items()}


def _passes(inp, causal, scale, split=True):
    q, k, v = inp["q"], inp["k"], inp["v"]
    o, lse2, _ = _lib.attn_fwd(q, k, v, causal, scale, split=split)
    dq, dk, dv, delta = _lib.attn_bwd(q, k, v, o, inp["do"], lse2, causal, scale, split=split)
    gq, gk, gv, _ = _lib.attn_bwd2(q, k, v, inp["do"], lse2, delta, inp["uq"], inp["uk"], inp["uv"], causal, scale,
                                   need_gdout=False, split=split)
    torch.cuda.synchronize()
    return {"o": o, "dq": dq, "dk": dk, "dv": dv, "gq": gq, "gk": gk, "gv": gv}


def test_small_causal_problems_split():
    lib = _lib.load_library()
    pb = _lib.Problem(1, 1, 16384, 64, 0, 1, 0.125)
    assert lib.ttt_attn_split_count(ctypes.byref(pb)) > 1
    assert lib.ttt_attn_work_bytes(ctypes.byref(pb)) > 16384 * 64 * 4  # split slices + the dQ accumulator
    big = _lib.Problem(8, 32, 16384, 128, 1, 1, 0.125)  # config 4: enough CTAs, no split
    assert lib.ttt_attn_split_count(ctypes.byref(big)) == 1
    assert lib.ttt_attn_work_bytes(ctypes.byref(big)) == 0
    band = _lib.Problem(1, 1, 16384, 64, 0, 1, 0.125, 512, 0)  # banded: CTAs of equal length
    assert lib.ttt_attn_split_count(ctypes.byref(band)) == 1
    assert lib.ttt_attn_work_bytes(ctypes.byref(band)) == 16384 * 64 * 4  # the dQ accumulator only


@pytest.mark.parametrize("dtype,shape", [
    (torch.float16, (1, 1, 1000, 64)),
    (torch.bfloat16, (1, 2, 777, 128)),
    (torch.float16, (1, 1, 4096, 64)),
])
def test_split_matches_oracle_and_unsplit(dtype, shape):
    b, h, t, d = shape
    causal, scale = True, 1.0 / math.sqrt(d)
    pb = _lib.Problem(b, h, t, d, _lib.TTT_BF16 if dtype == torch.bfloat16 else _lib.TTT_F16, 1, scale)
    assert _lib.load_library().ttt_attn_split_count(ctypes.byref(pb)) > 1
    inp = _inputs(b, h, t, d, dtype, seed=17)
    split = _passes(inp, causal, scale)
    unsplit = _passes(inp, causal, scale, split=False)
    for name in split:
        err = orc.normalized_err(split[name].float().cpu(), unsplit[name].float().cpu())
        assert err <= TOL[dtype] / 4, f"{name}: split vs unsplit {err:.3e}"
    if t <= 1024:
        ref = orc.closed_form_gradgrad(*(inp[n].double().cpu() for n in ("q", "k", "v", "do", "uq", "uk", "uv")),
                                       causal=causal, scale=scale)
        for name, key in (("dk", "dk"), ("dv", "dv"), ("gk", "gk"), ("gv", "gv")):
            err = orc.normalized_err(split[name].float().cpu(), torch.from_numpy(ref[key]).float())
            assert err <= TOL[dtype], f"{name}: {err:.3e}"
    _lib.check_device_errors()


@pytest.mark.parametrize("dtype,causal,shape", [
    (torch.float16, False, (1, 2, 257, 64)),
    (torch.bfloat16, False, (2, 1, 1000, 64)),
    (torch.float16, True, (1, 3, 448, 64)),
    (torch.bfloat16, True, (1, 1, 192, 64)),
])
def test_fused_dq_matches_two_passes_and_oracle(dtype, causal, shape):
    """d = 64 with the work space: dQ comes out of the key-major pass (pairs of query
    tiles, rows added into an fp32 accumulator); without it, from the query-major pass.
    Odd tile counts (257, 1000, 192 rows) leave a last pair with one tile."""
    b, h, t, d = shape
    scale = 1.0 / math.sqrt(d)
    inp = _inputs(b, h, t, d, dtype, seed=23)
    q, k, v = inp["q"], inp["k"], inp["v"]
    o, lse2, _ = _lib.attn_fwd(q, k, v, causal, scale, split=False)
    fused = _lib.attn_bwd(q, k, v, o, inp["do"], lse2, causal, scale)
    two = _lib.attn_bwd(q, k, v, o, inp["do"], lse2, causal, scale, split=False)
    torch.cuda.synchronize()
    ref = orc.closed_form_gradgrad(*(inp[n].double().cpu() for n in ("q", "k", "v", "do", "uq", "uk", "uv")),
                                   causal=causal, scale=scale)
    for i, name in enumerate(("dq", "dk", "dv")):
        err = orc.normalized_err(fused[i].float().cpu(), two[i].float().cpu())
        assert err <= TOL[dtype] / 4, f"{name}: fused vs two passes {err:.3e}"
        err = orc.normalized_err(fused[i].float().cpu(), torch.from_numpy(ref[name]).float())
        assert err <= TOL[dtype], f"{name}: {err:.3e}"
    _lib.check_device_errors()
