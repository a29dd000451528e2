"""GPU test of the allocation-free double backward, ttt_attn_bwd2_noalloc.

Some callers of this library may not allocate device memory while the op
runs, for example a host runtime that plans all of its memory ahead of time
and hands a plugin only its input and output buffers. For them the library
offers ttt_attn_bwd2_noalloc: the same double backward as ttt_attn_bwd2, but
its two scratch rows (gamma, rho) live in a fixed array inside the library
instead of being passed in. This file checks, through the C ABI, that it
returns the same results as ttt_attn_bwd2 on two calls in a row (the array
keeps the previous call's contents between calls), and that problems larger
than the array are refused before anything runs.

The file name makes pytest collect it last.
"""

import ctypes
import math

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
TTT_ERR_SCRATCH = 11


def _setup(b, h, t, d, dtype, causal, seed):
    inp = {n: x.to(dtype).cuda() for n, x in orc.seeded_inputs(b, h, t, d, seed=seed, scale_in=0.5).items()}
    scale = 1.0 / math.sqrt(d)
    o, lse2, _ = _lib.attn_fwd(inp["q"], inp["k"], inp["v"], causal, scale)
    _, _, _, delta = _lib.attn_bwd(inp["q"], inp["k"], inp["v"], o, inp["do"], lse2, causal, scale)
    return inp, lse2, delta, scale


def _call_noalloc(lib, inp, lse2, delta, causal, scale):
    """ttt_attn_bwd2_noalloc through ctypes; gamma and rho are passed as NULL."""
    q = inp["q"]
    gq, gk, gv, gdo = (torch.empty_like(q) for _ in range(4))
    args = _lib.Bwd2Args(_lib.problem(q, causal, scale), _lib.view(q), _lib.view(inp["k"]), _lib.view(inp["v"]),
                         _lib.view(inp["do"]), lse2.data_ptr(), delta.data_ptr(), _lib.view(inp["uq"]),
                         _lib.view(inp["uk"]), _lib.view(inp["uv"]), None, None, _lib.view(gq), _lib.view(gk),
                         _lib.view(gv), _lib.view(gdo), _lib.error_word(q.device).data_ptr())
    status = lib.ttt_attn_bwd2_noalloc(ctypes.byref(args),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == 0, lib.ttt_attn_status_string(status)
    return gq, gk, gv, gdo


@pytest.mark.parametrize("dtype,causal,shape", [
    (torch.float16, True, (1, 2, 300, 64)),
    (torch.bfloat16, False, (2, 1, 257, 128)),
])
def test_noalloc_matches_bwd2_on_two_calls(dtype, causal, shape):
    lib = _lib.load_library()
    b, h, t, d = shape
    inp, lse2, delta, scale = _setup(b, h, t, d, dtype, causal, seed=91)
    ref = _lib.attn_bwd2(inp["q"], inp["k"], inp["v"], inp["do"], lse2, delta, inp["uq"], inp["uk"], inp["uv"],
                         causal, scale, need_gdout=True)
    for _ in range(2):
        out = _call_noalloc(lib, inp, lse2, delta, causal, scale)
        torch.cuda.synchronize()
        for name, x, r in zip(("gq", "gk", "gv", "gdo"), out, ref):
            err = orc.normalized_err(x.float().cpu(), r.float().cpu())
            assert err <= TOL[dtype], f"{name}: {err:.3e}"
    _lib.check_device_errors()


def test_noalloc_refuses_problems_above_its_scratch():
    lib = _lib.load_library()
    # b*h*t_pad = 2^20 + 128 rows: one row block past the built-in array
    pb = _lib.Problem(1, 1, (1 << 20) + 1, 64, 0, 1, 0.125)
    args = _lib.Bwd2Args()
    args.pb = pb
    assert lib.ttt_attn_bwd2_noalloc(ctypes.byref(args), None) == TTT_ERR_SCRATCH
