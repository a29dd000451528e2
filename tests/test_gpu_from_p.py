"""Parity of the P-streaming kernels (ttt_attn_dv_from_p, ttt_attn_rowsum_from_p,
ttt_attn_dqdk_from_p, through the backward_stubs wrappers) with the oracle's
restatement of the reference's P-taking helpers (backward_stubs.py:124-425).

P comes from the attention forward of seeded inputs (causal: zero above the
diagonal, as the reference's softmax leaves it), in the input dtype. Errors
are max|x - ref| / max(1, max|ref|) against float64, within 2e-3 (fp16) and
1e-2 (bf16)."""

import math

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib
from ttt_kernels import backward_stubs as bs

pytestmark = pytest.mark.gpu
TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
SHAPES = [(1, 1, 64), (1, 2, 200), (2, 1, 257), (1, 1, 512), (1, 1, 1), (1, 2, 17), (1, 1, 129)]


def _case(b, h, t, d, dtype, causal, seed):
    inp = orc.seeded_inputs(b, h, t, d, seed=seed, scale_in=1.0)
    scale = 1.0 / math.sqrt(d)
    q, k, v, do = (inp[n].to(dtype) for n in ("q", "k", "v", "do"))
    s = torch.matmul(q.double(), k.double().transpose(-2, -1)) * scale
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(t, t, dtype=torch.bool), 1), float("-inf"))
    p = torch.softmax(s, dim=-1).to(dtype)
    return q, k, v, do, p, scale


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"b{b}h{h}t{t}" for b, h, t in SHAPES])
def test_from_p_kernels_match_oracle(d, dtype, causal, shape):
    b, h, t = shape
    q, k, v, do, p, scale = _case(b, h, t, d, dtype, causal, seed=t + d)
    cu = lambda x: x.cuda()  # noqa: E731
    dv = bs.triton_attn_bwd_dv_from_p(cu(p), cu(do))
    assert dv.dtype == dtype and dv.shape == do.shape
    assert orc.normalized_err(dv.float().cpu(), orc.dv_from_p(p, do)) <= TOL[dtype]
    rs = bs.triton_attn_rowsum_from_p(cu(p), cu(do), cu(v), causal=causal)
    assert rs.dtype == torch.float32 and rs.shape == (b, h, t)
    ors = orc.rowsum_from_p(p, do, v, causal)
    assert orc.normalized_err(rs.cpu(), ors) <= TOL[dtype]
    # dq, dk from the oracle's rowsum so that only this pass is under test
    ors_t = torch.from_numpy(ors).float()
    dq, dk = bs.triton_attn_bwd_dqdk_from_p(cu(q), cu(k), cu(v), cu(do), cu(p), cu(ors_t), causal=causal,
                                            scale=scale)
    odq, odk = orc.dqdk_from_p(q, k, v, do, p, ors_t, causal, scale)
    assert orc.normalized_err(dq.float().cpu(), odq) <= TOL[dtype]
    assert orc.normalized_err(dk.float().cpu(), odk) <= TOL[dtype]
    _lib.check_device_errors()


def test_from_p_gives_the_attention_gradients():
    """With P and rowsum from the forward, the from-P passes reproduce the
    LSE-recompute backward (same dq, dk, dv up to rounding)."""
    b, h, t, d, dtype = 1, 2, 384, 128, torch.bfloat16
    q, k, v, do, _, scale = _case(b, h, t, d, dtype, True, seed=5)
    q, k, v, do = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    o, lse2, p = _lib.attn_fwd(q, k, v, True, scale, save_p=True)
    dq, dk, dv, _ = _lib.attn_bwd(q, k, v, o, do, lse2, True, scale)
    rs = bs.triton_attn_rowsum_from_p(p, do, v, causal=True)
    dq2, dk2 = bs.triton_attn_bwd_dqdk_from_p(q, k, v, do, p, rs, causal=True, scale=scale)
    dv2 = bs.triton_attn_bwd_dv_from_p(p, do)
    for a, r in ((dq2, dq), (dk2, dk), (dv2, dv)):
        assert orc.normalized_err(a.float().cpu(), r.float().cpu()) <= 2e-2
    _lib.check_device_errors()


def test_function_forwards_on_gpu():
    b, h, t, d, dtype = 1, 1, 200, 64, torch.float16
    q, k, v, do, p, scale = _case(b, h, t, d, dtype, False, seed=9)
    q, k, v, do, p = (x.cuda() for x in (q, k, v, do, p))
    dv = bs.TritonDvFn.apply(p, do)
    rs = bs.TritonRowSumFn.apply(p, do, v, False)
    dq, dk = bs.TritonDqDkFn.apply(q, k, v, do, p, rs, scale, False)
    assert orc.normalized_err(dv.float().cpu(), orc.dv_from_p(p, do)) <= TOL[dtype]
    odq, odk = orc.dqdk_from_p(q, k, v, do, p, rs, False, scale)
    assert orc.normalized_err(dq.float().cpu(), odq) <= TOL[dtype]
    assert orc.normalized_err(dk.float().cpu(), odk) <= TOL[dtype]
    _lib.check_device_errors()
