"""The P-taking helpers of backward_stubs on CPU: the wrappers' math path
against the oracle restatement, and the three autograd Functions' backward
against the exact derivative of their forward (torch.autograd, float64).

tests/golden/from_p_function_backwards_t48_d16_fp64.npz holds the outputs of
the reference's own backward methods (TritonDvFn, TritonRowSumFn,
TritonDqDkFn; backward_stubs.py:428-514) on fixed inputs. They pin two facts:
the reference's TritonDvFn / TritonRowSumFn backward and the q/k gradients of
its TritonDqDkFn backward are exact, while TritonDqDkFn's gradients that flow
through dS from grad_dk (to v, do, P and rowsum) use the transpose of the
right term (grad_dk q^T instead of q grad_dk^T, backward_stubs.py:492-493).
The Functions here give the exact derivative throughout.
"""

import math
import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from ttt_kernels import backward_stubs as bs

FIXTURE = os.path.join(os.path.dirname(__file__), "golden", "from_p_function_backwards_t48_d16_fp64.npz")


def _fixture():
    z = np.load(FIXTURE)
    return z, {n: torch.from_numpy(z[n]) for n in ("q", "k", "v", "do", "p", "rowsum", "gdv", "gdq", "gdk", "grs")}


def _exact(x, scale):
    """Exact input gradients of the three Functions' forwards (autograd, float64)."""
    q, k, v, do, p, rs = (x[n].clone().requires_grad_(True) for n in ("q", "k", "v", "do", "p", "rowsum"))
    dv = torch.matmul(p.transpose(-2, -1), do)
    g_dv = torch.autograd.grad(dv, (p, do), x["gdv"])
    rsum = (torch.matmul(do, v.transpose(-2, -1)) * p).sum(-1)
    g_rs = torch.autograd.grad(rsum, (p, do, v), x["grs"])
    ds = (torch.matmul(do, v.transpose(-2, -1)) - rs.unsqueeze(-1)) * p
    dq, dk = scale * torch.matmul(ds, k), scale * torch.matmul(ds.transpose(-2, -1), q)
    g_dqdk = torch.autograd.grad((dq, dk), (q, k, v, do, p, rs), (x["gdq"], x["gdk"]))
    return g_dv, g_rs, g_dqdk


def _err(a, b):
    return orc.normalized_err(torch.as_tensor(a), torch.as_tensor(b))


def test_reference_function_backwards_pinned():
    z, x = _fixture()
    scale = float(z["scale"])
    g_dv, g_rs, g_dqdk = _exact(x, scale)
    assert _err(z["dvfn_grad_p"], g_dv[0]) < 1e-12 and _err(z["dvfn_grad_do"], g_dv[1]) < 1e-12
    for name, e in zip(("p", "do", "v"), g_rs):
        assert _err(z[f"rsfn_grad_{name}"], e) < 1e-12, name
    exact = dict(zip(("q", "k", "v", "do", "p", "rowsum"), g_dqdk))
    for name in ("q", "k"):
        assert _err(z[f"dqdkfn_grad_{name}"], exact[name]) < 1e-12, name
    # the reference's transposed grad_dk term: every gradient that flows through dS is off by O(1)
    for name in ("v", "do", "p", "rowsum"):
        assert _err(z[f"dqdkfn_grad_{name}"], exact[name]) > 1e-2, name


def test_function_backwards_are_exact():
    z, x = _fixture()
    scale = float(z["scale"])
    g_dv, g_rs, g_dqdk = _exact(x, scale)

    class Ctx:
        pass

    c = Ctx()
    c.saved_tensors = (x["p"], x["do"])
    out = bs.TritonDvFn.backward(c, x["gdv"])
    assert all(_err(a, b) < 1e-12 for a, b in zip(out, g_dv))
    c.saved_tensors, c.causal = (x["p"], x["do"], x["v"]), True
    out = bs.TritonRowSumFn.backward(c, x["grs"])
    assert all(_err(a, b) < 1e-12 for a, b in zip(out[:3], g_rs))
    c.saved_tensors, c.scale = (x["q"], x["k"], x["v"], x["do"], x["p"], x["rowsum"]), scale
    out = bs.TritonDqDkFn.backward(c, x["gdq"], x["gdk"])
    assert all(_err(a, b) < 1e-12 for a, b in zip(out[:6], g_dqdk))


def _softmax_p(q, k, causal, scale):
    s = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        t = s.shape[-1]
        s = s.masked_fill(torch.triu(torch.ones(t, t, dtype=torch.bool), 1), float("-inf"))
    return torch.softmax(s, dim=-1)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("t", [37, 130])
def test_from_p_wrappers_match_oracle_on_cpu(causal, t):
    inp = orc.seeded_inputs(1, 2, t, 16, seed=t, scale_in=1.0)
    q, k, v, do = (inp[n].double() for n in ("q", "k", "v", "do"))
    scale = 1.0 / math.sqrt(16)
    p = _softmax_p(q, k, causal, scale)
    assert _err(bs.triton_attn_bwd_dv_from_p(p, do), orc.dv_from_p(p, do)) < 1e-12
    # rowsum is fp32, as in the reference (backward_stubs.py:229)
    rs = bs.triton_attn_rowsum_from_p(p, do, v, causal=causal)
    assert rs.dtype == torch.float32
    assert _err(rs, orc.rowsum_from_p(p, do, v, causal)) < 1e-6
    dq, dk = bs.triton_attn_bwd_dqdk_from_p(q, k, v, do, p, rs, causal=causal, scale=scale)
    odq, odk = orc.dqdk_from_p(q, k, v, do, p, rs, causal, scale)
    assert _err(dq, odq) < 1e-6 and _err(dk, odk) < 1e-6
    # with P from the forward, rowsum(P o dO V^T) = rowsum(dO o O) and (dq, dk) are the attention gradients
    o = orc.attention_math(q, k, v, causal, scale)
    assert _err(rs, (do * o).sum(-1)) < 1e-6
    ref = orc.math_gradgrad(*(inp[n] for n in ("q", "k", "v", "do", "uq", "uk", "uv")), causal=causal, scale=scale)
    assert _err(dq, ref["dq"]) < 1e-6 and _err(dk, ref["dk"]) < 1e-6


def test_causal_block_skip_matches_reference_granularity():
    # entries above the diagonal inside a visited 64 x 64 block are used, blocks past it are not
    t = 130
    m = orc._causal_block_mask(t)
    assert m[0, 63] == 1 and m[0, 64] == 0 and m[64, 127] == 1 and m[63, 64] == 0 and m[129, 129] == 1
    mask = bs._causal_blocks(t, "cpu").numpy().astype(np.float64)
    assert np.array_equal(mask, m)
