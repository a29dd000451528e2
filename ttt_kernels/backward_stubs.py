"""Drop-in for ``ttt_kernels/backward_stubs.py`` of the reference.

The reference module holds its Triton backward kernels, three autograd
Functions whose backward is its (incomplete) double backward, and
NotImplementedError stubs for dq/dk and the bwd2 kernels
(backward_stubs.py:20-548). Here the same names are thin wrappers over the
sm_100a ops of libttt_attn.so:

* ``triton_attn_bwd_dv`` / ``_dq`` / ``_dk`` and ``triton_attn_bwd2_*`` take
  (q, k, v, do[, probes]) and recompute P from the row log-sum-exp; the
  reference's stubs for dq/dk and bwd2 (backward_stubs.py:529-548) are
  implemented.
* ``triton_attn_bwd_dv_from_p``, ``triton_attn_rowsum_from_p`` and
  ``triton_attn_bwd_dqdk_from_p`` take the materialized P and run the
  P-streaming kernels (HBM-bound on P).
* ``TritonDvFn``, ``TritonRowSumFn`` and ``TritonDqDkFn`` keep their
  signatures: forward = the from-P kernel, backward = the derivative of that
  forward with respect to each input (P included), in differentiable torch
  ops as in the reference. ``TritonDqDkFn.backward`` differs from the
  reference's in one term: the gradient reaching dS from grad_dk is
  scale * q grad_dk^T ([t_q, t_k]); the reference adds grad_dk q^T
  (backward_stubs.py:492-493), its transpose.

CPU tensors run the same formulas in torch ops.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
from torch.autograd import Function

from testtimeideas_b200 import _lib


def _scale(q: torch.Tensor, scale: Optional[float]) -> float:
    return 1.0 / math.sqrt(q.size(-1)) if scale is None else float(scale)


def _first_order(q, k, v, do, causal: bool, scale: Optional[float]):
    s = _scale(q, scale)
    o, lse2, _ = _lib.attn_fwd(q, k, v, causal, s)
    dq, dk, dv, delta = _lib.attn_bwd(q, k, v, o, do, lse2, causal, s)
    return dq, dk, dv, lse2, delta, s


def triton_attn_bwd_dv(q, k, v, do, *, causal: bool, scale: float):
    """dV = P^T dO with P recomputed on the fly (reference: backward_stubs.py:86-121)."""
    return _first_order(q, k, v, do, causal, scale)[2]


def triton_attn_bwd_dq(q, k, v, do, *, causal: bool, scale: float):
    """dQ (stub in the reference, backward_stubs.py:529-530)."""
    return _first_order(q, k, v, do, causal, scale)[0]


def triton_attn_bwd_dk(q, k, v, do, *, causal: bool, scale: float):
    """dK (stub in the reference, backward_stubs.py:533-534)."""
    return _first_order(q, k, v, do, causal, scale)[1]


def _second_order(q, k, v, do, uq, uk, uv, causal: bool, scale: Optional[float]):
    s = _scale(q, scale)
    o, lse2, _ = _lib.attn_fwd(q, k, v, causal, s)
    _, _, _, delta = _lib.attn_bwd(q, k, v, o, do, lse2, causal, s)
    return _lib.attn_bwd2(q, k, v, do, lse2, delta, uq, uk, uv, causal, s, need_gdout=False)


def triton_attn_bwd2_dq(q, k, v, do, uq, uk, uv, *, causal: bool = False, scale: Optional[float] = None):
    """d<dq,uq>+<dk,uk>+<dv,uv>/dq (stub in the reference, backward_stubs.py:539-540)."""
    return _second_order(q, k, v, do, uq, uk, uv, causal, scale)[0]


def triton_attn_bwd2_dk(q, k, v, do, uq, uk, uv, *, causal: bool = False, scale: Optional[float] = None):
    """... /dk (stub in the reference, backward_stubs.py:543-544)."""
    return _second_order(q, k, v, do, uq, uk, uv, causal, scale)[1]


def triton_attn_bwd2_dv(q, k, v, do, uq, uk, uv, *, causal: bool = False, scale: Optional[float] = None):
    """... /dv (stub in the reference, backward_stubs.py:547-548)."""
    return _second_order(q, k, v, do, uq, uk, uv, causal, scale)[2]


# ---------------------------------------------------------------- passes over materialized P
def triton_attn_bwd_dv_from_p(p, do):
    """dV = P^T dO for P [b, h, t, t] (reference: backward_stubs.py:154-181)."""
    if not do.is_cuda:
        return torch.matmul(p.transpose(-2, -1).to(do.dtype), do)
    return _lib.dv_from_p(p, do)


def _causal_blocks(t: int, device) -> torch.Tensor:
    """Entries of the 64 x 64 blocks the reference visits under causal=True
    (a block whose last query row is at or past its first key column)."""
    i = torch.arange(t, device=device)
    return (i // 64 * 64 + 63)[:, None] >= (i // 64 * 64)[None, :]


def triton_attn_rowsum_from_p(p, do, v, *, causal: bool):
    """rowsum[b, h, i] = sum_j P_ij (dO_i . V_j), fp32 (reference: backward_stubs.py:224-255)."""
    if not do.is_cuda:
        pp = p.float()
        if causal:
            pp = pp * _causal_blocks(p.shape[-1], p.device)
        return (torch.matmul(do.float(), v.float().transpose(-2, -1)) * pp).sum(-1)
    return _lib.rowsum_from_p(p, do, v, causal)


def triton_attn_bwd_dqdk_from_p(q, k, v, do, p, rowsum, *, causal: bool, scale: float):
    """dQ = scale dS K, dK = scale dS^T Q with dS = (dO V^T - rowsum) o P
    (reference: backward_stubs.py:362-425)."""
    if not q.is_cuda:
        pp = p.float()
        if causal:
            pp = pp * _causal_blocks(p.shape[-1], p.device)
        ds = (torch.matmul(do.float(), v.float().transpose(-2, -1)) - rowsum.float().unsqueeze(-1)) * pp
        return ((scale * torch.matmul(ds, k.float())).to(q.dtype),
                (scale * torch.matmul(ds.transpose(-2, -1), q.float())).to(q.dtype))
    return _lib.dqdk_from_p(q, k, v, do, p, rowsum, causal, scale)


class TritonDvFn(Function):
    """dV = P^T dO as a differentiable op (reference: backward_stubs.py:428-439)."""

    @staticmethod
    def forward(ctx, p, do):
        ctx.save_for_backward(p, do)
        return triton_attn_bwd_dv_from_p(p, do)

    @staticmethod
    def backward(ctx, grad_dv):
        p, do = ctx.saved_tensors
        grad_p = torch.matmul(do, grad_dv.transpose(-2, -1))
        grad_do = torch.matmul(p, grad_dv)
        return grad_p, grad_do


class TritonRowSumFn(Function):
    """rowsum(P o (dO V^T)) as a differentiable op (reference: backward_stubs.py:442-459)."""

    @staticmethod
    def forward(ctx, p, do, v, causal: bool):
        ctx.save_for_backward(p, do, v)
        ctx.causal = causal
        return triton_attn_rowsum_from_p(p, do, v, causal=causal)

    @staticmethod
    def backward(ctx, grad_rs):
        p, do, v = ctx.saved_tensors
        g = grad_rs.to(p.dtype).unsqueeze(-1)
        grad_p = g * torch.matmul(do, v.transpose(-2, -1))
        grad_do = g * torch.matmul(p, v)
        grad_v = torch.matmul(p.transpose(-2, -1), g * do)
        return grad_p.to(p.dtype), grad_do.to(p.dtype), grad_v.to(p.dtype), None


class TritonDqDkFn(Function):
    """(dQ, dK) from P as a differentiable op (reference: backward_stubs.py:462-514)."""

    @staticmethod
    def forward(ctx, q, k, v, do, p, rowsum, scale: float, causal: bool):
        ctx.save_for_backward(q, k, v, do, p, rowsum)
        ctx.scale = scale
        ctx.causal = causal
        return triton_attn_bwd_dqdk_from_p(q, k, v, do, p, rowsum, causal=causal, scale=scale)

    @staticmethod
    def backward(ctx, grad_dq, grad_dk):
        q, k, v, do, p, rowsum = ctx.saved_tensors
        scale, dt = ctx.scale, p.dtype
        gdq = (grad_dq if grad_dq is not None else torch.zeros_like(q)).to(dt)
        gdk = (grad_dk if grad_dk is not None else torch.zeros_like(k)).to(dt)
        rs = rowsum.to(dt).unsqueeze(-1)
        dp = torch.matmul(do, v.transpose(-2, -1))
        ds = (dp - rs) * p
        # dq = scale dS k and dk = scale dS^T q, so dS receives scale (gdq k^T + q gdk^T)
        grad_ds = (torch.matmul(gdq, k.transpose(-2, -1)) + torch.matmul(q, gdk.transpose(-2, -1))) * scale
        grad_q = torch.matmul(ds, gdk) * scale
        grad_k = torch.matmul(ds.transpose(-2, -1), gdq) * scale
        grad_dp = grad_ds * p
        grad_p = grad_ds * (dp - rs)
        grad_rowsum = -grad_dp.sum(dim=-1)
        grad_do = torch.matmul(grad_dp, v)
        grad_v = torch.matmul(grad_dp.transpose(-2, -1), do)
        return (grad_q.to(q.dtype), grad_k.to(k.dtype), grad_v.to(v.dtype), grad_do.to(do.dtype),
                grad_p.to(dt), grad_rowsum.to(rowsum.dtype), None, None)
