"""Drop-in for ``ttt_kernels/backward_stubs.py`` of the reference.

The reference module holds its Triton backward kernels, three autograd
Functions whose backward is its (incomplete) double backward, and
NotImplementedError stubs for dq/dk and the bwd2 kernels
(backward_stubs.py:20-548). Here the same names are thin wrappers over the
sm_100a ops of libttt_attn.so. The LSE-recompute entry points take (q, k, v,
do) as in the reference; the dq/dk and bwd2 stubs that the reference leaves
unimplemented (backward_stubs.py:529-548) are implemented.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

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
