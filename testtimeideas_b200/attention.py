"""Autograd surface of the B200 attention kernels.

``TritonAttentionFn`` keeps the signature and mode strings of the reference's
``ttt_kernels.triton_attention.TritonAttentionFn`` (triton_attention.py:259-420):
``apply(q, k, v, causal, scale, bwd_mode)`` with a backward that returns six
gradients. Differences, all deliberate:

* On CUDA the forward, backward and double backward always run the sm_100a
  kernels of libttt_attn.so; fp16/bf16 with d in {64, 128} is required and
  anything else raises (no silent math fallback on the GPU path).
* Every ``bwd_mode`` yields the complete second-order gradient. The
  reference's ``save_p*`` modes store P as a constant and drop the terms
  through P's dependence on q and k (backward_stubs.py:428-514); here the
  double backward is the closed form of d<dq,u_q>+<dk,u_k>+<dv,u_v>.
* The ``save_p`` / ``save_p_triton`` / ``save_p_triton_bwd`` /
  ``save_p_triton_full`` modes run the same kernels as ``recompute`` and do
  not materialize P. The reference saves the T x T probabilities in the
  forward (triton_attention.py:270-273) and streams them in its backward
  (:354-362) to avoid recomputing them; on B200 recomputing a score tile
  from the saved row log-sum-exp costs a fraction of streaming it from HBM
  (2*d flops against 2 bytes per entry: at d=64, 128 flops at ~1.3 PFLOP/s
  against 2 bytes at ~6.5 TB/s, a quarter of the time), and the complete
  second-order terms need the scores again anyway. The passes that do read
  a materialized P remain available as the reference's from-P helpers
  (``ttt_kernels.backward_stubs``), with the P-writing forward in
  ``_lib.attn_fwd(..., save_p=True)``.
* CPU tensors (and fp32 tensors on CPU) take the reference's math path:
  forward without a graph, backward recomputing ``_attention_math`` under
  autograd (triton_attention.py:416-420), so create_graph works there too.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
from torch.autograd.function import once_differentiable

from . import _lib

BWD_MODES = (
    "recompute", "recompute_manual", "recompute_sdp", "recompute_sdp_mem", "recompute_sdp_auto", "save_p",
    "save_p_triton", "save_p_triton_bwd", "save_p_triton_full", "recompute_compiled", "dv_only", "custom",
)
SAVE_P_MODES = ("save_p", "save_p_triton", "save_p_triton_bwd", "save_p_triton_full")


def attention_math(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, scale: float) -> torch.Tensor:
    """Dense softmax attention with the reference's mask convention (triu(1) -> -inf),
    triton_attention.py:18-25. Used only for CPU tensors."""
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        t = scores.size(-1)
        mask = torch.triu(torch.ones((t, t), device=scores.device, dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), v)


def _kernel_path(q: torch.Tensor) -> bool:
    """True when the call runs the CUDA kernels (every CUDA tensor); CPU tensors
    take the reference's math path. Host-logic tests on CPU replace this seam
    together with the ops of ``_lib``."""
    return q.is_cuda


class _AttnBwdFn(torch.autograd.Function):
    """First-order backward as a differentiable op: forward = (dq, dk, dv),
    backward = the complete double backward (grads w.r.t. q, k, v and dO)."""

    @staticmethod
    def forward(ctx, q, k, v, dout, o, lse2, causal: bool, scale: float, window=0):
        dq, dk, dv, delta = _lib.attn_bwd(q, k, v, o, dout, lse2, causal, scale, window=window)
        ctx.save_for_backward(q, k, v, dout, lse2, delta)
        ctx.causal = causal
        ctx.scale = scale
        ctx.window = window
        return dq, dk, dv

    @staticmethod
    @once_differentiable
    def backward(ctx, gdq, gdk, gdv):
        q, k, v, dout, lse2, delta = ctx.saved_tensors
        need_gdo = bool(ctx.needs_input_grad[3])
        gq, gk, gv, gdo = _lib.attn_bwd2(q, k, v, dout, lse2, delta, gdq, gdk, gdv, ctx.causal, ctx.scale, need_gdo,
                                         window=ctx.window)
        return gq, gk, gv, gdo, None, None, None, None, None


class TritonAttentionFn(torch.autograd.Function):
    """Drop-in for the reference ``TritonAttentionFn`` backed by libttt_attn.so."""

    @staticmethod
    def forward(ctx, q, k, v, causal: bool = False, scale: Optional[float] = None, bwd_mode: str = "recompute"):
        if scale is None:
            scale = 1.0 / math.sqrt(q.size(-1))
        ctx.causal = bool(causal)
        ctx.scale = float(scale)
        ctx.bwd_mode = bwd_mode
        ctx.on_gpu = _kernel_path(q)
        if not ctx.on_gpu:
            ctx.save_for_backward(q, k, v)
            return attention_math(q, k, v, causal, scale)
        o, lse2, _ = _lib.attn_fwd(q, k, v, ctx.causal, ctx.scale)
        ctx.save_for_backward(q, k, v, o, lse2)
        return o

    @staticmethod
    def backward(ctx, grad_out):
        if not ctx.on_gpu:
            q, k, v = ctx.saved_tensors
            with torch.enable_grad():
                qq = q if q.requires_grad else q.detach().requires_grad_(True)
                kk = k if k.requires_grad else k.detach().requires_grad_(True)
                vv = v if v.requires_grad else v.detach().requires_grad_(True)
                out = attention_math(qq, kk, vv, ctx.causal, ctx.scale)
                dq, dk, dv = torch.autograd.grad(out, (qq, kk, vv), grad_out, create_graph=torch.is_grad_enabled())
            return dq, dk, dv, None, None, None
        q, k, v, o, lse2 = ctx.saved_tensors
        if torch.is_grad_enabled():
            dq, dk, dv = _AttnBwdFn.apply(q, k, v, grad_out, o.detach(), lse2, ctx.causal, ctx.scale)
        else:
            dq, dk, dv, _ = _lib.attn_bwd(q, k, v, o, grad_out, lse2, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None, None


def triton_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = False,
                     scale: Optional[float] = None, bwd_mode: str = "recompute") -> torch.Tensor:
    """Same signature as the reference entry point (triton_attention.py:423-424)."""
    return TritonAttentionFn.apply(q, k, v, causal, scale, bwd_mode)
