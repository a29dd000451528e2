"""Drop-in attention for the TTT-E2E model of the reference
(cloud_ttt_e2e/ttt_e2e/attention.py and utils.make_window_mask).

The reference computes its grad-grad-safe attention in PyTorch: an additive
[t, t] mask (0 visible, -inf masked) added to the scores, and for sequences
longer than the window a Python loop over chunks. Here the same three names
run the sm_100a kernels on CUDA tensors, with the mask expressed as a band of
visible keys per row (no [t, t] tensor, tiles outside the band are never
computed):

* ``make_window_mask(seq_len, window_size, device, dtype)`` - the reference's
  additive mask (utils.py:40-54), for callers that build one.
* ``GradGradAttentionFn.apply(q, k, v, attn_mask)`` - attention.py:21-53. On
  CUDA the mask must be one ``make_window_mask`` produces (possibly viewed as
  [1, 1, t, t]); it is checked on the device and turned into a sliding band;
  any other mask raises (there is no dense-mask fallback on the GPU path). The
  first- and second-order gradients are complete whether or not the upstream
  gradient requires grad (the reference keeps a graph only when it does,
  attention.py:32).
* ``WindowedSelfAttention`` - attention.py:72-131, same constructor, weights
  and forward. For t > window the reference's chunk loop restricts each query
  to keys of its own chunk (the last partial chunk sees the last ``window``
  keys); that rule is the kernels' chunk-local band, so one call covers the
  whole sequence.

CPU tensors run the reference's PyTorch formulation (dense additive mask).
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from .attention import _AttnBwdFn


def make_window_mask(seq_len: int, window_size: Optional[int], device, dtype) -> torch.Tensor:
    """Additive [seq_len, seq_len] mask: 0 where key j <= query i (and i - j <
    window_size when given), -inf elsewhere (utils.py:40-54)."""
    i = torch.arange(seq_len, device=device)
    masked = i[None, :] > i[:, None]
    if window_size is not None:
        masked = masked | ((i[:, None] - i[None, :]) >= window_size)
    return torch.zeros((seq_len, seq_len), device=device, dtype=dtype).masked_fill(masked, float("-inf"))


def window_of_mask(attn_mask: torch.Tensor, t: int) -> int:
    """The window of a mask made by make_window_mask(t, window): 0 for the plain
    causal mask (window None or >= t), else the window. Raises ValueError for
    any other mask."""
    m = attn_mask
    if m.dim() < 2 or tuple(m.shape[-2:]) != (t, t) or m[..., :1, :1].numel() != 1:
        raise ValueError(f"attention mask must be [t, t] (or [1, 1, t, t]) with t={t}, got {tuple(m.shape)}")
    m = m.reshape(t, t)
    visible_last_row = int(torch.isfinite(m[-1]).sum().item())
    window = 0 if visible_last_row >= t else visible_last_row
    expected = make_window_mask(t, window or None, m.device, m.dtype)
    if not torch.equal(m, expected):
        raise ValueError("the sm_100a path takes only masks built by make_window_mask (causal, optionally windowed)")
    return window


def _math(q, k, v, attn_mask):
    """attention.py:9-18: softmax(q k^T / sqrt(d) + attn_mask) v."""
    scores = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(q.size(-1)))
    if attn_mask is not None:
        scores = scores + attn_mask
    return torch.matmul(torch.softmax(scores, dim=-1), v)


class _MathFn(torch.autograd.Function):
    """CPU path: the reference's Function, recomputing the math under autograd in
    backward (differentiable when grad mode is on)."""

    @staticmethod
    def forward(ctx, q, k, v, attn_mask):
        ctx.save_for_backward(q, k, v, attn_mask)
        with torch.no_grad():
            return _math(q, k, v, attn_mask)

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, attn_mask = ctx.saved_tensors
        with torch.enable_grad():
            qq, kk, vv = (x if x.requires_grad else x.detach().requires_grad_(True) for x in (q, k, v))
            out = _math(qq, kk, vv, attn_mask)
            grads = torch.autograd.grad(out, (qq, kk, vv), grad_out, create_graph=torch.is_grad_enabled())
        return grads[0], grads[1], grads[2], None


class BandAttentionFn(torch.autograd.Function):
    """Causal attention over a band of keys on the sm_100a kernels:
    apply(q, k, v, window, kind) with kind "sliding" or "chunk" (window 0: plain
    causal); scale 1/sqrt(d). Backward is differentiable (double backward,
    including the gradient with respect to the upstream gradient)."""

    @staticmethod
    def forward(ctx, q, k, v, window: int, kind: str):
        scale = 1.0 / math.sqrt(q.size(-1))
        band = (int(window), kind) if window else 0
        o, lse2, _ = _lib.attn_fwd(q, k, v, True, scale, window=band)
        ctx.save_for_backward(q, k, v, o, lse2)
        ctx.scale, ctx.band = scale, band
        return o

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, o, lse2 = ctx.saved_tensors
        if torch.is_grad_enabled():
            dq, dk, dv = _AttnBwdFn.apply(q, k, v, grad_out, o.detach(), lse2, True, ctx.scale, ctx.band)
        else:
            dq, dk, dv, _ = _lib.attn_bwd(q, k, v, o, grad_out, lse2, True, ctx.scale, window=ctx.band)
        return dq, dk, dv, None, None


class GradGradAttentionFn:
    """Same call as the reference's autograd Function (attention.py:21-53):
    ``GradGradAttentionFn.apply(q, k, v, attn_mask)``."""

    @staticmethod
    def apply(q, k, v, attn_mask):
        if not q.is_cuda:
            return _MathFn.apply(q, k, v, attn_mask)
        window = window_of_mask(attn_mask, q.size(-2))
        return BandAttentionFn.apply(q, k, v, window, "sliding")


class WindowedSelfAttention(nn.Module):
    """attention.py:72-131 with the attention on the kernels (CUDA) or the
    reference's PyTorch formulation (CPU, or use_gradgrad=False)."""

    def __init__(self, d_model: int, n_heads: int, window_size: Optional[int], use_gradgrad: bool = True):
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.window_size = window_size
        self.use_gradgrad = use_gradgrad
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)

    def _split_heads(self, x):
        b, t, _ = x.shape
        return x.view(b, t, self.n_heads, self.head_dim).transpose(1, 2)  # [B, H, T, HD]

    def _merge_heads(self, x):
        b, h, t, d = x.shape
        return x.transpose(1, 2).contiguous().view(b, t, h * d)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, t, _ = x.shape
        q = self._split_heads(self.q_proj(x))
        k = self._split_heads(self.k_proj(x))
        v = self._split_heads(self.v_proj(x))
        chunked = self.window_size is not None and t > self.window_size
        if self.use_gradgrad and x.is_cuda:
            out = BandAttentionFn.apply(q, k, v, self.window_size if chunked else 0, "chunk")
        elif not chunked:
            if self.use_gradgrad:
                mask = make_window_mask(t, self.window_size, x.device, x.dtype).view(1, 1, t, t)
                out = _MathFn.apply(q, k, v, mask)
            else:
                out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            # the reference's chunk loop: queries [start, end) against keys [max(0, end - w), end)
            w, outs = self.window_size, []
            for start in range(0, t, w):
                end = min(t, start + w)
                kv0 = max(0, end - w)
                qi = torch.arange(start, end, device=x.device)[:, None]
                kj = torch.arange(kv0, end, device=x.device)[None, :]
                mask = torch.zeros((end - start, end - kv0), device=x.device, dtype=x.dtype).masked_fill(
                    (kj > qi) | ((qi - kj) >= w), float("-inf")).view(1, 1, end - start, end - kv0)
                qc, kc, vc = q[:, :, start:end], k[:, :, kv0:end], v[:, :, kv0:end]
                if self.use_gradgrad:
                    outs.append(_MathFn.apply(qc, kc, vc, mask))
                else:
                    outs.append(F.scaled_dot_product_attention(qc, kc, vc, attn_mask=mask))
            out = torch.cat(outs, dim=2)
        return self.out_proj(self._merge_heads(out))
