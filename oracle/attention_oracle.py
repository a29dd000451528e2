"""CPU oracle for the grad-grad attention path.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs import this module, and only as the checker or
the timed CPU baseline; the product path (testtimeideas_b200, ttt_kernels)
never imports it.

It restates the reference's math path in two independent ways:

1. ``math_gradgrad``: ``_attention_math`` (ttt_kernels/triton_attention.py:18-25)
   differentiated twice with torch.autograd, exactly what the reference's
   ``recompute`` backward does (triton_attention.py:416-420) and what its
   benchmarks time as "math" (tests/bench_gradgrad_sweep.py:49-54).
2. ``closed_form_gradgrad``: the closed-form first- and second-order
   derivatives of softmax attention in numpy float64, with the probes
   u_q, u_k, u_v as the upstream gradients of dq, dk, dv:

       dP = dO V^T,  delta = rowsum(dO o O),  dS = P o (dP - delta)
       G_dS = scale (u_q K^T + Q u_k^T),  gamma = rowsum(P o G_dS)
       G_dP = P o (G_dS - gamma)
       G_P  = G_dS o (dP - delta) - gamma o dP + dO u_v^T
       rho  = rowsum(P o G_P),  G_S = P o (G_P - rho)
       dd_Q = scale (dS u_k + G_S K),  dd_K = scale (dS^T u_q + G_S^T Q)
       dd_V = G_dP^T dO,  dd_dO = G_dP V + P u_v

Both are pinned against tests/golden/*.npz, which tests/golden/make_golden.py
generated from the reference's own public entry point
(``triton_attention(..., bwd_mode='recompute')`` on CPU) in this container.
"""

from __future__ import annotations

import math

import numpy as np
import torch


def band_visible(t: int, window: int = 0, kind: str = "sliding") -> np.ndarray:
    """[t, t] bool: key j visible to query i under a causal mask restricted to a band.

    window 0: plain causal (j <= i). kind "sliding": i - window < j <= i, the
    additive mask of make_window_mask (cloud_ttt_e2e/ttt_e2e/utils.py:40-54).
    kind "chunk": the attention WindowedSelfAttention computes for t > window
    with its chunk loop (cloud_ttt_e2e/ttt_e2e/attention.py:112-127): queries of
    chunk [start, end) see keys max(0, end - window) .. i.
    """
    i = np.arange(t)[:, None]
    j = np.arange(t)[None, :]
    vis = j <= i
    if window and kind == "sliding":
        vis &= (i - j) < window
    elif window and kind == "chunk":
        start = (i // window) * window
        end = np.minimum(t, start + window)
        vis &= j >= np.maximum(0, end - window)
    return vis


def attention_math(q, k, v, causal: bool, scale: float, window: int = 0, window_kind: str = "sliding"):
    """softmax(scale * q k^T, causal triu(1) -> -inf) v  (triton_attention.py:18-25);
    with window > 0 (causal) the mask of band_visible."""
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        t = scores.size(-1)
        vis = torch.from_numpy(band_visible(t, window, window_kind)).to(scores.device)
        scores = scores.masked_fill(~vis, float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), v)


def math_gradgrad(q, k, v, do, uq, uk, uv, causal: bool, scale: float | None = None,
                  dtype: torch.dtype = torch.float64, need_gdo: bool = False, window: int = 0,
                  window_kind: str = "sliding") -> dict:
    """Forward, first-order grads of <O, dO> and second-order grads of
    <dq,uq> + <dk,uk> + <dv,uv>, via torch.autograd on the math path."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    cast = lambda x: x.detach().to(dtype)  # noqa: E731
    q_, k_, v_ = (cast(x).requires_grad_(True) for x in (q, k, v))
    do_ = cast(do).requires_grad_(need_gdo)
    uq_, uk_, uv_ = cast(uq), cast(uk), cast(uv)
    with torch.enable_grad():
        o = attention_math(q_, k_, v_, causal, scale, window, window_kind)
        dq, dk, dv = torch.autograd.grad(o, (q_, k_, v_), do_, create_graph=True)
        l2 = (dq * uq_).sum() + (dk * uk_).sum() + (dv * uv_).sum()
        wrt = (q_, k_, v_, do_) if need_gdo else (q_, k_, v_)
        gg = torch.autograd.grad(l2, wrt)
    out = {"o": o.detach(), "dq": dq.detach(), "dk": dk.detach(), "dv": dv.detach(),
           "gq": gg[0], "gk": gg[1], "gv": gg[2]}
    if need_gdo:
        out["gdo"] = gg[3]
    return out


def mean_loss_gradgrad(q, k, v, causal: bool, scale: float | None = None, dtype: torch.dtype = torch.float64) -> dict:
    """The reference benchmark's objective (tests/bench_gradgrad_sweep.py:50-54):
    loss = mean(O); grads = d loss / d(q,k,v) with create_graph; s = sum_g mean(g^2);
    returns grads and d s / d(q,k,v)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    q_, k_, v_ = (x.detach().to(dtype).requires_grad_(True) for x in (q, k, v))
    with torch.enable_grad():
        o = attention_math(q_, k_, v_, causal, scale)
        # out.float().mean() exactly as the reference (it casts fp64 outputs to fp32 too)
        grads = torch.autograd.grad(o.float().mean(), (q_, k_, v_), create_graph=True)
        s = sum(g.pow(2).mean() for g in grads)
        gg = torch.autograd.grad(s, (q_, k_, v_))
    return {"o": o.detach(), "dq": grads[0].detach(), "dk": grads[1].detach(), "dv": grads[2].detach(),
            "gq": gg[0], "gk": gg[1], "gv": gg[2]}


def _softmax_rows(s: np.ndarray) -> np.ndarray:
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def closed_form_gradgrad(q, k, v, do, uq, uk, uv, causal: bool, scale: float | None = None, window: int = 0,
                         window_kind: str = "sliding") -> dict:
    """numpy float64 closed form of the same quantities (see module docstring).
    Inputs are [..., t, d] arrays (any leading batch dims)."""
    q, k, v, do, uq, uk, uv = (np.asarray(x, dtype=np.float64) for x in (q, k, v, do, uq, uk, uv))
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    tr = lambda x: np.swapaxes(x, -1, -2)  # noqa: E731
    s = scale * (q @ tr(k))
    if causal:
        s = np.where(band_visible(s.shape[-1], window, window_kind), s, -np.inf)
    p = _softmax_rows(s)
    o = p @ v
    dp = do @ tr(v)
    delta = np.sum(do * o, axis=-1, keepdims=True)
    ds = p * (dp - delta)
    dq = scale * (ds @ k)
    dk = scale * (tr(ds) @ q)
    dv = tr(p) @ do
    g_ds = scale * (uq @ tr(k) + q @ tr(uk))
    gamma = np.sum(p * g_ds, axis=-1, keepdims=True)
    g_dp = p * (g_ds - gamma)
    g_p = g_ds * (dp - delta) - gamma * dp + do @ tr(uv)
    rho = np.sum(p * g_p, axis=-1, keepdims=True)
    g_s = p * (g_p - rho)
    gq = scale * (ds @ uk + g_s @ k)
    gk = scale * (tr(ds) @ uq + tr(g_s) @ q)
    gv = tr(g_dp) @ do
    gdo = g_dp @ v + p @ uv
    return {"o": o, "dq": dq, "dk": dk, "dv": dv, "gq": gq, "gk": gk, "gv": gv, "gdo": gdo,
            "lse": np.log(np.sum(np.exp(s - np.max(s, -1, keepdims=True)), -1)) + np.max(s, -1),
            "delta": delta[..., 0], "gamma": gamma[..., 0], "rho": rho[..., 0]}


# ---------------------------------------------------------------- passes over a given P
# Restatements of the reference's P-taking helpers (backward_stubs.py), numpy
# float64 on [b, h, t, t] P and [b, h, t, d] tensors. ``causal`` follows the
# reference's block skip: a 64 x 64 block of P is used only if its last query
# row is at or past its first key column (backward_stubs.py:212-215, 291-294,
# 336-337); inside a used block P is taken as given.
_BLOCK = 64


def _causal_block_mask(t: int) -> np.ndarray:
    """[t, t] 0/1 mask of the (query, key) entries inside blocks the reference visits."""
    i = np.arange(t)
    last_q = (i // _BLOCK) * _BLOCK + _BLOCK - 1          # last query row of each query block
    first_k = (i // _BLOCK) * _BLOCK                      # first key of each key block
    return (last_q[:, None] >= first_k[None, :]).astype(np.float64)


def dv_from_p(p, do):
    """dV = P^T dO  (backward_stubs.py:124-181)."""
    p64, do64 = _np64(p), _np64(do)
    return np.einsum("bhqk,bhqd->bhkd", p64, do64)


def rowsum_from_p(p, do, v, causal: bool):
    """rowsum_i = sum_j P_ij (dO_i . V_j)  (backward_stubs.py:184-255)."""
    p64, do64, v64 = _np64(p), _np64(do), _np64(v)
    if causal:
        p64 = p64 * _causal_block_mask(p64.shape[-1])
    dp = np.einsum("bhqd,bhkd->bhqk", do64, v64)
    return (dp * p64).sum(-1)


def dqdk_from_p(q, k, v, do, p, rowsum, causal: bool, scale: float):
    """dS = (dO V^T - rowsum) o P; dQ = scale dS K; dK = scale dS^T Q  (backward_stubs.py:259-425)."""
    q64, k64, v64, do64, p64, rs64 = (_np64(x) for x in (q, k, v, do, p, rowsum))
    if causal:
        p64 = p64 * _causal_block_mask(p64.shape[-1])
    ds = (np.einsum("bhqd,bhkd->bhqk", do64, v64) - rs64[..., None]) * p64
    return scale * np.einsum("bhqk,bhkd->bhqd", ds, k64), scale * np.einsum("bhqk,bhqd->bhkd", ds, q64)


def _np64(x):
    if isinstance(x, torch.Tensor):
        return x.detach().to("cpu", torch.float64).numpy()
    return np.asarray(x, dtype=np.float64)


def seeded_inputs(b: int, h: int, t: int, d: int, seed: int, scale_in: float = 1.0,
                  dtype: torch.dtype = torch.float32) -> dict:
    """q, k, v, do, uq, uk, uv iid N(0,1) * scale_in from one CPU generator
    (the synthetic inputs of every benchmark configuration)."""
    g = torch.Generator().manual_seed(seed)
    names = ("q", "k", "v", "do", "uq", "uk", "uv")
    return {n: (torch.randn(b, h, t, d, generator=g, dtype=torch.float32) * scale_in).to(dtype) for n in names}


def max_abs_err(x, ref) -> float:
    x = torch.as_tensor(x).double()
    ref = torch.as_tensor(ref).double()
    return float((x - ref).abs().max()) if x.numel() else 0.0


def normalized_err(x, ref) -> float:
    """max |x - ref| / max(1, max |ref|): the absolute error for O(1) outputs and
    the relative error for large ones."""
    ref_t = torch.as_tensor(ref).double()
    scale = max(1.0, float(ref_t.abs().max())) if ref_t.numel() else 1.0
    return max_abs_err(x, ref_t) / scale
