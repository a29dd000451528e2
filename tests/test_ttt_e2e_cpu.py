"""The TTT-E2E attention drop-in (testtimeideas_b200.ttt_e2e) on CPU, pinned to
outputs of the reference's own module (tests/golden/ttt_e2e_windows_fp64.npz,
made by tests/golden/make_golden.py from cloud_ttt_e2e/ttt_e2e):

* GradGradAttentionFn with a binding sliding-window mask from make_window_mask:
  forward, first-order grads (create_graph) and second-order grads including
  the one with respect to the upstream gradient;
* WindowedSelfAttention on a sequence longer than its window (its chunk loop,
  with a partial last chunk): output, first- and second-order input grads.

The oracle's banded masks ("sliding", "chunk") are pinned by the same vectors,
so the GPU tests that compare the kernels with the oracle test the reference's
semantics."""

import math
import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import ttt_e2e

FIX = os.path.join(os.path.dirname(__file__), "golden", "ttt_e2e_windows_fp64.npz")


def _z():
    return np.load(FIX)


def test_make_window_mask_matches_band():
    for t, w in ((48, 12), (40, 16), (10, None), (10, 20)):
        m = ttt_e2e.make_window_mask(t, w, "cpu", torch.float32)
        vis = orc.band_visible(t, w or 0, "sliding")
        assert np.array_equal(torch.isfinite(m).numpy(), vis)
        assert ttt_e2e.window_of_mask(m.view(1, 1, t, t), t) == (w if w is not None and w < t else 0)


def test_window_of_mask_rejects_other_masks():
    t = 16
    with pytest.raises(ValueError):
        ttt_e2e.window_of_mask(torch.zeros(t, t), t)  # non-causal
    m = ttt_e2e.make_window_mask(t, 4, "cpu", torch.float32)
    m[5, 5] = float("-inf")
    with pytest.raises(ValueError):
        ttt_e2e.window_of_mask(m, t)
    with pytest.raises(ValueError):
        ttt_e2e.window_of_mask(torch.zeros(2, 1, t, t), t)  # per-batch masks


def test_sliding_window_gradgrad_matches_reference():
    z = _z()
    b, h, t, d, w = (int(x) for x in z["sw_meta"])
    x = {n: torch.from_numpy(z[f"sw_in_{n}"]) for n in ("q", "k", "v", "do", "uq", "uk", "uv")}
    ref = orc.math_gradgrad(*(x[n] for n in ("q", "k", "v", "do", "uq", "uk", "uv")), causal=True,
                            need_gdo=True, window=w, window_kind="sliding")
    for key in ("o", "dq", "dk", "dv", "gq", "gk", "gv", "gdo"):
        assert orc.normalized_err(ref[key], z[f"sw_{key}"]) < 1e-12, key
    # the drop-in's CPU path, through autograd, with a dO that does not require grad
    q, k, v = (x[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    mask = ttt_e2e.make_window_mask(t, w, "cpu", torch.float64).view(1, 1, t, t)
    out = ttt_e2e.GradGradAttentionFn.apply(q, k, v, mask)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), x["do"], create_graph=True)
    gq, gk, gv = torch.autograd.grad((dq * x["uq"]).sum() + (dk * x["uk"]).sum() + (dv * x["uv"]).sum(), (q, k, v))
    for key, val in (("o", out), ("dq", dq), ("gq", gq), ("gk", gk), ("gv", gv)):
        assert orc.normalized_err(val.detach(), z[f"sw_{key}"]) < 1e-12, key


def _module_from_fixture(z):
    d_model, n_heads, w, t = (int(x) for x in z["wsa_meta"])
    mod = ttt_e2e.WindowedSelfAttention(d_model, n_heads, w, use_gradgrad=True).double()
    mod.load_state_dict({n[4:]: torch.from_numpy(z[n]) for n in z.files
                         if n.startswith("wsa_") and (n.endswith(".weight") or n.endswith(".bias"))})
    return mod, w, t


def test_windowed_self_attention_matches_reference():
    z = _z()
    mod, w, t = _module_from_fixture(z)
    x = torch.from_numpy(z["wsa_x"]).clone().requires_grad_(True)
    y = mod(x)
    (gx,) = torch.autograd.grad(y, x, torch.from_numpy(z["wsa_g"]), create_graph=True)
    (ggx,) = torch.autograd.grad((gx * torch.from_numpy(z["wsa_u"])).sum(), x)
    assert orc.normalized_err(y.detach(), z["wsa_y"]) < 1e-12
    assert orc.normalized_err(gx.detach(), z["wsa_gx"]) < 1e-12
    assert orc.normalized_err(ggx, z["wsa_ggx"]) < 1e-12


def test_chunk_band_is_the_reference_chunk_loop():
    """One attention over the whole sequence with the oracle's "chunk" band
    reproduces the reference module's output (chunk loop + partial last chunk)."""
    z = _z()
    mod, w, t = _module_from_fixture(z)
    x = torch.from_numpy(z["wsa_x"])
    with torch.no_grad():
        q, k, v = (mod._split_heads(proj(x)) for proj in (mod.q_proj, mod.k_proj, mod.v_proj))
        o = orc.attention_math(q, k, v, True, 1.0 / math.sqrt(q.size(-1)), window=w, window_kind="chunk")
        y = mod.out_proj(mod._merge_heads(o))
    assert orc.normalized_err(y, z["wsa_y"]) < 1e-12
    # and it is not the sliding window of the same width
    with torch.no_grad():
        o2 = orc.attention_math(q, k, v, True, 1.0 / math.sqrt(q.size(-1)), window=w, window_kind="sliding")
        y2 = mod.out_proj(mod._merge_heads(o2))
    assert orc.normalized_err(y2, z["wsa_y"]) > 1e-3
