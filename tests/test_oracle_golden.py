"""Pin the CPU oracle against golden vectors generated from the reference.

tests/golden/*.npz were produced by tests/golden/make_golden.py from the
reference's public entry point (ttt_kernels.triton_attention with
bwd_mode='recompute', i.e. its math path) on CPU. Both oracle restatements
(autograd over the math definition, and the numpy closed form) must match
them; the reference's save_p mode is recorded too, to pin the finding that
its q/k second-order gradients are incomplete.
"""

import glob
import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc

# attention-path cases (the P-taking Function fixture is covered by test_from_p_cpu.py,
# the TTT-E2E window fixture by test_ttt_e2e_cpu.py)
GOLDEN = sorted(p for p in glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz"))
                if not os.path.basename(p).startswith(("from_p_", "ttt_e2e_")))
NAMES = ("q", "k", "v", "do", "uq", "uk", "uv")


def _load(path):
    z = np.load(path)
    b, h, t, d, causal, seed = (int(x) for x in z["meta"])
    inputs = {n: torch.from_numpy(z[f"in_{n}"]) for n in NAMES}
    return z, inputs, bool(causal), float(z["scale"])


def _tol(z):
    return 1e-10 if z["in_q"].dtype == np.float64 else 2e-5


def test_golden_present():
    assert len(GOLDEN) >= 6


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_math_oracle_matches_reference(path):
    z, inp, causal, scale = _load(path)
    dtype = torch.float64 if z["in_q"].dtype == np.float64 else torch.float32
    out = orc.math_gradgrad(*(inp[n] for n in NAMES), causal=causal, scale=scale, dtype=dtype)
    for key in ("o", "dq", "dk", "dv", "gq", "gk", "gv"):
        ref = z[f"ref_{key}"]
        assert orc.normalized_err(out[key], ref) <= _tol(z), key


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_closed_form_matches_reference(path):
    z, inp, causal, scale = _load(path)
    out = orc.closed_form_gradgrad(*(inp[n].numpy() for n in NAMES), causal=causal, scale=scale)
    tol = 1e-10 if z["in_q"].dtype == np.float64 else 1e-4
    for key in ("o", "dq", "dk", "dv", "gq", "gk", "gv"):
        assert orc.normalized_err(out[key], z[f"ref_{key}"]) <= tol, key


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_mean_loss_objective_matches_reference(path):
    z, inp, causal, scale = _load(path)
    dtype = torch.float64 if z["in_q"].dtype == np.float64 else torch.float32
    out = orc.mean_loss_gradgrad(inp["q"], inp["k"], inp["v"], causal=causal, scale=scale, dtype=dtype)
    for key in ("gq", "gk", "gv"):
        ref = z[f"meanloss_{key}"]
        err = orc.max_abs_err(out[key], ref) / max(1e-30, float(np.abs(ref).max()))
        assert err <= (1e-9 if dtype == torch.float64 else 1e-4), key


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_reference_save_p_drops_q_k_terms(path):
    """The reference save_p grad-grad: exact for v, wrong for q and k."""
    z, _, _, _ = _load(path)
    assert orc.normalized_err(z["savep_gv"], z["ref_gv"]) <= _tol(z) * 10
    err_qk = max(orc.normalized_err(z["savep_gq"], z["ref_gq"]), orc.normalized_err(z["savep_gk"], z["ref_gk"]))
    assert err_qk > 1e-2


def test_closed_form_stats_consistent():
    """delta = rowsum(dO o O) and the gamma/rho identities the kernels use."""
    inp = orc.seeded_inputs(1, 2, 40, 16, seed=11, dtype=torch.float64)
    a = {n: inp[n].numpy() for n in NAMES}
    out = orc.closed_form_gradgrad(*(a[n] for n in NAMES), causal=True)
    o = out["o"]
    assert np.allclose(out["delta"], np.sum(a["do"] * o, -1))


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_gradgradcheck_fp64(causal):
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 2, 9, 4, generator=g, dtype=torch.float64, requires_grad=True) for _ in range(3))
    fn = lambda q, k, v: orc.attention_math(q, k, v, causal, 0.5)  # noqa: E731
    assert torch.autograd.gradcheck(fn, (q, k, v))
    assert torch.autograd.gradgradcheck(fn, (q, k, v))


def test_closed_form_gdo_matches_autograd():
    inp = orc.seeded_inputs(2, 1, 33, 8, seed=3, dtype=torch.float64)
    auto = orc.math_gradgrad(*(inp[n] for n in NAMES), causal=True, need_gdo=True)
    cf = orc.closed_form_gradgrad(*(inp[n].numpy() for n in NAMES), causal=True)
    for key in ("gq", "gk", "gv", "gdo"):
        assert orc.normalized_err(auto[key], cf[key]) <= 1e-10, key
