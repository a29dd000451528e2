"""Generate the golden vectors in tests/golden/ from the reference itself.

Runs only where a reference checkout exists: pass its directory with
--reference DIR or in $TTT_REFERENCE_DIR. It imports the reference's ``ttt_kernels`` package under
the alias ``ref_ttt_kernels`` (its own name is taken by the drop-in package of
this repository) and calls its public entry point
``triton_attention(q, k, v, causal=..., bwd_mode=...)`` on CPU tensors, where
the reference runs its math path (triton_attention.py:275-280 forward,
416-420 recompute backward). Outputs: forward O, first-order grads of
<O, dO> (create_graph=True) and second-order grads of <dq,uq>+<dk,uk>+<dv,uv>.

Also records the reference's TTT-E2E attention (GradGradAttentionFn with a
sliding-window mask, and WindowedSelfAttention's chunk loop) and meta step on
tiny models, the backward
methods of the reference's P-taking autograd
Functions (TritonDvFn, TritonRowSumFn, TritonDqDkFn) on fixed inputs, and the
reference's ``save_p`` mode on the same inputs as the math path; its
grad-grad for q and k differs from the math path because P is saved as a
constant (backward_stubs.py:428-514); the tests pin that difference too.

    python tests/golden/make_golden.py --reference <checkout of ry2009/TestTimeIdeas>
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("TTT_REFERENCE_DIR", "")) if os.environ.get("TTT_REFERENCE_DIR") else None

# (name, b, h, t, d, causal, dtype, seed, input scale)
CASES = [
    ("config1_noncausal_t64_d64_fp32", 1, 1, 64, 64, False, torch.float32, 0, 1.0),
    ("config1_causal_t64_d64_fp32", 1, 1, 64, 64, True, torch.float32, 1, 1.0),
    ("ragged_causal_b2h2_t37_d16_fp64", 2, 2, 37, 16, True, torch.float64, 2, 1.0),
    ("noncausal_b1h2_t48_d16_fp64", 1, 2, 48, 16, False, torch.float64, 3, 1.0),
    ("causal_b1h1_t130_d16_fp64", 1, 1, 130, 16, True, torch.float64, 4, 0.5),
    ("noncausal_b1h1_t64_d128_fp32", 1, 1, 64, 128, False, torch.float32, 5, 0.5),
]


def load_reference():
    pkg_dir = REF / "ttt_kernels"
    spec = importlib.util.spec_from_file_location("ref_ttt_kernels", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_ttt_kernels"] = mod
    spec.loader.exec_module(mod)
    # the package re-exports the function under the submodule's name
    return sys.modules["ref_ttt_kernels.triton_attention"]


def run_reference(ta, inputs, causal, mode):
    q, k, v = (inputs[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    out = ta.triton_attention(q, k, v, causal=causal, bwd_mode=mode)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), inputs["do"], create_graph=True)
    l2 = (dq * inputs["uq"]).sum() + (dk * inputs["uk"]).sum() + (dv * inputs["uv"]).sum()
    gq, gk, gv = torch.autograd.grad(l2, (q, k, v))
    return {"o": out, "dq": dq, "dk": dk, "dv": dv, "gq": gq, "gk": gk, "gv": gv}


def run_reference_mean_loss(ta, inputs, causal):
    """The reference benchmark objective (tests/bench_gradgrad_sweep.py:56-61)."""
    q, k, v = (inputs[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    out = ta.triton_attention(q, k, v, causal=causal, bwd_mode="recompute")
    grads = torch.autograd.grad(out.float().mean(), (q, k, v), create_graph=True)
    s = sum(g.pow(2).mean() for g in grads)
    gg = torch.autograd.grad(s, (q, k, v))
    return {"gq": gg[0], "gk": gg[1], "gv": gg[2]}


class _Ctx:
    """Stand-in for an autograd context: just the saved tensors and attributes."""

    def __init__(self, saved, **attrs):
        self.saved_tensors = saved
        self.__dict__.update(attrs)


def from_p_function_backwards(out_path: Path) -> None:
    """Outputs of the backward methods of the reference's TritonDvFn,
    TritonRowSumFn and TritonDqDkFn (backward_stubs.py:428-514). Those methods
    are plain torch code, so they run on CPU with a stand-in context; their
    forwards are Triton kernels and are not run here."""
    bs = sys.modules["ref_ttt_kernels.backward_stubs"]
    b, h, t, d, causal = 1, 2, 48, 16, True
    scale = 1.0 / math.sqrt(d)
    g = torch.Generator().manual_seed(17)
    rnd = lambda *shape: torch.randn(*shape, generator=g, dtype=torch.float64)  # noqa: E731
    q, k, v, do = (rnd(b, h, t, d) for _ in range(4))
    s = torch.matmul(q, k.transpose(-2, -1)) * scale
    s = s.masked_fill(torch.triu(torch.ones(t, t, dtype=torch.bool), 1), float("-inf"))
    p = torch.softmax(s, dim=-1)
    rowsum = (torch.matmul(do, v.transpose(-2, -1)) * p).sum(-1)
    gdv, gdq, gdk = rnd(b, h, t, d), rnd(b, h, t, d), rnd(b, h, t, d)
    grs = rnd(b, h, t)
    rec = {"q": q, "k": k, "v": v, "do": do, "p": p, "rowsum": rowsum, "gdv": gdv, "gdq": gdq, "gdk": gdk,
           "grs": grs}
    out = bs.TritonDvFn.backward(_Ctx((p, do)), gdv)
    rec.update({"dvfn_grad_p": out[0], "dvfn_grad_do": out[1]})
    out = bs.TritonRowSumFn.backward(_Ctx((p, do, v), causal=causal), grs)
    rec.update({"rsfn_grad_p": out[0], "rsfn_grad_do": out[1], "rsfn_grad_v": out[2]})
    out = bs.TritonDqDkFn.backward(_Ctx((q, k, v, do, p, rowsum), scale=scale, causal=causal), gdq, gdk)
    for name, x in zip(("q", "k", "v", "do", "p", "rowsum"), out[:6]):
        rec[f"dqdkfn_grad_{name}"] = x
    rec = {n: x.detach().numpy() for n, x in rec.items()}
    rec["meta"] = np.array([b, h, t, d, int(causal)], dtype=np.int64)
    rec["scale"] = np.array(scale)
    np.savez_compressed(out_path, **rec)
    print(f"wrote {out_path.name}")


def load_reference_ttt_e2e():
    """The reference's TTT-E2E package (cloud_ttt_e2e/ttt_e2e) under the alias ref_ttt_e2e."""
    pkg_dir = REF / "cloud_ttt_e2e" / "ttt_e2e"
    spec = importlib.util.spec_from_file_location("ref_ttt_e2e", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_ttt_e2e"] = mod
    spec.loader.exec_module(mod)
    return sys.modules["ref_ttt_e2e.attention"], sys.modules["ref_ttt_e2e.utils"]


def ttt_e2e_window_cases(out_path: Path) -> None:
    """The reference's TTT-E2E attention on CPU (pure torch there):
    * GradGradAttentionFn.apply(q, k, v, make_window_mask(t, W)) with a binding
      sliding window (W < t): forward, first-order grads with create_graph and the
      second-order grads of <dq,uq>+<dk,uk>+<dv,uv>;
    * WindowedSelfAttention(window_size=W) on a sequence longer than W, so that
      its chunk loop runs (attention.py:112-127), with a partial last chunk:
      output, d<out,g>/dx with create_graph, and d<that,u>/dx. Its seeded
      initial weights are saved with the outputs."""
    attn, utils = load_reference_ttt_e2e()
    rec = {}
    b, h, t, d, w = 1, 2, 48, 16, 12
    g = torch.Generator().manual_seed(21)
    x = {n: torch.randn(b, h, t, d, generator=g, dtype=torch.float64) for n in ("q", "k", "v", "do", "uq", "uk", "uv")}
    q, k, v = (x[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    # GradGradAttentionFn keeps a graph only when the upstream gradient requires grad
    # (need_higher = grad_out.requires_grad, attention.py:32), as in the TTT meta step
    do = x["do"].clone().requires_grad_(True)
    mask = utils.make_window_mask(t, w, torch.device("cpu"), torch.float64).view(1, 1, t, t)
    out = attn.GradGradAttentionFn.apply(q, k, v, mask)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), do, create_graph=True)
    l2 = (dq * x["uq"]).sum() + (dk * x["uk"]).sum() + (dv * x["uv"]).sum()
    gq, gk, gv, gdo = torch.autograd.grad(l2, (q, k, v, do))
    rec.update({f"sw_in_{n}": t_.numpy() for n, t_ in x.items()})
    rec.update({f"sw_{n}": t_.detach().numpy() for n, t_ in
                (("o", out), ("dq", dq), ("dk", dk), ("dv", dv), ("gq", gq), ("gk", gk), ("gv", gv), ("gdo", gdo))})
    rec["sw_meta"] = np.array([b, h, t, d, w], dtype=np.int64)

    d_model, n_heads, w2, t2 = 32, 2, 16, 40
    torch.manual_seed(5)
    mod = attn.WindowedSelfAttention(d_model, n_heads, w2, use_gradgrad=True).double()
    g2 = torch.Generator().manual_seed(22)
    xin = torch.randn(1, t2, d_model, generator=g2, dtype=torch.float64).requires_grad_(True)
    gout = torch.randn(1, t2, d_model, generator=g2, dtype=torch.float64)
    uin = torch.randn(1, t2, d_model, generator=g2, dtype=torch.float64)
    y = mod(xin)
    (gx,) = torch.autograd.grad(y, xin, gout, create_graph=True)
    (ggx,) = torch.autograd.grad((gx * uin).sum(), xin)
    rec.update({f"wsa_{n}": p_.detach().numpy() for n, p_ in mod.state_dict().items()})
    rec.update({"wsa_x": xin.detach().numpy(), "wsa_g": gout.numpy(), "wsa_u": uin.numpy(), "wsa_y": y.detach().numpy(),
                "wsa_gx": gx.detach().numpy(), "wsa_ggx": ggx.numpy()})
    rec["wsa_meta"] = np.array([d_model, n_heads, w2, t2], dtype=np.int64)
    np.savez_compressed(out_path, **rec)
    print(f"wrote {out_path.name}")


# (name, cfg overrides, t, inner_steps, inner_lr, param_filter, chunk_size)
META_CASES = [
    ("meta_full", dict(window_size=None, suffix_layers=-1), 24, 1, 0.1, None, None),
    ("meta_chunked", dict(window_size=8, suffix_layers=1), 24, 2, 0.05, "mlp_fast", 12),
]


def ttt_e2e_meta_cases(out_path: Path) -> None:
    """The reference's meta_step (cloud_ttt_e2e/ttt_e2e/meta.py:148-184) on tiny
    float64 TTT models on CPU: inner and outer losses and the meta-gradient
    (d outer_loss / d every parameter), with the seeded initial weights."""
    load_reference_ttt_e2e()
    model_mod, meta_mod = sys.modules["ref_ttt_e2e.model"], sys.modules["ref_ttt_e2e.meta"]
    rec = {}
    for name, over, t, steps, lr, pfilter, chunk in META_CASES:
        cfg = model_mod.ModelConfig(vocab_size=64, max_seq_len=64, d_model=32, n_heads=2, n_layers=2, d_ff=64,
                                    **over)
        torch.manual_seed(11)
        model = model_mod.TTTModel(cfg).double()
        g = torch.Generator().manual_seed(12)
        ids = torch.randint(0, cfg.vocab_size, (2, t), generator=g)
        tgt = torch.randint(0, cfg.vocab_size, (2, t), generator=g)
        inner_mask = (torch.rand(2, t, generator=g) < 0.7).to(torch.float64)
        outer_mask = 1.0 - inner_mask
        inner, outer = meta_mod.meta_step(model, ids, tgt, inner_mask, outer_mask, inner_lr=lr, inner_steps=steps,
                                          param_filter=pfilter, chunk_size=chunk)
        outer.backward()
        rec.update({f"{name}/w/{n}": p_.detach().numpy() for n, p_ in model.state_dict().items()})
        rec.update({f"{name}/g/{n}": p_.grad.numpy() for n, p_ in model.named_parameters() if p_.grad is not None})
        rec.update({f"{name}/ids": ids.numpy(), f"{name}/tgt": tgt.numpy(), f"{name}/inner_mask": inner_mask.numpy(),
                    f"{name}/outer_mask": outer_mask.numpy(),
                    f"{name}/losses": np.array([inner.item(), outer.item()])})
    np.savez_compressed(out_path, **rec)
    print(f"wrote {out_path.name}")


# name, config overrides, t, inner_steps, inner_lr, param_filter, chunk_size, stream window/chunk
INFER_CASES = [
    ("infer_chunked", dict(window_size=8, suffix_layers=1), 24, 2, 0.05, "suffix_blocks,ln_f,head", 8, (8, 8)),
    ("infer_full", dict(window_size=None, suffix_layers=-1), 16, 1, 0.1, None, None, (12, 4)),
]


def ttt_e2e_infer_cases(out_path: Path) -> None:
    """Test-time adaptation at inference with the reference's ttt_apply and
    ttt_logits (cloud_ttt_e2e/ttt_e2e/meta.py:180-224) on tiny float64 TTT models
    on CPU, and streaming forwards as its latency demo runs them
    (cloud_ttt_e2e/scripts/demo_infer.py:11-27): the adapted model's logits and
    each streaming call's logits."""
    load_reference_ttt_e2e()
    model_mod, meta_mod = sys.modules["ref_ttt_e2e.model"], sys.modules["ref_ttt_e2e.meta"]
    rec = {}
    for name, over, t, steps, lr, pfilter, chunk, (window, schunk) in INFER_CASES:
        cfg = model_mod.ModelConfig(vocab_size=64, max_seq_len=64, d_model=32, n_heads=2, n_layers=2, d_ff=64,
                                    dropout=0.0, **over)
        torch.manual_seed(21)
        model = model_mod.TTTModel(cfg).double().eval()
        g = torch.Generator().manual_seed(22)
        ids = torch.randint(0, cfg.vocab_size, (1, t), generator=g)
        tgt = torch.randint(0, cfg.vocab_size, (1, t), generator=g)
        inner_mask = (torch.rand(1, t, generator=g) < 0.7).to(torch.float64)
        params = meta_mod.ttt_apply(model, ids, tgt, inner_mask, inner_lr=lr, inner_steps=steps,
                                    param_filter=pfilter, chunk_size=chunk)
        with torch.no_grad():
            logits = meta_mod.ttt_logits(model, params, ids, chunk_size=chunk)
            stream = [model(ids[:, max(0, end - window):end])
                      for end in (min(t, s0 + schunk) for s0 in range(0, t, schunk))]
        rec.update({f"{name}/w/{n}": p_.detach().numpy() for n, p_ in model.state_dict().items()})
        rec.update({f"{name}/ids": ids.numpy(), f"{name}/tgt": tgt.numpy(), f"{name}/inner_mask": inner_mask.numpy(),
                    f"{name}/logits": logits.numpy()})
        rec.update({f"{name}/stream{i}": x.numpy() for i, x in enumerate(stream)})
    np.savez_compressed(out_path, **rec)
    print(f"wrote {out_path.name}")


def main() -> None:
    import argparse
    global REF
    ap = argparse.ArgumentParser(description="regenerate tests/golden/*.npz from a reference checkout")
    ap.add_argument("--reference", type=Path, default=REF,
                    help="directory of the ry2009/TestTimeIdeas checkout (default: $TTT_REFERENCE_DIR)")
    args = ap.parse_args()
    if args.reference is None or not (args.reference / "ttt_kernels").is_dir():
        raise SystemExit("give the reference checkout with --reference DIR or $TTT_REFERENCE_DIR")
    REF = args.reference
    ttt_e2e_window_cases(HERE / "ttt_e2e_windows_fp64.npz")
    ttt_e2e_meta_cases(HERE / "ttt_e2e_meta_fp64.npz")
    ttt_e2e_infer_cases(HERE / "ttt_e2e_infer_fp64.npz")
    ta = load_reference()
    importlib.import_module("ref_ttt_kernels.backward_stubs")
    from_p_function_backwards(HERE / "from_p_function_backwards_t48_d16_fp64.npz")
    for name, b, h, t, d, causal, dtype, seed, sc in CASES:
        g = torch.Generator().manual_seed(seed)
        inputs = {n: (torch.randn(b, h, t, d, generator=g, dtype=torch.float64) * sc).to(dtype)
                  for n in ("q", "k", "v", "do", "uq", "uk", "uv")}
        ref = run_reference(ta, inputs, causal, "recompute")
        rec = {f"in_{n}": x.numpy() for n, x in inputs.items()}
        rec.update({f"ref_{n}": x.detach().numpy() for n, x in ref.items()})
        savep = run_reference(ta, inputs, causal, "save_p")
        rec.update({f"savep_{n}": x.detach().numpy() for n, x in savep.items() if n.startswith("g")})
        ml = run_reference_mean_loss(ta, inputs, causal)
        rec.update({f"meanloss_{n}": x.detach().numpy() for n, x in ml.items()})
        rec["meta"] = np.array([b, h, t, d, int(causal), seed], dtype=np.int64)
        rec["scale"] = np.array(1.0 / math.sqrt(d))
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(f"wrote {name}.npz")


if __name__ == "__main__":
    main()
