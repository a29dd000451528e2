"""The TTT-E2E model and meta step (testtimeideas_b200.ttt_model) on CPU in
float64 against the reference's own meta_step on the same weights and data
(tests/golden/ttt_e2e_meta_fp64.npz, made by tests/golden/make_golden.py from
cloud_ttt_e2e/ttt_e2e): inner and outer losses and the meta-gradient of every
parameter. Cases: all layers updated, full-sequence attention; and one suffix
layer, a window shorter than the sequence (chunk loop), two inner steps on
chunks, only the fast MLPs updated."""

import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import ttt_model

FIX = os.path.join(os.path.dirname(__file__), "golden", "ttt_e2e_meta_fp64.npz")
CASES = {
    "meta_full": (dict(window_size=None, suffix_layers=-1), 1, 0.1, None, None),
    "meta_chunked": (dict(window_size=8, suffix_layers=1), 2, 0.05, "mlp_fast", 12),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_meta_step_matches_reference(name):
    z = np.load(FIX)
    over, steps, lr, pfilter, chunk = CASES[name]
    cfg = ttt_model.ModelConfig(vocab_size=64, max_seq_len=64, d_model=32, n_heads=2, n_layers=2, d_ff=64, **over)
    model = ttt_model.TTTModel(cfg).double()
    prefix = f"{name}/w/"
    model.load_state_dict({k[len(prefix):]: torch.from_numpy(z[k]) for k in z.files if k.startswith(prefix)})
    get = lambda key: torch.from_numpy(z[f"{name}/{key}"])  # noqa: E731
    inner, outer = ttt_model.meta_step(model, get("ids"), get("tgt"), get("inner_mask"), get("outer_mask"),
                                       inner_lr=lr, inner_steps=steps, param_filter=pfilter, chunk_size=chunk)
    outer.backward()
    ref_inner, ref_outer = z[f"{name}/losses"]
    assert abs(inner.item() - ref_inner) < 1e-12 and abs(outer.item() - ref_outer) < 1e-12
    grads = {f"{name}/g/{n}": p.grad for n, p in model.named_parameters() if p.grad is not None}
    assert set(grads) == {k for k in z.files if k.startswith(f"{name}/g/")}
    for key, g in grads.items():
        assert orc.normalized_err(g, z[key]) < 1e-10, key


INFER_FIX = os.path.join(os.path.dirname(__file__), "golden", "ttt_e2e_infer_fp64.npz")
INFER_CASES = {
    # config overrides, inner steps, inner lr, param filter, chunk size, stream (window, chunk)
    "infer_chunked": (dict(window_size=8, suffix_layers=1), 2, 0.05, "suffix_blocks,ln_f,head", 8, (8, 8)),
    "infer_full": (dict(window_size=None, suffix_layers=-1), 1, 0.1, None, None, (12, 4)),
}


@pytest.mark.parametrize("name", sorted(INFER_CASES))
def test_inference_adaptation_and_streaming_match_reference(name):
    """ttt_apply + ttt_logits (test-time adaptation without create_graph) and the
    streaming forwards of the reference's latency demo, against the reference's
    own functions on the same weights (tests/golden/ttt_e2e_infer_fp64.npz)."""
    z = np.load(INFER_FIX)
    over, steps, lr, pfilter, chunk, (window, schunk) = INFER_CASES[name]
    cfg = ttt_model.ModelConfig(vocab_size=64, max_seq_len=64, d_model=32, n_heads=2, n_layers=2, d_ff=64,
                                dropout=0.0, **over)
    model = ttt_model.TTTModel(cfg).double().eval()
    prefix = f"{name}/w/"
    model.load_state_dict({k[len(prefix):]: torch.from_numpy(z[k]) for k in z.files if k.startswith(prefix)})
    get = lambda key: torch.from_numpy(z[f"{name}/{key}"])  # noqa: E731
    params = ttt_model.ttt_apply(model, get("ids"), get("tgt"), get("inner_mask"), inner_lr=lr, inner_steps=steps,
                                 param_filter=pfilter, chunk_size=chunk)
    with torch.no_grad():
        logits = ttt_model.ttt_logits(model, params, get("ids"), chunk_size=chunk)
    assert orc.normalized_err(logits, z[f"{name}/logits"]) < 1e-12
    stream = ttt_model.stream_logits(model, get("ids"), window, schunk)
    refs = sorted((k for k in z.files if k.startswith(f"{name}/stream")), key=lambda k: int(k.rsplit("stream", 1)[1]))
    assert len(stream) == len(refs)
    for x, k in zip(stream, refs):
        assert orc.normalized_err(x, z[k]) < 1e-12, k
