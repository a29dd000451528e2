"""The TTT-E2E meta step on CUDA (bf16 model, every attention call on the
sm_100a kernels) against the same model in float64 on CPU, where the step is
the reference's formulation (pinned by tests/test_ttt_model_cpu.py). Checks the
losses, the meta-gradient, and that the grad-grad kernels ran."""

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib, ttt_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("window,suffix,chunk,pfilter", [(None, -1, None, None), (96, 1, 128, "mlp_fast")])
def test_meta_step_cuda_matches_cpu(window, suffix, chunk, pfilter):
    cfg = ttt_model.ModelConfig(vocab_size=256, max_seq_len=512, d_model=128, n_heads=2, n_layers=2, d_ff=256,
                                window_size=window, suffix_layers=suffix)
    torch.manual_seed(3)
    cpu = ttt_model.TTTModel(cfg).double()
    gpu = ttt_model.TTTModel(cfg).to("cuda", torch.bfloat16)
    gpu.load_state_dict({n: p.to(torch.bfloat16) for n, p in cpu.state_dict().items()})
    t = 256
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (1, t), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (1, t), generator=g)
    inner_mask = torch.zeros(1, t)
    inner_mask[:, : 3 * t // 4] = 1.0
    outer_mask = 1.0 - inner_mask

    def run(model, dev):
        args = [x.to(dev) for x in (ids, tgt, inner_mask, outer_mask)]
        inner, outer = ttt_model.meta_step(model, *args, inner_lr=0.05, inner_steps=1, param_filter=pfilter,
                                           chunk_size=chunk)
        outer.backward()
        return inner.item(), outer.item(), {n: p.grad for n, p in model.named_parameters() if p.grad is not None}

    ri, ro, rg = run(cpu, "cpu")
    _lib.profile_collect()
    _lib.profile_enable(True)
    gi, go, gg = run(gpu, "cuda")
    torch.cuda.synchronize()
    _lib.profile_enable(False)
    prof = _lib.profile_collect()
    _lib.check_device_errors()
    assert abs(gi - ri) < 2e-2 * abs(ri) and abs(go - ro) < 2e-2 * abs(ro)
    assert set(gg) == set(rg)
    # bf16 weights and activations through the whole model: compare the meta-gradient in aggregate
    num = sum(float((gg[n].double().cpu() - rg[n]).pow(2).sum()) for n in rg)
    den = sum(float(rg[n].pow(2).sum()) for n in rg)
    assert (num / den) ** 0.5 < 5e-2
    # the double backward runs when the inner gradient passes through attention (all
    # parameters updated); with only the last block's fast MLP updated it does not
    # (head dim 64: dQ comes out of the key-major pass, so no separate query-major dQ pass runs)
    kinds = ("fwd", "bwd_kv") + (("bwd2_stats", "bwd2_q", "bwd2_kv") if pfilter is None else ())
    for kind in kinds:
        assert prof[kind][0] > 0, kind
    if pfilter is not None:
        assert prof["bwd2_q"][0] == 0


def test_inference_adaptation_and_streaming_cuda_matches_cpu():
    """ttt_apply + ttt_logits and streaming forwards (the forward-only path) on a bf16
    CUDA model against float64 on CPU; the forward and first-order backward kernels run,
    the double backward does not (no create_graph at inference)."""
    cfg = ttt_model.ModelConfig(vocab_size=256, max_seq_len=512, d_model=128, n_heads=2, n_layers=2, d_ff=256,
                                window_size=128, suffix_layers=1, dropout=0.0)
    torch.manual_seed(5)
    cpu = ttt_model.TTTModel(cfg).double().eval()
    gpu = ttt_model.TTTModel(cfg).to("cuda", torch.bfloat16).eval()
    gpu.load_state_dict({n: p.to(torch.bfloat16) for n, p in cpu.state_dict().items()})
    t = 256
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, cfg.vocab_size, (1, t), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (1, t), generator=g)
    inner_mask = (torch.rand(1, t, generator=g) < 0.7).float()

    def run(model, dev):
        a = [x.to(dev) for x in (ids, tgt, inner_mask)]
        params = ttt_model.ttt_apply(model, *a, inner_lr=0.05, inner_steps=2, param_filter="suffix_blocks,ln_f,head",
                                     chunk_size=128)
        with torch.no_grad():
            logits = ttt_model.ttt_logits(model, params, a[0], chunk_size=128)
        return logits, ttt_model.stream_logits(model, a[0], window_size=128, chunk_size=64)

    ref_logits, ref_stream = run(cpu, "cpu")
    _lib.profile_collect()
    _lib.profile_enable(True)
    logits, stream = run(gpu, "cuda")
    torch.cuda.synchronize()
    _lib.profile_enable(False)
    prof = _lib.profile_collect()
    _lib.check_device_errors()
    rel = lambda x, r: float((x.double().cpu() - r).norm() / r.norm())  # noqa: E731
    assert rel(logits, ref_logits) < 3e-2
    assert len(stream) == len(ref_stream)
    for x, r in zip(stream, ref_stream):
        assert rel(x, r) < 3e-2
    for kind in ("fwd", "bwd_kv"):
        assert prof[kind][0] > 0, kind
    assert prof["bwd2_stats"][0] == 0
