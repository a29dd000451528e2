"""GPU tests of failure detection (bounded waits), without faulting the GPU.

Every mbarrier wait in the kernels is bounded; a wait that runs out records a
code in the pass's device error word and in the host mirror the binding
registers, and the kernel returns normally. Here a self-test kernel runs that
same wait (tc100.cuh mbar_wait) on a barrier nothing completes, with a 1 ms
limit and no TMA or tensor-core work in flight, so the wait is made to run out
on purpose. The tests check that the code lands in the error word, that the
next op raises KernelError without a synchronization of its own, and that the
context and library work normally afterwards.
"""

import math

import pytest
import torch

from oracle import attention_oracle as orc
from testtimeideas_b200 import _lib

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms


def _small_inputs():
    inp = orc.seeded_inputs(1, 1, 128, 64, seed=5, scale_in=0.5)
    return {n: x.to(torch.float16).cuda() for n, x in inp.items()}


def _expected_code(code: int) -> bool:
    return (code & _lib.ERR_WORD_TIMEOUT) != 0 and ((code >> 8) & 0xFF) == _lib.SELFTEST_WAIT_SITE


def test_bounded_wait_runs_out_and_check_raises():
    dev = torch.device("cuda", 0)
    _lib.check_device_errors(dev)  # starts clean
    _lib.selftest_wait(LIMIT_NS, dev)
    torch.cuda.synchronize(dev)
    code = int(_lib.error_word(dev).item())
    assert _expected_code(code), hex(code)
    with pytest.raises(_lib.KernelError, match="error word"):
        _lib.check_device_errors(dev)
    assert int(_lib.error_word(dev).item()) == 0  # cleared by the report
    _lib.check_device_errors(dev)


def test_timeout_surfaces_at_the_next_op_and_library_recovers():
    dev = torch.device("cuda", 0)
    _lib.check_device_errors(dev)
    x = _small_inputs()
    scale = 1.0 / math.sqrt(64)
    _lib.attn_fwd(x["q"], x["k"], x["v"], True, scale)  # creates the error word and registers its host mirror
    torch.cuda.synchronize(dev)
    _lib.selftest_wait(LIMIT_NS, dev)
    torch.cuda.synchronize(dev)  # the failing kernel has finished; the next op issues no sync of its own
    with pytest.raises(_lib.KernelError, match="bounded wait"):
        _lib.attn_fwd(x["q"], x["k"], x["v"], True, scale)
    # the report cleared both words: the same op now runs and is correct
    o, _, _ = _lib.attn_fwd(x["q"], x["k"], x["v"], True, scale)
    ref = orc.closed_form_gradgrad(*(x[n].cpu().double().numpy() for n in ("q", "k", "v", "do", "uq", "uk", "uv")),
                                   causal=True, scale=scale)
    assert orc.normalized_err(o.float().cpu(), ref["o"]) <= 2e-3
    _lib.check_device_errors(dev)


def test_timeout_surfaces_through_the_public_autograd_path():
    import ttt_kernels
    dev = torch.device("cuda", 0)
    _lib.check_device_errors(dev)
    x = _small_inputs()
    q, k, v = (x[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    o = ttt_kernels.triton_attention(q, k, v, causal=True)
    torch.cuda.synchronize(dev)
    _lib.selftest_wait(LIMIT_NS, dev)
    torch.cuda.synchronize(dev)
    # the autograd engine re-raises the backward's exception (KernelError is a RuntimeError)
    with pytest.raises(RuntimeError, match="bounded wait"):
        torch.autograd.grad(o, (q, k, v), x["do"], create_graph=True)
    _lib.check_device_errors(dev)
