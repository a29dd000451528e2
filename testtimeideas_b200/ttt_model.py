"""The TTT-E2E model and its meta step, with every attention call on the
sm_100a kernels (the f3 row: the driver of BASELINE config 5).

Same configuration fields, module and parameter names as the reference
(cloud_ttt_e2e/ttt_e2e/model.py:9-143), so its state dicts load here, and the
same meta step (cloud_ttt_e2e/ttt_e2e/meta.py:148-184): prefix blocks run once,
the inner loop takes ``inner_steps`` SGD steps on the suffix loss per chunk with
``create_graph=True`` for the parameters ``param_filter`` selects, and the
outer loss is the masked loss of the updated model. Backpropagating the outer
loss differentiates through the inner step, i.e. through the first-order
attention backward: that is the grad-grad attention step, including the
gradient with respect to the upstream gradient (∂dO), which the kernels'
double backward provides.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import nn
from torch.func import functional_call

from .ttt_e2e import WindowedSelfAttention


@dataclass
class ModelConfig:
    vocab_size: int = 4096
    max_seq_len: int = 8192
    window_size: Optional[int] = 512
    d_model: int = 512
    n_heads: int = 8
    n_layers: int = 8
    d_ff: int = 2048
    dropout: float = 0.0
    use_gradgrad_attention: bool = True
    suffix_layers: int = -1  # layers updated by the inner loop (-1: all); the rest form the prefix
    dual_mlp: bool = True    # suffix blocks add a slow MLP to the fast one


def _mlp(cfg: ModelConfig) -> nn.Sequential:
    return nn.Sequential(nn.Linear(cfg.d_model, cfg.d_ff), nn.GELU(), nn.Linear(cfg.d_ff, cfg.d_model))


class PrefixBlock(nn.Module):
    """Pre-norm block: x + attn(ln1 x), then x + mlp(ln2 x)."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = WindowedSelfAttention(cfg.d_model, cfg.n_heads, cfg.window_size, cfg.use_gradgrad_attention)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.mlp = _mlp(cfg)
        self.dropout = nn.Dropout(cfg.dropout)

    def forward(self, x):
        x = x + self.dropout(self.attn(self.ln1(x)))
        return x + self.dropout(self.mlp(self.ln2(x)))


class SuffixBlock(nn.Module):
    """Pre-norm block whose MLP is a fast MLP (plus a slow one with dual_mlp)."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = WindowedSelfAttention(cfg.d_model, cfg.n_heads, cfg.window_size, cfg.use_gradgrad_attention)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.mlp_fast = _mlp(cfg)
        self.mlp_slow = _mlp(cfg) if cfg.dual_mlp else None
        self.dropout = nn.Dropout(cfg.dropout)

    def forward(self, x):
        x = x + self.dropout(self.attn(self.ln1(x)))
        h = self.ln2(x)
        y = self.mlp_fast(h)
        if self.mlp_slow is not None:
            y = y + self.mlp_slow(h)
        return x + self.dropout(y)


class TTTModel(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.pos = nn.Embedding(cfg.max_seq_len, cfg.d_model)
        n_suffix = cfg.n_layers if cfg.suffix_layers < 0 or cfg.suffix_layers > cfg.n_layers else cfg.suffix_layers
        self.suffix_layers = n_suffix
        self.prefix_layers = cfg.n_layers - n_suffix
        self.prefix_blocks = nn.ModuleList(PrefixBlock(cfg) for _ in range(self.prefix_layers))
        self.suffix_blocks = nn.ModuleList(SuffixBlock(cfg) for _ in range(n_suffix))
        self.ln_f = nn.LayerNorm(cfg.d_model)
        self.head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)

    def prefix_forward(self, input_ids):
        t = input_ids.shape[1]
        x = self.embed(input_ids) + self.pos(torch.arange(t, device=input_ids.device))[None]
        for blk in self.prefix_blocks:
            x = blk(x)
        return x

    def suffix_forward(self, hidden):
        x = hidden
        for blk in self.suffix_blocks:
            x = blk(x)
        return self.head(self.ln_f(x))

    def forward(self, input_ids=None, *, mode: str = "full", prefix_hidden=None):
        """Token ids to logits. mode="prefix" stops after the prefix blocks and returns
        their hidden states; mode="suffix" starts from such states (prefix_hidden);
        any other mode runs the whole model, as the reference's does."""
        start_from_hidden = mode == "suffix"
        given, what = (prefix_hidden, "prefix_hidden") if start_from_hidden else (input_ids, "input_ids")
        if given is None:
            raise ValueError(f"TTTModel.forward(mode={mode!r}) needs {what}")
        hidden = prefix_hidden if start_from_hidden else self.prefix_forward(input_ids)
        return hidden if mode == "prefix" else self.suffix_forward(hidden)


def compute_loss(logits, targets, mask=None):
    """Token cross-entropy, averaged over the positions where mask is set."""
    ce = F.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1), reduction="none")
    if mask is None:
        return ce.mean()
    m = mask.reshape(-1).float()
    return (ce * m).sum() / m.sum().clamp_min(1.0)


def _fast_names(model: nn.Module, param_filter) -> List[str]:
    """Parameters the inner loop updates: names containing any filter string
    (comma-separated or a sequence), or all parameters when none matches."""
    names = [n for n, _ in model.named_parameters()]
    if param_filter is None:
        return names
    keys = param_filter.split(",") if isinstance(param_filter, str) else [str(x) for x in param_filter]
    keys = [k.strip() for k in keys if k.strip()]
    chosen = [n for n in names if any(k in n for k in keys)]
    return chosen or names


def _chunks(x: torch.Tensor, size: Optional[int]) -> Sequence[torch.Tensor]:
    if size is None or x.dim() < 2:
        return [x]
    if x.shape[1] % size:
        raise ValueError(f"seq len {x.shape[1]} not divisible by chunk_size {size}")
    return x.split(size, dim=1)


def _suffix_logits(model: TTTModel, params: Dict[str, torch.Tensor], hidden: torch.Tensor) -> torch.Tensor:
    return functional_call(model, params, (None,), {"mode": "suffix", "prefix_hidden": hidden})


def _inner_scan(model: TTTModel, params: Dict[str, torch.Tensor], fast: List[str], prefix: torch.Tensor, targets,
                inner_mask, inner_lr: float, inner_steps: int, chunk_size: Optional[int],
                create_graph: bool) -> Tuple[Dict[str, torch.Tensor], torch.Tensor]:
    """``inner_steps`` SGD steps on each chunk's suffix loss, chunk after chunk, for
    the parameters named in ``fast`` (cloud_ttt_e2e/ttt_e2e/meta.py:44-109); with
    create_graph the updates stay differentiable (the meta step), without it they
    are plain tensors (test-time adaptation at inference)."""
    inner_losses = []
    for hid, tgt, msk in zip(_chunks(prefix, chunk_size), _chunks(targets, chunk_size), _chunks(inner_mask, chunk_size)):
        for _ in range(inner_steps):
            loss = compute_loss(_suffix_logits(model, params, hid), tgt, msk)
            grads = torch.autograd.grad(loss, [params[n] for n in fast], create_graph=create_graph,
                                        retain_graph=create_graph)
            params = dict(params)
            for n, g in zip(fast, grads):
                params[n] = params[n] - inner_lr * g
        inner_losses.append(loss)
    inner_loss = torch.stack(inner_losses).mean() if inner_losses else torch.zeros((), device=targets.device)
    return params, inner_loss


def meta_step(model: TTTModel, input_ids, targets, inner_mask, outer_mask, inner_lr: float, inner_steps: int,
              param_filter=None, chunk_size: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(inner_loss, outer_loss) of one meta step; outer_loss.backward() gives the meta-gradient."""
    params: Dict[str, torch.Tensor] = dict(model.named_parameters())
    fast = _fast_names(model, param_filter)
    prefix = functional_call(model, params, (input_ids,), {"mode": "prefix"})
    params, inner_loss = _inner_scan(model, params, fast, prefix, targets, inner_mask, inner_lr, inner_steps,
                                     chunk_size, create_graph=True)
    total, weight = torch.zeros((), device=targets.device), torch.zeros((), device=targets.device)
    for hid, tgt, msk in zip(_chunks(prefix, chunk_size), _chunks(targets, chunk_size), _chunks(outer_mask, chunk_size)):
        w = msk.sum()
        if w.item() <= 0:
            continue
        total = total + compute_loss(_suffix_logits(model, params, hid), tgt, msk) * w
        weight = weight + w
    return inner_loss, total / weight.clamp_min(1.0)


def ttt_apply(model: TTTModel, input_ids, targets, inner_mask, inner_lr: float, inner_steps: int,
              param_filter=None, chunk_size: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Test-time adaptation at inference (cloud_ttt_e2e/ttt_e2e/meta.py:180-204): the
    inner loop without create_graph; returns the adapted parameters by name. Each
    inner step is an attention forward and first-order backward on the kernels."""
    params: Dict[str, torch.Tensor] = dict(model.named_parameters())
    fast = _fast_names(model, param_filter)
    prefix = functional_call(model, params, (input_ids,), {"mode": "prefix"})
    params, _ = _inner_scan(model, params, fast, prefix, targets, inner_mask, inner_lr, inner_steps, chunk_size,
                            create_graph=False)
    return params


def ttt_logits(model: TTTModel, params: Dict[str, torch.Tensor], input_ids,
               chunk_size: Optional[int] = None) -> torch.Tensor:
    """Logits of the model with parameters ``params`` (cloud_ttt_e2e/ttt_e2e/meta.py:207-224):
    the prefix over the whole sequence, the suffix over each chunk of it."""
    prefix = functional_call(model, params, (input_ids,), {"mode": "prefix"})
    return torch.cat([_suffix_logits(model, params, h) for h in _chunks(prefix, chunk_size)], dim=1)


@torch.no_grad()
def stream_logits(model: TTTModel, tokens: torch.Tensor, window_size: int, chunk_size: int) -> List[torch.Tensor]:
    """Streaming inference as the reference's latency demo runs it
    (cloud_ttt_e2e/scripts/demo_infer.py:11-27): for each chunk of ``chunk_size``
    new tokens, one forward over the last ``window_size`` tokens up to the
    chunk's end (forward-only attention on the kernels). Returns each call's logits."""
    out = []
    t = tokens.shape[1]
    for start in range(0, t, chunk_size):
        end = min(t, start + chunk_size)
        out.append(model(tokens[:, max(0, end - window_size):end]))
    return out
