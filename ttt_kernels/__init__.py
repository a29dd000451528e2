"""Drop-in replacement for the reference package ``ttt_kernels``
(ttt_kernels/__init__.py:1-3): same module path, same exported name."""

from .triton_attention import triton_attention

__all__ = ["triton_attention"]
