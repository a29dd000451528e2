"""Drop-in for ``ttt_kernels/triton_attention.py`` of the reference.

``triton_attention`` and ``TritonAttentionFn`` keep the reference signatures
(triton_attention.py:259-261, 423-424) but run the sm_100a kernels of
``libttt_attn.so``. ``_attention_math`` keeps the reference's math definition
(triton_attention.py:18-25) for callers that import it.
"""

from testtimeideas_b200.attention import (  # noqa: F401
    BWD_MODES,
    SAVE_P_MODES,
    TritonAttentionFn,
    attention_math as _attention_math,
    triton_attention,
)

from . import backward_stubs  # noqa: F401

__all__ = ["triton_attention", "TritonAttentionFn"]
