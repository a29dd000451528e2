"""B200-native (sm_100a) grad-grad-safe attention.

The public surface mirrors the reference's ``ttt_kernels`` package; the
kernels live in ``libttt_attn.so`` (C ABI: ``include/ttt_attn.h``).
"""

from .attention import TritonAttentionFn, triton_attention, BWD_MODES, SAVE_P_MODES

__all__ = ["triton_attention", "TritonAttentionFn", "BWD_MODES", "SAVE_P_MODES"]
