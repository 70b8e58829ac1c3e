"""triangleops_b200 — B200-native (sm_100a) TriangleOps.

Drop-in for the ``triangle_ops`` Python API (``triangle_ops/__init__.py:17-31``):

    attention_pair_bias            — QKV proj + LN(Z) bias + attention, then gate + W_o
    triangle_attention             — LN + Q/K/V/bias proj + attention, then gate + W_o
    triangle_multiplicative_update — LN + gated proj, triangular contraction, LN + gated proj

Each op module exposes ``precompute(...)`` (one-time weight prep -> opaque dict),
``forward(x, pre, ...)`` (per call) and the one-shot ``<op_name>(...)``.
``pairformer.pair_update`` chains the triangle ops of one Pairformer block
in place (residual adds fused, ending node without a transpose copy);
``transition`` is the Pairformer pair transition MLP (one fused kernel).
All compute runs in hand-written sm_100a kernels behind a C-ABI library
(``libtriangleops_b200.so``); there is no CPU fallback.
"""

from . import attn_pair_bias, pairformer, transition, triangle_attn, triangle_mul
from .attn_pair_bias import attention_pair_bias
from .triangle_attn import triangle_attention
from .triangle_mul import triangle_multiplicative_update

__version__ = "0.1.0"

__all__ = [
    "attn_pair_bias",
    "attention_pair_bias",
    "pairformer",
    "transition",
    "triangle_attn",
    "triangle_mul",
    "triangle_attention",
    "triangle_multiplicative_update",
]
