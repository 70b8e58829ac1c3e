"""Public API of attention with pair bias (``triangle_ops/attn_pair_bias/module.py``).

Per call: [LN(z) + bias projection] -> [Q/K/V projection] -> [flash attention]
-> [gate + W_o] (the reference runs the last step as two torch linears,
``module.py:65-66``; here it is one fused tcgen05 kernel with the biases in its
epilogues). ``mask`` is an optional (M,) key mask — an extension for padded
token sequences; ``None`` keeps the reference behaviour.
"""

from __future__ import annotations

import torch

from .._common.layouts import interleave_qkv, qkv_rows
from .. import _f32
from .._common.ln_absorption import absorb_ln_matmul
from ..triangle_attn.kernel import gate_forward
from .kernel import apb_core


def precompute(WQ, WK, WV, W_ln, B_ln, W_proj_z, B_proj_z, H, D):
    """One-time fusion (``module.py:18-42``): W_QKV interleave, LN(z) folded into the
    bias projection in fp32."""
    W_QKV = interleave_qkv(WQ, WK, WV, H, D)
    W_combined, sum_W_combined, B_const = absorb_ln_matmul(W_proj_z, W_ln, B_ln, weight_dtype=torch.float32)
    W_combined = W_combined.t().contiguous()  # (C_z, H) -> (H, C_z)
    if B_proj_z is not None:
        B_const = B_const + B_proj_z.float()
    return {
        "W_QKV": W_QKV,
        "W_combined": W_combined,
        "sum_W_combined": sum_W_combined,
        "B_const": B_const.contiguous(),
        "w_rows": qkv_rows(WQ, WK, WV),
        "H": H,
        "D": D,
        # fp32 IO path: the unfolded weights
        "f32": (WQ, WK, WV, W_ln, B_ln, W_proj_z, B_proj_z),
    }


def forward(X, Z, pre, *, scale=1.0, eps=1e-5, W_proj_g, B_proj_g, W_proj_o, B_proj_o, mask=None):
    """Per-call forward (``module.py:45-66``). X (M, c_s), Z (M, M, C_z) -> (M, c_s)."""
    M = X.shape[0]
    H, D = pre["H"], pre["D"]
    if X.dtype == torch.float32:
        WQ, WK, WV, W_ln, B_ln, W_pz, B_pz = pre["f32"]
        return _f32.attention_pair_bias(X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_proj_g, B_proj_g, W_proj_o,
                                        B_proj_o, H, D, scale, eps, mask)
    if (X.shape[-1], Z.shape[-1], H, D) != (128, 128, 4, 32):
        # the tcgen05 path is built for c_s = C_z = 128, H = 4, D = 32; other shapes run on
        # the CUDA-core fp32 kernels and round back once
        WQ, WK, WV, W_ln, B_ln, W_pz, B_pz = pre["f32"]
        return _f32.attention_pair_bias(X.float(), WQ, WK, WV, Z.float(), W_ln, B_ln, W_pz, B_pz, W_proj_g, B_proj_g,
                                        W_proj_o, B_proj_o, H, D, scale, eps, mask).to(X.dtype)
    w = pre["w_rows"]
    if w.dtype != X.dtype:
        w = w.to(X.dtype)
    Og = torch.empty(M, H * D, device=X.device, dtype=X.dtype)
    apb_core(X, w, Z, pre["W_combined"], pre["sum_W_combined"], pre["B_const"], Og, H, D, scale=scale, eps=eps,
             key_mask=mask)
    return gate_forward(Og, X, W_proj_g, W_proj_o, B_proj_g, B_proj_o)


def attention_pair_bias(X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o, H,
                        D, scale=1.0, eps=1e-5, mask=None):
    """One-shot (precompute included), ``module.py:69-101``."""
    pre = precompute(WQ, WK, WV, W_ln, B_ln, W_proj_z, B_proj_z, H, D)
    return forward(X, Z, pre, scale=scale, eps=eps, W_proj_g=W_proj_g, B_proj_g=B_proj_g, W_proj_o=W_proj_o,
                   B_proj_o=B_proj_o, mask=mask)
