"""Public API of the triangle multiplicative update (``triangle_ops/triangle_mul/module.py``).

LN_in / LN_out affines are folded into all four projections at ``precompute``
(``module.py:17-52``; note g_out absorbs LN_in because it gates on LN_in(x)).
Per call: [LN_in + gated input projection] -> [triangular contraction] ->
[LN_out + gated output projection], three sm_100a kernels behind one C-ABI call.
x is (B, L, L, C) with C == hidden (the reference's single-constexpr constraint).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _f32
from .._common.ln_absorption import absorb_ln
from .kernel import direction_code, fused_forward


def precompute(norm_in_weight, norm_in_bias, p_in_weight, g_in_weight, norm_out_weight, norm_out_bias,
               p_out_weight, g_out_weight):
    """One-time fusion of LN affines into the projections. Weights are (out, in):
    p_in, g_in (2D, C); p_out (C, D); g_out (C, C)."""
    wd = p_in_weight.dtype
    p_in_c, sWp_in, Bp_in = absorb_ln(p_in_weight, norm_in_weight, norm_in_bias, weight_dtype=wd)
    g_in_c, sWg_in, Bg_in = absorb_ln(g_in_weight, norm_in_weight, norm_in_bias, weight_dtype=wd)
    p_out_c, sWp_out, Bp_out = absorb_ln(p_out_weight, norm_out_weight, norm_out_bias, weight_dtype=wd)
    g_out_c, sWg_out, Bg_out = absorb_ln(g_out_weight, norm_in_weight, norm_in_bias, weight_dtype=wd)
    return {
        # reference keys
        "p_in_combined": p_in_c,
        "g_in_combined": g_in_c,
        "p_out_combined": p_out_c,
        "g_out_combined": g_out_c,
        "sum_W_p_in": sWp_in,
        "sum_W_g_in": sWg_in,
        "sum_W_p_out": sWp_out,
        "sum_W_g_out": sWg_out,
        "B_p_in_const": Bp_in,
        "B_g_in_const": Bg_in,
        "B_p_out_const": Bp_out,
        "B_g_out_const": Bg_out,
        # B200 kernel operands (stacked K-major weights, fp32 folds)
        "w_in": torch.cat([p_in_c, g_in_c], 0).contiguous(),
        "sum_in": torch.cat([sWp_in, sWg_in]).contiguous(),
        "b_in": torch.cat([Bp_in, Bg_in]).contiguous(),
        "w_out": torch.cat([p_out_c, g_out_c], 0).contiguous(),
        "sum_out": torch.cat([sWp_out, sWg_out]).contiguous(),
        "b_out": torch.cat([Bp_out, Bg_out]).contiguous(),
        # fp32 IO path: the unfolded weights
        "f32": {"norm_in_weight": norm_in_weight, "norm_in_bias": norm_in_bias, "p_in_weight": p_in_weight,
                "g_in_weight": g_in_weight, "norm_out_weight": norm_out_weight, "norm_out_bias": norm_out_bias,
                "p_out_weight": p_out_weight, "g_out_weight": g_out_weight},
    }


def forward(x, pre, *, direction, mask=None, eps=1e-5):
    """Per-call forward (``module.py:55-88``). x (B, L, L, C) -> (B, L, L, C)."""
    direction_code(direction)  # ValueError on an unknown direction, before any launch
    B, L, _, C = x.shape
    if x.dtype == torch.float32:
        return _f32.triangle_multiplicative_update(x, pre["f32"], direction, mask, eps)
    if C not in (64, 128):
        # the tcgen05 kernels are built for C = 64 and 128; other widths run on the
        # CUDA-core fp32 kernels and round back once
        return _f32.triangle_multiplicative_update(x.float(), pre["f32"], direction, mask, eps).to(x.dtype)
    Lp = (L + 7) // 8 * 8
    if Lp == L:
        return fused_forward(x, pre, direction, mask=mask, eps=eps)
    # TMA row strides must be 16-byte multiples: pad the pair dims to a multiple of 8
    # with masked (zero-contribution) positions and slice the result back.
    xp = F.pad(x, (0, 0, 0, Lp - L, 0, Lp - L))
    if mask is None:
        mp = torch.zeros(B, Lp, Lp, dtype=torch.int8, device=x.device)
        mp[:, :L, :L] = 1
    else:
        mp = F.pad(mask.reshape(B, L, L).to(torch.int8), (0, Lp - L, 0, Lp - L), value=0)
    out = fused_forward(xp, pre, direction, mask=mp, eps=eps)
    return out[:, :L, :L].contiguous()


def triangle_multiplicative_update(x, *, direction, mask=None, eps=1e-5, norm_in_weight, norm_in_bias, p_in_weight,
                                   g_in_weight, norm_out_weight, norm_out_bias, p_out_weight, g_out_weight):
    """One-shot (precompute included), ``module.py:91-118``."""
    pre = precompute(norm_in_weight, norm_in_bias, p_in_weight, g_in_weight, norm_out_weight, norm_out_bias,
                     p_out_weight, g_out_weight)
    return forward(x, pre, direction=direction, mask=mask, eps=eps)
