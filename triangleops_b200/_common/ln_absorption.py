"""LayerNorm-affine absorption (``triangle_ops/_common/ln_absorption.py:1-63``).

LN(x)[i] = (x[i]-mean)*rstd*w[i] + b[i], so for a projection W (out, in):

    (LN(x) W^T)[o] = rstd * (sum_i x[i] Wc[o,i] - mean * sumW[o]) + Bc[o]
    Wc[o,i] = w[i] W[o,i],   sumW[o] = sum_i Wc[o,i],   Bc[o] = sum_i b[i] W[o,i]

The kernels then need only the per-token (mean, rstd). ``sumW`` and ``Bc`` are
fp32 (they feed fp32 accumulators); ``Wc`` is cast to ``weight_dtype``
(default: the weight's dtype) so it stays 16-bit for the tensor cores.
"""

import torch


def absorb_ln(weight: torch.Tensor, w_ln: torch.Tensor, b_ln: torch.Tensor, *, weight_dtype=None):
    """(out, in) nn.Linear weight -> Wc (out, in) [weight_dtype], sumW (out,) fp32, Bc (out,) fp32."""
    W = weight.float()
    Wc = W * w_ln.float()[None, :]
    sum_W = Wc.sum(dim=1).contiguous()
    B_const = torch.mv(W, b_ln.float()).contiguous()
    return Wc.to(weight_dtype or weight.dtype).contiguous(), sum_W, B_const


def absorb_ln_matmul(weight: torch.Tensor, w_ln: torch.Tensor, b_ln: torch.Tensor, *, weight_dtype=None):
    """(in, out) matmul weight -> Wc (in, out) [weight_dtype], sumW (out,) fp32, Bc (out,) fp32."""
    W = weight.float()
    Wc = W * w_ln.float()[:, None]
    sum_W = Wc.sum(dim=0).contiguous()
    B_const = torch.mv(W.t(), b_ln.float()).contiguous()
    return Wc.to(weight_dtype or weight.dtype).contiguous(), sum_W, B_const
