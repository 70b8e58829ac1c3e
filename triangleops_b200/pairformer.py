"""The pair-update chain of a Pairformer block, on one GPU, in place:

    x += triangle_multiplicative_update(x, "outgoing")
    x += triangle_multiplicative_update(x, "incoming")
    x += triangle_attention(x)                       (starting node)
    x += triangle_attention(x^T)^T                   (ending node)

    x += transition(x)                               (optional stage "transition")

The reference ships the three primitives, not the block; this is the glue a
Pairformer trunk puts around them (AlphaFold-3-style ordering). The pair transition
(:mod:`triangleops_b200.transition`) runs as a fifth stage when its weights are
given; the single-representation update is not part of the pair path.
Every residual add is fused into the epilogue of the op's last kernel (the
triangle-mul output phase, the gate), which writes x in place. The ending node
reads x column-wise through a 3-D tensor map (no transposed copy) and its gate
writes each result token back to its untransposed position; its mask is mask^T.
"""

from __future__ import annotations

import torch

from .triangle_attn import module as _ta
from .triangle_attn.kernel import attend_rows, gate_forward, project_rows
from .triangle_mul import module as _tm
from .triangle_mul.kernel import residual_update
from . import transition as _tr


def precompute(tri_mul_out, tri_mul_in, tri_attn_start, tri_attn_end, transition=None):
    """Weights of the four ops. ``tri_mul_*``: dicts of the eight
    ``triangle_mul.precompute`` arguments; ``tri_attn_*``: dicts with the
    ``triangle_attn.precompute`` arguments (W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z,
    H, D) plus W_proj_g and W_proj_o; ``transition`` (optional): a dict of the
    ``transition.precompute`` arguments (norm_weight, norm_bias, w1, w2, w3)."""
    keys_tm = ("norm_in_weight", "norm_in_bias", "p_in_weight", "g_in_weight", "norm_out_weight", "norm_out_bias",
               "p_out_weight", "g_out_weight")
    keys_ta = ("W_ln", "B_ln", "WQ", "WK", "WV", "W_proj_z", "B_proj_z", "H", "D")
    out = {}
    for name, w in (("tri_mul_out", tri_mul_out), ("tri_mul_in", tri_mul_in)):
        out[name] = _tm.precompute(*[w[k] for k in keys_tm])
    for name, w in (("tri_attn_start", tri_attn_start), ("tri_attn_end", tri_attn_end)):
        pre = _ta.precompute(*[w[k] for k in keys_ta])
        pre["W_proj_g"] = w["W_proj_g"]
        pre["W_proj_o"] = w["W_proj_o"]
        out[name] = pre
    if transition is not None:
        out["transition"] = _tr.precompute(**transition)
    return out


def _tri_attn_residual(x, pre, mask, scale, eps, ending):
    N = x.shape[0]
    H, D = pre["H"], pre["D"]
    w = pre["W_qkvz"] if pre["W_qkvz"].dtype == x.dtype else pre["W_qkvz"].to(x.dtype)
    src = x.transpose(0, 1) if ending else x
    m = None if mask is None else (mask.t() if ending else mask)
    ws = project_rows(src, w, pre["ln_w32"], pre["ln_b32"], pre["BZ"], H, D, N=N, mask_rows=m, scale=scale, eps=eps)
    O = attend_rows(ws, ws["bias"], H, D)
    gate_forward(O, ws["xln"], pre["W_proj_g"], pre["W_proj_o"], out=x, residual=x, trans_n=N if ending else 0)
    return x


STAGES = ("tri_mul_out", "tri_mul_in", "tri_attn_start", "tri_attn_end")
ALL_STAGES = STAGES + ("transition",)


def pair_update(x, pre, *, mask=None, scale=None, eps=1e-5, stages=STAGES):
    """One pass of the chain over the pair tensor x (N, N, C) or (1, N, N, C),
    contiguous, N % 8 == 0; x is updated in place and returned. ``mask`` (N, N)
    (pair mask; multiplicative in the triangle multiplications, key mask in the
    attentions). ``scale`` defaults to 1/sqrt(D). ``stages`` selects a sub-sequence
    of :data:`STAGES` (in that order)."""
    x4 = x if x.dim() == 4 else x.unsqueeze(0)
    assert x4.shape[0] == 1 and x4.is_contiguous(), "one contiguous pair tensor"
    N = x4.shape[1]
    assert N % 8 == 0, "N must be a multiple of 8"
    assert all(st in ALL_STAGES for st in stages), f"stages must be drawn from {ALL_STAGES}"
    m = None if mask is None else mask.reshape(N, N)
    m3 = None if m is None else m.reshape(1, N, N)
    for name in ALL_STAGES:
        if name not in stages:
            continue
        if name == "transition":
            _tr.forward(x4, pre["transition"], eps=eps, out=x4)
        elif name.startswith("tri_mul"):
            residual_update(x4, pre[name], "outgoing" if name == "tri_mul_out" else "incoming", mask=m3, eps=eps)
        else:
            p = pre[name]
            sc = p["D"] ** -0.5 if scale is None else scale
            _tri_attn_residual(x4[0], p, m, sc, eps, name == "tri_attn_end")
    return x


@torch.no_grad()
def pair_update_unfused(x, pre, *, mask=None, scale=None, eps=1e-5):
    """The same chain through the public per-op API (out-of-place ops, separate
    adds, explicit transposes): the composition a user of the reference writes."""
    x4 = x if x.dim() == 4 else x.unsqueeze(0)
    N = x4.shape[1]
    m = None if mask is None else mask.reshape(N, N)
    m3 = None if m is None else m.reshape(1, N, N)
    x4 = x4 + _tm.forward(x4, pre["tri_mul_out"], direction="outgoing", mask=m3, eps=eps)
    x4 = x4 + _tm.forward(x4, pre["tri_mul_in"], direction="incoming", mask=m3, eps=eps)
    x3 = x4[0]
    for name, ending in (("tri_attn_start", False), ("tri_attn_end", True)):
        p = pre[name]
        sc = p["D"] ** -0.5 if scale is None else scale
        src = x3.transpose(0, 1).contiguous() if ending else x3
        mm = None if m is None else (m.t().contiguous() if ending else m)
        o = _ta.forward(src, p, mask=mm, scale=sc, eps=eps, W_proj_g=p["W_proj_g"], B_proj_g=None,
                        W_proj_o=p["W_proj_o"], B_proj_o=None)
        x3 = x3 + (o.transpose(0, 1) if ending else o)
    return x3.reshape(x.shape)
