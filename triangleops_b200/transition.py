"""Pairformer pair transition: x + W3 (silu(LN(x) W1^T) * (LN(x) W2^T)), hidden 4C.

The reference ships the triangle primitives only; a Pairformer block also needs this
transition MLP after the four triangle updates (the AlphaFold-3 transition layer:
LayerNorm, two bias-free linears to 4C combined by SwiGLU, a bias-free linear back
to C). Same calling pattern as the triangle ops: ``precompute`` once (the LN affine
folded into W1 and W2, the weights interleaved per 64-wide hidden chunk for the
kernel), ``forward`` per call, ``transition`` one-shot. One fused sm_100a kernel per
call (LayerNorm, both GEMMs, SwiGLU and the residual add; the 4C-wide hidden
activation never leaves the SM). C = 128, bf16 or fp16 IO.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_lib.register("tops_transition_forward", [_I, _I64, _I64, _P, _P, _P, _P, _F, _P, _P])

CHUNK = 64


def precompute(norm_weight, norm_bias, w1, w2, w3):
    """norm_weight/norm_bias (C,), w1/w2 (nC, C), w3 (C, nC) (nn.Linear layouts).
    Returns the opaque dict for :func:`forward`."""
    NH, C = w1.shape
    assert C == 128 and NH == 4 * C, "the transition kernel takes C = 128 with hidden width 4C"
    assert w2.shape == (NH, C) and w3.shape == (C, NH)
    io = w1.dtype
    g = norm_weight.float()
    b = norm_bias.float()
    W1, W2 = w1.float(), w2.float()
    # per hidden chunk h: rows W1[h]*gamma then W2[h]*gamma; biases W1[h] beta | W2[h] beta
    w12 = torch.stack([(W1 * g).view(NH // CHUNK, CHUNK, C), (W2 * g).view(NH // CHUNK, CHUNK, C)], 1)
    b12 = torch.stack([torch.mv(W1, b).view(NH // CHUNK, CHUNK), torch.mv(W2, b).view(NH // CHUNK, CHUNK)], 1)
    return {"w12": w12.reshape(2 * NH, C).to(io).contiguous(), "b12": b12.reshape(NH // CHUNK, 2 * CHUNK).contiguous(),
            "w3": w3.to(io).contiguous(), "C": C}


def forward(x, pre, *, eps=1e-5, out=None):
    """x (..., C) contiguous -> x + transition(x) (a new tensor, or ``out``; ``out=x``
    updates x in place)."""
    _lib.require_cuda(x)
    C = x.shape[-1]
    assert C == pre["C"] and x.is_contiguous(), "x must be contiguous (..., C)"
    dt = _lib.dtype_code(x.dtype)
    if dt == _lib.F32:
        raise ValueError("the transition takes bf16 or fp16 IO")
    M = x.numel() // C
    if out is None:
        out = torch.empty_like(x)
    assert out.is_contiguous() and out.shape == x.shape and out.dtype == x.dtype
    w12 = pre["w12"] if pre["w12"].dtype == x.dtype else pre["w12"].to(x.dtype)
    w3 = pre["w3"] if pre["w3"].dtype == x.dtype else pre["w3"].to(x.dtype)
    _lib.call("tops_transition_forward", dt, M, C, x.data_ptr(), w12.data_ptr(), w3.data_ptr(), pre["b12"].data_ptr(),
              float(eps), out.data_ptr(), _lib.stream_ptr(x.device))
    return out


def transition(x, norm_weight, norm_bias, w1, w2, w3, eps=1e-5):
    """One-shot (precompute included)."""
    return forward(x, precompute(norm_weight, norm_bias, w1, w2, w3), eps=eps)
