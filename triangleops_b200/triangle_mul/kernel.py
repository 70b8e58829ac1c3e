"""Low-level triangle-multiplicative-update launchers over the C-ABI (replaces the
reference's Triton ``triangle_ops/triangle_mul/kernel.py`` and its cuBLAS einsum).

``input_phase`` / ``output_phase`` keep the reference signatures
(``kernel.py:235-279``, ``:282-326``); ``contract`` is the triangular einsum of
``module.py:70-76`` as a tcgen05 batched GEMM (one L x L x L GEMM per channel).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib

_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_lib.register("tops_trimul_input_phase", [_I, _I64, _I64, _P, _P, _P, _P, _P, _F, _P, _P])
_lib.register("tops_trimul_contract", [_I, _I, _I64, _I64, _P, _P, _P, _P])
_lib.register("tops_trimul_contract_slab", [_I, _I, _I64, _I64, _I64, _I64, _P, _P, _P, _P])
_lib.register("tops_trimul_contract_slab_cols", [_I, _I, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P])
_lib.register("tops_trimul_output_phase", [_I, _I64, _I64, _P, _P, _P, _P, _P, _F, _P, _P])
_lib.register("tops_trimul_output_phase_residual", [_I, _I64, _I64, _P, _P, _P, _P, _P, _F, _P, _P, _P])
_lib.register("tops_trimul_forward",
              [_I, _I, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _F, _P, _P, _P, _P])

DIRECTIONS = {"outgoing": 0, "incoming": 1}


def direction_code(direction) -> int:
    try:
        return DIRECTIONS[direction]
    except (KeyError, TypeError):
        raise ValueError(f"unknown direction: {direction!r} (expected 'outgoing'/'incoming')") from None


def mask_u8(mask, M):
    """Reference semantics: the mask is cast to int8 (``kernel.py:252``) and that int8
    value multiplies the gated projection (``kernel.py:128,158``); a float mask
    therefore truncates toward zero. The kernel reads the int8 bytes as signed."""
    if mask is None:
        return None
    return mask.reshape(M).to(torch.int8).contiguous()


def input_phase(x, mask, p_in_combined, g_in_combined, sum_W_p_in, sum_W_g_in, B_p_in_const, B_g_in_const, eps,
                out=None):
    """LN_in + p_in * sigmoid(g_in) (+ mask) -> ab (2D, B, L, L), D-major."""
    _lib.require_cuda(x)
    B, L, _, C = x.shape
    D_OUT = p_in_combined.shape[0]
    assert D_OUT == 2 * C and g_in_combined.shape == p_in_combined.shape == (2 * C, C)
    M = B * L * L
    dt = _lib.dtype_code(x.dtype)
    w = torch.cat([p_in_combined, g_in_combined], 0).to(x.dtype).contiguous()
    s = torch.cat([sum_W_p_in, sum_W_g_in]).float().contiguous()
    b = torch.cat([B_p_in_const, B_g_in_const]).float().contiguous()
    xf = x.reshape(M, C).contiguous()
    if out is None:
        out = torch.empty(D_OUT, M, device=x.device, dtype=x.dtype)
    m = mask_u8(mask, M)
    _lib.call("tops_trimul_input_phase", dt, M, C, xf.data_ptr(), _lib.ptr(m), w.data_ptr(), s.data_ptr(),
              b.data_ptr(), float(eps), out.data_ptr(), _lib.stream_ptr(x.device))
    return out.view(D_OUT, B, L, L)


def contract(a, b, direction, out=None):
    """outgoing y[d,b,i,j] = sum_k a[d,b,i,k] b[d,b,j,k]; incoming sum_k a[d,b,k,i] b[d,b,k,j]."""
    code = direction_code(direction)
    _lib.require_cuda(a, b)
    D, B, L, L2 = a.shape
    assert L == L2 and b.shape == a.shape
    dt = _lib.dtype_code(a.dtype)
    a = a.contiguous()
    b = b.contiguous()
    if out is None:
        out = torch.empty(D, B, L, L, device=a.device, dtype=a.dtype)
    _lib.call("tops_trimul_contract", dt, code, D * B, L, a.data_ptr(), b.data_ptr(), out.data_ptr(),
              _lib.stream_ptr(a.device))
    return out


def output_phase(y_t, x, p_out_combined, g_out_combined, sum_W_p_out, sum_W_g_out, B_p_out_const, B_g_out_const,
                 eps, out=None):
    """sigmoid(g_out(LN_in(x))) * p_out(LN_out(y)) -> (B, L, L, C); y is (D, B, L, L) D-major."""
    _lib.require_cuda(x, y_t)
    B, L, _, C = x.shape
    M = B * L * L
    dt = _lib.dtype_code(x.dtype)
    assert p_out_combined.shape[0] == C and g_out_combined.shape == (C, C)
    w = torch.cat([p_out_combined, g_out_combined], 0).to(x.dtype).contiguous()
    s = torch.cat([sum_W_p_out, sum_W_g_out]).float().contiguous()
    b = torch.cat([B_p_out_const, B_g_out_const]).float().contiguous()
    yf = y_t.reshape(C, M).contiguous()
    xf = x.reshape(M, C).contiguous()
    if out is None:
        out = torch.empty(M, C, device=x.device, dtype=x.dtype)
    _lib.call("tops_trimul_output_phase", dt, M, C, yf.data_ptr(), xf.data_ptr(), w.data_ptr(), s.data_ptr(),
              b.data_ptr(), float(eps), out.data_ptr(), _lib.stream_ptr(x.device))
    return out.view(B, L, L, C)


def fused_forward(x, pre, direction, mask=None, eps=1e-5, out=None, ab_ws=None, y_ws=None):
    """All three phases through one C-ABI call (x is (B, L, L, C) with L % 8 == 0)."""
    code = direction_code(direction)
    _lib.require_cuda(x)
    B, L, _, C = x.shape
    M = B * L * L
    dt = _lib.dtype_code(x.dtype)
    x = x.contiguous()
    if ab_ws is None:
        ab_ws = torch.empty(2 * C, M, device=x.device, dtype=x.dtype)
    if y_ws is None:
        y_ws = torch.empty(C, M, device=x.device, dtype=x.dtype)
    if out is None:
        out = torch.empty(B, L, L, C, device=x.device, dtype=x.dtype)
    w_in, w_out = pre["w_in"], pre["w_out"]
    if w_in.dtype != x.dtype:
        w_in, w_out = w_in.to(x.dtype), w_out.to(x.dtype)
    m = mask_u8(mask, M)
    _lib.call("tops_trimul_forward", dt, code, B, L, C, x.data_ptr(), _lib.ptr(m), w_in.data_ptr(),
              pre["sum_in"].data_ptr(), pre["b_in"].data_ptr(), w_out.data_ptr(), pre["sum_out"].data_ptr(),
              pre["b_out"].data_ptr(), float(eps), ab_ws.data_ptr(), y_ws.data_ptr(), out.data_ptr(),
              _lib.stream_ptr(x.device))
    return out


def input_phase_tokens(x_tokens, mask_tokens, pre, eps=1e-5):
    """Input phase over an arbitrary contiguous token set x_tokens (M, C) -> ab (2C, M)."""
    _lib.require_cuda(x_tokens)
    M, C = x_tokens.shape
    dt = _lib.dtype_code(x_tokens.dtype)
    w_in = pre["w_in"] if pre["w_in"].dtype == x_tokens.dtype else pre["w_in"].to(x_tokens.dtype)
    out = torch.empty(2 * C, M, device=x_tokens.device, dtype=x_tokens.dtype)
    m = mask_u8(mask_tokens, M)
    _lib.call("tops_trimul_input_phase", dt, M, C, x_tokens.data_ptr(), _lib.ptr(m), w_in.data_ptr(),
              pre["sum_in"].data_ptr(), pre["b_in"].data_ptr(), float(eps), out.data_ptr(),
              _lib.stream_ptr(x_tokens.device))
    return out


def contract_slab(a, b_chunks, direction, Mi, L, P):
    """Row-slab contraction: a (C, Mi, L) outgoing / (C, L, Mi) incoming; b_chunks the
    all-gathered (P, C, L/P, L) / (P, C, L, L/P). Returns y (C, Mi, L)."""
    code = direction_code(direction)
    C = a.shape[0]
    dt = _lib.dtype_code(a.dtype)
    y = torch.empty(C, Mi, L, device=a.device, dtype=a.dtype)
    a = a.contiguous()
    b_chunks = b_chunks.contiguous()
    _lib.call("tops_trimul_contract_slab", dt, code, C, Mi, L, P, a.data_ptr(), b_chunks.data_ptr(), y.data_ptr(),
              _lib.stream_ptr(a.device))
    return y


def contract_slab_cols(a, b_flat, direction, Mi, L, P, j_begin, j_count, y):
    """Output columns [j_begin, j_begin + j_count) of :func:`contract_slab` into the
    caller's y (C, Mi, L); b_flat is the full (P, C, ...) chunk buffer, of which only
    the chunks covering the range are read."""
    code = direction_code(direction)
    C = a.shape[0]
    dt = _lib.dtype_code(a.dtype)
    assert y.is_contiguous() and y.shape == (C, Mi, L) and a.is_contiguous() and b_flat.is_contiguous()
    _lib.call("tops_trimul_contract_slab_cols", dt, code, C, Mi, L, P, j_begin, j_count, a.data_ptr(),
              b_flat.data_ptr(), y.data_ptr(), _lib.stream_ptr(a.device))
    return y


def output_phase_tokens(y_dmajor, x_tokens, pre, eps=1e-5):
    """Output phase: y (C, M) D-major and x_tokens (M, C) -> (M, C)."""
    M, C = x_tokens.shape
    dt = _lib.dtype_code(x_tokens.dtype)
    w_out = pre["w_out"] if pre["w_out"].dtype == x_tokens.dtype else pre["w_out"].to(x_tokens.dtype)
    out = torch.empty(M, C, device=x_tokens.device, dtype=x_tokens.dtype)
    _lib.call("tops_trimul_output_phase", dt, M, C, y_dmajor.data_ptr(), x_tokens.data_ptr(), w_out.data_ptr(),
              pre["sum_out"].data_ptr(), pre["b_out"].data_ptr(), float(eps), out.data_ptr(),
              _lib.stream_ptr(x_tokens.device))
    return out


def residual_update(x, pre, direction, mask=None, eps=1e-5, ab_ws=None, y_ws=None):
    """x += triangle_multiplicative_update(x), in place (the Pairformer residual
    update): input phase -> contraction -> output phase with the residual added in
    its epilogue. x (B, L, L, C) contiguous, L % 8 == 0."""
    code = direction_code(direction)
    _lib.require_cuda(x)
    assert x.is_contiguous(), "the in-place update needs a contiguous x"
    B, L, _, C = x.shape
    M = B * L * L
    dt = _lib.dtype_code(x.dtype)
    if ab_ws is None:
        ab_ws = torch.empty(2 * C, M, device=x.device, dtype=x.dtype)
    if y_ws is None:
        y_ws = torch.empty(C, M, device=x.device, dtype=x.dtype)
    w_in, w_out = pre["w_in"], pre["w_out"]
    if w_in.dtype != x.dtype:
        w_in, w_out = w_in.to(x.dtype), w_out.to(x.dtype)
    m = mask_u8(mask, M)
    st = _lib.stream_ptr(x.device)
    _lib.call("tops_trimul_input_phase", dt, M, C, x.data_ptr(), _lib.ptr(m), w_in.data_ptr(),
              pre["sum_in"].data_ptr(), pre["b_in"].data_ptr(), float(eps), ab_ws.data_ptr(), st)
    _lib.call("tops_trimul_contract", dt, code, C * B, L, ab_ws.data_ptr(), ab_ws[C:].data_ptr(), y_ws.data_ptr(),
              st)
    _lib.call("tops_trimul_output_phase_residual", dt, M, C, y_ws.data_ptr(), x.data_ptr(), w_out.data_ptr(),
              pre["sum_out"].data_ptr(), pre["b_out"].data_ptr(), float(eps), x.data_ptr(), x.data_ptr(), st)
    return x
