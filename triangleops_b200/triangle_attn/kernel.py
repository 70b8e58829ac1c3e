"""Low-level triangle-attention launchers over the C-ABI (replaces the reference's
Triton ``triangle_ops/triangle_attn/kernel.py``).

``triangle_attn_forward`` keeps the reference signature (``kernel.py:256-374``):
it takes the pre-normalised x~ = LN(x) and writes the attention output into the
caller's ``out`` (N, N, H*D). ``fused_gate_forward`` keeps ``kernel.py:438-470``.
``triangle_attn_fused_forward`` is the path ``module.forward`` uses: LN is fused
into the projection kernel and x~ is produced as a by-product for the gate.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib
from .._common.layouts import deinterleave_kv, qkv_rows

_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_lib.register("tops_triangle_attn_forward",
              [_I, _I64, _I64, _I64, _I64, _P, _I, _P, _P, _P, _P, _P, _F, _F, _P, _P, _P, _P, _P, _P, _P, _P])
_lib.register("tops_fused_gate_forward", [_I, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P])
_lib.register("tops_fused_gate_residual", [_I, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _P])


def _mask_u8(mask, shape):
    """Reference semantics: the mask is cast to int8 and compared with 0
    (``triangle_attn/kernel.py:326``, ``:235``)."""
    if mask is None:
        return None
    m = mask.reshape(shape)
    if m.dtype != torch.bool:
        m = m.to(torch.int8) != 0
    return m.to(torch.uint8).contiguous()


def _workspaces(N, C, H, D, dtype, device, Bias_buf=None):
    nkp = (N + 7) // 8 * 8
    q = torch.empty(N, H, N, D, dtype=torch.float16, device=device)
    k = torch.empty(N, H, N, D, dtype=torch.float16, device=device)
    vt = torch.empty(N, H, D, nkp, dtype=torch.float16, device=device)
    pen = torch.empty(N, nkp, dtype=torch.float16, device=device)  # key penalty (0 / -inf), masked calls
    # the shared bias is kept in f16, pre-scaled by log2(e) (the attention kernel works in log2 units)
    if Bias_buf is not None and nkp == N and Bias_buf.is_contiguous() and Bias_buf.shape == (H, N, N) \
            and Bias_buf.dtype == torch.float16:
        bias = Bias_buf
    else:
        bias = torch.empty(H, N, nkp, dtype=torch.float16, device=device)
    return q, k, vt, pen, bias


def triangle_attn_fused_forward(X, w_qkvz, ln_w, ln_b, bz, H, D, *, mask=None, scale=1.0, eps=1e-5, out=None,
                                xln_out=None):
    """LN(x) fused into the projection; returns (O (N,N,H*D), x~ (N,N,C))."""
    _lib.require_cuda(X, w_qkvz)
    dt = _lib.dtype_code(X.dtype)
    N, N2, C = X.shape
    assert N == N2, "X must be (N, N, C)"
    X = X.contiguous()
    if out is None:
        out = torch.empty(N, N, H * D, dtype=X.dtype, device=X.device)
    if xln_out is None:
        xln_out = torch.empty(N, N, C, dtype=X.dtype, device=X.device)
    q, k, vt, pen, bias = _workspaces(N, C, H, D, X.dtype, X.device)
    m = _mask_u8(mask, (N, N))
    _lib.call("tops_triangle_attn_forward", dt, N, C, H, D, X.data_ptr(), 1, ln_w.data_ptr(), ln_b.data_ptr(),
              w_qkvz.data_ptr(), bz.data_ptr(), _lib.ptr(m), float(scale), float(eps), xln_out.data_ptr(),
              q.data_ptr(), k.data_ptr(), vt.data_ptr(), pen.data_ptr(), bias.data_ptr(), out.data_ptr(),
              _lib.stream_ptr(X.device))
    return out, xln_out


def triangle_attn_forward(X_ln, WQ_c, WKV_c, WZ_c, BZ, out, scale=1.0, mask=None, Bias_buf=None, *, WK_c=None,
                          WV_c=None):
    """Attention on a pre-normalised x~ (N, N, C) into ``out`` (N, N, H*D)."""
    _lib.require_cuda(X_ln, WQ_c, out)
    N, N2, C = X_ln.shape
    assert N == N2
    H = WZ_c.shape[0]
    D = WQ_c.shape[1] // H
    assert WKV_c.shape == (C, 2 * H * D)
    assert out.shape == (N, N, H * D)
    dt = _lib.dtype_code(X_ln.dtype)
    if WK_c is None or WV_c is None:
        WK_c, WV_c = deinterleave_kv(WKV_c, H, D)
    w = qkv_rows(WQ_c.to(X_ln.dtype), WK_c.to(X_ln.dtype), WV_c.to(X_ln.dtype), WZ_c.to(X_ln.dtype))
    bz = BZ.float().contiguous()
    X_ln = X_ln.contiguous()
    dst = out if out.is_contiguous() else torch.empty(N, N, H * D, dtype=X_ln.dtype, device=X_ln.device)
    q, k, vt, pen, bias = _workspaces(N, C, H, D, X_ln.dtype, X_ln.device, Bias_buf)
    m = _mask_u8(mask, (N, N))
    _lib.call("tops_triangle_attn_forward", dt, N, C, H, D, X_ln.data_ptr(), 0, None, None, w.data_ptr(),
              bz.data_ptr(), _lib.ptr(m), float(scale), 1e-5, None, q.data_ptr(), k.data_ptr(), vt.data_ptr(),
              pen.data_ptr(), bias.data_ptr(), dst.data_ptr(), _lib.stream_ptr(X_ln.device))
    if dst is not out:
        out.copy_(dst)
    return out


def gate_forward(o, gin, WG, WO, BG=None, BO=None, out=None, residual=None, trans_n=0):
    """out = (o * sigmoid(gin WG^T + BG)) WO^T + BO over (T, C) token rows.

    ``residual`` (same layout as ``out``, may be ``out`` itself) is added in the
    epilogue. ``trans_n`` = n > 0 writes token t = i*n + k to out row k*n + i, i.e.
    the result of an ending-node (transposed) problem lands in the untransposed
    pair layout."""
    _lib.require_cuda(o, gin, WG, WO)
    dt = _lib.dtype_code(gin.dtype)
    C = gin.shape[-1]
    T = gin.numel() // C
    o2 = o.reshape(T, C)
    if not o2.is_contiguous():
        o2 = o2.contiguous()
    g2 = gin.reshape(T, C).contiguous()
    wg = WG.to(gin.dtype).contiguous()
    wo = WO.to(gin.dtype).contiguous()
    assert wg.shape == (C, C) and wo.shape == (C, C), "gate requires square (C, C) weights"
    bg = None if BG is None else BG.float().contiguous()
    bo = None if BO is None else BO.float().contiguous()
    if out is None:
        out = torch.empty(T, C, dtype=gin.dtype, device=gin.device)
    if residual is None and trans_n == 0:
        _lib.call("tops_fused_gate_forward", dt, T, C, o2.data_ptr(), g2.data_ptr(), wg.data_ptr(), wo.data_ptr(),
                  _lib.ptr(bg), _lib.ptr(bo), out.data_ptr(), _lib.stream_ptr(gin.device))
        return out
    assert out.is_contiguous() and out.numel() == T * C
    assert residual is None or (residual.is_contiguous() and residual.numel() == T * C
                                and residual.dtype == gin.dtype)
    _lib.call("tops_fused_gate_residual", dt, T, C, o2.data_ptr(), g2.data_ptr(), wg.data_ptr(), wo.data_ptr(),
              _lib.ptr(bg), _lib.ptr(bo), _lib.ptr(residual), out.data_ptr(), int(trans_n),
              _lib.stream_ptr(gin.device))
    return out


def fused_gate_forward(o_attn, qx_ln, WG, WO):
    """Triangle wrap-up: (o_attn * sigmoid(qx_ln WG^T)) WO^T -> (N1, N2, C)."""
    N1, N2, H, D = o_attn.shape
    C = H * D
    return gate_forward(o_attn.reshape(N1, N2, C), qx_ln, WG, WO).view(N1, N2, C)


_lib.register("tops_triangle_attn_project",
              [_I, _I64, _I64, _I64, _I64, _I64, _P, _I, _P, _P, _P, _P, _P, _F, _F, _P, _P, _P, _P, _P, _P, _P])
_lib.register("tops_triangle_attn_project_transposed",
              [_I, _I64, _I64, _I64, _I64, _I64, _P, _I, _P, _P, _P, _P, _P, _F, _F, _P, _P, _P, _P, _P, _P, _P])
_lib.register("tops_triangle_attn_attend", [_I, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P])


def is_transposed_rows(X_rows):
    """True for rows of the transposed view of a contiguous square (N, N, C) pair
    tensor: strides (C, N*C, 1) with more than one row."""
    R, N, C = X_rows.shape
    return R > 1 and N > 1 and X_rows.stride() == (C, N * C, 1)


def project_rows(X_rows, w_qkvz, ln_w, ln_b, bz, H, D, *, N, mask_rows=None, scale=1.0, eps=1e-5):
    """LN + Q/K/V/bias projection of R pair rows X_rows (R, N, C).

    Returns dict(q, k, vt, pen, bias, xln): bias holds this slab's rows of the
    shared bias, (H, R, Np) f16 in log2 units; the others are row-local attention
    operands (vt f16; pen, the f16 key penalty 0 / -inf, or None without a mask). X_rows may be rows of a transposed view
    (``X.transpose(0, 1)[r0:r1]`` of a contiguous square X, the ending node): the
    projection then reads X column-wise through a 3-D tensor map, without a copy."""
    _lib.require_cuda(X_rows)
    R, N2, C = X_rows.shape
    assert N2 == N
    if is_transposed_rows(X_rows) and N % 8 == 0:
        entry = "tops_triangle_attn_project_transposed"
    else:
        entry = "tops_triangle_attn_project"
        X_rows = X_rows.contiguous()
    dt = _lib.dtype_code(X_rows.dtype)
    nkp = (N + 7) // 8 * 8
    dev, dty = X_rows.device, X_rows.dtype
    ws = dict(q=torch.empty(R, H, N, D, dtype=torch.float16, device=dev),
              k=torch.empty(R, H, N, D, dtype=torch.float16, device=dev),
              vt=torch.empty(R, H, D, nkp, dtype=torch.float16, device=dev),
              pen=None if mask_rows is None else torch.empty(R, nkp, dtype=torch.float16, device=dev),
              bias=torch.empty(H, R, nkp, dtype=torch.float16, device=dev),
              xln=torch.empty(R, N, C, dtype=dty, device=dev))
    m = _mask_u8(mask_rows, (R, N))
    _lib.call(entry, dt, R, N, C, H, D, X_rows.data_ptr(), 1, ln_w.data_ptr(),
              ln_b.data_ptr(), w_qkvz.data_ptr(), bz.data_ptr(), _lib.ptr(m), float(scale), float(eps),
              ws["xln"].data_ptr(), ws["q"].data_ptr(), ws["k"].data_ptr(), ws["vt"].data_ptr(),
              _lib.ptr(ws["pen"]), ws["bias"].data_ptr(), _lib.stream_ptr(dev))
    return ws


def attend_rows(ws, bias_full, H, D, out=None):
    """Flash attention of the R projected rows in ``ws`` against the full shared bias
    (H, N, Np) -> O (R, N, H*D)."""
    R, _, N, _ = ws["q"].shape
    io = ws["xln"].dtype  # Q/K/V^T workspaces are f16; the output is in the IO dtype
    dt = _lib.dtype_code(io)
    if out is None:
        out = torch.empty(R, N, H * D, dtype=io, device=ws["q"].device)
    _lib.call("tops_triangle_attn_attend", dt, R, N, H, D, ws["q"].data_ptr(), ws["k"].data_ptr(),
              ws["vt"].data_ptr(), _lib.ptr(ws["pen"]), bias_full.data_ptr(), out.data_ptr(),
              _lib.stream_ptr(out.device))
    return out
