"""Low-level attention-with-pair-bias launcher over the C-ABI (replaces the
reference's Triton ``triangle_ops/attn_pair_bias/kernel.py``).

``apb_forward`` keeps the reference signature (``kernel.py:205-257``): it writes the
pre-gate attention output into the caller's ``Og`` (M, H*D). Internally:
[LN(z) + bias projection, z read once for all heads] -> [Q/K/V projection] ->
[flash attention]. ``key_mask`` (optional, (M,) bool) is an extension used by the
masked configuration; ``None`` is the reference behaviour (no mask).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib

_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_lib.register("tops_apb_forward",
              [_I, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _F, _F, _P, _P, _P, _P, _P, _P, _P])
_lib.register("tops_apb_forward_rows",
              [_I, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _F, _F, _P, _P, _P, _P, _P,
               _P, _P])


def qkv_rows_from_interleaved(W_QKV, H, D):
    """(C, 3*H*D) per-head [Q_h | K_h | V_h] -> K-major rows [WQ^T; WK^T; WV^T] (3*H*D, C)."""
    C = W_QKV.shape[0]
    w = W_QKV.reshape(C, H, 3, D)
    return torch.cat([w[:, :, i, :].reshape(C, H * D).t() for i in range(3)], 0).contiguous()


def apb_core(X, w_rows, Z, W_combined, sum_W_combined, B_const, Og, H, D, *, scale=1.0, eps=1e-5, key_mask=None,
             q0=0):
    """Pre-gate attention output of query rows [q0, q0 + Z.shape[0]) into ``Og``
    (Z.shape[0], H*D). X (M, C) holds every token (keys and values need all of
    them); Z holds the pair rows of those queries, (Mq, M, C_z)."""
    _lib.require_cuda(X, Z, Og)
    M, C = X.shape
    Mq = Z.shape[0]
    assert Z.shape == (Mq, M, Z.shape[-1])
    assert 0 <= q0 and q0 + Mq <= M
    assert W_combined.shape == (H, Z.shape[-1])
    assert B_const.shape == (H,)
    assert Og.shape == (Mq, H * D)
    dt = _lib.dtype_code(X.dtype)
    mkp = (M + 7) // 8 * 8
    dev = X.device
    q = torch.empty(1, H, M, D, dtype=torch.float16, device=dev)
    k = torch.empty(1, H, M, D, dtype=torch.float16, device=dev)
    vt = torch.empty(1, H, D, mkp, dtype=torch.float16, device=dev)
    pen = torch.empty(1, mkp, dtype=torch.float16, device=dev) if key_mask is not None else None
    bias = torch.empty(H, Mq, mkp, dtype=torch.float16, device=dev)  # logits in log2 units
    km = None
    if key_mask is not None:
        km = key_mask.reshape(M)
        if km.dtype != torch.bool:
            km = km != 0
        km = km.to(torch.uint8).contiguous()
    X = X.contiguous()
    Z = Z.contiguous()
    wc = W_combined.float().contiguous()
    sw = sum_W_combined.float().contiguous()
    bc = B_const.float().contiguous()
    dst = Og if Og.is_contiguous() else torch.empty(Mq, H * D, dtype=X.dtype, device=dev)
    _lib.call("tops_apb_forward_rows", dt, M, q0, Mq, C, Z.shape[-1], H, D, X.data_ptr(), w_rows.data_ptr(),
              Z.data_ptr(), wc.data_ptr(), sw.data_ptr(), bc.data_ptr(), _lib.ptr(km), float(scale), float(eps), q.data_ptr(),
              k.data_ptr(), vt.data_ptr(), _lib.ptr(pen), bias.data_ptr(), dst.data_ptr(), _lib.stream_ptr(dev))
    if dst is not Og:
        Og.copy_(dst)
    return Og


def apb_forward(X, W_QKV, Z, W_combined, sum_W_combined, B_const, Og, scale=1.0, eps=1e-5, key_mask=None):
    """Pre-gate attention output into ``Og`` (M, H*D).

    X (M, C); W_QKV (C, 3*H*D) per-head interleaved; Z (M, M, C_z) raw;
    W_combined (H, C_z) fp32 LN-folded bias weight; sum_W_combined, B_const (H,) fp32."""
    H = sum_W_combined.shape[0]
    D = W_QKV.shape[1] // (3 * H)
    assert W_QKV.shape == (X.shape[1], 3 * H * D)
    w_rows = qkv_rows_from_interleaved(W_QKV.to(X.dtype), H, D)
    return apb_core(X, w_rows, Z, W_combined, sum_W_combined, B_const, Og, H, D, scale=scale, eps=eps,
                    key_mask=key_mask)
