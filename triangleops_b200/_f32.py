"""fp32 IO path of the three ops, composed from the fp32 CUDA-core kernels of
``csrc/f32.cu`` (LayerNorm, strided batched GEMM, attention, gated multiply).

The reference admits fp32 IO (``_common/dtype.py:7-19``); the tensor-core kernels are
16-bit, so fp32 inputs take this path. It follows the reference's pure-torch formulas
(``benchmarks/references.py:143-221``) with every intermediate in fp32.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_lib.register("tops_f32_layernorm", [_I64, _I64, _P, _P, _P, _F, _P, _P])
_lib.register("tops_f32_gemm", [_I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P])
_lib.register("tops_f32_attention",
              [_I64, _I64, _I64, _I64, _I64, _P, _P, _P, _I64, _I64, _I64, _P, _P, _F, _I, _P, _P])
_lib.register("tops_f32_gated_mul", [_I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I64, _P])


def _f(t):
    return None if t is None else t.float().contiguous()


def layernorm(x2, w, b, eps):
    T, C = x2.shape
    y = torch.empty_like(x2)
    w, b = _f(w), _f(b)
    _lib.call("tops_f32_layernorm", T, C, x2.data_ptr(), _lib.ptr(w), _lib.ptr(b), float(eps), y.data_ptr(),
              _lib.stream_ptr(x2.device))
    return y


def gemm(batch, M, N, K, A, B, out, strides, bias=None):
    """out[b, m, n] = sum_k A(b, m, k) B(b, n, k) (+ bias[n]); strides (A b,m,k, B b,n,k, C b,m,n)."""
    st = (ctypes.c_int64 * 9)(*[int(v) for v in strides])
    _lib.call("tops_f32_gemm", batch, M, N, K, A.data_ptr(), B.data_ptr(), _lib.ptr(bias), out.data_ptr(), st,
              _lib.stream_ptr(out.device))
    return out


def linear(x2, W, bias=None):
    """x2 (T, Cin) times W (Cout, Cin)^T (nn.Linear layout) (+ bias)."""
    T, Cin = x2.shape
    Cout = W.shape[0]
    W = _f(W)
    out = torch.empty(T, Cout, device=x2.device, dtype=torch.float32)
    return gemm(1, T, Cout, Cin, x2, W, out, (0, Cin, 1, 0, Cin, 1, 0, Cout, 1), _f(bias))


def matmul(x2, W, bias=None):
    """x2 (T, Cin) @ W (Cin, Cout) (matmul layout) (+ bias)."""
    T, Cin = x2.shape
    Cout = W.shape[1]
    W = _f(W)
    out = torch.empty(T, Cout, device=x2.device, dtype=torch.float32)
    return gemm(1, T, Cout, Cin, x2, W, out, (0, Cin, 1, 0, 1, Cout, 0, Cout, 1), _f(bias))


def gated_mul(a, lda, g, ldg, rows, cols, bg=None, mask=None):
    y = torch.empty(rows, cols, device=a.device, dtype=torch.float32)
    _lib.call("tops_f32_gated_mul", rows, cols, a.data_ptr(), lda, g.data_ptr(), ldg, _lib.ptr(_f(bg)),
              _lib.ptr(mask), y.data_ptr(), cols, _lib.stream_ptr(a.device))
    return y


def attention(q, k, v, R, H, Nq, Nk, D, bias, mask_u8, scale, mask_mode):
    """q/k/v token-major (R, N, H*D) fp32; bias (H, Nq, Nk); returns (R, Nq, H*D)."""
    out = torch.empty(R, Nq, H * D, device=q.device, dtype=torch.float32)
    _lib.call("tops_f32_attention", R, H, Nq, Nk, D, q.data_ptr(), k.data_ptr(), v.data_ptr(), Nq * H * D, D,
              H * D, bias.data_ptr(), _lib.ptr(mask_u8), float(scale), mask_mode, out.data_ptr(),
              _lib.stream_ptr(q.device))
    return out


def triangle_attention(X, W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g, W_proj_o, H, D, scale, eps, mask):
    _lib.require_cuda(X)
    N, _, C = X.shape
    xln = layernorm(X.reshape(N * N, C).contiguous(), W_ln, B_ln, eps)
    q, k, v = matmul(xln, WQ), matmul(xln, WK), matmul(xln, WV)
    bias = torch.empty(H, N, N, device=X.device, dtype=torch.float32)
    bz = torch.zeros(H, device=X.device) if B_proj_z is None else B_proj_z
    # bias[h, q, k] = xln[(q, k)] . W_proj_z[:, h] + bz[h]: C element (t, h) at h*N*N + t
    gemm(1, N * N, H, C, xln, _f(W_proj_z), bias, (0, C, 1, 0, 1, H, 0, 1, N * N), _f(bz))
    m = None if mask is None else (mask.reshape(N, N).to(torch.int8) != 0).to(torch.uint8).contiguous()
    o = attention(q, k, v, N, H, N, N, D, bias, m, scale, 0)
    g = linear(xln, W_proj_g)
    y = gated_mul(o.reshape(N * N, H * D), H * D, g, H * D, N * N, H * D)
    return linear(y, W_proj_o).reshape(N, N, -1)


def triangle_multiplicative_update(x, w, direction, mask, eps):
    _lib.require_cuda(x)
    B, L, _, C = x.shape
    M = B * L * L
    xln = layernorm(x.reshape(M, C).contiguous(), w["norm_in_weight"], w["norm_in_bias"], eps)
    Dh = w["p_in_weight"].shape[0] // 2
    pg = linear(xln, torch.cat([w["p_in_weight"], w["g_in_weight"]], 0))  # (M, 4Dh): p | g
    m = None if mask is None else mask.reshape(M).to(torch.int8).contiguous()
    ab = gated_mul(pg, 4 * Dh, pg[:, 2 * Dh:], 4 * Dh, M, 2 * Dh, mask=m)  # (M, 2Dh): a | b, token-major
    y = torch.empty(M, Dh, device=x.device, dtype=torch.float32)
    W2 = 2 * Dh
    for bb in range(B):
        base = bb * L * L
        a0 = ab[base:]
        b0 = ab[base:, Dh:]
        y0 = y[base:]
        if direction == "outgoing":  # y[i,j,d] = sum_k a[i,k,d] b[j,k,d]
            st = (1, L * W2, W2, 1, L * W2, W2, 1, L * Dh, Dh)
        else:  # y[i,j,d] = sum_k a[k,i,d] b[k,j,d]
            st = (1, W2, L * W2, 1, W2, L * W2, 1, L * Dh, Dh)
        gemm(Dh, L, L, L, a0, b0, y0, st)
    yln = layernorm(y, w["norm_out_weight"], w["norm_out_bias"], eps)
    p = linear(yln, w["p_out_weight"])
    g = linear(xln, w["g_out_weight"])
    return gated_mul(p, C, g, C, M, C).reshape(B, L, L, C)


def attention_pair_bias(X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o, H,
                        D, scale, eps, key_mask):
    _lib.require_cuda(X, Z)
    M, C = X.shape
    Cz = Z.shape[-1]
    zln = layernorm(Z.reshape(M * M, Cz).contiguous(), W_ln, B_ln, eps)
    bias = torch.empty(H, M, M, device=X.device, dtype=torch.float32)
    bz = torch.zeros(H, device=X.device) if B_proj_z is None else B_proj_z
    gemm(1, M * M, H, Cz, zln, _f(W_proj_z), bias, (0, Cz, 1, 0, 1, H, 0, 1, M * M), _f(bz))
    X = X.contiguous()
    q, k, v = matmul(X, WQ), matmul(X, WK), matmul(X, WV)
    km = None if key_mask is None else (key_mask.reshape(M) != 0).to(torch.uint8).contiguous()
    o = attention(q, k, v, 1, H, M, M, D, bias, km, scale, 1)
    g = linear(X, W_proj_g)
    y = gated_mul(o.reshape(M, H * D), H * D, g, H * D, M, H * D, bg=B_proj_g)
    return linear(y, W_proj_o, B_proj_o)
