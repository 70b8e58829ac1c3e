"""CPU fp32 oracle for the TriangleOps hot path — TEST INFRASTRUCTURE ONLY.

This module is the parity checker. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference legs may import it, and only to
check or to time the reference algorithm on the host; the product path
(``triangleops_b200``) never calls it and has no CPU fallback.

Each function restates, in plain fp32 torch on the CPU, the reference's pure-torch
implementation of one op (youngchan2/TriangleOps ``benchmarks/references.py``):

* :func:`triangle_attention`              <- ``references.py:174-205``
* :func:`triangle_attention_chunked`      <- same formula, applied to blocks of pair rows
* :func:`triangle_multiplicative_update`  <- ``references.py:208-221``
* :func:`attention_pair_bias`             <- ``references.py:143-171``
* :func:`attention_pair_bias_masked`      <- ``references.py:224-277`` with ``b_q=0``, no qk-norm
* :func:`pair_update`                     <- the four triangle ops chained with residual adds
  (out, in, starting, ending = transposed view), composed from
  the functions above
* :func:`transition`                      <- the Pairformer pair transition (no counterpart in
  the reference, which ships only the triangle ops): the published AlphaFold-3 transition
  layer, x + W3 (silu(LN(x) W1^T) * (LN(x) W2^T)), hidden width 4C, no biases

plus the LN-affine fold of ``triangle_ops/_common/ln_absorption.py:28-63``
(:func:`absorb_ln`, :func:`absorb_ln_matmul`).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own functions
(imported from a reference checkout) on seeded inputs and stores inputs and
outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this
module against those fixtures.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _f32(*ts):
    return [None if t is None else t.detach().to("cpu", torch.float32) for t in ts]


# --------------------------------------------------------------------------- #
# LN-affine absorption (triangle_ops/_common/ln_absorption.py)
# --------------------------------------------------------------------------- #
def absorb_ln(weight, w_ln, b_ln):
    """(out,in) weight: Wc = W * w_ln, sumW = rowsum(Wc), Bc = W @ b_ln
    (``_common/ln_absorption.py:28-44``). All fp32."""
    Wf, w, b = _f32(weight, w_ln, b_ln)
    Wc = Wf * w.unsqueeze(0)
    return Wc, Wc.sum(dim=1), Wf @ b


def absorb_ln_matmul(weight, w_ln, b_ln):
    """(in,out) weight: Wc = W * w_ln[:,None], sumW = colsum(Wc), Bc = b_ln @ W
    (``_common/ln_absorption.py:47-63``). All fp32."""
    Wf, w, b = _f32(weight, w_ln, b_ln)
    Wc = Wf * w.unsqueeze(-1)
    return Wc, Wc.sum(dim=0), b @ Wf


# --------------------------------------------------------------------------- #
# triangle attention (references.py:174-205)
# --------------------------------------------------------------------------- #
def triangle_attention(X, W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o,
                       H, D, scale=1.0, eps=1e-5, mask=None, io_round=None):
    """Starting-node triangle attention on a (N, N, C) pair tensor, fp32 CPU.

    LN(x) -> Q/K/V = LN(x) @ W (matmul convention), bias Bp[h,q,k] = LN(x)[q,k] @ W_proj_z + B_proj_z,
    S = (Q*scale) K^T + Bp (+ -1e9 where mask[i,k] is False, ``references.py:200-201``),
    O = softmax(S) V, gate sigma(LN(x) @ W_g^T) (``references.py:203``), then W_o.

    ``io_round`` additionally rounds what the reference stores or casts to the IO
    dtype: LN(x) (``module.py:73``), scaled Q, K, V (``kernel.py:195,219-220``), the bias
    (``kernel.py:96``), O (``kernel.py:250``) and the gated product (``kernel.py:434``).
    """
    (X, W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o) = _f32(
        X, W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o)
    N, _, Cin = X.shape
    r = io_round
    xln = _rt(F.layer_norm(X, (Cin,), W_ln, B_ln, eps=eps), r)
    q = _rt((xln @ WQ) * scale, r).view(N, N, H, D).permute(0, 2, 1, 3)
    k = _rt(xln @ WK, r).view(N, N, H, D).permute(0, 2, 1, 3)
    v = _rt(xln @ WV, r).view(N, N, H, D).permute(0, 2, 1, 3)
    bz = B_proj_z if B_proj_z is not None else torch.zeros(H)
    bp = _rt(xln @ W_proj_z + bz, r).permute(2, 0, 1).unsqueeze(0)
    scores = torch.matmul(q, k.transpose(-1, -2)) + bp
    if mask is not None:
        m = mask.detach().to("cpu").bool()
        scores = scores + torch.where(m[:, None, None, :], 0.0, -1e9)
    o = _rt(torch.matmul(torch.softmax(scores, -1), v).permute(0, 2, 1, 3).reshape(N, N, H * D), r)
    g = torch.sigmoid(F.linear(xln, W_proj_g, B_proj_g)).view(N, N, H, D)
    o = _rt((o.view(N, N, H, D) * g).reshape(N, N, H * D), r)
    return F.linear(o, W_proj_o, B_proj_o)


def triangle_attention_chunked(X, W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o,
                               B_proj_o, H, D, scale=1.0, eps=1e-5, mask=None, rows=None, row_block=16):
    """Same formula as :func:`triangle_attention`, applied to blocks of pair rows so
    that large N fits in host memory (rows are independent given the shared bias).
    ``rows`` optionally restricts the output to a subset of row indices (returned in
    that order), which is how bounded CPU samples of a large workload are taken."""
    (X, W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o) = _f32(
        X, W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o)
    N, _, Cin = X.shape
    xln = F.layer_norm(X, (Cin,), W_ln, B_ln, eps=eps)
    bz = B_proj_z if B_proj_z is not None else torch.zeros(H)
    bp = (xln @ W_proj_z + bz).permute(2, 0, 1).unsqueeze(0)  # (1,H,N,N), shared by every row
    m = None if mask is None else mask.detach().to("cpu").bool()
    row_ids = torch.arange(N) if rows is None else torch.as_tensor(rows)
    outs = []
    for s in range(0, len(row_ids), row_block):
        ids = row_ids[s:s + row_block]
        xr = xln[ids]  # (R, N, C)
        R = xr.shape[0]
        q = (xr @ WQ).view(R, N, H, D).permute(0, 2, 1, 3)
        k = (xr @ WK).view(R, N, H, D).permute(0, 2, 1, 3)
        v = (xr @ WV).view(R, N, H, D).permute(0, 2, 1, 3)
        scores = torch.matmul(q * scale, k.transpose(-1, -2)) + bp
        if m is not None:
            scores = scores + torch.where(m[ids][:, None, None, :], 0.0, -1e9)
        o = torch.matmul(torch.softmax(scores, -1), v).permute(0, 2, 1, 3).reshape(R, N, H * D)
        g = torch.sigmoid(F.linear(xr, W_proj_g, B_proj_g)).view(R, N, H, D)
        o = (o.view(R, N, H, D) * g).reshape(R, N, H * D)
        outs.append(F.linear(o, W_proj_o, B_proj_o))
    return torch.cat(outs, 0)


# --------------------------------------------------------------------------- #
# triangle multiplicative update (references.py:208-221)
# --------------------------------------------------------------------------- #
def _rt(t, io):
    """Round to the IO dtype and back (emulates a store/load in that dtype)."""
    return t if io is None else t.to(io).float()


def triangle_multiplicative_update(x, *, direction, mask=None, eps=1e-5, io_round=None, **w):
    """(B, L, L, C) -> (B, L, L, C), fp32 CPU.

    ``io_round`` (e.g. torch.bfloat16) additionally rounds the two intermediates the
    reference stores in the IO dtype: the gated projection ``ab``
    (``triangle_mul/kernel.py:148-162``) and the einsum output ``y`` (cuBLAS output in
    the IO dtype, ``module.py:71-74``). ``None`` = pure fp32.

    g = (LN_in(x) p_in^T) * sigma(LN_in(x) g_in^T) [* mask] (``references.py:210-214``);
    a, b = chunk(g, 2); outgoing y = einsum(bikd,bjkd->bijd), incoming einsum(bkid,bkjd->bijd);
    out = (LN_out(y) p_out^T) * sigma(LN_in(x) g_out^T) (``references.py:221``).
    """
    if direction not in ("outgoing", "incoming"):
        raise ValueError(f"unknown direction: {direction!r} (expected 'outgoing'/'incoming')")
    (x,) = _f32(x)
    w = {k: _f32(v)[0] for k, v in w.items()}
    C = x.shape[-1]
    xln = F.layer_norm(x, (C,), w["norm_in_weight"], w["norm_in_bias"], eps=eps)
    if io_round is None:
        lin_in = lambda name: F.linear(xln, w[name])  # noqa: E731
    else:
        # the reference folds the LayerNorm affine into each projection and stores the
        # folded weight in the IO dtype (triangle_mul/module.py:34-38,
        # _common/ln_absorption.py:28-63): LN(x) W^T = xhat (W*gamma)^T + W beta
        xhat = F.layer_norm(x, (C,), None, None, eps=eps)
        lin_in = lambda name: _folded_linear(xhat, w[name], w["norm_in_weight"], w["norm_in_bias"], io_round)  # noqa
    g = lin_in("p_in_weight") * lin_in("g_in_weight").sigmoid()
    if mask is not None:
        g = g * mask.detach().to("cpu", torch.float32).unsqueeze(-1)
    g = _rt(g, io_round)
    a, b = torch.chunk(g, 2, dim=-1)
    if direction == "outgoing":
        y = torch.einsum("bikd,bjkd->bijd", a, b)
    else:
        y = torch.einsum("bkid,bkjd->bijd", a, b)
    y = _rt(y, io_round)
    if io_round is None:
        yln = F.layer_norm(y, y.shape[-1:], w["norm_out_weight"], w["norm_out_bias"], eps=eps)
        return F.linear(yln, w["p_out_weight"]) * F.linear(xln, w["g_out_weight"]).sigmoid()
    yhat = F.layer_norm(y, y.shape[-1:], None, None, eps=eps)
    p = _folded_linear(yhat, w["p_out_weight"], w["norm_out_weight"], w["norm_out_bias"], io_round)
    return p * lin_in("g_out_weight").sigmoid()


def _folded_linear(xhat, W, gamma, beta, io):
    """xhat (W*gamma)^T + W beta with the folded weight rounded to ``io`` (the
    reference's absorb_ln with weight_dtype = the IO dtype)."""
    Wc = (W * gamma[None, :]).to(io).float()
    return F.linear(xhat, Wc) + torch.mv(W, beta)


def triangle_multiplicative_update_rows(x, *, direction, rows, mask=None, eps=1e-5, **w):
    """Output rows ``rows`` (pair-row indices i) of :func:`triangle_multiplicative_update`
    for batch 0, computed without materialising the full output — used for bounded
    CPU samples at large L. Same formula as the full function."""
    (x,) = _f32(x)
    w = {k: _f32(v)[0] for k, v in w.items()}
    C = x.shape[-1]
    xln = F.layer_norm(x[0], (C,), w["norm_in_weight"], w["norm_in_bias"], eps=eps)  # (L,L,C)
    g = F.linear(xln, w["p_in_weight"]) * F.linear(xln, w["g_in_weight"]).sigmoid()
    if mask is not None:
        g = g * mask.detach().to("cpu", torch.float32)[0].unsqueeze(-1)
    a, b = torch.chunk(g, 2, dim=-1)
    ids = torch.as_tensor(rows)
    if direction == "outgoing":
        y = torch.einsum("ikd,jkd->ijd", a[ids], b)
    elif direction == "incoming":
        y = torch.einsum("kid,kjd->ijd", a[:, ids], b)
    else:
        raise ValueError(f"unknown direction: {direction!r} (expected 'outgoing'/'incoming')")
    yln = F.layer_norm(y, y.shape[-1:], w["norm_out_weight"], w["norm_out_bias"], eps=eps)
    return F.linear(yln, w["p_out_weight"]) * F.linear(xln[ids], w["g_out_weight"]).sigmoid()


# --------------------------------------------------------------------------- #
# attention with pair bias (references.py:143-171, 224-277)
# --------------------------------------------------------------------------- #
def _apb(X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o, H, D, scale,
         eps, key_mask, io_round):
    (X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o) = _f32(
        X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o)
    r = io_round
    M, _ = X.shape
    Cz = Z.shape[-1]
    q = _rt(X @ WQ, r).view(M, H, D).permute(1, 0, 2)
    k = _rt(X @ WK, r).view(M, H, D).permute(1, 0, 2)
    v = _rt(X @ WV, r).view(M, H, D).permute(1, 0, 2)
    bz = B_proj_z if B_proj_z is not None else torch.zeros(H)
    bp = (F.layer_norm(Z, (Cz,), W_ln, B_ln, eps=eps) @ W_proj_z + bz).permute(2, 0, 1)
    scores = torch.matmul(q, k.transpose(-1, -2)) * scale + bp
    if key_mask is not None:
        scores = scores.masked_fill(~key_mask.detach().to("cpu").bool().reshape(-1)[None, None, :], float("-inf"))
    o = _rt(torch.matmul(torch.softmax(scores, -1), v).permute(1, 0, 2).reshape(M, H * D), r)
    g = _rt(torch.sigmoid(_rt(F.linear(X, W_proj_g, B_proj_g), r)), r)
    return F.linear(_rt(g * o, r), W_proj_o, B_proj_o)


def attention_pair_bias(X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o,
                        H, D, scale=1.0, eps=1e-5, io_round=None):
    """(M, c_s), (M, M, C_z) -> (M, c_s), fp32 CPU (``references.py:143-171``): q, k, v = X W,
    S = (q k^T) * scale + LN(Z) W_proj_z + B_proj_z, softmax, gate sigmoid(X W_g^T + b_g) on raw X.

    ``io_round`` additionally rounds what the reference stores or casts to the IO dtype:
    q, k, v (``attn_pair_bias/kernel.py:116-131``), the attention output Og
    (``kernel.py:197-202``) and the torch gate path of ``module.py:65-66`` (linear output,
    sigmoid, product). The bias logits stay fp32 as in the reference kernel."""
    return _apb(X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o, H, D,
                scale, eps, None, io_round)


def attention_pair_bias_masked(X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, W_proj_o, H, D, *,
                               key_mask=None, scale=1.0, eps=1e-5, B_proj_g=None, B_proj_o=None, io_round=None):
    """Key-masked attention with pair bias (``references.py:224-277`` with b_q = 0 and no
    qk-norm): masked keys get -inf before the softmax (``references.py:273-274``)."""
    return _apb(X, WQ, WK, WV, Z, W_ln, B_ln, W_proj_z, B_proj_z, W_proj_g, B_proj_g, W_proj_o, B_proj_o, H, D,
                scale, eps, key_mask, io_round)


# --------------------------------------------------------------------------- #
# Pairformer pair-update chain (composition of the functions above)
# --------------------------------------------------------------------------- #
def pair_update(x, *, tri_mul_out, tri_mul_in, tri_attn_start, tri_attn_end, mask=None, scale=None, eps=1e-5,
                io_round=None, stages=("tri_mul_out", "tri_mul_in", "tri_attn_start", "tri_attn_end"),
                transition=None):
    """x (N, N, C) -> x + the four triangle updates in order, fp32 CPU:
    x += trimul_out(x); x += trimul_in(x); x += tri_attn(x); x += tri_attn(x^T)^T with
    mask^T (ending node as the transposed view). ``tri_mul_*``: the eight trimul
    weights; ``tri_attn_*``: W_ln, B_ln, WQ, WK, WV, W_proj_z, B_proj_z, W_proj_g,
    W_proj_o, H, D; ``transition``: the weights of the optional fifth stage
    "transition" (:func:`transition`). ``stages`` selects a sub-sequence. ``io_round`` rounds what a chain in the IO dtype stores: each op's
    intermediates (the ops' own ``io_round``), each op's output and x after every add."""
    (x,) = _f32(x)
    r = io_round
    N = x.shape[0]
    m = None if mask is None else mask.detach().to("cpu").reshape(N, N)
    m3 = None if m is None else m.reshape(1, N, N)
    for w, direction, name in ((tri_mul_out, "outgoing", "tri_mul_out"), (tri_mul_in, "incoming", "tri_mul_in")):
        if name not in stages:
            continue
        x = _rt(x + _rt(triangle_multiplicative_update(x[None], direction=direction, mask=m3, eps=eps, io_round=r,
                                                       **w)[0], r), r)
    for w, ending, name in ((tri_attn_start, False, "tri_attn_start"), (tri_attn_end, True, "tri_attn_end")):
        if name not in stages:
            continue
        sc = w["D"] ** -0.5 if scale is None else scale
        src = x.transpose(0, 1) if ending else x
        mm = None if m is None else (m.t() if ending else m)
        o = triangle_attention(src, w["W_ln"], w["B_ln"], w["WQ"], w["WK"], w["WV"], w["W_proj_z"], w["B_proj_z"],
                               w["W_proj_g"], None, w["W_proj_o"], None, w["H"], w["D"], scale=sc, eps=eps, mask=mm,
                               io_round=r)
        x = _rt(x + _rt(o.transpose(0, 1) if ending else o, r), r)
    if "transition" in stages:
        x = _transition_layer(x, eps=eps, io_round=r, **transition)
    return x


# --------------------------------------------------------------------------- #
# Pairformer pair transition (AlphaFold 3 supplementary, Algorithm 11 "Transition")
# --------------------------------------------------------------------------- #
def transition(x, *, norm_weight, norm_bias, w1, w2, w3, eps=1e-5, io_round=None):
    """x (..., C) -> x + transition(x), fp32 CPU: a = LN(x); h = silu(a W1^T) * (a W2^T)
    with W1, W2 (nC, C); out = x + h W3^T with W3 (C, nC). ``io_round`` rounds what a
    16-bit kernel stores: the LN-folded weights (W1*gamma, W2*gamma), the hidden h and
    the output."""
    (x, norm_weight, norm_bias, w1, w2, w3) = _f32(x, norm_weight, norm_bias, w1, w2, w3)
    C = x.shape[-1]
    if io_round is None:
        a = F.layer_norm(x, (C,), norm_weight, norm_bias, eps=eps)
        u, v = F.linear(a, w1), F.linear(a, w2)
    else:
        xhat = _rt(F.layer_norm(x, (C,), None, None, eps=eps), io_round)
        u = _folded_linear(xhat, w1, norm_weight, norm_bias, io_round)
        v = _folded_linear(xhat, w2, norm_weight, norm_bias, io_round)
        w3 = _rt(w3, io_round)
    h = _rt(F.silu(u) * v, io_round)
    return _rt(x + F.linear(h, w3), io_round)


_transition_layer = transition  # pair_update's keyword of the same name holds the weights
