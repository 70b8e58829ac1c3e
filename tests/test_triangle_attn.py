"""Triangle attention parity vs the CPU oracle (case matrix of the reference's
tests/test_triangle_attn.py: N in {128, 130, 256}, masked, general affine, D=16)."""
import math

import pytest
import torch

from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu


def _inputs(N, H, D, Cin, dtype, device, general=False, masked=False):
    X = rnd(N, N, Cin, dtype=dtype, device=device, seed=1)
    if general:
        W_ln = 1.0 + rnd(Cin, dtype=dtype, device=device, sd=0.2, seed=21)
        B_ln = rnd(Cin, dtype=dtype, device=device, sd=0.1, seed=22)
        B_pz = rnd(H, dtype=dtype, device=device, sd=0.1, seed=23)
    else:
        W_ln = torch.ones(Cin, device=device, dtype=dtype)
        B_ln = torch.zeros(Cin, device=device, dtype=dtype)
        B_pz = torch.zeros(H, device=device, dtype=dtype)
    WQ, WK, WV = (rnd(Cin, H * D, dtype=dtype, device=device, sd=Cin**-0.5, seed=s) for s in (3, 4, 5))
    W_pz = rnd(Cin, H, dtype=dtype, device=device, sd=Cin**-0.5, seed=6)
    W_pg = rnd(Cin, H * D, dtype=dtype, device=device, sd=Cin**-0.5, seed=7)
    W_po = rnd(Cin, H * D, dtype=dtype, device=device, sd=(H * D) ** -0.5, seed=8)
    mask = None
    if masked:
        g = torch.Generator().manual_seed(N)
        mask = (torch.rand(N, N, generator=g) > 0.2).to(device)
    return (X, W_ln, B_ln, WQ, WK, WV, W_pz, B_pz, W_pg, None, W_po, None, H, D), mask


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N", [128, 130, 256])
@pytest.mark.parametrize("masked", [False, True])
def test_matches_oracle(device, dtype, N, masked):
    args, mask = _inputs(N, 4, 32, 128, dtype, device, masked=masked)
    scale = 1.0 / math.sqrt(32)
    out = tops.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask)
    ref = oracle.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask)
    rio = oracle.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask, io_round=dtype)
    assert_parity(out, ref, dtype, f"N={N} masked={masked}", ref_io=rio)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("masked", [False, True])
def test_general_affine(device, dtype, masked):
    args, mask = _inputs(256, 4, 32, 128, dtype, device, general=True, masked=masked)
    scale = 1.0 / math.sqrt(32)
    out = tops.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask)
    ref = oracle.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask)
    rio = oracle.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask, io_round=dtype)
    assert_parity(out, ref, dtype, f"general masked={masked}", ref_io=rio)


@pytest.mark.parametrize("masked", [False, True])
def test_apo_d16(device, masked):
    """K-Fold Apo shape: N=33, H=4, D=16, C=64."""
    args, mask = _inputs(33, 4, 16, 64, torch.bfloat16, device, general=True, masked=masked)
    out = tops.triangle_attention(*args, scale=0.25, eps=1e-5, mask=mask)
    ref = oracle.triangle_attention(*args, scale=0.25, eps=1e-5, mask=mask)
    assert_parity(out, ref, torch.bfloat16, f"apo masked={masked}")


def test_fully_masked_row(device):
    args, mask = _inputs(130, 4, 32, 128, torch.bfloat16, device, masked=True)
    mask[7] = False
    mask[129] = False
    out = tops.triangle_attention(*args, scale=32**-0.5, eps=1e-5, mask=mask)
    ref = oracle.triangle_attention(*args, scale=32**-0.5, eps=1e-5, mask=mask)
    assert_parity(out, ref, torch.bfloat16, "fully masked rows")


def test_precompute_forward_matches_oneshot(device):
    args, mask = _inputs(128, 4, 32, 128, torch.bfloat16, device, masked=True)
    (X, W_ln, B_ln, WQ, WK, WV, W_pz, B_pz, W_pg, _, W_po, _, H, D) = args
    pre = tops.triangle_attn.precompute(W_ln, B_ln, WQ, WK, WV, W_pz, B_pz, H, D)
    a = tops.triangle_attn.forward(X, pre, mask=mask, scale=0.2, W_proj_g=W_pg, B_proj_g=None, W_proj_o=W_po,
                                   B_proj_o=None)
    b = tops.triangle_attention(*args, scale=0.2, mask=mask)
    assert torch.equal(a, b)


def test_lowlevel_triangle_attn_forward(device):
    """x~ given (no LN inside), reference kernel.py signature with caller-owned out."""
    args, mask = _inputs(130, 4, 32, 128, torch.bfloat16, device, masked=True)
    (X, W_ln, B_ln, WQ, WK, WV, W_pz, B_pz, W_pg, _, W_po, _, H, D) = args
    pre = tops.triangle_attn.precompute(W_ln, B_ln, WQ, WK, WV, W_pz, B_pz, H, D)
    X_ln = torch.nn.functional.layer_norm(X, (128,), W_ln, B_ln, 1e-5)
    out = torch.empty(130, 130, H * D, device=device, dtype=X.dtype)
    tops.triangle_attn.triangle_attn_forward(X_ln, pre["WQ_c"], pre["WKV_c"], pre["WZ_c"], pre["BZ"], out,
                                             scale=0.2, mask=mask)
    o = tops.triangle_attn.fused_gate_forward(out.view(130, 130, H, D), X_ln, W_pg, W_po)
    ref = oracle.triangle_attention(*args, scale=0.2, mask=mask)
    assert_parity(o, ref, torch.bfloat16, "low-level")


def test_host_pipeline_matches_forward(device):
    """HostPipeline (pinned host tensors, slab-streamed copies, calls overlapping) gives the
    device forward's result, including a fully masked row, over back-to-back calls."""
    N, H, D, C = 256, 4, 32, 128
    args, mask = _inputs(N, H, D, C, torch.bfloat16, device, general=True, masked=True)
    (X, W_ln, B_ln, WQ, WK, WV, W_pz, B_pz, W_pg, _, W_po, _, H, D) = args
    mask[5] = False
    pre = tops.triangle_attn.precompute(W_ln, B_ln, WQ, WK, WV, W_pz, B_pz, H, D)
    kw = dict(scale=D**-0.5, W_proj_g=W_pg, W_proj_o=W_po)
    pipe = tops.triangle_attn.HostPipeline(pre, slabs=4, **kw)
    X2 = rnd(N, N, C, dtype=torch.bfloat16, device=device, seed=77)
    outs = []
    for Xi in (X, X2, X):
        outs.append(pipe(Xi.cpu().pin_memory(), mask.cpu().pin_memory()))
    pipe.wait()
    torch.cuda.synchronize()
    for Xi, o in zip((X, X2, X), outs):
        ref = tops.triangle_attn.forward(Xi, pre, mask=mask, B_proj_g=None, B_proj_o=None, **kw)
        assert torch.equal(o, ref.cpu()), (o.float() - ref.cpu().float()).abs().max()
