"""Pairformer pair-update chain (BASELINE configuration 4's op order): the fused
in-place chain (residual adds in the epilogues, ending node read column-wise) vs
the fp32 oracle composition, vs the same chain through the per-op public API, and
the zero-copy transposed-view input of triangle_attn.forward."""
import math

import pytest
import torch

from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu


def _tm_weights(C, dev, seed):
    r = lambda *s, sd, k: rnd(*s, dtype=torch.bfloat16, device=dev, sd=sd, seed=seed * 100 + k)  # noqa: E731
    return dict(norm_in_weight=1 + r(C, sd=0.1, k=1), norm_in_bias=r(C, sd=0.1, k=2),
                p_in_weight=r(2 * C, C, sd=C**-0.5, k=3), g_in_weight=r(2 * C, C, sd=C**-0.5, k=4),
                norm_out_weight=1 + r(C, sd=0.1, k=5), norm_out_bias=r(C, sd=0.1, k=6),
                p_out_weight=r(C, C, sd=C**-0.5, k=7), g_out_weight=r(C, C, sd=C**-0.5, k=8))


def _ta_weights(C, H, D, dev, seed):
    r = lambda *s, sd, k: rnd(*s, dtype=torch.bfloat16, device=dev, sd=sd, seed=seed * 100 + k)  # noqa: E731
    return dict(W_ln=1 + r(C, sd=0.1, k=1), B_ln=r(C, sd=0.1, k=2), WQ=r(C, H * D, sd=C**-0.5, k=3),
                WK=r(C, H * D, sd=C**-0.5, k=4), WV=r(C, H * D, sd=C**-0.5, k=5), W_proj_z=r(C, H, sd=C**-0.5, k=6),
                B_proj_z=r(H, sd=0.1, k=7), W_proj_g=r(C, C, sd=C**-0.5, k=8), W_proj_o=r(C, C, sd=C**-0.5, k=9),
                H=H, D=D)


def _setup(N, dev, masked):
    C, H, D = 128, 4, 32
    w = dict(tri_mul_out=_tm_weights(C, dev, 10), tri_mul_in=_tm_weights(C, dev, 11),
             tri_attn_start=_ta_weights(C, H, D, dev, 12), tri_attn_end=_ta_weights(C, H, D, dev, 13))
    x = rnd(N, N, C, dtype=torch.bfloat16, device=dev, sd=1.0, seed=4)
    mask = None
    if masked:
        g = torch.Generator().manual_seed(N)
        mask = (torch.rand(N, N, generator=g) > 0.1).to(dev)
    return x, w, mask


@pytest.mark.parametrize("N", [128, 136])
@pytest.mark.parametrize("masked", [False, True])
def test_each_stage_matches_oracle(device, N, masked):
    """Stage by stage: the GPU chain's x before a stage, advanced by that stage on the GPU
    (fused residual, in place) and by the oracle, agree to the per-op bar."""
    x, w, mask = _setup(N, device, masked)
    pre = tops.pairformer.precompute(**w)
    cur = x.clone()
    for st in tops.pairformer.STAGES:
        ref = oracle.pair_update(cur, mask=mask, stages=(st,), **w)
        rio = oracle.pair_update(cur, mask=mask, stages=(st,), io_round=torch.bfloat16, **w)
        tops.pairformer.pair_update(cur, pre, mask=mask, stages=(st,))
        assert_parity(cur, ref, torch.bfloat16, f"stage {st} N={N} masked={masked}", ref_io=rio)


@pytest.mark.parametrize("N", [128, 136])
@pytest.mark.parametrize("masked", [False, True])
def test_chain_matches_oracle(device, N, masked):
    x, w, mask = _setup(N, device, masked)
    pre = tops.pairformer.precompute(**w)
    ref = oracle.pair_update(x, mask=mask, **w)
    rio = oracle.pair_update(x, mask=mask, io_round=torch.bfloat16, **w)
    out = tops.pairformer.pair_update(x.clone(), pre, mask=mask)
    # Whole chain: the bar is max(2e-2, the reference's own bf16 chain deviation from fp32)
    # on the same inputs (each op's deviation feeds the next ops in both)
    assert_parity(out, ref, torch.bfloat16, f"chain N={N} masked={masked}", ref_io=rio)
    unfused = tops.pairformer.pair_update_unfused(x, pre, mask=mask)
    du = (out.float() - unfused.float()).abs().max().item()
    assert du < 0.1, f"fused vs per-op chain: {du}"


def test_transposed_view_input(device):
    """triangle_attn.forward on X.transpose(0, 1) (ending node) reads X in place and
    equals the call on the contiguous transposed copy."""
    N, C, H, D = 256, 128, 4, 32
    X = rnd(N, N, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=9)
    w = _ta_weights(C, H, D, device, 14)
    g = torch.Generator().manual_seed(3)
    mask = (torch.rand(N, N, generator=g) > 0.1).to(device)
    pre = tops.triangle_attn.precompute(*[w[k] for k in ("W_ln", "B_ln", "WQ", "WK", "WV", "W_proj_z",
                                                           "B_proj_z", "H", "D")])
    kw = dict(scale=1 / math.sqrt(D), W_proj_g=w["W_proj_g"], B_proj_g=None, W_proj_o=w["W_proj_o"], B_proj_o=None)
    a = tops.triangle_attn.forward(X.transpose(0, 1), pre, mask=mask.t(), **kw)
    b = tops.triangle_attn.forward(X.transpose(0, 1).contiguous(), pre, mask=mask.t().contiguous(), **kw)
    assert torch.equal(a, b)


def test_residual_gate_transposed_store(device):
    """gate_forward(residual=, trans_n=) equals out-of-place gate + transpose + add."""
    from triangleops_b200.triangle_attn.kernel import gate_forward

    N, C = 136, 128
    o = rnd(N * N, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=1)
    gin = rnd(N * N, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=2)
    wg = rnd(C, C, dtype=torch.bfloat16, device=device, sd=C**-0.5, seed=3)
    wo = rnd(C, C, dtype=torch.bfloat16, device=device, sd=C**-0.5, seed=4)
    x = rnd(N, N, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=5)
    plain = gate_forward(o, gin, wg, wo).view(N, N, C)
    ref = x.float() + plain.float().transpose(0, 1)
    out = x.clone()
    gate_forward(o, gin, wg, wo, out=out, residual=out, trans_n=N)
    d = (out.float() - ref).abs() - 2.0**-7 * ref.abs()
    assert d.max().item() <= 2.0**-7, d.max().item()
