"""Pairformer pair transition (the fused LN + SwiGLU MLP + residual kernel) against the
fp32 oracle and its 16-bit emulation; the chain with the transition as fifth stage."""
import pytest
import torch

from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu


def _weights(dtype, device, seed=5, C=128):
    r = lambda *s, sd, k: rnd(*s, dtype=dtype, device=device, sd=sd, seed=seed * 100 + k)  # noqa: E731
    return dict(norm_weight=1 + r(C, sd=0.1, k=1), norm_bias=r(C, sd=0.1, k=2), w1=r(4 * C, C, sd=C**-0.5, k=3),
                w2=r(4 * C, C, sd=C**-0.5, k=4), w3=r(C, 4 * C, sd=(4 * C) ** -0.5, k=5))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(64, 64), (200,), (3, 37)])
def test_matches_oracle(device, dtype, shape):
    x = rnd(*shape, 128, dtype=dtype, device=device, sd=1.0, seed=2)
    w = _weights(dtype, device)
    out = tops.transition.transition(x, **w)
    ref = oracle.transition(x, **w)
    rio = oracle.transition(x, io_round=dtype, **w)
    assert_parity(out, ref, dtype, f"transition {shape}", ref_io=rio)


def test_in_place_and_precompute(device):
    x = rnd(1, 96, 96, 128, dtype=torch.bfloat16, device=device, sd=1.0, seed=3)
    w = _weights(torch.bfloat16, device, seed=6)
    pre = tops.transition.precompute(**w)
    a = tops.transition.forward(x, pre)
    y = x.clone()
    tops.transition.forward(y, pre, out=y)
    assert torch.equal(a, y)
    assert torch.equal(a, tops.transition.transition(x, **w))


def test_chain_with_transition_stage(device):
    from test_pairformer import _setup

    N = 128
    x, w, mask = _setup(N, device, masked=True)
    tw = _weights(torch.bfloat16, device, seed=7)
    pre = tops.pairformer.precompute(**w, transition=tw)
    stages = tops.pairformer.ALL_STAGES
    out = tops.pairformer.pair_update(x.clone(), pre, mask=mask, stages=stages)
    ref = oracle.pair_update(x, mask=mask, stages=stages, transition=tw, **w)
    rio = oracle.pair_update(x, mask=mask, stages=stages, transition=tw, io_round=torch.bfloat16, **w)
    assert_parity(out, ref, torch.bfloat16, "chain + transition", ref_io=rio)
