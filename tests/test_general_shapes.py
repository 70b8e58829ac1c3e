"""Shapes the reference accepts but the tcgen05 kernels are not built for (any C = H*D for
the attentions, any C for the multiplication): they run on the fp32 CUDA-core kernels
and round back to the IO dtype once, so they must match the fp32 oracle closely."""
import math

import pytest
import torch

from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("C,H,D,N", [(128, 8, 16, 40), (48, 2, 24, 33), (256, 8, 32, 24)])
def test_triangle_attention_other_shapes(device, C, H, D, N):
    dt = torch.bfloat16
    r = lambda *s, sd, k: rnd(*s, dtype=dt, device=device, sd=sd, seed=70 + k)  # noqa: E731
    args = (rnd(N, N, C, dtype=dt, device=device, sd=1.0, seed=7), 1 + r(C, sd=0.1, k=1), r(C, sd=0.1, k=2),
            r(C, H * D, sd=C**-0.5, k=3), r(C, H * D, sd=C**-0.5, k=4), r(C, H * D, sd=C**-0.5, k=5),
            r(C, H, sd=C**-0.5, k=6), r(H, sd=0.1, k=7), r(C, H * D, sd=C**-0.5, k=8), None,
            r(H * D, C, sd=(H * D) ** -0.5, k=9), None, H, D)
    g = torch.Generator().manual_seed(N)
    mask = (torch.rand(N, N, generator=g) > 0.2).to(device)
    out = tops.triangle_attention(*args, scale=1 / math.sqrt(D), mask=mask)
    ref = oracle.triangle_attention(*args, scale=1 / math.sqrt(D), mask=mask)
    assert out.dtype == dt
    assert_parity(out, ref, dt, f"C={C} H={H} D={D}")


@pytest.mark.parametrize("C", [32, 96])
@pytest.mark.parametrize("direction", ["outgoing", "incoming"])
def test_triangle_mul_other_widths(device, C, direction):
    dt = torch.bfloat16
    L = 37
    r = lambda *s, sd, k: rnd(*s, dtype=dt, device=device, sd=sd, seed=90 + k)  # noqa: E731
    w = dict(norm_in_weight=1 + r(C, sd=0.1, k=1), norm_in_bias=r(C, sd=0.1, k=2),
             p_in_weight=r(2 * C, C, sd=C**-0.5, k=3), g_in_weight=r(2 * C, C, sd=C**-0.5, k=4),
             norm_out_weight=1 + r(C, sd=0.1, k=5), norm_out_bias=r(C, sd=0.1, k=6),
             p_out_weight=r(C, C, sd=C**-0.5, k=7), g_out_weight=r(C, C, sd=C**-0.5, k=8))
    x = rnd(1, L, L, C, dtype=dt, device=device, sd=1.0, seed=9)
    mask = (torch.rand(1, L, L, generator=torch.Generator().manual_seed(1)) > 0.2).to(device)
    out = tops.triangle_multiplicative_update(x, direction=direction, mask=mask, **w)
    ref = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, **w)
    assert out.dtype == dt
    assert_parity(out, ref, dt, f"C={C} {direction}")


def test_attention_pair_bias_other_shapes(device):
    dt = torch.bfloat16
    M, C, Cz, H, D = 96, 128, 64, 8, 16
    r = lambda *s, sd, k: rnd(*s, dtype=dt, device=device, sd=sd, seed=110 + k)  # noqa: E731
    X, Z = r(M, C, sd=1.0, k=1), r(M, M, Cz, sd=1.0, k=2)
    args = (X, r(C, H * D, sd=C**-0.5, k=3), r(C, H * D, sd=C**-0.5, k=4), r(C, H * D, sd=C**-0.5, k=5), Z,
            1 + r(Cz, sd=0.1, k=6), r(Cz, sd=0.1, k=7), r(Cz, H, sd=Cz**-0.5, k=8), None,
            r(C, H * D, sd=C**-0.5, k=9), None, r(H * D, C, sd=(H * D) ** -0.5, k=10), None, H, D)
    out = tops.attention_pair_bias(*args, scale=1 / math.sqrt(D))
    ref = oracle.attention_pair_bias(*args, scale=1 / math.sqrt(D))
    assert out.dtype == dt
    assert_parity(out, ref, dt, "apb H=8 D=16 C_z=64")
