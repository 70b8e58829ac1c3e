"""Triangle multiplicative update parity vs the CPU oracle (case matrix of the
reference's tests/test_triangle_mul.py: L in {64, 130, 256}, both directions,
masked, general affine, precompute == one-shot)."""
import pytest
import torch

from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu


def _weights(C, dtype, device, general=False):
    w = {
        "norm_in_weight": torch.ones(C, device=device, dtype=dtype),
        "norm_in_bias": torch.zeros(C, device=device, dtype=dtype),
        "p_in_weight": rnd(2 * C, C, dtype=dtype, device=device, sd=C**-0.5, seed=11),
        "g_in_weight": rnd(2 * C, C, dtype=dtype, device=device, sd=C**-0.5, seed=12),
        "norm_out_weight": torch.ones(C, device=device, dtype=dtype),
        "norm_out_bias": torch.zeros(C, device=device, dtype=dtype),
        "p_out_weight": rnd(C, C, dtype=dtype, device=device, sd=C**-0.5, seed=13),
        "g_out_weight": rnd(C, C, dtype=dtype, device=device, sd=C**-0.5, seed=14),
    }
    if general:
        w["norm_in_weight"] = 1.0 + rnd(C, dtype=dtype, device=device, sd=0.2, seed=21)
        w["norm_in_bias"] = rnd(C, dtype=dtype, device=device, sd=0.1, seed=22)
        w["norm_out_weight"] = 1.0 + rnd(C, dtype=dtype, device=device, sd=0.2, seed=23)
        w["norm_out_bias"] = rnd(C, dtype=dtype, device=device, sd=0.1, seed=24)
    return w


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("L", [64, 130, 256])
@pytest.mark.parametrize("direction", ["outgoing", "incoming"])
@pytest.mark.parametrize("masked", [False, True])
def test_matches_oracle(device, dtype, L, direction, masked):
    C = 128
    x = rnd(1, L, L, C, dtype=dtype, device=device, seed=1)
    if masked:
        g = torch.Generator().manual_seed(L)
        mask = (torch.rand(1, L, L, generator=g) > 0.2).to(device)
    else:
        mask = torch.ones(1, L, L, dtype=torch.bool, device=device)
    w = _weights(C, dtype, device)
    out = tops.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, **w)
    ref = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, **w)
    rio = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, io_round=dtype, **w)
    assert_parity(out, ref, dtype, f"L={L} {direction} masked={masked}", ref_io=rio)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("L", [128, 256])
@pytest.mark.parametrize("direction", ["outgoing", "incoming"])
def test_general_affine(device, dtype, L, direction):
    C = 128
    x = rnd(1, L, L, C, dtype=dtype, device=device, seed=1)
    mask = torch.ones(1, L, L, dtype=torch.bool, device=device)
    w = _weights(C, dtype, device, general=True)
    out = tops.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, **w)
    ref = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, **w)
    rio = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, io_round=dtype, **w)
    assert_parity(out, ref, dtype, f"general L={L} {direction}", ref_io=rio)


def test_precompute_forward_matches_oneshot(device):
    C, L = 128, 256
    x = rnd(1, L, L, C, dtype=torch.bfloat16, device=device, seed=1)
    mask = torch.ones(1, L, L, dtype=torch.bool, device=device)
    w = _weights(C, torch.bfloat16, device)
    pre = tops.triangle_mul.precompute(*[w[k] for k in ("norm_in_weight", "norm_in_bias", "p_in_weight",
                                                        "g_in_weight", "norm_out_weight", "norm_out_bias",
                                                        "p_out_weight", "g_out_weight")])
    a = tops.triangle_mul.forward(x, pre, direction="outgoing", mask=mask)
    b = tops.triangle_multiplicative_update(x, direction="outgoing", mask=mask, **w)
    assert torch.equal(a, b)


def test_padded_tail_mask_batch2(device):
    """Config-3 style 2D outer-product mask with a padded tail, and batch B=2."""
    C, L = 128, 192
    x = rnd(2, L, L, C, dtype=torch.bfloat16, device=device, seed=3)
    v = torch.ones(L)
    v[170:] = 0
    mask = (v[:, None] * v[None, :]).expand(2, L, L).to(device)
    w = _weights(C, torch.bfloat16, device, general=True)
    for direction in ("outgoing", "incoming"):
        out = tops.triangle_multiplicative_update(x, direction=direction, mask=mask, **w)
        ref = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, **w)
        rio = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, io_round=torch.bfloat16, **w)
        assert_parity(out, ref, torch.bfloat16, f"tail {direction}", ref_io=rio)


def test_lowlevel_phases(device):
    """input_phase -> contract -> output_phase (reference kernel.py signatures)."""
    C, L = 128, 128
    x = rnd(1, L, L, C, dtype=torch.bfloat16, device=device, seed=5)
    w = _weights(C, torch.bfloat16, device, general=True)
    pre = tops.triangle_mul.precompute(*[w[k] for k in ("norm_in_weight", "norm_in_bias", "p_in_weight",
                                                        "g_in_weight", "norm_out_weight", "norm_out_bias",
                                                        "p_out_weight", "g_out_weight")])
    ab = tops.triangle_mul.input_phase(x, None, pre["p_in_combined"], pre["g_in_combined"], pre["sum_W_p_in"],
                                       pre["sum_W_g_in"], pre["B_p_in_const"], pre["B_g_in_const"], 1e-5)
    a, b = torch.chunk(ab, 2, dim=0)
    # the contraction alone vs torch's einsum on the same bf16 operands
    y = tops.triangle_mul.contract(a, b, "incoming")
    yref = torch.einsum("dbki,dbkj->dbij", a.float(), b.float())
    assert (y.float() - yref).abs().max().item() <= 2e-2 * max(1.0, yref.abs().max().item())
    y = tops.triangle_mul.contract(a, b, "outgoing")
    out = tops.triangle_mul.output_phase(y, x, pre["p_out_combined"], pre["g_out_combined"], pre["sum_W_p_out"],
                                         pre["sum_W_g_out"], pre["B_p_out_const"], pre["B_g_out_const"], 1e-5)
    ref = oracle.triangle_multiplicative_update(x, direction="outgoing", **w)
    rio = oracle.triangle_multiplicative_update(x, direction="outgoing", io_round=torch.bfloat16, **w)
    assert_parity(out, ref, torch.bfloat16, "low-level", ref_io=rio)


def test_bad_direction(device):
    x = rnd(1, 16, 16, 128, dtype=torch.bfloat16, device=device, seed=1)
    with pytest.raises(ValueError):
        tops.triangle_multiplicative_update(x, direction="sideways", **_weights(128, torch.bfloat16, device))
