"""fp32 IO parity vs the CPU oracle: all three ops take fp32 inputs through the fp32
CUDA-core kernels (the reference's dtype contract admits fp32, ``_common/dtype.py``).
Bar: max|delta| <= 1e-4 of max|ref| and cos > 0.9999."""
import math

import pytest
import torch

import test_attn_pair_bias as apb_t
import test_triangle_attn as ta_t
import test_triangle_mul as tm_t
from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu
F32 = torch.float32


@pytest.mark.parametrize("N", [33, 130])
@pytest.mark.parametrize("masked", [False, True])
def test_triangle_attention_f32(device, N, masked):
    args, mask = ta_t._inputs(N, 4, 32, 128, F32, device, general=True, masked=masked)
    if masked:
        mask[3] = False  # one fully masked row: the -1e9 path gives a uniform average
    scale = 1.0 / math.sqrt(32)
    out = tops.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask)
    assert out.dtype == F32
    ref = oracle.triangle_attention(*args, scale=scale, eps=1e-5, mask=mask)
    assert_parity(out, ref, F32, f"tri_attn f32 N={N} masked={masked}")


@pytest.mark.parametrize("L", [37, 96])
@pytest.mark.parametrize("direction", ["outgoing", "incoming"])
def test_triangle_mul_f32(device, L, direction):
    C = 64
    x = rnd(2, L, L, C, dtype=F32, device=device, seed=1)
    g = torch.Generator().manual_seed(L)
    mask = (torch.rand(2, L, L, generator=g) > 0.2).to(device)
    w = tm_t._weights(C, F32, device, general=True)
    out = tops.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, **w)
    assert out.dtype == F32
    ref = oracle.triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, **w)
    assert_parity(out, ref, F32, f"trimul f32 L={L} {direction}")


@pytest.mark.parametrize("M", [100, 256])
def test_attention_pair_bias_f32(device, M):
    args = apb_t._inputs(M, F32, device, general=True)
    out = tops.attention_pair_bias(*args, scale=0.5)
    assert out.dtype == F32
    ref = oracle.attention_pair_bias(*args, scale=0.5)
    assert_parity(out, ref, F32, f"apb f32 M={M}")


def test_attention_pair_bias_f32_key_mask(device):
    M = 200
    (X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, B_pg, W_po, B_po, H, D) = apb_t._inputs(M, F32, device,
                                                                                           general=True)
    km = torch.ones(M, dtype=torch.bool, device=device)
    km[-40:] = False
    pre = tops.attn_pair_bias.precompute(WQ, WK, WV, W_ln, B_ln, W_pz, B_pz, H, D)
    out = tops.attn_pair_bias.forward(X, Z, pre, scale=1.0, W_proj_g=W_pg, B_proj_g=B_pg, W_proj_o=W_po,
                                      B_proj_o=B_po, mask=km)
    ref = oracle.attention_pair_bias_masked(X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, W_po, H, D, key_mask=km,
                                            scale=1.0, B_proj_g=B_pg, B_proj_o=B_po)
    assert_parity(out, ref, F32, "apb f32 key-masked")
