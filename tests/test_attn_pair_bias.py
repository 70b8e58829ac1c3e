"""Attention-with-pair-bias parity vs the CPU oracle (case matrix of the
reference's tests/test_attn_pair_bias.py: M in {128, 256, 512}, general affine +
biases, precompute == one-shot) plus the key-masked configuration."""
import pytest
import torch

from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu


def _inputs(M, dtype, device, H=4, D=32, Cz=128, general=False):
    N = H * D
    X = rnd(M, N, dtype=dtype, device=device, sd=1.0, seed=1)
    Z = rnd(M, M, Cz, dtype=dtype, device=device, sd=1.0, seed=2)
    WQ, WK, WV = (rnd(N, N, dtype=dtype, device=device, sd=N**-0.5, seed=s) for s in (3, 4, 5))
    if general:
        W_ln = 1.0 + rnd(Cz, dtype=dtype, device=device, sd=0.2, seed=21)
        B_ln = rnd(Cz, dtype=dtype, device=device, sd=0.1, seed=22)
        B_pz = rnd(H, dtype=dtype, device=device, sd=0.1, seed=23)
        B_pg = rnd(N, dtype=dtype, device=device, sd=0.1, seed=24)
        B_po = rnd(N, dtype=dtype, device=device, sd=0.1, seed=25)
    else:
        W_ln = torch.ones(Cz, device=device, dtype=dtype)
        B_ln = torch.zeros(Cz, device=device, dtype=dtype)
        B_pz = torch.zeros(H, device=device, dtype=dtype)
        B_pg = torch.zeros(N, device=device, dtype=dtype)
        B_po = torch.zeros(N, device=device, dtype=dtype)
    W_pz = rnd(Cz, H, dtype=dtype, device=device, sd=Cz**-0.5, seed=6)
    W_pg = rnd(N, N, dtype=dtype, device=device, sd=N**-0.5, seed=7)
    W_po = rnd(N, N, dtype=dtype, device=device, sd=N**-0.5, seed=8)
    return (X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, B_pg, W_po, B_po, H, D)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M", [128, 256, 512])
def test_matches_oracle(device, dtype, M):
    args = _inputs(M, dtype, device)
    out = tops.attention_pair_bias(*args, scale=1.0)
    ref = oracle.attention_pair_bias(*args, scale=1.0)
    rio = oracle.attention_pair_bias(*args, scale=1.0, io_round=dtype)
    assert_parity(out, ref, dtype, f"M={M}", ref_io=rio)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_general_affine(device, dtype):
    args = _inputs(256, dtype, device, general=True)
    out = tops.attention_pair_bias(*args, scale=0.5)
    ref = oracle.attention_pair_bias(*args, scale=0.5)
    rio = oracle.attention_pair_bias(*args, scale=0.5, io_round=dtype)
    assert_parity(out, ref, dtype, "general", ref_io=rio)


def test_precompute_forward_matches_oneshot(device):
    args = _inputs(256, torch.bfloat16, device, general=True)
    (X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, B_pg, W_po, B_po, H, D) = args
    pre = tops.attn_pair_bias.precompute(WQ, WK, WV, W_ln, B_ln, W_pz, B_pz, H, D)
    a = tops.attn_pair_bias.forward(X, Z, pre, scale=1.0, W_proj_g=W_pg, B_proj_g=B_pg, W_proj_o=W_po, B_proj_o=B_po)
    b = tops.attention_pair_bias(*args, scale=1.0)
    assert torch.equal(a, b)


@pytest.mark.parametrize("M", [200, 1024])
def test_key_masked(device, M):
    """Config-2 style: token mask with a padded tail (last 64 keys masked), ragged M."""
    args = _inputs(M, torch.bfloat16, device)
    (X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, B_pg, W_po, B_po, H, D) = args
    km = torch.ones(M, dtype=torch.bool, device=device)
    km[-64:] = False
    out = tops.attention_pair_bias(*args, scale=1.0, mask=km)
    kw = dict(key_mask=km, scale=1.0, B_proj_g=B_pg, B_proj_o=B_po)
    ref = oracle.attention_pair_bias_masked(X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, W_po, H, D, **kw)
    rio = oracle.attention_pair_bias_masked(X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, W_po, H, D,
                                            io_round=torch.bfloat16, **kw)
    assert_parity(out, ref, torch.bfloat16, f"masked M={M}", ref_io=rio)


def test_lowlevel_apb_forward(device):
    args = _inputs(256, torch.bfloat16, device, general=True)
    (X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, B_pg, W_po, B_po, H, D) = args
    pre = tops.attn_pair_bias.precompute(WQ, WK, WV, W_ln, B_ln, W_pz, B_pz, H, D)
    Og = torch.empty(256, H * D, device=device, dtype=X.dtype)
    tops.attn_pair_bias.apb_forward(X, pre["W_QKV"], Z, pre["W_combined"], pre["sum_W_combined"], pre["B_const"], Og,
                                    scale=1.0)
    g = torch.sigmoid(torch.nn.functional.linear(X, W_pg, B_pg))
    out = torch.nn.functional.linear(g * Og, W_po, B_po)  # the reference's torch gate path (bf16)
    ref = oracle.attention_pair_bias(*args, scale=1.0)
    rio = oracle.attention_pair_bias(*args, scale=1.0, io_round=torch.bfloat16)
    assert_parity(out, ref, torch.bfloat16, "low-level", ref_io=rio)


@pytest.mark.parametrize("M", [256, 1000])
def test_query_row_windows(device, M):
    """tops_apb_forward_rows: query windows (ragged, unaligned starts) of the row-sharded
    entry point reproduce the corresponding rows of the whole-sequence call."""
    from triangleops_b200.attn_pair_bias.kernel import apb_core

    args = _inputs(M, torch.bfloat16, device, general=True)
    (X, WQ, WK, WV, Z, W_ln, B_ln, W_pz, B_pz, W_pg, B_pg, W_po, B_po, H, D) = args
    km = torch.ones(M, dtype=torch.bool, device=device)
    km[-24:] = False
    pre = tops.attn_pair_bias.precompute(WQ, WK, WV, W_ln, B_ln, W_pz, B_pz, H, D)
    core = lambda Zr, Og, q0: apb_core(X, pre["w_rows"], Zr, pre["W_combined"], pre["sum_W_combined"],  # noqa: E731
                                       pre["B_const"], Og, H, D, key_mask=km, q0=q0)
    full = core(Z, torch.empty(M, H * D, device=device, dtype=X.dtype), 0)
    for q0, q1 in ((0, M // 2), (M // 2, M), (37, 37 + 131), (M - 5, M)):
        part = core(Z[q0:q1], torch.empty(q1 - q0, H * D, device=device, dtype=X.dtype), q0)
        assert torch.equal(part, full[q0:q1]), f"window [{q0}, {q1})"
