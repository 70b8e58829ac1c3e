"""Numerics of the attention softmax beyond N(0,1) inputs.

* the two 2^x paths of the softmax (FMA-pipe polynomial and MUFU) over every f16 input
  in the range the softmax feeds them, against fp64 exp2;
* large logits (scaled Q/K and pair bias, |S| up to ~30 in log2 units), where the f16
  S accumulator must stay within the reference's own bf16 error;
* shift invariance: a large negative per-head bias offset with out-of-range tail keys
  and masked keys, and a masked key that carries the row's largest logit — masked and
  out-of-range keys must take no part in the row max (the reference adds -1e9 / -inf
  before its max, ``triangle_attn/kernel.py:230-239``).
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from helpers import assert_parity, rnd
from oracle import oracle
import triangleops_b200 as tops
from triangleops_b200 import _lib

pytestmark = pytest.mark.gpu

_lib.register("tops_selftest_ex2", [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                     ctypes.c_void_p])


def _f16_range(lo, hi):
    """Every finite f16 value in [lo, hi] (as float16 tensor)."""
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16)
    v = bits.view(torch.float16)
    keep = torch.isfinite(v) & (v >= lo) & (v <= hi)
    return torch.sort(v[keep].float()).values.to(torch.float16).contiguous()


def test_ex2_paths_exhaustive(device):
    x = _f16_range(-16.0, 8.0)
    xd = x.to(device)
    poly = torch.empty_like(xd)
    mufu = torch.empty_like(xd)
    _lib.call("tops_selftest_ex2", xd.data_ptr(), poly.data_ptr(), mufu.data_ptr(), xd.numel(),
              _lib.stream_ptr(device))
    torch.cuda.synchronize()
    xf = x.double()
    exact = torch.exp2(xf)
    p, m = poly.cpu().double(), mufu.cpu().double()
    normal = xf >= -14.0  # results are normal f16 numbers
    rel_p = ((p - exact).abs() / exact)[normal].max().item()
    rel_m = ((m - exact).abs() / exact)[normal].max().item()
    # f16 rounding alone is 2^-11 = 4.9e-4; the degree-3 polynomial evaluated in f16 adds
    # a few ulp, the MUFU path one or two
    assert rel_p <= 2.5e-3, f"polynomial 2^x: max relative error {rel_p:.3e}"
    assert rel_m <= 2.5e-3, f"MUFU 2^x: max relative error {rel_m:.3e}"
    # below 2^-14 both paths give a subnormal or zero: absolute error under the smallest normal
    sub = ~normal
    assert (p - exact)[sub].abs().max().item() <= 2.0**-14
    assert (m - exact)[sub].abs().max().item() <= 2.0**-14
    # -inf (masked or out-of-range key) gives exactly 0 on both paths
    ninf = torch.tensor([float("-inf"), float("-inf")], dtype=torch.float16, device=device)
    po, mo = torch.empty_like(ninf), torch.empty_like(ninf)
    _lib.call("tops_selftest_ex2", ninf.data_ptr(), po.data_ptr(), mo.data_ptr(), 2, _lib.stream_ptr(device))
    torch.cuda.synchronize()
    assert po.float().abs().max().item() == 0.0 and mo.float().abs().max().item() == 0.0
    # monotone over the softmax range up to one f16 ulp (the polynomial's range
    # reduction rounds x to an integer, and at f = +-0.5 neighbouring inputs may swap by
    # one rounding step)
    assert ((p[1:] - p[:-1]) + 2.0**-10 * p[1:]).min().item() >= 0.0


def _ta_inputs(N, device, seed=12, qs=1.0, bz=None, masked=True):
    C, H, D = 128, 4, 32
    r = lambda *s, sd, k: rnd(*s, dtype=torch.bfloat16, device=device, sd=sd, seed=seed * 100 + k)  # noqa: E731
    W_pz = r(C, H, sd=qs * C**-0.5, k=6)
    B_pz = r(H, sd=0.1, k=7) if bz is None else torch.tensor(bz, dtype=torch.bfloat16, device=device)
    args = (rnd(N, N, C, dtype=torch.bfloat16, device=device, sd=1.0, seed=seed), 1 + r(C, sd=0.1, k=1),
            r(C, sd=0.1, k=2), r(C, H * D, sd=qs * C**-0.5, k=3), r(C, H * D, sd=qs * C**-0.5, k=4),
            r(C, H * D, sd=C**-0.5, k=5), W_pz, B_pz, r(C, C, sd=C**-0.5, k=8), None, r(C, C, sd=C**-0.5, k=9),
            None, H, D)
    mask = None
    if masked:
        g = torch.Generator().manual_seed(N + seed)
        mask = (torch.rand(N, N, generator=g) > 0.1).to(device)
    return args, mask


def _check(args, mask, what):
    scale = 1 / math.sqrt(32)
    out = tops.triangle_attention(*args, scale=scale, mask=mask)
    ref = oracle.triangle_attention(*args, scale=scale, mask=mask)
    rio = oracle.triangle_attention(*args, scale=scale, mask=mask, io_round=torch.bfloat16)
    assert _lib.device_error()[0] == 0
    return assert_parity(out, ref, torch.bfloat16, what, ref_io=rio)


@pytest.mark.parametrize("qs", [3.0, 6.0])
@pytest.mark.parametrize("masked", [False, True])
def test_large_logits(device, qs, masked):
    """Q, K and the pair bias scaled by qs: logits of a few tens in log2 units."""
    args, mask = _ta_inputs(200, device, qs=qs, masked=masked)
    _check(args, mask, f"qs={qs} masked={masked}")


def test_negative_bias_offset_with_tail_and_masked_keys(device):
    """B_proj_z = -20 for every head, N = 130 (two out-of-range tail keys in the last
    64-key block) and masked keys: every real logit sits far below 0, the value that
    zero-filled tail keys would carry if they entered the row max."""
    args, mask = _ta_inputs(130, device, bz=[-20.0, -20.0, -20.0, -20.0])
    _check(args, mask, "B_proj_z=-20 N=130")


def test_large_positive_offsets_unmasked_tail(device):
    args, _ = _ta_inputs(130, device, bz=[30.0, -30.0, 25.0, -25.0], masked=False)
    _check(args, None, "B_proj_z=+-30 N=130")


def test_masked_key_carries_the_largest_logit(device):
    """Keys 5 and 77 get a pair-bias logit far above every other key (their x rows are
    aligned with W_proj_z), and are masked in every row: they must not set the row max."""
    N = 136
    args, _ = _ta_inputs(N, device, qs=3.0, masked=False)
    X, W_pz = args[0].clone(), args[6]
    big = (W_pz.float().sum(dim=1) / W_pz.float().norm(dim=1).clamp_min(1e-6))
    big = 12.0 * big / big.norm() * math.sqrt(128)
    X[:, 5, :] = big.to(X.dtype)
    X[:, 77, :] = big.to(X.dtype)
    args = (X,) + args[1:]
    mask = torch.ones(N, N, dtype=torch.bool, device=device)
    mask[:, 5] = False
    mask[:, 77] = False
    mask[3, 10:20] = False
    _check(args, mask, "masked largest-logit keys")
