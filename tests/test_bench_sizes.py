"""Parity at the sizes the benchmark numbers are quoted on, through sampled rows of the
fp32 oracle (rows of these ops are independent given the tensors every row shares, so
a handful of rows checks the full-size launch configuration, tails and all):

* config 1 — triangle attention, starting node, N = 2048, mask Bernoulli(0.9);
* config 3 — triangle multiplication, incoming, L = 2048, 1900-residue tail mask;
* config 4 — the Pairformer pair-update chain at N = 2048, stage by stage: before each
  stage the GPU chain's own state is copied, and rows of that stage's oracle update are
  compared with the GPU state after the stage (every stage runs at full size).

The generators are bench.py's, so these are the same inputs the bench line times.
"""
import math

import pytest
import torch

import bench
from helpers import assert_parity
from oracle import oracle
import triangleops_b200 as tops

pytestmark = pytest.mark.gpu

ROWS = [0, 1, 777, 1024, 1899, 1900, 2047]


def test_config1_triangle_attention_n2048(device):
    N, H, D = 2048, bench.H, bench.D
    inp = bench.make_inputs(N, device)
    pre = tops.triangle_attn.precompute(inp["W_ln"], inp["B_ln"], inp["WQ"], inp["WK"], inp["WV"], inp["W_proj_z"],
                                        None, H, D)
    out = tops.triangle_attn.forward(inp["X"], pre, mask=inp["mask"], scale=1 / math.sqrt(D),
                                     W_proj_g=inp["W_proj_g"], B_proj_g=None, W_proj_o=inp["W_proj_o"], B_proj_o=None)
    got = out[ROWS].cpu()
    del out
    cpu = {k: v.cpu() for k, v in inp.items()}
    ref = oracle.triangle_attention_chunked(cpu["X"], cpu["W_ln"], cpu["B_ln"], cpu["WQ"], cpu["WK"], cpu["WV"],
                                            cpu["W_proj_z"], None, cpu["W_proj_g"], None, cpu["W_proj_o"], None, H, D,
                                            scale=1 / math.sqrt(D), mask=cpu["mask"], rows=ROWS)
    assert_parity(got, ref, torch.bfloat16, "config 1 N=2048 rows")


def test_config3_triangle_mul_incoming_l2048(device):
    x, mask, w = bench.config3_inputs(device)
    pre = tops.triangle_mul.precompute(*w)
    out = tops.triangle_mul.forward(x, pre, direction="incoming", mask=mask)
    got = out[0, ROWS].cpu()
    del out
    names = ("norm_in_weight", "norm_in_bias", "p_in_weight", "g_in_weight", "norm_out_weight", "norm_out_bias",
             "p_out_weight", "g_out_weight")
    wd = {k: v.cpu() for k, v in zip(names, w)}
    ref = oracle.triangle_multiplicative_update_rows(x.cpu(), direction="incoming", rows=ROWS, mask=mask.cpu(), **wd)
    assert_parity(got, ref, torch.bfloat16, "config 3 L=2048 rows")


def _tm_dict(p):
    return {k: v.cpu() for k, v in p.items()}


def test_config4_chain_n2048_stagewise(device):
    N = 2048
    params, x = bench.chain_inputs(device, N)
    pre = tops.pairformer.precompute(*params)
    ones = torch.ones(N, N, dtype=torch.bool, device=device)
    cur = x.clone()
    for st, p in zip(tops.pairformer.STAGES, params):
        before = cur.cpu()
        tops.pairformer.pair_update(cur, pre, mask=ones, stages=(st,))
        if st.startswith("tri_mul"):
            upd = oracle.triangle_multiplicative_update_rows(before[None], rows=ROWS, direction="outgoing"
                                                             if st == "tri_mul_out" else "incoming", **_tm_dict(p))
            ref = before[ROWS].float() + upd
            got = cur[ROWS].cpu()
        else:
            src = before.transpose(0, 1) if st == "tri_attn_end" else before
            q = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in p.items()}
            upd = oracle.triangle_attention_chunked(src, q["W_ln"], q["B_ln"], q["WQ"], q["WK"], q["WV"],
                                                    q["W_proj_z"], q["B_proj_z"], q["W_proj_g"], None, q["W_proj_o"],
                                                    None, q["H"], q["D"], scale=q["D"] ** -0.5, rows=ROWS)
            ref = src[ROWS].float() + upd
            got = (cur.transpose(0, 1) if st == "tri_attn_end" else cur)[ROWS].cpu()
        # x is stored in bf16 after the add: one more rounding (half an ulp of |x|) than the op alone
        assert_parity(got, ref, torch.bfloat16, f"config 4 stage {st} rows", rtol_scale=1.5)
