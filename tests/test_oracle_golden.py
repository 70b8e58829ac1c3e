"""Pin the CPU oracle against golden outputs of the reference's own torch functions."""
import os

import pytest
import torch

from oracle import oracle

GOLD = torch.load(os.path.join(os.path.dirname(__file__), "golden", "golden.pt"), weights_only=False)


def _close(a, b, tol=2e-5):
    assert a.shape == b.shape
    err = (a.float() - b.float()).abs().max().item()
    assert err <= tol * max(1.0, b.abs().max().item()), err


@pytest.mark.parametrize("masked", [0, 1])
def test_triangle_attention(masked):
    c = GOLD[f"tri_attn_masked{masked}"]
    a = c["inputs"]
    args = (a["X"], a["W_ln"], a["B_ln"], a["WQ"], a["WK"], a["WV"], a["W_proj_z"], a["B_proj_z"], a["W_proj_g"],
            None, a["W_proj_o"], None, c["H"], c["D"])
    _close(oracle.triangle_attention(*args, scale=c["scale"], mask=c["mask"]), c["out"])
    _close(oracle.triangle_attention_chunked(*args, scale=c["scale"], mask=c["mask"], row_block=3), c["out"])
    sub = oracle.triangle_attention_chunked(*args, scale=c["scale"], mask=c["mask"], rows=[7, 2])
    _close(sub, c["out"][[7, 2]])


@pytest.mark.parametrize("direction", ["outgoing", "incoming"])
def test_triangle_mul(direction):
    c = GOLD[f"tri_mul_{direction}"]
    out = oracle.triangle_multiplicative_update(c["x"], direction=direction, mask=c["mask"], **c["weights"])
    _close(out, c["out"])
    rows = oracle.triangle_multiplicative_update_rows(c["x"], direction=direction, rows=[3, 0, 11], mask=c["mask"],
                                                      **c["weights"])
    _close(rows, c["out"][0, [3, 0, 11]])


def test_triangle_mul_bad_direction():
    c = GOLD["tri_mul_outgoing"]
    with pytest.raises(ValueError):
        oracle.triangle_multiplicative_update(c["x"], direction="sideways", **c["weights"])


def test_attention_pair_bias():
    c = GOLD["apb"]
    a = c["inputs"]
    out = oracle.attention_pair_bias(a["X"], a["WQ"], a["WK"], a["WV"], a["Z"], a["W_ln"], a["B_ln"], a["W_proj_z"],
                                     a["B_proj_z"], a["W_proj_g"], a["B_proj_g"], a["W_proj_o"], a["B_proj_o"], c["H"],
                                     c["D"], scale=c["scale"])
    _close(out, c["out"])


def test_attention_pair_bias_masked():
    c = GOLD["apb_masked"]
    a = c["inputs"]
    out = oracle.attention_pair_bias_masked(a["X"], a["WQ"], a["WK"], a["WV"], a["Z"], a["W_ln"], a["B_ln"],
                                            a["W_proj_z"], a["B_proj_z"], a["W_proj_g"], a["W_proj_o"], c["H"], c["D"],
                                            key_mask=c["key_mask"], scale=c["scale"])
    _close(out, c["out"])


def test_absorb_ln():
    for name, fn in (("absorb_ln", oracle.absorb_ln), ("absorb_ln_matmul", oracle.absorb_ln_matmul)):
        c = GOLD[name]
        for mine, ref in zip(fn(c["W"], c["w_ln"], c["b_ln"]), c["out"]):
            _close(mine, ref, 1e-6)
