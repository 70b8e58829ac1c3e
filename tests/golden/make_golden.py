"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run where a checkout of youngchan2/TriangleOps is available, its path in
``TRIANGLEOPS_REF``::

    TRIANGLEOPS_REF=<path to the checkout> python tests/golden/make_golden.py

It imports the reference's own pure-torch functions
(``benchmarks/references.py``: ``torch_triangle_attention`` :174-205,
``torch_triangle_multiplicative_update`` :208-221, ``torch_attn_pair_bias``
:143-171, ``torch_attn_pair_bias_qknorm`` :224-277) and its LN-affine fold
(``triangle_ops/_common/ln_absorption.py:28-63``), evaluates them in fp32 on
seeded small inputs (ragged sizes, masks, non-identity LN affines, biases) and
writes inputs + outputs to ``tests/golden/golden.pt``. The tests never read the
reference checkout; they only read this committed file.
"""

import importlib.util
import os
import sys

import torch

REF = os.environ.get("TRIANGLEOPS_REF", "")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.pt")


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    if not REF or not os.path.isdir(REF):
        sys.exit("set TRIANGLEOPS_REF to a checkout of youngchan2/TriangleOps")
    refs = _load("ref_references", os.path.join(REF, "benchmarks", "references.py"))
    lnabs = _load("ref_ln_absorption", os.path.join(REF, "triangle_ops", "_common", "ln_absorption.py"))
    g = torch.Generator().manual_seed(1234)

    def rn(*s, sd=1.0):
        return torch.randn(*s, generator=g) * sd

    cases = {}

    # triangle attention: ragged N, general affine, with and without mask
    for masked in (False, True):
        N, H, D, C = 10, 2, 8, 16
        a = dict(X=rn(N, N, C), W_ln=1 + 0.2 * rn(C), B_ln=0.1 * rn(C), WQ=rn(C, H * D, sd=C**-0.5),
                 WK=rn(C, H * D, sd=C**-0.5), WV=rn(C, H * D, sd=C**-0.5), W_proj_z=rn(C, H, sd=C**-0.5),
                 B_proj_z=0.1 * rn(H), W_proj_g=rn(C, H * D, sd=C**-0.5), W_proj_o=rn(C, H * D, sd=(H * D) ** -0.5))
        mask = (torch.rand(N, N, generator=g) > 0.3) if masked else None
        out = refs.torch_triangle_attention(a["X"], a["W_ln"], a["B_ln"], a["WQ"], a["WK"], a["WV"], a["W_proj_z"],
                                            a["B_proj_z"], a["W_proj_g"], None, a["W_proj_o"], None, H, D,
                                            scale=D**-0.5, eps=1e-5, mask=mask)
        cases[f"tri_attn_masked{int(masked)}"] = dict(inputs=a, mask=mask, H=H, D=D, scale=D**-0.5, out=out)

    # triangle multiplicative update: both directions, masked, general affine
    for direction in ("outgoing", "incoming"):
        B, L, C = 1, 12, 16
        w = dict(norm_in_weight=1 + 0.2 * rn(C), norm_in_bias=0.1 * rn(C), p_in_weight=rn(2 * C, C, sd=C**-0.5),
                 g_in_weight=rn(2 * C, C, sd=C**-0.5), norm_out_weight=1 + 0.2 * rn(C), norm_out_bias=0.1 * rn(C),
                 p_out_weight=rn(C, C, sd=C**-0.5), g_out_weight=rn(C, C, sd=C**-0.5))
        x = rn(B, L, L, C)
        mask = (torch.rand(B, L, L, generator=g) > 0.2)
        out = refs.torch_triangle_multiplicative_update(x, direction=direction, mask=mask, eps=1e-5, **w)
        cases[f"tri_mul_{direction}"] = dict(x=x, mask=mask, weights=w, direction=direction, out=out)

    # attention with pair bias: unmasked with biases, and key-masked (qknorm variant, b_q=0)
    M, H, D, Cz = 12, 2, 8, 16
    N = H * D
    a = dict(X=rn(M, N), WQ=rn(N, N, sd=N**-0.5), WK=rn(N, N, sd=N**-0.5), WV=rn(N, N, sd=N**-0.5),
             Z=rn(M, M, Cz), W_ln=1 + 0.2 * rn(Cz), B_ln=0.1 * rn(Cz), W_proj_z=rn(Cz, H, sd=Cz**-0.5),
             B_proj_z=0.1 * rn(H), W_proj_g=rn(N, N, sd=N**-0.5), B_proj_g=0.1 * rn(N), W_proj_o=rn(N, N, sd=N**-0.5),
             B_proj_o=0.1 * rn(N))
    out = refs.torch_attn_pair_bias(a["X"], a["WQ"], a["WK"], a["WV"], a["Z"], a["W_ln"], a["B_ln"], a["W_proj_z"],
                                    a["B_proj_z"], a["W_proj_g"], a["B_proj_g"], a["W_proj_o"], a["B_proj_o"], H, D,
                                    scale=0.7, eps=1e-5)
    cases["apb"] = dict(inputs=a, H=H, D=D, scale=0.7, out=out)
    key_mask = torch.ones(M, dtype=torch.bool)
    key_mask[-3:] = False
    out_m = refs.torch_attn_pair_bias_qknorm(a["X"], a["WQ"], torch.zeros(N), a["WK"], a["WV"], a["Z"], a["W_ln"],
                                             a["B_ln"], a["W_proj_z"], a["B_proj_z"], a["W_proj_g"], a["W_proj_o"],
                                             H, D, key_mask=key_mask, scale=1.0, eps=1e-5)
    cases["apb_masked"] = dict(inputs=a, H=H, D=D, scale=1.0, key_mask=key_mask, out=out_m)

    # LN-affine fold
    W = rn(6, 16)
    wl, bl = 1 + 0.2 * rn(16), 0.1 * rn(16)
    cases["absorb_ln"] = dict(W=W, w_ln=wl, b_ln=bl, out=lnabs.absorb_ln(W, wl, bl))
    Wm = rn(16, 6)
    cases["absorb_ln_matmul"] = dict(W=Wm, w_ln=wl, b_ln=bl, out=lnabs.absorb_ln_matmul(Wm, wl, bl))

    torch.save(cases, OUT)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(cases)} cases)")


if __name__ == "__main__":
    sys.exit(main())
