"""Host-only checks of the C-ABI library: it loads, exports every symbol the
public header declares, and rejects bad arguments before touching the GPU."""
import ctypes
import os
import re

import pytest
import torch

from triangleops_b200 import _build, _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "triangleops_b200.h")


def _declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(tops_\w+)\s*\(", txt, re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("tops_triangle_attn_forward", "tops_fused_gate_forward", "tops_trimul_forward", "tops_apb_forward"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_build.build())
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_version_and_status_strings():
    assert _lib.lib().tops_version() == 100
    assert _lib.status_string(0) == "ok"
    assert "shape" in _lib.status_string(_lib.ERR_SHAPE)


def test_errors_map_to_reference_exceptions():
    with pytest.raises(AssertionError):
        _lib.check(_lib.ERR_SHAPE, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_DTYPE, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_ARG, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_TIMEOUT, "x")


def test_argument_validation_before_launch():
    """Bad dtype / direction / shape are rejected on the host (no device needed)."""
    lib = _lib.lib()
    f = lib.tops_trimul_contract
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64] + [ctypes.c_void_p] * 4
    assert f(5, 0, 1, 8, 16, 16, 16, None) == _lib.ERR_DTYPE
    assert f(_lib.BF16, 7, 1, 8, 16, 16, 16, None) == _lib.ERR_ARG
    assert f(_lib.BF16, 0, 1, 10, 16, 16, 16, None) == _lib.ERR_ALIGN
    assert f(_lib.BF16, 0, 1, 8, 0, 16, 16, None) == _lib.ERR_ALIGN
    g = lib.tops_fused_gate_forward
    g.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int64] + [ctypes.c_void_p] * 8
    assert g(_lib.BF16, 128, 96, 16, 16, 16, 16, None, None, 16, None) == _lib.ERR_SHAPE


def test_no_cpu_fallback():
    import torch
    import triangleops_b200 as tops
    x = torch.zeros(1, 8, 8, 128)
    w = {k: torch.zeros(s) for k, s in (("norm_in_weight", 128), ("norm_in_bias", 128),
                                        ("p_in_weight", (256, 128)), ("g_in_weight", (256, 128)),
                                        ("norm_out_weight", 128), ("norm_out_bias", 128),
                                        ("p_out_weight", (128, 128)), ("g_out_weight", (128, 128)))}
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        tops.triangle_multiplicative_update(x.bfloat16(), direction="outgoing", **w)


def test_drop_in_import_name():
    import triangle_ops
    import triangle_ops.triangle_mul as tm

    assert triangle_ops.triangle_attention is not None
    assert tm.precompute is triangle_ops.triangle_mul.precompute
    for name in ("triangle_attention", "triangle_multiplicative_update", "attention_pair_bias"):
        assert hasattr(triangle_ops, name)


def test_workspace_bytes_match_the_python_layer():
    """The host-only size queries agree with the workspaces the Python layer allocates
    (triangle_attn/kernel.py, triangle_mul/kernel.py, attn_pair_bias/kernel.py) and
    reject bad shapes; they need no GPU."""
    lib = ctypes.CDLL(_build.build())
    I64 = ctypes.c_int64
    out = (I64 * 6)()
    N, C, H, D = 130, 128, 4, 32
    np_ = (N + 7) // 8 * 8
    assert lib.tops_triangle_attn_workspace_bytes(1, I64(N), I64(N), I64(C), I64(H), I64(D), out) == 0
    assert list(out) == [N * N * C * 2, N * H * N * D * 2, N * H * N * D * 2, N * H * D * np_ * 2, N * np_ * 2,
                         H * N * np_ * 2]
    assert lib.tops_triangle_attn_workspace_bytes(1, I64(N + 1), I64(N), I64(C), I64(H), I64(D), out) == _lib.ERR_SHAPE
    assert lib.tops_triangle_attn_workspace_bytes(2, I64(N), I64(N), I64(C), I64(H), I64(D), out) == _lib.ERR_DTYPE
    B, L = 2, 64
    assert lib.tops_trimul_workspace_bytes(0, I64(B), I64(L), I64(C), out) == 0
    assert list(out)[:2] == [2 * C * B * L * L * 2, C * B * L * L * 2]
    M, Mq = 200, 100
    mp = (M + 7) // 8 * 8
    assert lib.tops_apb_workspace_bytes(I64(M), I64(Mq), I64(H), I64(D), out) == 0
    assert list(out)[:5] == [H * M * D * 2, H * M * D * 2, H * D * mp * 2, mp * 2, H * Mq * mp * 2]
    assert lib.tops_apb_workspace_bytes(I64(M), I64(M + 1), I64(H), I64(D), out) == _lib.ERR_SHAPE
    assert lib.tops_apb_workspace_bytes(I64(M), I64(M), I64(H), I64(D), None) == _lib.ERR_ARG


def test_extension_entry_points_validate_on_the_host():
    """The entry points without a reference counterpart reject bad arguments before any
    device work (so these run without a GPU)."""
    lib = ctypes.CDLL(_build.build())
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    f = lib.tops_apb_forward_rows
    f.argtypes = [I, I64, I64, I64, I64, I64, I64, I64] + [P] * 7 + [F, F] + [P] * 7
    base = [P(16)] * 7
    ws = [P(16)] * 7
    assert f(_lib.BF16, 256, 200, 100, 128, 128, 4, 32, *base, 1.0, 1e-5, *ws) == _lib.ERR_SHAPE  # q0 + Mq > M
    assert f(2, 256, 0, 256, 128, 128, 4, 32, *base, 1.0, 1e-5, *ws) == _lib.ERR_DTYPE
    g = lib.tops_trimul_input_phase
    g.argtypes = [I, I64, I64, P, P, P, P, P, F, P, P]
    assert g(_lib.BF16, 10, 128, 16, None, 16, 16, 16, 1e-5, 16, None) == _lib.ERR_ALIGN  # M % 8 != 0
    h = lib.tops_triangle_attn_project_transposed
    h.argtypes = [I, I64, I64, I64, I64, I64, P, I, P, P, P, P, P, F, F] + [P] * 7
    assert h(_lib.BF16, 10, 130, 128, 4, 32, 16, 1, 16, 16, 16, 16, None, 1.0, 1e-5, *([P(16)] * 6), None) == \
        _lib.ERR_ALIGN  # column stride N*C*2 must be a multiple of 16
    k = lib.tops_fused_gate_residual
    k.argtypes = [I, I64, I64, P, P, P, P, P, P, P, P, I64, P]
    assert k(_lib.BF16, 100, 128, 16, 16, 16, 16, None, None, 16, 16, 7, None) == _lib.ERR_SHAPE  # T % trans_n
    o = lib.tops_trimul_output_phase_residual
    o.argtypes = [I, I64, I64, P, P, P, P, P, F, P, P, P]
    assert o(_lib.BF16, 64, 128, 16, 16, 16, 16, 16, 1e-5, None, 16, None) == _lib.ERR_ALIGN  # no residual


def test_pairformer_shape_checks_on_host():
    import torch
    import triangleops_b200 as tops

    with pytest.raises(AssertionError):
        tops.pairformer.pair_update(torch.zeros(10, 10, 128), {}, mask=None)  # N % 8
    with pytest.raises(AssertionError):
        tops.pairformer.pair_update(torch.zeros(8, 8, 128), {}, stages=("tri_mul_sideways",))


def test_transition_precompute_on_host():
    """The transition's host-side weight prep: LN affine folded per hidden chunk."""
    import triangleops_b200 as tops

    C = 128
    g = torch.Generator().manual_seed(0)
    w1, w2 = torch.randn(4 * C, C, generator=g), torch.randn(4 * C, C, generator=g)
    gamma, beta = torch.randn(C, generator=g), torch.randn(C, generator=g)
    pre = tops.transition.precompute(gamma, beta, w1, w2, torch.randn(C, 4 * C, generator=g))
    assert pre["w12"].shape == (8 * C, C) and pre["b12"].shape == (8, 2 * 64)
    # chunk 3: rows 384..447 of w12 are W1[192:256]*gamma, rows 448..511 W2[192:256]*gamma
    assert torch.allclose(pre["w12"][384:448], w1[192:256] * gamma)
    assert torch.allclose(pre["w12"][448:512], w2[192:256] * gamma)
    assert torch.allclose(pre["b12"][3, :64], w1[192:256] @ beta, atol=1e-4)
    with pytest.raises(AssertionError):
        tops.transition.precompute(gamma, beta, w1[:, :64], w2[:, :64], torch.randn(C, 4 * C))
