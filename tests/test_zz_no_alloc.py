"""The allocation-free attention-with-pair-bias entry point.

Some hosts of this library cannot hand it device workspaces: a serving runtime
or embedding framework that owns a fixed device-memory budget and forbids any
allocation once it is running. ``tops_apb_forward_noalloc`` serves them by
keeping its workspaces in a library-owned static device array (M <= 512). This
test calls it through the C ABI, twice in a row with different inputs, and
checks that each result is bit-identical to the regular ``tops_apb_forward`` on the
same inputs.
The file name sorts last so a stop-at-first-failure run has run everything else.
"""
import ctypes

import pytest
import torch

from triangleops_b200 import _lib
from triangleops_b200.attn_pair_bias.kernel import apb_core
from triangleops_b200._common.layouts import qkv_rows
from triangleops_b200._common.ln_absorption import absorb_ln_matmul

pytestmark = pytest.mark.gpu

_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_lib.register("tops_apb_forward_noalloc",
              [_I, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _F, _F, _P, _P])


def _case(M, seed, device, masked):
    g = torch.Generator().manual_seed(seed)
    C, H, D = 128, 4, 32
    r = lambda *s, sd=1.0: (torch.randn(*s, generator=g) * sd).to(device, torch.bfloat16)  # noqa: E731
    X, Z = r(M, C), r(M, M, C)
    WQ, WK, WV = (r(C, C, sd=C**-0.5) for _ in range(3))
    Wc, sW, Bc = absorb_ln_matmul(r(C, H, sd=C**-0.5), 1 + 0.1 * r(C), 0.1 * r(C), weight_dtype=torch.float32)
    km = None
    if masked:
        km = torch.ones(M, dtype=torch.bool, device=device)
        km[-37:] = False
    return X, qkv_rows(WQ, WK, WV), Z, Wc.t().contiguous(), sW, Bc.contiguous(), km


def _noalloc(X, w, Z, Wc, sW, Bc, km, scale):
    M = X.shape[0]
    og = torch.full((M, 128), float("nan"), device=X.device, dtype=X.dtype)
    m = None if km is None else km.to(torch.uint8).contiguous()
    _lib.call("tops_apb_forward_noalloc", _lib.BF16, M, 128, 128, 4, 32, X.data_ptr(), w.data_ptr(), Z.data_ptr(),
              Wc.data_ptr(), sW.data_ptr(), Bc.data_ptr(), _lib.ptr(m), scale, 1e-5, og.data_ptr(),
              _lib.stream_ptr(X.device))
    return og


def test_noalloc_matches_regular_entry_point_twice(device):
    for M, seed, masked, scale in ((512, 11, False, 1.0), (200, 12, True, 0.5)):
        X, w, Z, Wc, sW, Bc, km = _case(M, seed, device, masked)
        got = _noalloc(X, w, Z, Wc, sW, Bc, km, scale)
        ref = torch.empty(M, 128, device=device, dtype=X.dtype)
        apb_core(X, w, Z, Wc, sW, Bc, ref, 4, 32, scale=scale, key_mask=km)
        torch.cuda.synchronize()
        assert _lib.device_error()[0] == 0
        assert torch.isfinite(got).all()
        # the same kernels with the same launch shapes run on the same inputs: any
        # difference would come from the static scratch carve-up, so the bar is bit-equality
        assert torch.equal(got, ref), f"M={M}: noalloc differs from tops_apb_forward " \
            f"(max |d| {(got.double() - ref.double()).abs().max().item():.3e})"


def test_noalloc_rejects_oversize(device):
    X, w, Z, Wc, sW, Bc, km = _case(8, 1, device, False)
    rc = _lib.lib().tops_apb_forward_noalloc(_lib.BF16, 513, 128, 128, 4, 32, X.data_ptr(), w.data_ptr(),
                                             Z.data_ptr(), Wc.data_ptr(), sW.data_ptr(), Bc.data_ptr(), None, 1.0,
                                             1e-5, X.data_ptr(), _lib.stream_ptr(device))
    assert rc == _lib.ERR_CAPACITY
    assert "capacity" in _lib.status_string(rc)
