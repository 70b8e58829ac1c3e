"""Single-tile checks of each tcgen05 operand mode against a plain fp32 matmul."""
import ctypes

import pytest
import torch

from triangleops_b200 import _lib

pytestmark = pytest.mark.gpu


def _run(mode, a, b, n_out):
    d = torch.full((128, n_out), float("nan"), device=a.device, dtype=torch.float32)
    _lib.call("tops_selftest_umma", mode, a.data_ptr(), b.data_ptr(), d.data_ptr(), _lib.stream_ptr())
    torch.cuda.synchronize()
    st, site = _lib.device_error()
    assert st == 0, f"device wait timeout at site {site}"
    return d


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_umma_mode(device, mode):
    g = torch.Generator(device="cpu").manual_seed(mode)
    if mode == 0:
        a = torch.randn(128, 64, generator=g)
        b = torch.randn(128, 64, generator=g)
        ref = a.bfloat16().float() @ b.bfloat16().float().T
        n = 128
    elif mode == 1:
        a = torch.randn(128, 32, generator=g)
        b = torch.randn(64, 32, generator=g)
        ref = a.bfloat16().float() @ b.bfloat16().float().T
        n = 64
    elif mode == 2:
        a = torch.randn(64, 128, generator=g)
        b = torch.randn(64, 128, generator=g)
        ref = a.bfloat16().float().T @ b.bfloat16().float()
        n = 128
    else:
        a = torch.randn(128, 64, generator=g)
        b = torch.randn(48, 64, generator=g)
        ref = a.bfloat16().float() @ b.bfloat16().float().T
        n = 48
    out = _run(mode, a.bfloat16().to(device).contiguous(), b.bfloat16().to(device).contiguous(), n)
    err = (out.cpu() - ref).abs().max().item()
    assert err < 1e-3, f"mode {mode}: max|err|={err}"
