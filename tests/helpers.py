"""Shared test helpers: seeded inputs and the parity gate.

Parity bar (bf16/fp16 IO vs the fp32 CPU oracle fed the same rounded inputs):
max|delta| <= 2e-2 and cosine similarity > 0.9999 (fp16: 1e-2).
"""
import torch

TOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2, torch.float32: 1e-4}
COS = 0.9999


def rnd(*shape, dtype, device, sd=0.05, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * sd).to(device=device, dtype=dtype)


def assert_parity(out, ref, dtype, what=""):
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert out.shape == ref.shape, (out.shape, ref.shape)
    assert torch.isfinite(out).all(), f"{what}: non-finite output"
    d = (out - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(out.flatten(), ref.flatten(), dim=0).item()
    if dtype == torch.float32:
        rel = d / max(ref.abs().max().item(), 1e-12)
        assert rel <= TOL[dtype], f"{what}: rel max err {rel:.3e}"
    else:
        assert d <= TOL[dtype], f"{what}: max|d|={d:.3e} cos={cos:.6f}"
    assert cos > COS, f"{what}: cos={cos:.6f} max|d|={d:.3e}"
    return d, cos
