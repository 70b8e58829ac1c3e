"""Shared test helpers: seeded inputs and the parity gate.

Parity bar for bf16/fp16 IO (the oracle is fed the same rounded inputs):
  * cosine similarity > 0.9999 against the pure-fp32 oracle, and
  * element-wise |delta| <= ATOL + RTOL * |ref|, where ref is either the pure-fp32
    oracle or the oracle evaluated with the reference's own IO-dtype rounding points
    (``io_round=dtype``, what the reference's kernels compute): every element must be
    within the bar of at least one of the two. ATOL = 2e-2 (fp16 1e-2) is the absolute
    bar; RTOL = 2^-7 (fp16 2^-10) is one ulp of the IO dtype, so outputs of magnitude
    > 2 may differ by one rounding step.
fp32 IO: max relative error <= 1e-4 against the fp32 oracle.
"""
import torch

TOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2, torch.float32: 1e-4}
RTOL = {torch.bfloat16: 2.0**-7, torch.float16: 2.0**-10}
COS = 0.9999


def rnd(*shape, dtype, device, sd=0.05, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * sd).to(device=device, dtype=dtype)


def assert_parity(out, ref, dtype, what="", ref_io=None, rtol_scale=1.0):
    out = out.detach().double().cpu()
    ref = ref.detach().double().cpu()
    assert out.shape == ref.shape, (out.shape, ref.shape)
    assert torch.isfinite(out).all(), f"{what}: non-finite output"
    cos = torch.nn.functional.cosine_similarity(out.flatten(), ref.flatten(), dim=0).item()
    if dtype == torch.float32:
        d = (out - ref).abs().max().item()
        rel = d / max(ref.abs().max().item(), 1e-12)
        assert rel <= TOL[dtype], f"{what}: rel max err {rel:.3e}"
    else:
        rt = RTOL[dtype] * rtol_scale
        ex32 = (out - ref).abs() - (TOL[dtype] + rt * ref.abs())
        d = d32 = (out - ref).abs().max().item()
        if ref_io is not None:
            rio = ref_io.detach().double().cpu()
            exio = (out - rio).abs() - (TOL[dtype] + rt * rio.abs())
            excess = torch.minimum(ex32, exio).max().item()
            d = (out - rio).abs().max().item()
        else:
            excess = ex32.max().item()
        assert excess <= 0, (f"{what}: |d| exceeds {TOL[dtype]}+{rt:.4g}|ref| by {excess:.3e} "
                             f"(max|d| vs io-rounded {d:.3e}, vs fp32 {d32:.3e}, cos={cos:.7f})")
    assert cos > COS, f"{what}: cos={cos:.7f} max|d|={d:.3e}"
    return d, cos
