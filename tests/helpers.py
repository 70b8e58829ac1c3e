"""Shared test helpers: seeded inputs and the parity gate.

Parity bar for bf16/fp16 IO (the oracle is fed the same rounded inputs):
  * cosine similarity > 0.9999 against the pure-fp32 oracle, and
  * with the reference's own IO-dtype emulation at hand (the oracle evaluated with the
    reference kernels' rounding points, ``io_round=dtype``), element-wise
        |ours - fp32 oracle| <= max(ATOL, max |emulation - fp32 oracle|) + ulp(ref)
    i.e. the north-star bar ATOL = 2e-2 (fp16 1e-2) against fp32, relaxed only as far
    as the reference's own 16-bit path needs on the same inputs, plus one ulp of the IO
    dtype at the element: half for the final store into the IO dtype (the emulation
    keeps its output in fp32) and half for a different summation order at the same
    16-bit rounding points;
  * without an emulation: element-wise |delta| <= ATOL + RTOL * |ref|, RTOL = 2^-7
    (fp16 2^-10) being one ulp of the IO dtype.
fp32 IO: max relative error <= 1e-4 against the fp32 oracle.
"""
import torch

TOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2, torch.float32: 1e-4}
RTOL = {torch.bfloat16: 2.0**-7, torch.float16: 2.0**-10}
COS = 0.9999


def rnd(*shape, dtype, device, sd=0.05, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * sd).to(device=device, dtype=dtype)


def half_ulp(ref, dtype):
    """Half an ulp of the IO dtype at |ref| (element-wise): the most a correctly rounded
    store of the exact value can differ from it."""
    mant = {torch.bfloat16: 7, torch.float16: 10}[dtype]
    e = torch.floor(torch.log2(ref.abs().clamp_min(2.0**-14)))
    return torch.pow(2.0, e - mant - 1)


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
    elif ref_io is not None:
        rio = ref_io.detach().double().cpu()
        d = (out - ref).abs().max().item()
        d_ref = (rio - ref).abs().max().item()
        bar = max(TOL[dtype], d_ref) * rtol_scale + 2 * half_ulp(ref, dtype)
        excess = ((out - ref).abs() - bar).max().item()
        assert excess <= 0, (f"{what}: max|ours - fp32| = {d:.3e} exceeds max({TOL[dtype]}, reference "
                             f"emulation's {d_ref:.3e}) + ulp by {excess:.3e} (cos={cos:.7f})")
    else:
        rt = RTOL[dtype] * rtol_scale
        ex = (out - ref).abs() - (TOL[dtype] + rt * ref.abs())
        d = (out - ref).abs().max().item()
        assert ex.max().item() <= 0, f"{what}: |d| exceeds {TOL[dtype]}+{rt:.4g}|ref| (max|d| {d:.3e}, cos={cos:.7f})"
    cos_bar = COS
    if ref_io is not None and dtype != torch.float32:
        # the reference's own 16-bit path sets the bar where it is below 0.9999 itself
        cos_rio = torch.nn.functional.cosine_similarity(ref_io.detach().double().cpu().flatten(), ref.flatten(),
                                                         dim=0).item()
        cos_bar = min(COS, 1.0 - 1.5 * (1.0 - cos_rio))
    assert cos > cos_bar, f"{what}: cos={cos:.7f} (bar {cos_bar:.7f}) max|d|={d:.3e}"
    return d, cos
