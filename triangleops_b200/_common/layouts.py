"""Per-head weight layouts (``triangle_ops/_common/layouts.py:11-31``).

Kept for API compatibility: the reference's ``precompute`` dicts expose these
layouts. The B200 kernels themselves consume a K-major concatenation built by
each op's ``precompute`` (see ``qkv_rows``).
"""

import torch


def interleave_qkv(WQ: torch.Tensor, WK: torch.Tensor, WV: torch.Tensor, H: int, D: int) -> torch.Tensor:
    """(C, H*D) x3 -> (C, 3*H*D); columns [3hD, 3(h+1)D) hold [Q_h | K_h | V_h]."""
    C = WQ.shape[0]
    assert WQ.shape == WK.shape == WV.shape == (C, H * D)
    parts = [W.reshape(C, H, 1, D) for W in (WQ, WK, WV)]
    return torch.cat(parts, dim=2).reshape(C, 3 * H * D).contiguous()


def interleave_kv(WK: torch.Tensor, WV: torch.Tensor, H: int, D: int) -> torch.Tensor:
    """(C, H*D) x2 -> (C, 2*H*D) feature-interleaved per head: [K0, V0, K1, V1, ...]."""
    C = WK.shape[0]
    assert WK.shape == WV.shape == (C, H * D)
    out = torch.empty(C, H, D, 2, dtype=WK.dtype, device=WK.device)
    out[..., 0] = WK.reshape(C, H, D)
    out[..., 1] = WV.reshape(C, H, D)
    return out.reshape(C, 2 * H * D)


def deinterleave_kv(WKV: torch.Tensor, H: int, D: int):
    """Inverse of :func:`interleave_kv`: (C, 2*H*D) -> WK, WV each (C, H*D)."""
    C = WKV.shape[0]
    v = WKV.reshape(C, H, D, 2)
    return v[..., 0].reshape(C, H * D), v[..., 1].reshape(C, H * D)


def qkv_rows(WQ: torch.Tensor, WK: torch.Tensor, WV: torch.Tensor, extra: torch.Tensor | None = None,
             pad_to: int = 16) -> torch.Tensor:
    """K-major concatenation consumed by the projection kernel: rows WQ^T, WK^T, WV^T
    (each (H*D, C)), then ``extra`` rows (e.g. the (H, C) bias projection), zero-padded
    to a multiple of ``pad_to`` extra rows. Matmul-convention (C, out) inputs."""
    rows = [WQ.t(), WK.t(), WV.t()]
    if extra is not None:
        pad = (-extra.shape[0]) % pad_to
        rows.append(extra)
        if pad:
            rows.append(torch.zeros(pad, extra.shape[1], dtype=extra.dtype, device=extra.device))
    return torch.cat([r.to(WQ.dtype) for r in rows], dim=0).contiguous()
