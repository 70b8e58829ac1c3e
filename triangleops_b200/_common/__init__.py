"""Shared host-side helpers of the three ops (mirrors ``triangle_ops/_common``)."""

from .dtype import TORCH_TO_IO, TORCH_TO_TL, io_dtype, tl_io_dtype
from .layouts import interleave_kv, interleave_qkv
from .ln_absorption import absorb_ln, absorb_ln_matmul

__all__ = [
    "TORCH_TO_IO",
    "TORCH_TO_TL",
    "io_dtype",
    "tl_io_dtype",
    "absorb_ln",
    "absorb_ln_matmul",
    "interleave_qkv",
    "interleave_kv",
]
