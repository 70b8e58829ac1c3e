"""IO dtype contract (``triangle_ops/_common/dtype.py:7-19``).

The kernels accept fp16, bf16 and fp32 IO; anything else raises ``ValueError``
exactly as the reference does. The reference maps torch dtypes to Triton
constexprs; here they map to the C-ABI dtype codes of ``include/triangleops_b200.h``.
``TORCH_TO_TL`` / ``tl_io_dtype`` keep the reference's names for drop-in imports.
"""

import torch

from .._lib import BF16, F16, F32

TORCH_TO_IO = {
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.float32: F32,
}
TORCH_TO_TL = TORCH_TO_IO


def io_dtype(dtype: torch.dtype) -> int:
    """Return the C-ABI dtype code for a torch IO dtype, raising on unsupported."""
    try:
        return TORCH_TO_IO[dtype]
    except KeyError as e:
        raise ValueError(f"unsupported IO dtype {dtype}; expected one of {list(TORCH_TO_IO)}") from e


tl_io_dtype = io_dtype
