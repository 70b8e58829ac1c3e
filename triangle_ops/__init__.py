"""Drop-in import name: ``import triangle_ops`` resolves to the B200 implementation.

The reference's package is ``triangle_ops`` (``triangle_ops/__init__.py:17-31``); this
alias exposes ``triangleops_b200`` under that name, including its submodules
(``triangle_ops.triangle_attn``, ``triangle_ops.triangle_mul``,
``triangle_ops.attn_pair_bias``, ``triangle_ops._common``)."""

import sys as _sys

import triangleops_b200 as _impl
from triangleops_b200 import *  # noqa: F401,F403
from triangleops_b200 import _common, attn_pair_bias, triangle_attn, triangle_mul  # noqa: F401

__version__ = _impl.__version__
__all__ = list(_impl.__all__)

for _name in ("_common", "attn_pair_bias", "triangle_attn", "triangle_mul"):
    _sys.modules[f"{__name__}.{_name}"] = getattr(_impl, _name)
