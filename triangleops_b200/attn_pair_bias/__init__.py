from .kernel import apb_forward
from .module import attention_pair_bias, forward, precompute

__all__ = ["attention_pair_bias", "precompute", "forward", "apb_forward"]
