from .host import HostPipeline
from .kernel import fused_gate_forward, triangle_attn_forward
from .module import forward, precompute, triangle_attention

__all__ = ["triangle_attention", "precompute", "forward", "triangle_attn_forward", "fused_gate_forward",
           "HostPipeline"]
