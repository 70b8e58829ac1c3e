from .kernel import contract, input_phase, output_phase
from .module import forward, precompute, triangle_multiplicative_update

__all__ = ["triangle_multiplicative_update", "precompute", "forward", "input_phase", "output_phase", "contract"]
