"""triangleops_b200 — B200-native (sm_100a) TriangleOps."""
__version__ = "0.1.0"
