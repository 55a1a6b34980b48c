"""CUDA primitives of the masked-selection path (no CPU fallback)."""
