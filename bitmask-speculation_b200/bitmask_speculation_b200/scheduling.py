"""Draft budgets from grammar-mask density, on the host and on the device.

``DensityPolicy`` is the reference's three-band policy (decoding/scheduling.py:
21-46) with identical fields, validation and ``budget``; ``LinearDensityPolicy``
is the linear schedule (K = max below ``low_density``, K = min above
``high_density``, ``max - floor((max - min) * (d - low) / (high - low))`` in
between).  ``device_budgets`` evaluates either policy for a batch of packed
masks on the GPU (popcount, ``count / V`` in IEEE double, budget), bit-identical
to ``policy.budget(packed_mask_count(mask, V) / V)``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from . import _native


def _density(value) -> None:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError("density must be numeric")
    if not math.isfinite(value) or not 0 <= value <= 1:
        raise ValueError("density must be finite and within [0, 1]")


def _budget(value) -> None:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError("draft budgets must be integers")
    if value < 1:
        raise ValueError("draft budgets must be positive")


@dataclass(frozen=True, slots=True)
class DensityPolicy:
    """Three configurable density bands; thresholds are experiment parameters."""

    low_density: float = 0.005
    high_density: float = 0.02
    min_budget: int = 1
    max_budget: int = 8

    def __post_init__(self) -> None:
        _density(self.low_density)
        _density(self.high_density)
        if self.low_density >= self.high_density:
            raise ValueError("density thresholds must be strictly increasing")
        _budget(self.min_budget)
        _budget(self.max_budget)
        if self.min_budget > self.max_budget:
            raise ValueError("min_budget cannot exceed max_budget")

    def budget(self, density: float) -> int:
        _density(density)
        if density < self.low_density:
            return self.max_budget
        if density < self.high_density:
            return (self.min_budget + self.max_budget) // 2
        return self.min_budget

    def native(self) -> _native.Policy:
        return _native.Policy(0, self.min_budget, self.max_budget, 0, float(self.low_density),
                              float(self.high_density))


@dataclass(frozen=True, slots=True)
class LinearDensityPolicy:
    """K = max_budget below low_density, min_budget above high_density, linear between."""

    low_density: float = 1e-3
    high_density: float = 0.1
    min_budget: int = 1
    max_budget: int = 8

    def __post_init__(self) -> None:
        DensityPolicy.__post_init__(self)  # same field contract

    def budget(self, density: float) -> int:
        _density(density)
        if density < self.low_density:
            return self.max_budget
        if density > self.high_density:
            return self.min_budget
        span = float(self.max_budget - self.min_budget)
        frac = (density - self.low_density) / (self.high_density - self.low_density)
        return self.max_budget - int(math.floor(span * frac))

    def native(self) -> _native.Policy:
        return _native.Policy(1, self.min_budget, self.max_budget, 0, float(self.low_density),
                              float(self.high_density))


def device_budgets(masks, vocab_size: int, policy=None):
    """Per-row (count int64, density float64, budget int32) CUDA tensors for [B, W] masks."""
    from .kernels._extension import load_extension
    policy = DensityPolicy() if policy is None else policy
    return load_extension().mask_budget(masks, vocab_size, policy.native())
