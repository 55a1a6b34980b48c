"""Draft budgets from grammar-mask density, on the host and on the device.

The reference sizes each speculative round from how permissive the committed grammar state is
(decoding/scheduling.py:21-46): a mask that admits few tokens makes long drafts cheap to get
right, a permissive one does not.  ``DensityPolicy`` keeps that policy's public contract -- field
names and defaults, the constructor's checks and their exception types and messages, and the
three-band ``budget`` -- because the reference's callers construct and inspect it.
``LinearDensityPolicy`` is the benchmark configuration's linear rule.

Both reach the device through ``native_policy``, which also accepts the reference's own
``DensityPolicy`` objects (anything with the four fields), so a caller that already holds one
passes it unchanged.  ``device_budgets`` evaluates a policy for a batch of packed masks on the
GPU: popcount, ``count / V`` as one IEEE double division, then the bands -- the same value as
``policy.budget(packed_mask_count(mask, V) / V)`` on the host.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from . import _native


def _check_density(value) -> None:
    # Messages and exception types match the reference's validators; its tests match on them.
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError("density must be numeric")
    if not (math.isfinite(value) and 0 <= value <= 1):
        raise ValueError("density must be finite and within [0, 1]")


def _check_budget(value) -> None:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError("draft budgets must be integers")
    if value < 1:
        raise ValueError("draft budgets must be positive")


def _check_fields(policy) -> None:
    for d in (policy.low_density, policy.high_density):
        _check_density(d)
    if not policy.low_density < policy.high_density:
        raise ValueError("density thresholds must be strictly increasing")
    for b in (policy.min_budget, policy.max_budget):
        _check_budget(b)
    if policy.max_budget < policy.min_budget:
        raise ValueError("min_budget cannot exceed max_budget")


@dataclass(frozen=True, slots=True)
class DensityPolicy:
    """Round budget K from mask density d: ``max_budget`` when d < ``low_density``, the midpoint
    ``(min_budget + max_budget) // 2`` when d < ``high_density``, else ``min_budget``."""

    low_density: float = 0.005
    high_density: float = 0.02
    min_budget: int = 1
    max_budget: int = 8

    def __post_init__(self) -> None:
        _check_fields(self)

    def budget(self, density: float) -> int:
        _check_density(density)
        if density >= self.high_density:
            return self.min_budget
        if density >= self.low_density:
            return (self.min_budget + self.max_budget) // 2
        return self.max_budget

    def native(self) -> _native.Policy:
        return native_policy(self)


@dataclass(frozen=True, slots=True)
class LinearDensityPolicy:
    """K = max_budget below low_density, min_budget above high_density, linear between."""

    low_density: float = 1e-3
    high_density: float = 0.1
    min_budget: int = 1
    max_budget: int = 8

    def __post_init__(self) -> None:
        _check_fields(self)

    def budget(self, density: float) -> int:
        _check_density(density)
        if density < self.low_density:
            return self.max_budget
        if density > self.high_density:
            return self.min_budget
        span = float(self.max_budget - self.min_budget)
        frac = (density - self.low_density) / (self.high_density - self.low_density)
        return self.max_budget - int(math.floor(span * frac))

    def native(self) -> _native.Policy:
        return native_policy(self)


def native_policy(policy) -> _native.Policy:
    """The ``bms_policy`` struct of a policy: ``LinearDensityPolicy`` -> kind 1; any other object
    with ``low_density``, ``high_density``, ``min_budget`` and ``max_budget`` (this module's
    ``DensityPolicy`` or the reference's) -> the three-band kind 0.  The fields are checked with
    the policy constructor's rules first."""
    _check_fields(policy)
    kind = 1 if isinstance(policy, LinearDensityPolicy) else 0
    return _native.Policy(kind, int(policy.min_budget), int(policy.max_budget), 0, float(policy.low_density),
                          float(policy.high_density))


def device_budgets(masks, vocab_size: int, policy=None):
    """Per-row (count int64, density float64, budget int32) CUDA tensors for [B, W] masks."""
    from .kernels._extension import load_extension
    return load_extension().mask_budget(masks, vocab_size, native_policy(DensityPolicy() if policy is None else policy))
