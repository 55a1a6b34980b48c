"""Explicit CUDA primitives; no implicit fallback or tensor copies.

Same functions, arguments, return types and errors as the reference's
kernels/cuda.py:7-69 (``mask_count``, ``mask_density``, ``masked_argmax``,
``masked_sample``, ``batched_masked_reduce``), backed by the sm_100a library,
plus ``batched_masked_sample``.
"""

from __future__ import annotations

from dataclasses import dataclass

from ._extension import load_extension
from ._validation import (batched_selection_inputs, mask_input, selection_inputs,
                          temperature_input, uniforms_input)

_MESSAGES = {
    1: "mask has no valid token",
    2: "logits contain NaN",
    3: "uniform must be finite and in [0, 1)",
    4: "valid logits have no finite probability mass",
    5: "positive infinity is unsupported for stochastic sampling",
    7: "device wait timed out",
}


def mask_count(mask, vocab_size: int):
    """Return an owned scalar int64 CUDA tensor; no host synchronization."""
    vocab_size = mask_input(mask, vocab_size)
    return load_extension().mask_count(mask, vocab_size)


def mask_density(mask, vocab_size: int):
    """Return a scalar float64 CUDA tensor including the count and division."""
    import torch
    return mask_count(mask, vocab_size).to(torch.float64) / vocab_size


def _checked_selection(result):
    output, status = result[0], result[-1]
    code = status.item()  # Explicit host synchronization to surface value errors.
    if code in _MESSAGES:
        raise ValueError(_MESSAGES[code])
    if code != 0:
        raise RuntimeError(f"unknown native selection status: {code}")
    return output


def masked_argmax(logits, mask):
    """Return the lowest-ID valid maximum as an owned scalar int64 CUDA tensor."""
    selection_inputs(logits, mask)
    return _checked_selection(load_extension().masked_argmax(logits, mask))


def masked_sample(logits, mask, *, temperature: float = 1.0, generator=None):
    """Sample masked softmax; temperature zero uses deterministic argmax.

    Positive temperatures draw one float64 uniform on the input device using the
    supplied PyTorch generator (or its default). Checked status synchronizes.
    This is a standalone primitive, not stochastic speculative decoding.
    """
    import torch
    temperature = temperature_input(temperature)
    selection_inputs(logits, mask)
    if temperature == 0:
        return masked_argmax(logits, mask)
    native = load_extension()  # Load errors must not consume generator state.
    uniform = torch.rand((), dtype=torch.float64, device=logits.device, generator=generator)
    return _checked_selection(native.masked_sample(logits, mask, temperature, uniform))


@dataclass(frozen=True, slots=True)
class BatchedMaskedReduction:
    """Owned vectors, with one independent status per input row."""

    token_ids: object
    valid_counts: object
    status: object

    def check(self) -> "BatchedMaskedReduction":
        codes = self.status.tolist()  # One explicit device-to-host synchronization.
        errors = [(row, code) for row, code in enumerate(codes) if code]
        if errors:
            raise ValueError(f"invalid reduction rows (row, status): {errors}")
        return self


def batched_masked_reduce(logits, mask):
    """Reduce [B,V] logits and [B,ceil(V/32)] masks: argmax, valid count, status per row.

    One launch regardless of B; outputs are owned [B] tensors. No host synchronization.
    """
    batched_selection_inputs(logits, mask)
    tokens, counts, status = load_extension().masked_reduce_batch(logits, mask)
    return BatchedMaskedReduction(tokens, counts, status)


def batched_masked_sample(logits, mask, *, temperature: float, uniforms=None, generator=None):
    """Sample every row of a batch; one float64 uniform per row (drawn if not given).

    Returns a ``BatchedMaskedReduction`` (token, valid count, status per row).
    """
    import torch
    temperature = temperature_input(temperature)
    batch, _ = batched_selection_inputs(logits, mask)
    native = load_extension()
    if temperature == 0:
        tokens, counts, status = native.masked_reduce_batch(logits, mask)
        return BatchedMaskedReduction(tokens, counts, status)
    if uniforms is None:
        uniforms = torch.rand(batch, dtype=torch.float64, device=logits.device, generator=generator)
    uniforms_input(uniforms, batch, logits.device)
    tokens, counts, status = native.masked_sample_batch(logits, mask, temperature, uniforms)
    return BatchedMaskedReduction(tokens, counts, status)
