"""Tensor-level selection calls over the sm_100a library.

The functions a caller of the reference imports from kernels/cuda.py:7-69 --
``mask_count``, ``mask_density``, ``masked_argmax``, ``masked_sample`` and
``batched_masked_reduce`` -- with the same arguments, return types and errors,
plus ``batched_masked_sample`` (one uniform per row).  Inputs must already be on
the GPU: nothing here copies, widens or moves a tensor, and a missing library is
an error, never a CPU computation.
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
    """Valid tokens of one packed mask row, as a new 0-d int64 tensor on the mask's device.
    Enqueued on the current stream; the host does not wait."""
    vocab_size = mask_input(mask, vocab_size)
    return load_extension().mask_count(mask, vocab_size)


def mask_density(mask, vocab_size: int):
    """``mask_count / vocab_size`` as a 0-d float64 tensor on the device (no host wait)."""
    import torch
    return mask_count(mask, vocab_size).to(torch.float64) / vocab_size


def _checked_selection(result):
    output, status = result[0], result[-1]
    code = status.item()  # the one device->host read of the call
    if code in _MESSAGES:
        raise ValueError(_MESSAGES[code])
    if code != 0:
        raise RuntimeError(f"unknown native selection status: {code}")
    return output


def masked_argmax(logits, mask):
    """Highest-scoring allowed token of one row (ties: smallest ID) as a new 0-d int64 tensor.
    Reads the status back to the host once, raising ValueError for NaN or an empty mask."""
    selection_inputs(logits, mask)
    return _checked_selection(load_extension().masked_argmax(logits, mask))


def masked_sample(logits, mask, *, temperature: float = 1.0, generator=None):
    """Draw one allowed token from softmax(logits / temperature) by inverse CDF.

    ``temperature == 0`` is ``masked_argmax``.  Otherwise one float64 uniform is
    drawn on the logits' device from ``generator`` (the device default if None),
    after the library is loaded so that a load failure leaves the generator
    untouched.  The status is read back once (ValueError on a data error).  One
    row, one draw: speculative acceptance lives elsewhere.
    """
    import torch
    temperature = temperature_input(temperature)
    selection_inputs(logits, mask)
    if temperature == 0:
        return masked_argmax(logits, mask)
    native = load_extension()  # before the draw: a failed load leaves the generator as it was
    uniform = torch.rand((), dtype=torch.float64, device=logits.device, generator=generator)
    return _checked_selection(native.masked_sample(logits, mask, temperature, uniform))


@dataclass(frozen=True, slots=True)
class BatchedMaskedReduction:
    """Per-row results of a batched call: token (-1 on error), valid count, status code.
    ``check()`` reads the statuses back once and raises ValueError listing failed rows."""

    token_ids: object
    valid_counts: object
    status: object

    def check(self) -> "BatchedMaskedReduction":
        codes = self.status.tolist()  # reads every row's status back in one transfer
        errors = [(row, code) for row, code in enumerate(codes) if code]
        if errors:
            raise ValueError(f"invalid reduction rows (row, status): {errors}")
        return self


def batched_masked_reduce(logits, mask):
    """Masked argmax, valid-token count and status of every row of a [B, V] batch under its
    [B, ceil(V/32)] masks, as new [B] tensors on the device.  The whole batch is one selection
    launch; the host does not wait."""
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
