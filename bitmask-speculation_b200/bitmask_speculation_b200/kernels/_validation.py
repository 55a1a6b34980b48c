"""Argument checks that run before anything is launched (tensor metadata only: no data is read,
copied or moved).

The checks, their order, exception types and messages are the reference's (kernels/_validation.py:
6-60), because its callers and tests match on them.  Two checks are relaxed on purpose: float16 and
bfloat16 logits pass (the kernels read them as they are), and a batch may hold more than 65,535
rows.  ``uniforms_input`` is new: the batched sampler takes one float64 uniform per row.
"""

from __future__ import annotations

import math

_FLOAT_DTYPES = None


def _float_dtypes():
    global _FLOAT_DTYPES
    if _FLOAT_DTYPES is None:
        import torch
        _FLOAT_DTYPES = (torch.float32, torch.bfloat16, torch.float16)
    return _FLOAT_DTYPES


def vocabulary_size(value) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError("vocab_size must be an integer")
    if value <= 0:
        raise ValueError("vocab_size must be positive")
    return value


def token_id(value, vocab_size: int, name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{name} must be an integer token ID")
    if not 0 <= value < vocab_size:
        raise ValueError(f"{name} must be in [0, {vocab_size})")
    return value


def mask_input(mask, vocab_size):
    import torch
    vocab_size = vocabulary_size(vocab_size)
    if vocab_size > 2147483647:
        raise ValueError("vocab_size exceeds the native int32 index range")
    if not isinstance(mask, torch.Tensor) or mask.dtype != torch.int32:
        raise TypeError("mask must be an int32 tensor")
    if mask.layout != torch.strided or mask.ndim != 1 or not mask.is_contiguous():
        raise ValueError("mask must be a contiguous one-dimensional strided tensor")
    if mask.numel() != (vocab_size + 31) // 32:
        raise ValueError("mask word count must equal ceil(vocab_size / 32)")
    if mask.device.type != "cuda":
        raise ValueError("mask must be on CUDA; no implicit transfer")
    return vocab_size


def selection_inputs(logits, mask):
    import torch
    if not isinstance(logits, torch.Tensor) or logits.dtype not in _float_dtypes():
        raise TypeError("logits must be a float32, bfloat16 or float16 tensor")
    if logits.layout != torch.strided or logits.ndim != 1 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous one-dimensional strided tensor")
    vocab_size = mask_input(mask, logits.numel())
    if logits.device != mask.device:
        raise ValueError("logits and mask must be on the same CUDA device")
    return vocab_size


def temperature_input(temperature):
    if isinstance(temperature, bool) or not isinstance(temperature, (int, float)):
        raise TypeError("temperature must be numeric")
    if not math.isfinite(temperature) or temperature < 0:
        raise ValueError("temperature must be finite and nonnegative")
    return float(temperature)


def batched_selection_inputs(logits, mask):
    import torch
    if not isinstance(logits, torch.Tensor) or logits.dtype not in _float_dtypes():
        raise TypeError("logits must be a float32, bfloat16 or float16 tensor")
    if not isinstance(mask, torch.Tensor) or mask.dtype != torch.int32:
        raise TypeError("mask must be an int32 tensor")
    for value in (logits, mask):
        if value.layout != torch.strided or value.ndim != 2 or not value.is_contiguous():
            raise ValueError("batch inputs must be contiguous two-dimensional strided tensors")
    batch, vocab = logits.shape
    vocabulary_size(vocab)
    if vocab > 2147483647:
        raise ValueError("vocab_size exceeds the native int32 index range")
    if tuple(mask.shape) != (batch, (vocab + 31) // 32):
        raise ValueError("mask shape must be [batch, ceil(vocab_size / 32)]")
    if logits.device.type != "cuda" or logits.device != mask.device:
        raise ValueError("batch inputs must be on the same CUDA device")
    return batch, vocab


def uniforms_input(uniforms, batch: int, device):
    import torch
    if not isinstance(uniforms, torch.Tensor) or uniforms.dtype != torch.float64:
        raise TypeError("uniforms must be a float64 tensor")
    if uniforms.ndim != 1 or uniforms.numel() != batch or not uniforms.is_contiguous():
        raise ValueError("uniforms must be a contiguous [batch] tensor")
    if uniforms.device != device:
        raise ValueError("uniforms must be on the logits device")
    return uniforms
