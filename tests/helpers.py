"""Shared test utilities: device transfer of oracle-format inputs, sampler tolerance."""

from __future__ import annotations

import math

import numpy as np

TORCH_DTYPE_NAMES = ("float32", "bfloat16", "float16")


def to_device(values: np.ndarray, dtype: str, device="cuda"):
    """numpy float32 values or uint16 bit patterns -> torch tensor of ``dtype`` on ``device``."""
    import torch
    if dtype == "float32":
        return torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to(device)
    bits = torch.from_numpy(np.ascontiguousarray(values, dtype=np.uint16).view(np.int16))
    return bits.view(getattr(torch, dtype)).to(device)


def as_dtype_bits(values_f32: np.ndarray, dtype: str) -> np.ndarray:
    from bitmask_speculation_b200 import workloads as wl
    if dtype == "float32":
        return np.ascontiguousarray(values_f32, dtype=np.float32)
    if dtype == "bfloat16":
        return wl.to_bf16_bits(values_f32)
    return wl.to_f16_bits(values_f32)


def widened(values: np.ndarray, dtype: str) -> np.ndarray:
    import oracle
    if dtype == "float32":
        return np.ascontiguousarray(values, dtype=np.float32)
    return oracle.widen(values, dtype)


def cdf_interval(row_f32: np.ndarray, mask_row: np.ndarray, temperature: float, token: int):
    """Normalised CDF interval [F(token-), F(token)] of the reference sampler (fp64)."""
    vocab = row_f32.size
    words = np.ascontiguousarray(mask_row, dtype=np.int32).view(np.uint32)
    t = np.arange(vocab)
    valid = ((words[t >> 5] >> (t & 31).astype(np.uint32)) & 1).astype(bool)
    x = row_f32.astype(np.float64)
    finite = valid & np.isfinite(x)
    m = x[valid].max()
    w = np.zeros(vocab)
    with np.errstate(over="ignore", invalid="ignore"):
        w[finite] = np.exp((x[finite] - m) / temperature)
    total = math.fsum(w[valid])
    cum = np.cumsum(w)
    hi = cum[token] / total
    lo = (cum[token] - w[token]) / total
    return lo, hi


def sample_matches(row_f32, mask_row, temperature, uniform, gpu_token, ref_token, tol=1e-6) -> bool:
    """Identical, or u within ``tol`` (normalised) of a CDF boundary of the GPU's token."""
    if gpu_token == ref_token:
        return True
    if gpu_token < 0:
        return False
    lo, hi = cdf_interval(row_f32, mask_row, temperature, gpu_token)
    if hi <= lo:  # zero-weight token can never be drawn
        return False
    dist = 0.0 if lo <= uniform < hi else min(abs(uniform - lo), abs(uniform - hi))
    return dist <= tol
