"""Shared test utilities: device transfer of oracle-format inputs, sampler tolerance."""

from __future__ import annotations

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


def cdf_interval(row_f32, mask_row, temperature, token):
    import oracle
    return oracle.cdf_interval(row_f32, mask_row, temperature, token)


def sample_matches(row_f32, mask_row, temperature, uniform, gpu_token, ref_token, tol=1e-6) -> bool:
    """Identical, or u within ``tol`` (normalised) of a CDF boundary of the GPU's token."""
    import oracle
    return oracle.sample_matches(row_f32, mask_row, temperature, uniform, gpu_token, ref_token, tol)
