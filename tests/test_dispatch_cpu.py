"""Host logic of ``dispatch`` (no GPU): backend validation and the packed CPU mask of a grammar."""

from types import SimpleNamespace

import numpy as np
import pytest

from bitmask_speculation_b200 import workloads as wl

torch = pytest.importorskip("torch")


def test_backends_other_than_cuda_are_rejected():
    from bitmask_speculation_b200.dispatch import resolve_backend, validate_backend
    for backend in ("reference", "triton", "cpu"):
        with pytest.raises(ValueError, match="backend must be one of"):
            validate_backend(backend, torch.device("cuda"))
    if not torch.cuda.is_available():
        with pytest.raises(ValueError, match="requires NVIDIA CUDA"):
            resolve_backend("auto", torch.device("cuda"))
    with pytest.raises(ValueError, match="requires NVIDIA CUDA"):
        validate_backend("cuda", torch.device("cpu"))


def test_packed_mask_from_allowed_ids_and_from_packed_mask_agree():
    from bitmask_speculation_b200.dispatch import packed_mask
    g = wl.SyntheticDFAGrammar(1000, states=8, seed=2)
    ids = SimpleNamespace(vocab_size=1000, allowed_token_ids=g.allowed_token_ids)
    a, b = packed_mask(g), packed_mask(ids)
    assert a.dtype == torch.int32 and a.shape == ((1000 + 31) // 32,)
    assert torch.equal(a, b)
    assert a.data_ptr() != torch.from_numpy(g.packed_mask_np()).data_ptr()  # an owned copy
    bits = wl.unpack_bits_np(a.numpy()[None, :], 1000)[0]
    assert np.flatnonzero(bits).tolist() == sorted(g.allowed_token_ids())


def test_packed_mask_rejects_a_malformed_snapshot():
    from bitmask_speculation_b200.dispatch import packed_mask
    bad = SimpleNamespace(vocab_size=64, packed_mask=lambda: torch.zeros(3, dtype=torch.int32))
    with pytest.raises(ValueError, match="CPU int32 vocabulary row"):
        packed_mask(bad)
    with pytest.raises(ValueError, match="allowed token"):
        packed_mask(SimpleNamespace(vocab_size=64, allowed_token_ids=lambda: (64,)))
