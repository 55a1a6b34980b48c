"""Grammar-constrained token selection for one row of model scores.

The reference's ``select_token`` (kernels/dispatch.py:79-103) is what its Transformers adapter calls
for every draft step and every verified row (models/transformers.py:131-145).  On its CUDA backend
each call copies the grammar's CPU mask to the device, widens fp16/bf16 scores to a float32 copy,
launches the two-kernel argmax and reads the token back.  Here:

* scores stay in their own dtype (float32, bfloat16 or float16): the kernel reads them directly,
  so no widening copy is made (a non-contiguous row is made contiguous, nothing else);
* the mask reaches the device through a pinned staging row (one 31 KB asynchronous copy at
  V = 248,320), or not at all when the caller passes the grammar's ``DeviceMaskTable``: the state's
  mask is then a row of that table;
* one kernel selects, and the token and status come back in one synchronization.

Same arguments, result and exceptions as the reference for the ``cuda`` backend: the selected
token as an ``int``, ``TypeError`` for other score dtypes, ``ValueError`` for an empty mask or NaN
scores; the grammar is not advanced.  The other backends of the reference (its CPU ``reference``
path and Triton) are not part of this library, and no CPU fallback exists.
"""

from __future__ import annotations

import threading

import numpy as np

from .grammar_verification import _mask_row

BACKENDS = ("cuda",)
_STATUS_MESSAGES = {1: "mask has no valid token", 2: "logits contain NaN", 7: "device wait timed out"}
_local = threading.local()


def validate_backend(backend, device) -> None:
    """``ValueError`` unless ``backend`` is ``"cuda"`` and ``device`` is a CUDA device here."""
    import torch
    if backend not in BACKENDS:
        raise ValueError(f"backend must be one of {BACKENDS}")
    if device.type != "cuda" or not torch.cuda.is_available() or torch.version.hip is not None:
        raise ValueError(f"{backend} backend requires NVIDIA CUDA")


def resolve_backend(backend, device) -> str:
    """``"auto"`` and ``"cuda"`` resolve to ``"cuda"`` (validated); anything else is an error."""
    backend = "cuda" if backend == "auto" else backend
    validate_backend(backend, device)
    return backend


def packed_mask(grammar):
    """The grammar's allowed set as an owned CPU int32 row of ceil(V / 32) words: its own
    ``packed_mask()`` when it has one (checked and copied), else built from ``allowed_token_ids()``."""
    import torch
    from .kernels._validation import vocabulary_size
    vocab = vocabulary_size(grammar.vocab_size)
    snapshot = getattr(grammar, "packed_mask", None)
    if snapshot is not None:
        mask = snapshot()
        if (not isinstance(mask, torch.Tensor) or mask.dtype != torch.int32 or mask.device.type != "cpu"
                or mask.layout != torch.strided or mask.ndim != 1 or mask.numel() != (vocab + 31) // 32):
            raise ValueError("grammar packed_mask must return a CPU int32 vocabulary row")
        return mask.clone().contiguous()
    return torch.from_numpy(np.array(_mask_row(grammar, vocab), dtype=np.int32))


class _Staging:
    """Per-thread, per-device pinned rows for the mask upload and the (token, status) read-back."""

    def __init__(self, device, words: int):
        import torch
        self.words = words
        self.host_mask = torch.zeros(words, dtype=torch.int32).pin_memory()
        self.dev_mask = torch.empty(words, dtype=torch.int32, device=device)
        self.host_token = torch.zeros(1, dtype=torch.int64).pin_memory()
        self.host_status = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.mask_np = self.host_mask.numpy()


def _staging(device, words: int) -> _Staging:
    cache = getattr(_local, "staging", None)
    if cache is None:
        cache = _local.staging = {}
    key = (device.index, words)
    st = cache.get(key)
    if st is None:
        st = cache[key] = _Staging(device, words)
    return st


def select_token(scores, grammar, backend="cuda", *, workspace=None, table=None) -> int:
    """Masked argmax of one row of scores under the grammar's current state (lowest token ID on
    ties), without advancing the grammar.

    ``scores``: a 1-D CUDA tensor of V float32 / bfloat16 / float16 scores.  ``table``: optional
    ``DeviceMaskTable`` of a grammar with a finite state set (``state_index()``); the state's mask
    is then read on the device and nothing is uploaded.  Returns the token ID; raises
    ``ValueError`` for an empty mask or NaN anywhere in the row.
    """
    import torch
    from .kernels._extension import load_extension
    validate_backend(backend, scores.device)
    if workspace is not None:
        raise ValueError("workspace is only supported by the Triton backend")
    if scores.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("native selection accepts float16, bfloat16 or float32 logits")
    if scores.ndim != 1 or scores.numel() == 0:
        raise ValueError("scores must be a nonempty one-dimensional tensor")
    from .kernels._validation import vocabulary_size
    vocab = vocabulary_size(grammar.vocab_size)
    if scores.numel() != vocab:
        raise ValueError("scores and grammar vocabularies differ")
    dev = scores.device
    words = (vocab + 31) // 32
    native = load_extension()
    st = _staging(dev, words)
    stream = torch.cuda.current_stream(dev)
    try:
        if table is not None and hasattr(grammar, "state_index"):
            idx = grammar.state_index()
            mask = table.table[idx if idx >= 0 else table.empty]
        else:
            st.mask_np[:] = _mask_row(grammar, vocab)
            st.dev_mask.copy_(st.host_mask, non_blocking=True)
            mask = st.dev_mask
        token, status = native.masked_argmax(scores.contiguous(), mask)
        st.host_token.copy_(token.view(1), non_blocking=True)
        st.host_status.copy_(status.view(1), non_blocking=True)
    finally:
        stream.synchronize()  # the staging rows are free again, whatever happened
    code = int(st.host_status[0])
    if code:
        raise ValueError(_STATUS_MESSAGES.get(code, f"native selection status {code}"))
    return int(st.host_token[0])


__all__ = ["BACKENDS", "validate_backend", "resolve_backend", "packed_mask", "select_token"]
