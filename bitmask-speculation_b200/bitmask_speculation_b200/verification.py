"""Batched K+1-row verification: one launch pair per round instead of one per row.

The reference verifies lazily, one masked argmax per row with a host sync each
(models/transformers.py:181-201 feeding decoding/verification.py:18-48).  Here
all rows of all sequences are reduced in one streaming kernel and a small
epilogue applies longest-prefix acceptance on the device; the host receives,
per sequence, the accepted length, the correction / bonus / fallback token and a
status, plus per-row counts and draft budgets.

``events`` replays one sequence as the reference's ``VerifiedToken`` stream:
accepted proposals, then exactly one correction / bonus / fallback.  A failed
row that the reference would have consumed raises the reference's ``ValueError``
at the point the reference raised it; failed rows after the first mismatch are
never surfaced (tests/integration/test_transformers_verification.py:43-60).
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from dataclasses import dataclass
from typing import Literal

from .kernels._validation import batched_selection_inputs, token_id
from .scheduling import DensityPolicy, native_policy

KINDS = {0: "correction", 1: "bonus", 2: "fallback"}
_ROW_ERRORS = {
    1: "mask has no valid token",
    2: "next-token logits contain NaN",
    6: "proposal count outside [0, K]",
    7: "device wait timed out",
    8: "mask row index outside the mask table",
}


@dataclass(frozen=True, slots=True)
class VerifiedToken:
    """An event of a verified round: ``token_id`` and how the target confirmed it ("accepted"
    draft token, "correction" at the first mismatch, "bonus" after a fully accepted draft, or
    "fallback" for an empty draft).  Same fields and kinds as the reference's type
    (decoding/verification.py:10-15), so its request loops consume these events unchanged; EOS,
    length limits and grammar termination are the caller's business."""

    token_id: int
    kind: Literal["accepted", "correction", "bonus", "fallback"]


@dataclass(frozen=True, slots=True)
class BatchVerification:
    """Device tensors of one verification round (no host synchronization yet)."""

    row_tokens: object
    row_counts: object
    row_status: object
    row_budget: object
    accept_len: object
    token: object
    kind: object
    seq_status: object

    def to_host(self) -> "HostVerification":
        import torch
        with torch.cuda.device(self.token.device):
            torch.cuda.current_stream().synchronize()
        return HostVerification(**{f: getattr(self, f).tolist() for f in self.__slots__})


@dataclass(frozen=True, slots=True)
class HostVerification:
    row_tokens: list
    row_counts: list
    row_status: list
    row_budget: list
    accept_len: list
    token: list
    kind: list
    seq_status: list

    def events(self, seq: int, proposals: Sequence[int]) -> Iterator[VerifiedToken]:
        """Reference-ordered events of sequence ``seq`` (lazy failure on consumed rows)."""
        accepted = self.accept_len[seq]
        status = self.seq_status[seq]
        draft = tuple(proposals)

        def gen():
            for i in range(accepted):
                yield VerifiedToken(int(draft[i]), "accepted")
            if status:
                raise ValueError(_ROW_ERRORS.get(status, f"verification row status {status}"))
            yield VerifiedToken(int(self.token[seq]), KINDS[self.kind[seq]])

        return gen()


def verify_batch(logits, masks, proposals, lengths, *, policy=None, mask_rows=None) -> BatchVerification:
    """Verify S sequences of K drafts against S*(K+1) target rows.

    ``logits`` [S*(K+1), V] (float32 / bfloat16 / float16), ``masks``
    [S*(K+1), ceil(V/32)] int32 with row ``s*(K+1)+i`` the grammar state after
    ``proposals[s, :i]``, ``proposals`` int64 [S, K], ``lengths`` int32 [S]
    (live proposals per sequence, at most K).  ``policy`` (default
    ``DensityPolicy()``) turns each row's popcount into a draft budget.  With
    ``mask_rows`` (int32 [S*(K+1)] on the device), ``masks`` is a device-resident
    table of mask rows (e.g. one per grammar state) and row r uses ``masks[mask_rows[r]]``;
    an index outside the table fails the row with status 8.
    """
    from .kernels._extension import load_extension
    if mask_rows is None:
        batched_selection_inputs(logits, masks)
    policy = DensityPolicy() if policy is None else policy
    out = load_extension().verify_batch(logits, masks, proposals, lengths, native_policy(policy), mask_rows=mask_rows)
    return BatchVerification(**out)


def verify_rows(proposals: Sequence[int], logits, masks, *, policy=None) -> Iterator[VerifiedToken]:
    """One sequence: the batched equivalent of ``verify_prefix`` over ``len+1`` rows.

    ``logits``/``masks`` hold the rows the reference's ``_choices`` would select
    from, in order (row i predicts proposal i, row len(proposals) the bonus).
    Proposal IDs are validated before anything is launched.
    """
    import torch
    vocab = logits.shape[1]
    draft = tuple(token_id(t, vocab, "proposal token") for t in proposals)
    k = len(draft)
    if logits.shape[0] != k + 1 or masks.shape[0] != k + 1:
        raise ValueError("verification needs len(proposals) + 1 rows")
    prop = torch.tensor([draft], dtype=torch.int64, device=logits.device).reshape(1, k)
    lengths = torch.tensor([k], dtype=torch.int32, device=logits.device)
    host = verify_batch(logits, masks, prop, lengths, policy=policy).to_host()
    return host.events(0, draft)
