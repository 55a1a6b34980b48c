"""XGrammar grammar state whose masks are written straight into the verification's staging rows.

The reference's adapter (grammar/xgrammar.py:15-90) fills a private ``[1, W]`` bitmask per query
and hands out copies; a verification round then copies those rows again, one per draft-fork
position.  ``XGrammarState`` keeps that adapter's constructor, methods, exceptions and mask
semantics (an all-valid state leaves the matcher's bitmask untouched, which the adapter reports as
every bit set; padding bits past the vocabulary may be set, and every consumer ignores them) and
adds ``fill_mask_row(out, row)``: XGrammar's ``fill_next_token_bitmask`` writes the state's mask
directly into row ``row`` of a caller's ``[B, W]`` int32 buffer -- the pinned rows of
``grammar_verification.DraftForkMasks`` -- so a round's K+1 fork masks land in the upload buffer
with no intermediate copy.  Densities are counted on the host row with a vectorised popcount.
"""

from __future__ import annotations

import numpy as np

from .kernels._validation import token_id, vocabulary_size


class GrammarTerminatedError(ValueError):
    """A mask or a token was requested after the grammar terminated (the reference's exception
    type and base class)."""


class XGrammarState:
    """Request state over an already compiled XGrammar grammar (``xgrammar.CompiledGrammar``),
    whose tokenizer vocabulary must use the model's token-ID meanings.  As in XGrammar, a stop token
    is required after the grammar body unless ``terminate_without_stop_token`` is set."""

    def __init__(self, compiled_grammar, *, terminate_without_stop_token: bool = False) -> None:
        import xgrammar as xgr

        self._vocab_size = vocabulary_size(compiled_grammar.tokenizer_info.vocab_size)
        self._matcher = xgr.GrammarMatcher(compiled_grammar,
                                           terminate_without_stop_token=terminate_without_stop_token)
        self._row = np.zeros((1, (self._vocab_size + 31) // 32), dtype=np.int32)

    @property
    def vocab_size(self) -> int:
        return self._vocab_size

    def fork(self) -> "XGrammarState":
        """An independent copy of the matcher state (for one draft round) with its own mask row."""
        branch = object.__new__(XGrammarState)
        branch._vocab_size = self._vocab_size
        branch._matcher = self._matcher.fork()
        branch._row = np.zeros_like(self._row)
        return branch

    def is_terminated(self) -> bool:
        return self._matcher.is_terminated()

    def _live(self) -> None:
        if self._matcher.is_terminated():
            raise GrammarTerminatedError("grammar has terminated")

    def fill_mask_row(self, out, row: int) -> None:
        """Write the current state's packed mask into ``out[row]`` (``out``: a C-contiguous [B, W]
        int32 numpy array or CPU tensor) without advancing the matcher."""
        self._live()
        if not self._matcher.fill_next_token_bitmask(out, row):
            out[row] = -1  # every token allowed (XGrammar left the row as it was)

    def packed_mask_np(self) -> np.ndarray:
        """The current state's packed mask as a numpy row (a private buffer, valid until the next
        query on this state)."""
        self.fill_mask_row(self._row, 0)
        return self._row[0]

    def packed_mask(self):
        """An owned CPU int32 tensor row of the current mask."""
        import torch
        return torch.from_numpy(self.packed_mask_np().copy())

    def allowed_token_ids(self) -> tuple[int, ...]:
        words = self.packed_mask_np().view(np.uint32)
        bits = np.unpackbits(words.view(np.uint8), bitorder="little")[: self._vocab_size]
        return tuple(int(t) for t in np.flatnonzero(bits))

    def mask_density(self) -> float:
        """Allowed tokens / vocabulary size (padding bits excluded), without advancing."""
        self._live()
        if not self._matcher.fill_next_token_bitmask(self._row, 0):
            return 1.0
        words = self._row[0].view(np.uint32)
        count = int(np.bitwise_count(words[:-1]).sum())
        tail = self._vocab_size % 32 or 32
        count += int(words[-1] & np.uint32((1 << tail) - 1 if tail < 32 else 0xFFFFFFFF)).bit_count()
        return count / self._vocab_size

    def accept_token(self, token: int) -> bool:
        token = token_id(token, self._vocab_size, "grammar token")
        self._live()
        return self._matcher.accept_token(token)


__all__ = ["XGrammarState", "GrammarTerminatedError"]
