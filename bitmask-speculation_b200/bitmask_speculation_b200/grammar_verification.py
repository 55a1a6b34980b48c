"""Grammar-constrained verification of a draft in one batched round.

The reference verifies a draft lazily: ``_choices`` (models/transformers.py:181-201) selects row
``start + i`` under the committed grammar, advances it with ``accept_token`` and stops at the first
mismatch or at termination, with one host round trip per row and a CPU mask copied to the device
for every selection (kernels/dispatch.py:95-96).  Because every row the reference consumes before
the first mismatch selects the draft's own token, row i's grammar state is the state after
``proposals[:i]``.  Here the K+1 states are obtained by forking the grammar along the draft, their
packed masks are written into one pinned host buffer, copied to the device in one transfer and
verified with one ``verify_batch`` launch pair and one host synchronization; the events are then
replayed against the committed grammar exactly as the reference's loop produces them (each
selected token accepted in turn, stopping once the grammar terminates, a failed row raising
lazily when it is reached).
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence

import numpy as np

from .kernels._validation import token_id
from .verification import VerifiedToken, verify_batch


def _mask_row(grammar, vocab: int) -> np.ndarray:
    """The grammar's packed mask (reference dispatch.packed_mask semantics) as int32 words."""
    words = (vocab + 31) // 32
    fast = getattr(grammar, "packed_mask_np", None)
    if fast is not None:
        return fast()
    snapshot = getattr(grammar, "packed_mask", None)
    if snapshot is not None:
        mask = snapshot()
        arr = mask.numpy() if hasattr(mask, "numpy") else np.asarray(mask)
        if arr.dtype != np.int32 or arr.shape != (words,):
            raise ValueError("grammar packed_mask must return a CPU int32 vocabulary row")
        return arr
    ids = np.fromiter((token_id(t, vocab, "allowed token") for t in grammar.allowed_token_ids()), dtype=np.int64)
    row = np.zeros(words, dtype=np.uint32)
    np.bitwise_or.at(row, ids >> 5, (np.uint32(1) << (ids & 31).astype(np.uint32)))
    return row.view(np.int32)


def _write_mask_row(grammar, vocab: int, out: np.ndarray, row: int) -> None:
    """The grammar's mask into ``out[row]``: written in place by grammars that can
    (``fill_mask_row``, e.g. ``xgrammar_state.XGrammarState``), else copied from ``_mask_row``."""
    fill = getattr(grammar, "fill_mask_row", None)
    if fill is not None:
        fill(out, row)
    else:
        out[row] = _mask_row(grammar, vocab)


def fork_masks(grammar, draft: Sequence[int], vocab: int, out: np.ndarray) -> int:
    """Write into ``out[: len(draft) + 1]`` the packed masks of the committed state and of the
    state after each draft prefix (rows a fork cannot reach -- after a proposal it rejects, or
    after it terminates -- are empty; the reference never consumes them).  Returns the rows."""
    rows = len(draft) + 1
    if rows > out.shape[0]:
        raise ValueError("draft longer than the buffer")
    fork = grammar.fork()
    _write_mask_row(fork, vocab, out, 0)
    live = not fork.is_terminated()
    for i, proposal in enumerate(draft):
        live = live and fork.accept_token(proposal) and not fork.is_terminated()
        if live:
            _write_mask_row(fork, vocab, out, i + 1)
        else:
            out[i + 1] = 0
    return rows


def fork_state_indices(grammar, draft: Sequence[int], out: np.ndarray, empty: int) -> int:
    """Like ``fork_masks`` for a grammar with a finite state set (``mask_table()`` /
    ``state_index()``): write into ``out[: len(draft) + 1]`` the table rows of the fork states,
    ``empty`` for rows a fork cannot reach.  Returns the rows."""
    rows = len(draft) + 1
    fork = grammar.fork()
    idx = fork.state_index()
    out[0] = idx if idx >= 0 else empty
    live = idx >= 0
    for i, proposal in enumerate(draft):
        live = live and fork.accept_token(proposal) and not fork.is_terminated()
        out[i + 1] = fork.state_index() if live else empty
    return rows


class DeviceMaskTable:
    """Device-resident masks of a grammar's finite state set (plus one empty row), so that a round
    uploads one int32 table index per row instead of its mask words."""

    def __init__(self, table: np.ndarray, max_rows: int, device):
        import torch
        table = np.ascontiguousarray(table, dtype=np.int32)
        self.empty = table.shape[0]
        full = np.vstack([table, np.zeros((1, table.shape[1]), dtype=np.int32)])
        self.table = torch.from_numpy(full).to(device)
        self.host = torch.zeros(max_rows, dtype=torch.int32).pin_memory()
        self.device = torch.empty(max_rows, dtype=torch.int32, device=device)
        self._host_np = self.host.numpy()

    @classmethod
    def for_grammar(cls, grammar, max_rows: int, device) -> "DeviceMaskTable":
        return cls(grammar.mask_table(), max_rows, device)

    def upload(self, rows: int):
        dev = self.device[:rows]
        dev.copy_(self.host[:rows], non_blocking=True)
        return dev


class DraftForkMasks:
    """Pinned host staging and device buffer for the packed masks of K+1 draft-fork states."""

    def __init__(self, vocab: int, max_rows: int, device):
        import torch
        self.vocab = int(vocab)
        self.words = (self.vocab + 31) // 32
        self.host = torch.zeros((max_rows, self.words), dtype=torch.int32).pin_memory()
        self.device = torch.empty((max_rows, self.words), dtype=torch.int32, device=device)
        self._host_np = self.host.numpy()

    def fill(self, grammar, draft: Sequence[int]) -> int:
        """``fork_masks`` into the pinned staging buffer; returns len(draft) + 1."""
        return fork_masks(grammar, draft, self.vocab, self._host_np)

    def upload(self, rows: int):
        """One asynchronous host-to-device copy on the current stream."""
        dev = self.device[:rows]
        dev.copy_(self.host[:rows], non_blocking=True)
        return dev


def verify_with_grammar(draft: Sequence[int], logits, grammar, *, buffer: DraftForkMasks | None = None,
                        policy=None) -> Iterator[VerifiedToken]:
    """Batched equivalent of the reference's ``_choices(draft, logits, start, grammar)``.

    ``logits`` are the K+1 target rows (row i predicts proposal i, row K the bonus) on the
    device; ``grammar`` is the committed ``ForkableGrammarState`` and is advanced by the events
    as they are consumed, exactly as the reference advances it.  One host synchronization per
    round (the ``to_host`` of the batched result).
    """
    import torch
    vocab = logits.shape[1]
    draft = tuple(token_id(t, vocab, "proposal token") for t in draft)
    if logits.shape[0] != len(draft) + 1:
        raise ValueError("verification needs len(proposals) + 1 rows")
    if getattr(grammar, "vocab_size", vocab) != vocab:
        raise ValueError("grammar and model vocabularies differ")
    if grammar.is_terminated():
        return iter(())
    buf = buffer if buffer is not None else DraftForkMasks(vocab, len(draft) + 1, logits.device)
    masks = buf.upload(buf.fill(grammar, draft))
    k = len(draft)
    prop = torch.tensor([draft], dtype=torch.int64).reshape(1, k).to(logits.device, non_blocking=True)
    lengths = torch.tensor([k], dtype=torch.int32).to(logits.device, non_blocking=True)
    host = verify_batch(logits, masks, prop, lengths, policy=policy).to_host()
    events = host.events(0, draft)

    def constrained() -> Iterator[VerifiedToken]:
        while not grammar.is_terminated():
            event = next(events, None)
            if event is None:
                return
            if not grammar.accept_token(event.token_id):
                raise ValueError("grammar rejected its selected token")
            yield event

    return constrained()


def verify_with_grammars(drafts: Sequence[Sequence[int]], logits, grammars, *, k: int,
                         buffer: DraftForkMasks | None = None, table: DeviceMaskTable | None = None,
                         policy=None) -> list[Iterator[VerifiedToken]]:
    """One verification round for S sequences: one host-to-device mask copy, one ``verify_batch``
    launch pair and one host synchronization for the whole batch.

    ``logits`` [S*(k+1), V] on the device, row ``s*(k+1) + i`` predicting proposal i of sequence s
    (row ``s*(k+1) + len(drafts[s])`` its bonus); ``grammars[s]`` the committed grammar of sequence
    s, advanced by its iterator as the reference's loop would.  Sequences whose grammar has
    terminated get an empty iterator.  With ``table`` (grammars sharing one finite state set, see
    ``DeviceMaskTable``) the round uploads one int32 table index per row instead of mask words.
    """
    import torch
    seqs = len(drafts)
    if len(grammars) != seqs:
        raise ValueError("one grammar per sequence")
    vocab = logits.shape[1]
    if logits.shape[0] != seqs * (k + 1):
        raise ValueError("logits must hold S * (k + 1) rows")
    drafts = [tuple(token_id(t, vocab, "proposal token") for t in d) for d in drafts]
    if any(len(d) > k for d in drafts):
        raise ValueError("a draft is longer than k")
    rows = seqs * (k + 1)
    if table is None:
        buf = buffer if buffer is not None else DraftForkMasks(vocab, rows, logits.device)
        if buf.host.shape[0] < rows:
            raise ValueError("buffer too small for the batch")
    elif table.host.shape[0] < rows or table.table.shape[1] != (vocab + 31) // 32:
        raise ValueError("mask table too small for the batch or of another vocabulary")
    prop = np.zeros((seqs, k), dtype=np.int64)
    lens = np.zeros(seqs, dtype=np.int32)
    for s, (d, g) in enumerate(zip(drafts, grammars)):
        if getattr(g, "vocab_size", vocab) != vocab:
            raise ValueError("grammar and model vocabularies differ")
        base = s * (k + 1)
        if table is None:
            fork_masks(g, d, vocab, buf._host_np[base:base + k + 1])
            buf._host_np[base + len(d) + 1:base + k + 1] = 0
        else:
            fork_state_indices(g, d, table._host_np[base:base + k + 1], table.empty)
            table._host_np[base + len(d) + 1:base + k + 1] = table.empty
        prop[s, : len(d)] = d
        lens[s] = len(d)
    dev = logits.device
    prop_d = torch.from_numpy(prop).to(dev, non_blocking=True)
    lens_d = torch.from_numpy(lens).to(dev, non_blocking=True)
    if table is None:
        result = verify_batch(logits, buf.upload(rows), prop_d, lens_d, policy=policy)
    else:
        result = verify_batch(logits, table.table, prop_d, lens_d, policy=policy, mask_rows=table.upload(rows))
    host = result.to_host()

    def replay(s: int, grammar) -> Iterator[VerifiedToken]:
        events = host.events(s, drafts[s])
        while not grammar.is_terminated():
            event = next(events, None)
            if event is None:
                return
            if not grammar.accept_token(event.token_id):
                raise ValueError("grammar rejected its selected token")
            yield event

    return [iter(()) if g.is_terminated() else replay(s, g) for s, g in enumerate(grammars)]
