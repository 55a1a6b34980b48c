"""Compact host-to-device transfer of a batch of grammar masks.

The reference copies every selection's mask to the device as a full packed row, 31,040 bytes at
V = 248,320 (kernels/dispatch.py:95), and a batched verification round uploads one such row per
target row.  Grammar states with few allowed tokens (enumerations, fixed keywords) need far less:
their token IDs.  ``CompressedMasks`` keeps each row either as a token-ID list (rows with at most
``max_ids`` valid tokens) or as a packed bitmap, and ``upload`` moves the batch in two host-to-device
copies -- the bitmaps, then one int32 block of row indices, list offsets and IDs -- after which
``bms_expand_token_lists`` writes the list rows as packed rows after the bitmaps on the device.
The result is a mask table plus one table index per row: exactly the ``masks`` / ``mask_rows``
pair of ``verification.verify_batch``, which reads the table in place.  Rows are unchanged as
masks: a list row allows exactly its listed IDs.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _native


def _torch():
    import torch
    return torch


@dataclass
class DeviceTable:
    """Device buffers one upload fills: ``table`` [capacity rows, W] int32 and ``aux`` int32."""

    table: object
    aux: object
    bad: object


class CompressedMasks:
    """A batch of ``rows`` packed mask rows of ``vocab`` tokens, held as bitmaps and token-ID lists.

    ``bitmaps`` int32 [nb, W]; ``ids`` int32 (all lists concatenated) with ``offsets`` int32 [nl + 1];
    ``mask_rows`` int32 [rows]: row r is bitmap ``mask_rows[r]`` if it is below nb, else list
    ``mask_rows[r] - nb`` -- the row of the device table that ``upload`` builds.
    """

    def __init__(self, vocab: int, bitmaps: np.ndarray, ids: np.ndarray, offsets: np.ndarray, mask_rows: np.ndarray):
        self.vocab = int(vocab)
        self.words = (self.vocab + 31) // 32
        self.bitmaps = np.ascontiguousarray(bitmaps, dtype=np.int32).reshape(-1, self.words)
        self.ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        self.offsets = np.ascontiguousarray(offsets, dtype=np.int32).reshape(-1)
        self.mask_rows = np.ascontiguousarray(mask_rows, dtype=np.int32).reshape(-1)
        nb, nl = self.bitmaps.shape[0], self.offsets.size - 1
        if nl < 0 or self.offsets[0] != 0 or self.offsets[-1] != self.ids.size or np.any(np.diff(self.offsets) < 0):
            raise ValueError("offsets must start at 0, never decrease and end at the number of IDs")
        if self.ids.size and (self.ids.min() < 0 or self.ids.max() >= self.vocab):
            raise ValueError(f"token IDs must be in [0, {self.vocab})")
        if self.mask_rows.size and (self.mask_rows.min() < 0 or self.mask_rows.max() >= nb + nl):
            raise ValueError("mask_rows must index the bitmaps and lists")
        self._staging = None

    # ---------------------------------------------------------------- construction
    @classmethod
    def from_bitmaps(cls, masks: np.ndarray, vocab: int, max_ids: int | None = None) -> "CompressedMasks":
        """Rows of a packed [rows, W] batch with at most ``max_ids`` valid tokens (default W / 8, a
        list at most an eighth of a bitmap's bytes) become ID lists; bits past ``vocab`` are
        ignored, as the kernels ignore them."""
        m = np.ascontiguousarray(masks, dtype=np.int32)
        words = (int(vocab) + 31) // 32
        if m.ndim != 2 or m.shape[1] != words:
            raise ValueError("masks must be [rows, ceil(vocab / 32)] int32")
        max_ids = words // 8 if max_ids is None else int(max_ids)
        u = m.view(np.uint32).copy()
        if vocab % 32:
            u[:, -1] &= np.uint32((1 << (vocab % 32)) - 1)
        counts = np.bitwise_count(u).sum(axis=1, dtype=np.int64)
        sparse = counts <= max_ids
        dense_rows = np.flatnonzero(~sparse)
        sparse_rows = np.flatnonzero(sparse)
        mask_rows = np.empty(m.shape[0], dtype=np.int32)
        mask_rows[dense_rows] = np.arange(dense_rows.size, dtype=np.int32)
        mask_rows[sparse_rows] = dense_rows.size + np.arange(sparse_rows.size, dtype=np.int32)
        if sparse_rows.size:
            # Only the nonzero words of sparse rows are expanded to bits (row-major, so each row's
            # IDs come out ascending).
            sub = u[sparse_rows]
            r, w = np.nonzero(sub)
            bits = (sub[r, w][:, None] >> np.arange(32, dtype=np.uint32)) & np.uint32(1)
            k, b = np.nonzero(bits)
            ids = (w[k].astype(np.int64) * 32 + b).astype(np.int32)
            offsets = np.zeros(sparse_rows.size + 1, dtype=np.int32)
            np.cumsum(np.bincount(r[k], minlength=sparse_rows.size), out=offsets[1:])
        else:
            ids, offsets = np.zeros(0, np.int32), np.zeros(1, np.int32)
        return cls(vocab, m[dense_rows], ids, offsets, mask_rows)

    @classmethod
    def from_rows(cls, rows, vocab: int) -> "CompressedMasks":
        """Rows given one by one: a packed int32 row of ceil(vocab / 32) words, or a 1-D array of
        allowed token IDs (any other length)."""
        words = (int(vocab) + 31) // 32
        bitmaps, lists, index = [], [], []
        for row in rows:
            a = np.asarray(row)
            if a.ndim == 1 and a.size == words and a.dtype == np.int32:
                index.append(("b", len(bitmaps)))
                bitmaps.append(a)
            else:
                index.append(("l", len(lists)))
                lists.append(a.astype(np.int32).reshape(-1))
        nb = len(bitmaps)
        mask_rows = np.array([i if k == "b" else nb + i for k, i in index], dtype=np.int32)
        offsets = np.zeros(len(lists) + 1, dtype=np.int32)
        if lists:
            np.cumsum([x.size for x in lists], out=offsets[1:])
        ids = np.concatenate(lists) if lists else np.zeros(0, np.int32)
        bm = np.stack(bitmaps) if bitmaps else np.zeros((0, words), np.int32)
        return cls(vocab, bm, ids, offsets, mask_rows)

    # ---------------------------------------------------------------- sizes
    @property
    def rows(self) -> int:
        return self.mask_rows.size

    @property
    def table_rows(self) -> int:
        return self.bitmaps.shape[0] + self.offsets.size - 1

    @property
    def aux_words(self) -> int:
        return self.mask_rows.size + self.offsets.size + self.ids.size

    @property
    def h2d_bytes(self) -> int:
        """Bytes one upload copies from host to device."""
        return 4 * (self.bitmaps.size + self.aux_words)

    def to_bitmaps(self) -> np.ndarray:
        """The packed [rows, W] batch these rows stand for (host; for checks)."""
        table = np.zeros((self.table_rows, self.words), dtype=np.uint32)
        table[: self.bitmaps.shape[0]] = self.bitmaps.view(np.uint32)
        for l in range(self.offsets.size - 1):
            ids = self.ids[self.offsets[l]:self.offsets[l + 1]].astype(np.int64)
            np.bitwise_or.at(table[self.bitmaps.shape[0] + l], ids >> 5, np.uint32(1) << (ids & 31).astype(np.uint32))
        return table.view(np.int32)[self.mask_rows]

    # ---------------------------------------------------------------- device side
    def _pinned(self):
        if self._staging is None:
            torch = _torch()
            bm = torch.from_numpy(self.bitmaps).pin_memory()
            aux = torch.from_numpy(np.concatenate([self.mask_rows, self.offsets, self.ids])).pin_memory()
            self._staging = (bm, aux)
        return self._staging

    def allocate(self, device) -> DeviceTable:
        """Device buffers for one upload of this batch (reusable for batches of the same shape)."""
        torch = _torch()
        return DeviceTable(torch.empty((max(1, self.table_rows), self.words), dtype=torch.int32, device=device),
                           torch.empty(max(1, self.aux_words), dtype=torch.int32, device=device),
                           torch.empty(max(1, self.offsets.size - 1), dtype=torch.int32, device=device))

    def upload(self, device, buffers: DeviceTable | None = None, *, copy_stream=None):
        """Enqueue the two host-to-device copies (on ``copy_stream`` if given, which the current
        stream then waits for) and the list expansion (current stream).  Returns (table [table_rows,
        W] int32, mask_rows int32 [rows]) on the device, ready for ``verify_batch(..., mask_rows=)``;
        the host staging is pinned, so the copies are asynchronous."""
        torch = _torch()
        buf = buffers or self.allocate(device)
        bm, aux = self._pinned()
        nb, nl = self.bitmaps.shape[0], self.offsets.size - 1
        cur = torch.cuda.current_stream(device)
        side = copy_stream or cur
        with torch.cuda.stream(side):
            if nb:
                buf.table[:nb].copy_(bm, non_blocking=True)
            buf.aux[: aux.numel()].copy_(aux, non_blocking=True)
        if side is not cur:
            cur.wait_stream(side)
        rows = self.mask_rows.size
        offsets = buf.aux[rows: rows + nl + 1]
        ids = buf.aux[rows + nl + 1: rows + nl + 1 + self.ids.size]
        if nl:
            _native.check(_native.library().bms_expand_token_lists(
                ids.data_ptr() if self.ids.size else None, self.ids.size, offsets.data_ptr(), nl, self.vocab,
                buf.table[nb:].data_ptr(), buf.bad.data_ptr(), device.index, cur.cuda_stream))
        return buf.table[: max(1, self.table_rows)], buf.aux[:rows]


__all__ = ["CompressedMasks", "DeviceTable"]
