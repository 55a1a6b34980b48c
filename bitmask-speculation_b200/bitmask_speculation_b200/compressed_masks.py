"""Compact host-to-device transfer of a batch of grammar masks.

The reference copies every selection's mask to the device as a full packed row, 31,040 bytes at
V = 248,320 (kernels/dispatch.py:95), and a batched verification round uploads one such row per
target row.  Grammar states with few allowed tokens (enumerations, fixed keywords) need far less:
their token IDs, or for rows of a few percent density one byte per allowed token (the gap to the
previous one).  ``CompressedMasks`` keeps each row in the smallest of three forms -- a packed
bitmap, a token-ID list, or a byte-coded gap stream -- and ``upload`` moves the batch in two
host-to-device copies (the bitmaps, then one int32 block of row indices, list offsets, IDs, stream
offsets and stream bytes), after which ``bms_expand_token_lists`` and ``bms_expand_token_gaps`` write
the list and gap rows as packed rows after the bitmaps on the device.
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
    """A batch of ``rows`` packed mask rows of ``vocab`` tokens, held as bitmaps, token-ID lists and
    byte-coded gap streams.

    ``bitmaps`` int32 [nb, W]; ``ids`` int32 (all lists concatenated) with ``offsets`` int32 [nl + 1];
    ``gaps`` uint8 (all streams concatenated) with ``gap_offsets`` int32 [ng + 1] (a byte b > 0 advances
    b tokens and allows the token reached, 0 advances 255; streams start before token 0);
    ``mask_rows`` int32 [rows]: the table row of each mask row, tables rows being the bitmaps, then
    the lists, then the gap rows -- the device table that ``upload`` builds.
    """

    def __init__(self, vocab: int, bitmaps: np.ndarray, ids: np.ndarray, offsets: np.ndarray, mask_rows: np.ndarray,
                 gaps: np.ndarray | None = None, gap_offsets: np.ndarray | None = None):
        self.vocab = int(vocab)
        self.words = (self.vocab + 31) // 32
        self.bitmaps = np.ascontiguousarray(bitmaps, dtype=np.int32).reshape(-1, self.words)
        self.ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        self.offsets = np.ascontiguousarray(offsets, dtype=np.int32).reshape(-1)
        self.gaps = np.zeros(0, np.uint8) if gaps is None else np.ascontiguousarray(gaps, dtype=np.uint8).reshape(-1)
        self.gap_offsets = (np.zeros(1, np.int32) if gap_offsets is None
                            else np.ascontiguousarray(gap_offsets, dtype=np.int32).reshape(-1))
        self.mask_rows = np.ascontiguousarray(mask_rows, dtype=np.int32).reshape(-1)
        for off, n, what in ((self.offsets, self.ids.size, "offsets"), (self.gap_offsets, self.gaps.size, "gap_offsets")):
            if off.size < 1 or off[0] != 0 or off[-1] != n or np.any(np.diff(off) < 0):
                raise ValueError(f"{what} must start at 0, never decrease and end at the number of entries")
        if self.ids.size and (self.ids.min() < 0 or self.ids.max() >= self.vocab):
            raise ValueError(f"token IDs must be in [0, {self.vocab})")
        for g in range(self.gap_offsets.size - 1):
            last = self._decode_gaps(g)
            if last.size and last[-1] >= self.vocab:
                raise ValueError(f"a gap stream reaches past token {self.vocab - 1}")
        if self.mask_rows.size and (self.mask_rows.min() < 0 or self.mask_rows.max() >= self.table_rows):
            raise ValueError("mask_rows must index the bitmaps, lists and gap rows")
        self._staging = None

    # ---------------------------------------------------------------- construction
    @staticmethod
    def encode_gaps(ids: np.ndarray) -> np.ndarray:
        """The byte stream of ascending token IDs."""
        ids = np.asarray(ids, dtype=np.int64)
        gap = np.diff(ids, prepend=-1)
        z = (gap - 1) // 255
        out = np.zeros(int(ids.size + z.sum()), dtype=np.uint8)
        out[np.cumsum(z + 1) - 1] = (gap - 255 * z).astype(np.uint8)
        return out

    def _decode_gaps(self, g: int) -> np.ndarray:
        b = self.gaps[self.gap_offsets[g]:self.gap_offsets[g + 1]].astype(np.int64)
        pos = np.cumsum(np.where(b == 0, 255, b)) - 1
        return pos[b != 0]

    @classmethod
    def from_bitmaps(cls, masks: np.ndarray, vocab: int, kinds=("list", "gap")) -> "CompressedMasks":
        """Each row of a packed [rows, W] batch in its smallest form among the bitmap and ``kinds``
        (ties keep the bitmap, then the list); bits past ``vocab`` are ignored, as the kernels ignore
        them."""
        m = np.ascontiguousarray(masks, dtype=np.int32)
        words = (int(vocab) + 31) // 32
        if m.ndim != 2 or m.shape[1] != words:
            raise ValueError("masks must be [rows, ceil(vocab / 32)] int32")
        u = m.view(np.uint32).copy()
        if vocab % 32:
            u[:, -1] &= np.uint32((1 << (vocab % 32)) - 1)
        rows = m.shape[0]
        counts = np.bitwise_count(u).sum(axis=1, dtype=np.int64)
        kind = np.zeros(rows, dtype=np.int8)  # 0 bitmap, 1 list, 2 gap stream
        cand = np.flatnonzero(counts < 4 * words)  # a list or a stream can only win below this
        row_ids = {}
        if cand.size and ("list" in kinds or "gap" in kinds):
            # Only the nonzero words of candidate rows are expanded to bits (row-major, so each
            # row's IDs come out ascending).
            sub = u[cand]
            r, w = np.nonzero(sub)
            bits = (sub[r, w][:, None] >> np.arange(32, dtype=np.uint32)) & np.uint32(1)
            k, b = np.nonzero(bits)
            ids_all = w[k].astype(np.int64) * 32 + b
            rr = r[k]
            starts = np.concatenate([[0], np.cumsum(np.bincount(rr, minlength=cand.size))])
            prev = np.roll(ids_all, 1)
            if ids_all.size:
                prev[starts[:-1][starts[:-1] < ids_all.size]] = -1
            zeros = np.bincount(rr, weights=(ids_all - prev - 1) // 255, minlength=cand.size).astype(np.int64)
            for j, row in enumerate(cand):
                n = int(counts[row])
                sizes = [4 * words, 4 * n if "list" in kinds else None, n + int(zeros[j]) if "gap" in kinds else None]
                best = min((s, i) for i, s in enumerate(sizes) if s is not None)[1]
                kind[row] = best
                if best:
                    row_ids[row] = ids_all[starts[j]:starts[j + 1]]
        dense = np.flatnonzero(kind == 0)
        lists = np.flatnonzero(kind == 1)
        streams = np.flatnonzero(kind == 2)
        mask_rows = np.empty(rows, dtype=np.int32)
        mask_rows[dense] = np.arange(dense.size, dtype=np.int32)
        mask_rows[lists] = dense.size + np.arange(lists.size, dtype=np.int32)
        mask_rows[streams] = dense.size + lists.size + np.arange(streams.size, dtype=np.int32)
        ids = np.concatenate([row_ids[r] for r in lists]).astype(np.int32) if lists.size else np.zeros(0, np.int32)
        offsets = np.concatenate([[0], np.cumsum([row_ids[r].size for r in lists])]).astype(np.int32)
        enc = [cls.encode_gaps(row_ids[r]) for r in streams]
        gaps = np.concatenate(enc) if enc else np.zeros(0, np.uint8)
        gap_offsets = np.concatenate([[0], np.cumsum([e.size for e in enc])]).astype(np.int32)
        return cls(vocab, m[dense], ids, offsets, mask_rows, gaps, gap_offsets)

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
        return self.bitmaps.shape[0] + self.offsets.size - 1 + self.gap_offsets.size - 1

    @property
    def aux_words(self) -> int:
        return self.mask_rows.size + self.offsets.size + self.ids.size + self.gap_offsets.size + (self.gaps.size + 3) // 4

    @property
    def h2d_bytes(self) -> int:
        """Bytes one upload copies from host to device."""
        return 4 * (self.bitmaps.size + self.aux_words)

    def to_bitmaps(self) -> np.ndarray:
        """The packed [rows, W] batch these rows stand for (host; for checks)."""
        table = np.zeros((self.table_rows, self.words), dtype=np.uint32)
        nb, nl = self.bitmaps.shape[0], self.offsets.size - 1
        table[:nb] = self.bitmaps.view(np.uint32)
        sets = [self.ids[self.offsets[l]:self.offsets[l + 1]] for l in range(nl)]
        sets += [self._decode_gaps(g) for g in range(self.gap_offsets.size - 1)]
        for j, ids in enumerate(sets):
            ids = np.asarray(ids, dtype=np.int64)
            np.bitwise_or.at(table[nb + j], ids >> 5, np.uint32(1) << (ids & 31).astype(np.uint32))
        return table.view(np.int32)[self.mask_rows]

    # ---------------------------------------------------------------- device side
    def _pinned(self):
        if self._staging is None:
            torch = _torch()
            bm = torch.from_numpy(self.bitmaps).pin_memory()
            padded = np.zeros(((self.gaps.size + 3) // 4) * 4, dtype=np.uint8)
            padded[: self.gaps.size] = self.gaps
            aux = np.concatenate([self.mask_rows, self.offsets, self.ids, self.gap_offsets, padded.view(np.int32)])
            self._staging = (bm, torch.from_numpy(aux).pin_memory())
        return self._staging

    def allocate(self, device) -> DeviceTable:
        """Device buffers for one upload of this batch (reusable for batches of the same shape)."""
        torch = _torch()
        nbad = max(1, self.offsets.size - 1, self.gap_offsets.size - 1)
        return DeviceTable(torch.empty((max(1, self.table_rows), self.words), dtype=torch.int32, device=device),
                           torch.empty(max(1, self.aux_words), dtype=torch.int32, device=device),
                           torch.empty(nbad, dtype=torch.int32, device=device))

    def upload(self, device, buffers: DeviceTable | None = None, *, copy_stream=None):
        """Enqueue the two host-to-device copies (on ``copy_stream`` if given, which the current
        stream then waits for) and the expansions (current stream).  Returns (table [table_rows, W]
        int32, mask_rows int32 [rows]) on the device, ready for ``verify_batch(..., mask_rows=)``;
        the host staging is pinned, so the copies are asynchronous."""
        torch = _torch()
        buf = buffers or self.allocate(device)
        bm, aux = self._pinned()
        nb, nl, ng = self.bitmaps.shape[0], self.offsets.size - 1, self.gap_offsets.size - 1
        cur = torch.cuda.current_stream(device)
        side = copy_stream or cur
        with torch.cuda.stream(side):
            if nb:
                buf.table[:nb].copy_(bm, non_blocking=True)
            buf.aux[: aux.numel()].copy_(aux, non_blocking=True)
        if side is not cur:
            cur.wait_stream(side)
        lib = _native.library()
        rows = self.mask_rows.size
        at = rows
        offsets = buf.aux[at: at + nl + 1]
        at += nl + 1
        ids = buf.aux[at: at + self.ids.size]
        at += self.ids.size
        gap_offsets = buf.aux[at: at + ng + 1]
        at += ng + 1
        if nl:
            _native.check(lib.bms_expand_token_lists(
                ids.data_ptr() if self.ids.size else None, self.ids.size, offsets.data_ptr(), nl, self.vocab,
                buf.table[nb:].data_ptr(), buf.bad.data_ptr(), device.index, cur.cuda_stream))
        if ng:
            _native.check(lib.bms_expand_token_gaps(
                buf.aux.data_ptr() + 4 * at if self.gaps.size else None, self.gaps.size, gap_offsets.data_ptr(), ng,
                self.vocab, buf.table[nb + nl:].data_ptr(), buf.bad.data_ptr(), device.index, cur.cuda_stream))
        return buf.table[: max(1, self.table_rows)], buf.aux[:rows]


__all__ = ["CompressedMasks", "DeviceTable"]
