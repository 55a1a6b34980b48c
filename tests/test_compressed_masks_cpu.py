"""Host side of the compact mask transfer (no GPU): bitmaps <-> (bitmaps, ID lists, row indices)."""

import numpy as np
import pytest

from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.compressed_masks import CompressedMasks


@pytest.mark.parametrize("vocab", [248320, 50257, 96, 33])
def test_from_bitmaps_round_trip(vocab):
    rng = np.random.default_rng(vocab)
    rows = 40
    dens = rng.choice([0.0, 1e-4, 0.002, 0.05, 0.6, 1.0], size=rows)
    valid = rng.random((rows, vocab)) < dens[:, None]
    valid[3, :] = False                      # an empty row travels as an empty list
    valid[4, [0, vocab - 1]] = True          # the first and the last token
    masks = wl.pack_bits_np(valid)
    c = CompressedMasks.from_bitmaps(masks, vocab)
    assert np.array_equal(c.to_bitmaps(), masks)
    words = (vocab + 31) // 32
    counts = valid.sum(axis=1)
    assert c.bitmaps.shape[0] == int((counts > words // 8).sum())
    assert c.h2d_bytes == 4 * (c.bitmaps.size + rows + c.offsets.size + c.ids.size)
    lists = c.mask_rows >= c.bitmaps.shape[0]
    for r in np.flatnonzero(lists):
        l = c.mask_rows[r] - c.bitmaps.shape[0]
        assert c.ids[c.offsets[l]:c.offsets[l + 1]].tolist() == np.flatnonzero(valid[r]).tolist()


def test_padding_bits_past_the_vocabulary_are_dropped_from_lists():
    vocab = 40
    masks = np.full((1, 2), -1, dtype=np.int32)  # bits 40..63 set too
    c = CompressedMasks.from_bitmaps(masks, vocab, max_ids=64)
    assert c.ids.tolist() == list(range(40))


def test_from_rows_mixes_bitmaps_and_lists():
    vocab = 100
    words = 4
    bitmap = wl.pack_bits_np(np.arange(vocab)[None, :] % 3 == 0)[0]
    c = CompressedMasks.from_rows([bitmap, np.array([7, 3, 7, 99]), np.array([], dtype=np.int64), bitmap], vocab)
    back = c.to_bitmaps()
    assert back.shape == (4, words)
    assert np.array_equal(back[0], bitmap) and np.array_equal(back[3], bitmap)
    assert np.flatnonzero(wl.unpack_bits_np(back[1:2], vocab)[0]).tolist() == [3, 7, 99]
    assert not back[2].any()
    assert c.table_rows == 4 and c.mask_rows.tolist() == [0, 2, 3, 1]


def test_invalid_lists_are_rejected_on_the_host():
    with pytest.raises(ValueError, match=r"token IDs must be in \[0, 10\)"):
        CompressedMasks.from_rows([np.array([10])], 10)
    with pytest.raises(ValueError, match="offsets"):
        CompressedMasks(10, np.zeros((0, 1), np.int32), np.array([1, 2], np.int32), np.array([0, 3], np.int32),
                        np.array([0], np.int32))
    with pytest.raises(ValueError, match="mask_rows"):
        CompressedMasks(10, np.zeros((0, 1), np.int32), np.array([1], np.int32), np.array([0, 1], np.int32),
                        np.array([1], np.int32))
