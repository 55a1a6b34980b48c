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
    for kinds in (("list", "gap"), ("list",), ("gap",), ()):
        c = CompressedMasks.from_bitmaps(masks, vocab, kinds=kinds)
        assert np.array_equal(c.to_bitmaps(), masks), kinds
        words = (vocab + 31) // 32
        nb, nl = c.bitmaps.shape[0], c.offsets.size - 1
        assert c.h2d_bytes == 4 * (c.bitmaps.size + rows + c.offsets.size + c.ids.size + c.gap_offsets.size
                                   + (c.gaps.size + 3) // 4)
        assert c.h2d_bytes <= 4 * (rows * words + rows + 2)  # never larger than the bitmaps (plus headers)
        for r in range(rows):  # each row in its smallest allowed form
            n = int(valid[r].sum())
            t = c.mask_rows[r]
            if t < nb:
                size = 4 * words
            elif t < nb + nl:
                size = 4 * (c.offsets[t - nb + 1] - c.offsets[t - nb])
                assert c.ids[c.offsets[t - nb]:c.offsets[t - nb + 1]].tolist() == np.flatnonzero(valid[r]).tolist()
            else:
                g = t - nb - nl
                size = int(c.gap_offsets[g + 1] - c.gap_offsets[g])
            options = [4 * words] + ([4 * n] if "list" in kinds else [])
            if "gap" in kinds:
                options.append(CompressedMasks.encode_gaps(np.flatnonzero(valid[r])).size)
            assert size == min(options), (kinds, r)


def test_padding_bits_past_the_vocabulary_are_dropped_from_lists_and_streams():
    vocab = 1000
    masks = np.zeros((2, 32), dtype=np.int32)
    masks[:, 31] = -1                       # tokens 992..999 and the padding bits 1000..1023
    masks[:, 0] = 0b100010                  # tokens 1 and 5
    for kinds in (("list",), ("gap",)):
        c = CompressedMasks.from_bitmaps(masks, vocab, kinds=kinds)
        want = [1, 5] + list(range(992, 1000))
        back = c.to_bitmaps()
        assert [np.flatnonzero(wl.unpack_bits_np(back[i:i + 1], vocab)[0]).tolist() for i in range(2)] == [want, want]
        assert c.bitmaps.shape[0] == 0


def test_gap_stream_coding():
    ids = np.array([0, 1, 254, 255, 509, 510, 1020, 248319])
    enc = CompressedMasks.encode_gaps(ids)
    pos = np.cumsum(np.where(enc == 0, 255, enc).astype(np.int64)) - 1
    assert pos[enc != 0].tolist() == ids.tolist()
    assert CompressedMasks.encode_gaps(np.array([], dtype=np.int64)).size == 0
    with pytest.raises(ValueError, match="past token"):
        CompressedMasks(300, np.zeros((0, 10), np.int32), np.zeros(0, np.int32), np.zeros(1, np.int32),
                        np.array([0], np.int32), CompressedMasks.encode_gaps(np.array([3, 300])), np.array([0, 3]))


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
