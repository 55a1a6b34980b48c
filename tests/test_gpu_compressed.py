"""Compact mask transfer on the GPU: ``bms_expand_token_lists`` and ``bms_expand_token_gaps`` write
exactly the listed / coded bits, and a
verification round over the uploaded table (``mask_rows``) equals the round over full bitmaps and
the oracle -- configuration 3 at full size (256 sequences x 9 rows)."""

import ctypes

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import _native
from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.compressed_masks import CompressedMasks

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _expand(ids, offsets, vocab):
    lib = _native.library()
    lists = len(offsets) - 1
    words = (vocab + 31) // 32
    d_ids = torch.tensor(ids, dtype=torch.int32, device="cuda") if len(ids) else None
    d_off = torch.tensor(offsets, dtype=torch.int32, device="cuda")
    out = torch.full((lists, words), -1, dtype=torch.int32, device="cuda")  # dirty: every word is rewritten
    bad = torch.full((lists,), 7, dtype=torch.int32, device="cuda")
    _native.check(lib.bms_expand_token_lists(d_ids.data_ptr() if d_ids is not None else None, len(ids), d_off.data_ptr(),
                                             lists, vocab, out.data_ptr(), bad.data_ptr(), 0,
                                             torch.cuda.current_stream().cuda_stream))
    return out.cpu().numpy(), bad.cpu().numpy()


@pytest.mark.parametrize("vocab", [248320, 50257, 33])
def test_expansion_sets_exactly_the_listed_bits(cuda_module, vocab):
    rng = np.random.default_rng(vocab)
    lists = [rng.integers(0, vocab, size=n) for n in (0, 1, 2, 31, 32, 33, 700, 5000)]
    lists.append(np.array([vocab - 1, 0, vocab - 1, 0]))  # repeats, unsorted, both ends
    ids = np.concatenate(lists).astype(np.int32)
    offsets = np.concatenate([[0], np.cumsum([x.size for x in lists])]).astype(np.int32)
    out, bad = _expand(ids.tolist(), offsets.tolist(), vocab)
    want = CompressedMasks(vocab, np.zeros((0, (vocab + 31) // 32), np.int32), ids, offsets,
                           np.arange(len(lists), dtype=np.int32)).to_bitmaps()
    assert np.array_equal(out, want)
    assert not bad.any()


def test_ids_outside_the_vocabulary_set_nothing_and_flag_the_list(cuda_module):
    out, bad = _expand([5, 64, -1, 3, 63], [0, 2, 4, 5], 64)
    assert bad.tolist() == [1, 1, 0]
    assert wl.unpack_bits_np(out, 64).nonzero()[1].tolist() == [5, 3, 63]
    # Offsets past the ID array are clamped: nothing outside it is read.
    out, bad = _expand([1, 2], [0, 1, 9], 64)
    assert wl.unpack_bits_np(out, 64).nonzero()[1].tolist() == [1, 2]


def _expand_gaps(stream: np.ndarray, offsets, vocab):
    lib = _native.library()
    rows = len(offsets) - 1
    words = (vocab + 31) // 32
    d_bytes = torch.from_numpy(np.ascontiguousarray(stream, dtype=np.uint8)).cuda() if len(stream) else None
    d_off = torch.tensor(offsets, dtype=torch.int32, device="cuda")
    out = torch.full((rows, words), -1, dtype=torch.int32, device="cuda")
    bad = torch.full((rows,), 7, dtype=torch.int32, device="cuda")
    _native.check(lib.bms_expand_token_gaps(d_bytes.data_ptr() if d_bytes is not None else None, len(stream),
                                            d_off.data_ptr(), rows, vocab, out.data_ptr(), bad.data_ptr(), 0,
                                            torch.cuda.current_stream().cuda_stream))
    return out.cpu().numpy(), bad.cpu().numpy()


@pytest.mark.parametrize("vocab", [248320, 50257, 700, 1_300_000, 1_400_000])
def test_gap_expansion_sets_exactly_the_coded_tokens(cuda_module, vocab):
    """Shared-memory row bitmaps (up to 160 KB: 1,300,000 tokens takes more than the default 48 KB)
    and, past that, the global-atomic expansion (1,400,000 tokens)."""
    rng = np.random.default_rng(vocab + 1)
    sets = [np.flatnonzero(rng.random(vocab) < d) for d in (0.0, 0.0005, 0.004, 0.05, 0.12, 0.5)]
    sets.append(np.array([254, 509, 764, vocab - 1]) if vocab > 800 else np.array([254, 509, vocab - 1]))
    # (gaps of exactly 255, then a long run of them to the last token)
    sets.append(np.array([0]))
    enc = [CompressedMasks.encode_gaps(x) for x in sets]
    offsets = np.concatenate([[0], np.cumsum([e.size for e in enc])]).astype(np.int32)
    out, bad = _expand_gaps(np.concatenate(enc), offsets.tolist(), vocab)
    for r, x in enumerate(sets):
        assert np.flatnonzero(wl.unpack_bits_np(out[r:r + 1], vocab)[0]).tolist() == x.tolist(), r
    assert not bad.any()


def test_gap_streams_past_the_vocabulary_set_nothing_there_and_flag_the_row(cuda_module):
    stream = CompressedMasks.encode_gaps(np.array([3, 70, 64 + 255]))  # the last token is past V = 64
    out, bad = _expand_gaps(stream, [0, stream.size, stream.size + 5], 64)
    assert bad.tolist() == [1, 0]  # the second row's offsets are clamped to the stream: empty
    assert wl.unpack_bits_np(out, 64).nonzero()[1].tolist() == [3]


def test_configuration_3_round_over_the_compressed_upload(cuda_module):
    from bitmask_speculation_b200.verification import verify_batch
    logits, masks, proposals, lengths = wl.verify_batch_torch(256, seed=3, device="cuda")
    host_masks = masks.cpu().numpy()
    c = CompressedMasks.from_bitmaps(host_masks, wl.VOCAB)
    # enumeration rows travel as ID lists, the 5 % rows as gap streams
    assert c.h2d_bytes < 0.45 * host_masks.nbytes and c.gaps.size and c.ids.size
    copy = torch.cuda.Stream()
    buf = c.allocate(logits.device)
    for _ in range(2):  # the buffers are reusable
        table, mask_rows = c.upload(logits.device, buf, copy_stream=copy)
        got = verify_batch(logits, table, proposals, lengths, mask_rows=mask_rows).to_host()
    want = verify_batch(logits, masks, proposals, lengths).to_host()
    assert got == want
    bits = logits.cpu().view(torch.int16).numpy().view(np.uint16)
    tok, cnt, st = oracle.reduce_rows(bits, host_masks, dtype="bfloat16")
    acc, token, kind, sst = oracle.verify(tok, st, proposals.cpu().numpy(), lengths.cpu().numpy())
    assert got.row_tokens == tok.tolist() and got.row_counts == cnt.tolist()
    assert got.accept_len == acc.tolist() and got.token == token.tolist() and got.kind == kind.tolist()
