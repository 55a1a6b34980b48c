"""bms_masked_reduce_batch_noalloc: the argmax + count kernel on the dynamic schedule with its
workspace in a file-scope device array, for callers that cannot allocate device memory.  Two
consecutive calls on different batches must equal the oracle (the reference's torch_reduce
restated) and bms_masked_reduce_batch (fixed schedule, no workspace) on the same inputs, bit for
bit."""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import _native
from bitmask_speculation_b200 import workloads as wl
from helpers import as_dtype_bits, to_device

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu
CODES = {"float32": 0, "bfloat16": 1, "float16": 2}


def _batch(rng, rows, vocab, dtype):
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(3)
    values[0, :] = np.float32(0.5)  # ties everywhere: the lowest valid index wins
    dens = rng.choice([1.0, 0.3, 0.01, 1e-4], size=rows)
    valid = rng.random((rows, vocab)) < dens[:, None]
    valid[1, :] = False  # a row without a valid token
    bits, masks = as_dtype_bits(values, dtype), wl.pack_bits_np(valid)
    return (to_device(bits, dtype), torch.from_numpy(masks).cuda()), (bits, masks)


def _run(fn, logits, masks, dtype, extra):
    rows, vocab = logits.shape
    tokens = torch.empty(rows, dtype=torch.int64, device="cuda")
    counts = torch.empty(rows, dtype=torch.int64, device="cuda")
    status = torch.empty(rows, dtype=torch.int32, device="cuda")
    _native.check(fn(logits.data_ptr(), CODES[dtype], masks.data_ptr(), rows, vocab, tokens.data_ptr(),
                     counts.data_ptr(), status.data_ptr(), *extra, logits.device.index,
                     torch.cuda.current_stream().cuda_stream))
    return tokens.cpu().numpy(), counts.cpu().numpy(), status.cpu().numpy()


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("rows,vocab", [(300, 248320), (1000, 151936), (9, 50257)])
def test_two_consecutive_calls_match_the_workspace_free_entry_point(cuda_module, dtype, rows, vocab):
    lib = _native.library()
    rng = np.random.default_rng(rows + vocab)
    first, first_host = _batch(rng, rows, vocab, dtype)
    second, second_host = _batch(rng, rows, vocab, dtype)
    got_first = _run(lib.bms_masked_reduce_batch_noalloc, *first, dtype, [])
    got_second = _run(lib.bms_masked_reduce_batch_noalloc, *second, dtype, [])
    for got, batch, (bits, masks) in ((got_first, first, first_host), (got_second, second, second_host)):
        expect = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)
        want = _run(lib.bms_masked_reduce_batch, *batch, dtype, [None, 0])
        for g, e, w in zip(got, expect, want):
            assert np.array_equal(g, e)
            assert np.array_equal(g, w)


def test_rows_longer_than_the_static_workspace_splits_are_rejected(cuda_module):
    lib = _native.library()
    logits = torch.zeros((1, 64 * 8192 + 32), dtype=torch.bfloat16, device="cuda")
    masks = torch.zeros((1, logits.shape[1] // 32), dtype=torch.int32, device="cuda")
    out = torch.empty(1, dtype=torch.int64, device="cuda")
    st = torch.empty(1, dtype=torch.int32, device="cuda")
    rc = lib.bms_masked_reduce_batch_noalloc(logits.data_ptr(), 1, masks.data_ptr(), 1, logits.shape[1],
                                             out.data_ptr(), None, st.data_ptr(), 0,
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == _native.ERROR_UNSUPPORTED
    assert b"static workspace" in lib.bms_last_error()
