"""``dispatch.select_token``: the reference's per-row selection call (kernels/dispatch.py:79-103) on
the sm_100a kernel -- scores read in their own dtype, the mask uploaded from a pinned row or read
from a device-resident state table, one synchronization.  Cases of the reference's
tests/gpu/test_backend_dispatch.py plus full-vocabulary rows against the oracle."""

from types import SimpleNamespace

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl
from helpers import as_dtype_bits, to_device

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DTYPES = ["float32", "float16", "bfloat16"]


@pytest.mark.parametrize("dtype", DTYPES)
def test_lowest_valid_maximum_of_the_reference_case(cuda_module, dtype):
    from bitmask_speculation_b200.dispatch import select_token
    grammar = SimpleNamespace(vocab_size=65, allowed_token_ids=lambda: (31, 32, 64))
    scores = torch.zeros(65, device="cuda", dtype=getattr(torch, dtype))
    scores[31] = 2
    scores[32] = 2
    scores[0] = 100
    assert select_token(scores, grammar, "cuda") == 31


def test_float64_scores_are_rejected_not_rounded(cuda_module):
    from bitmask_speculation_b200.dispatch import select_token
    grammar = SimpleNamespace(vocab_size=2, allowed_token_ids=lambda: (0, 1))
    with pytest.raises(TypeError, match="float32"):
        select_token(torch.zeros(2, device="cuda", dtype=torch.float64), grammar, "cuda")


def test_data_errors_raise_value_error(cuda_module):
    from bitmask_speculation_b200.dispatch import select_token
    empty = SimpleNamespace(vocab_size=40, allowed_token_ids=lambda: ())
    with pytest.raises(ValueError, match="no valid token"):
        select_token(torch.zeros(40, device="cuda"), empty, "cuda")
    scores = torch.zeros(40, device="cuda")
    scores[3] = float("nan")  # NaN at an invalid position still fails the row
    with pytest.raises(ValueError, match="NaN"):
        select_token(scores, SimpleNamespace(vocab_size=40, allowed_token_ids=lambda: (5,)), "cuda")


@pytest.mark.parametrize("dtype", DTYPES)
def test_full_vocabulary_rows_match_the_oracle_with_uploaded_and_table_masks(cuda_module, dtype):
    from bitmask_speculation_b200.dispatch import select_token
    from bitmask_speculation_b200.grammar_verification import DeviceMaskTable
    rng = np.random.default_rng(17)
    vocab = wl.VOCAB
    grammar = wl.SyntheticDFAGrammar(vocab, states=64, seed=21)
    table = DeviceMaskTable.for_grammar(grammar, 4, torch.device("cuda"))
    values = rng.standard_normal((12, vocab), dtype=np.float32) * np.float32(3)
    values[5, :] = np.float32(1.25)  # a row of ties
    bits = as_dtype_bits(values, dtype)
    rows = to_device(bits, dtype)
    masks = np.zeros((12, wl.words_for(vocab)), dtype=np.int32)
    got_upload, got_table = [], []
    g = grammar.fork()
    for r in range(12):
        masks[r] = g.packed_mask_np()
        got_upload.append(select_token(rows[r], g, "cuda"))
        got_table.append(select_token(rows[r], g, "cuda", table=table))
        g.accept_token(got_upload[-1])
        if g.is_terminated():
            g = grammar.fork()
    want, _, status = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)
    assert (status == 0).all()
    assert got_upload == want.tolist() == got_table


def test_no_widened_copy_of_16_bit_scores(cuda_module):
    """A bf16 row is read in place: selecting does not allocate a float32 copy of the row."""
    from bitmask_speculation_b200.dispatch import select_token
    vocab = wl.VOCAB
    grammar = wl.SyntheticDFAGrammar(vocab, states=8, seed=3)
    scores = torch.randn(vocab, device="cuda").to(torch.bfloat16)
    select_token(scores, grammar, "cuda")  # staging rows exist from here on
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    before = torch.cuda.memory_allocated()
    select_token(scores, grammar, "cuda")
    assert torch.cuda.max_memory_allocated() - before < vocab * 4 // 2


def test_selection_does_not_advance_the_grammar(cuda_module):
    from bitmask_speculation_b200.dispatch import select_token
    grammar = wl.SyntheticDFAGrammar(8320, states=16, seed=5)
    state = grammar.state
    select_token(torch.randn(8320, device="cuda"), grammar, "cuda")
    assert grammar.state == state and not grammar.is_terminated()
