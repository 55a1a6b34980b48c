"""Host-side logic of stochastic speculative acceptance (``stochastic.py``): the draft rows' mask-row
table and the argument checks, which all run before any device work."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def test_draft_rows_read_the_rounds_mask_rows():
    from bitmask_speculation_b200.stochastic import _draft_mask_rows
    seqs, k = 5, 3
    table = _draft_mask_rows(seqs, k, torch.device("cpu")).numpy()
    want = np.array([s * (k + 1) + i for s in range(seqs) for i in range(k)], dtype=np.int32)
    assert table.dtype == np.int32 and np.array_equal(table, want)
    assert _draft_mask_rows(seqs, k, torch.device("cpu")) is _draft_mask_rows(seqs, k, torch.device("cpu"))


def _inputs(seqs=2, k=3, vocab=64, dtype=torch.bfloat16):
    words = (vocab + 31) // 32
    return (torch.zeros((seqs * (k + 1), vocab), dtype=dtype), torch.zeros((seqs * k, vocab), dtype=dtype),
            torch.zeros((seqs * (k + 1), words), dtype=torch.int32), torch.zeros((seqs, k), dtype=torch.int64),
            torch.zeros(seqs, dtype=torch.int32))


def test_argument_checks():
    from bitmask_speculation_b200.stochastic import speculative_accept
    t, d, m, p, l = _inputs()
    with pytest.raises(ValueError, match="positive temperature"):
        speculative_accept(t, d, m, p, l, temperature=0.0)
    with pytest.raises(ValueError, match=r"\[S\*\(K\+1\), V\]"):
        speculative_accept(t[1:], d, m, p, l, temperature=1.0)
    with pytest.raises(ValueError, match="share dtype"):
        speculative_accept(t, d.float(), m, p, l, temperature=1.0)
    with pytest.raises(ValueError, match="int32"):
        speculative_accept(t, d, m.long(), p, l, temperature=1.0)
    with pytest.raises(ValueError, match="int64"):
        speculative_accept(t, d, m, p.int(), l, temperature=1.0)


def test_lazy_needs_bulk_copyable_rows():
    """``lazy=True`` streams rows by 16-byte bulk copies: 1,001 bf16 logits (2,002 bytes) per row, or
    a row of 129 mask words, cannot."""
    from bitmask_speculation_b200.stochastic import speculative_accept
    for vocab in (1001, 4104):
        t, d, m, p, l = _inputs(vocab=vocab)
        with pytest.raises(ValueError, match="lazy acceptance needs"):
            speculative_accept(t, d, m, p, l, temperature=1.0, lazy=True)


def test_acceptance_policy_follows_the_mean_accepted_run():
    from bitmask_speculation_b200.stochastic import AcceptancePolicy
    pol = AcceptancePolicy(threshold=1.5, decay=0.5)
    assert not pol.lazy                      # nothing observed yet: every row's partials first
    pol.observe([0, 0, 1, 0])                # mean 0.25
    assert pol.lazy and pol.mean_run == 0.25
    pol.observe([8, 8, 8, 8])                # 0.5 * 0.25 + 0.5 * 8
    assert not pol.lazy and abs(pol.mean_run - 4.125) < 1e-12
    pol.observe([])                          # an empty round changes nothing
    assert abs(pol.mean_run - 4.125) < 1e-12
    assert AcceptancePolicy(initial=0.5).lazy
    with pytest.raises(ValueError):
        AcceptancePolicy(decay=1.0)
