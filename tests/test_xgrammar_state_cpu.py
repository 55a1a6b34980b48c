"""``xgrammar_state.XGrammarState`` on the host: the same masks, allowed IDs, densities, accepts and
termination as the reference's adapter (grammar/xgrammar.py) when the reference is importable, and
draft-fork masks written in place into the verification's staging rows."""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

from bitmask_speculation_b200 import workloads as wl
from xgrammar_cases import EOS, char, compiled

pytest.importorskip("xgrammar")
REF = Path(os.environ.get("BMS_REFERENCE_SRC", "/root/reference/src"))


def _walk(rng, g, steps):
    """A random walk through allowed tokens (never EOS unless nothing else is allowed)."""
    out = []
    for _ in range(steps):
        if g.is_terminated():
            break
        ids = [t for t in g.allowed_token_ids() if t != EOS] or list(g.allowed_token_ids())
        t = int(rng.choice(ids))
        assert g.accept_token(t)
        out.append(t)
    return out


def test_matches_the_reference_adapter():
    if not (REF / "bitmask_speculation" / "grammar" / "xgrammar.py").exists():
        pytest.skip("the reference's sources are not on this machine")
    sys.path.insert(0, str(REF))
    try:
        from bitmask_speculation.grammar.xgrammar import XGrammarState as RefState
    finally:
        sys.path.remove(str(REF))
    from bitmask_speculation_b200.xgrammar_state import XGrammarState
    comp = compiled(4096)
    rng = np.random.default_rng(1)
    for trial in range(6):
        ours, ref = XGrammarState(comp), RefState(comp)
        for _ in range(40):
            if ref.is_terminated():
                assert ours.is_terminated()
                break
            mine, theirs = ours.packed_mask_np(), ref.packed_mask().numpy()
            words = wl.unpack_bits_np(mine[None, :], 4096), wl.unpack_bits_np(theirs[None, :], 4096)
            assert np.array_equal(*words)
            assert ours.allowed_token_ids() == ref.allowed_token_ids()
            assert ours.mask_density() == ref.mask_density()
            fork = ours.fork()
            _walk(np.random.default_rng(trial), fork, 3)  # a fork never moves its parent
            assert np.array_equal(wl.unpack_bits_np(ours.packed_mask_np()[None, :], 4096), words[0])
            ids = [t for t in ref.allowed_token_ids() if t != EOS] or list(ref.allowed_token_ids())
            t = int(rng.choice(ids))
            assert ours.accept_token(t) == ref.accept_token(t)


def test_fork_masks_are_written_in_place_into_the_staging_rows():
    from bitmask_speculation_b200.grammar_verification import fork_masks
    from bitmask_speculation_b200.xgrammar_state import GrammarTerminatedError, XGrammarState
    vocab = 4096
    g = XGrammarState(compiled(vocab))
    draft = [char("{"), char('"'), char("a"), char("b"), char('"'), char(":"), char("7")]
    rows = np.zeros((len(draft) + 1, (vocab + 31) // 32), dtype=np.int32)
    fork_masks(g, draft, vocab, rows)
    step = g.fork()
    for i in range(len(draft) + 1):
        assert np.array_equal(rows[i], step.packed_mask_np()), i
        if i < len(draft):
            assert step.accept_token(draft[i])
    assert not g.is_terminated() and np.array_equal(g.packed_mask_np(), rows[0])  # the committed state is untouched
    done = g.fork()
    for t in [char("{"), char('"'), char("x"), char('"'), char(":"), char("1"), char("}"), EOS]:
        assert done.accept_token(t)
    assert done.is_terminated()
    with pytest.raises(GrammarTerminatedError):
        done.packed_mask_np()
