"""Grammar-constrained verification rounds over XGrammar states at V = 248,320: the draft-fork masks
are written by XGrammar straight into the pinned staging rows (``XGrammarState.fill_mask_row``),
uploaded once per round and verified in one launch pair; the events and the advanced grammars must
equal the reference's lazy per-row loop (models/transformers.py:181-201 over
decoding/verification.py:18-48) restated on the oracle."""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl
from xgrammar_cases import EOS, compiled

torch = pytest.importorskip("torch")
pytest.importorskip("xgrammar")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def grammar(cuda_module):
    return compiled(wl.VOCAB)


def _setup(comp, seqs, k, seed):
    from bitmask_speculation_b200.xgrammar_state import XGrammarState
    rng = np.random.default_rng(seed)
    grammars, drafts = [], []
    for s in range(seqs):
        g = XGrammarState(comp)
        for _ in range(int(rng.integers(0, 12))):  # a committed prefix
            ids = [t for t in g.allowed_token_ids() if t != EOS]
            if not ids:
                break
            g.accept_token(int(rng.choice(ids)))
        f, d = g.fork(), []
        for _ in range(int(rng.integers(0, k + 1))):  # a draft the grammar accepts
            if f.is_terminated():
                break
            ids = list(f.allowed_token_ids())
            t = int(rng.choice(ids))
            d.append(t)
            f.accept_token(t)
        grammars.append(g)
        drafts.append(d)
    vals = rng.standard_normal((seqs * (k + 1), wl.VOCAB), dtype=np.float32) * np.float32(3)
    for s, d in enumerate(drafts):  # the target agrees with the draft up to a random point
        agree = int(rng.integers(0, len(d) + 1))
        for i in range(agree):
            vals[s * (k + 1) + i, d[i]] = 50.0
    return grammars, drafts, wl.to_bf16_bits(vals)


def _state(g):
    return (g.is_terminated(), None if g.is_terminated() else g.packed_mask_np().tobytes())


def test_batched_rounds_match_the_reference_loop(grammar):
    from bitmask_speculation_b200.grammar_verification import DraftForkMasks, verify_with_grammars
    seqs, k = 24, 6
    grammars, drafts, bits = _setup(grammar, seqs, k, seed=3)
    logits = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    buf = DraftForkMasks(wl.VOCAB, seqs * (k + 1), logits.device)
    ours = [g.fork() for g in grammars]
    its = verify_with_grammars(drafts, logits, ours, k=k, buffer=buf)
    for s, (it, g) in enumerate(zip(its, grammars)):
        got = [(e.token_id, e.kind) for e in it]
        ref_g = g.fork()
        rows = bits[s * (k + 1): s * (k + 1) + len(drafts[s]) + 1]
        want = oracle.grammar_choices(drafts[s], rows, ref_g, dtype="bfloat16")
        assert got == want, s
        assert _state(ours[s]) == _state(ref_g), s
    assert any(len(d) for d in drafts)


def test_single_round_matches_the_reference_loop(grammar):
    from bitmask_speculation_b200.grammar_verification import verify_with_grammar
    grammars, drafts, bits = _setup(grammar, 6, 5, seed=9)
    for s, (g, d) in enumerate(zip(grammars, drafts)):
        rows = bits[s * 6: s * 6 + len(d) + 1]
        logits = torch.from_numpy(np.ascontiguousarray(rows).view(np.int16)).view(torch.bfloat16).cuda()
        mine = g.fork()
        got = [(e.token_id, e.kind) for e in verify_with_grammar(d, logits, mine)]
        ref_g = g.fork()
        assert got == oracle.grammar_choices(d, rows, ref_g, dtype="bfloat16"), s
        assert _state(mine) == _state(ref_g), s
