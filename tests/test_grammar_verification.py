"""Grammar-constrained batched verification (draft-fork masks, one launch and one sync per round)
against the reference's lazy per-row loop restated with the oracle: models/transformers.py:181-201
(`_choices` + `constrained_choices`) over decoding/verification.py:18-48 (`verify_prefix`), with
each row selected by the masked argmax under the committed grammar (grammar/selection.py:12-32)."""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.grammar_verification import fork_masks
from bitmask_speculation_b200.verification import VerifiedToken


def reference_choices(draft, rows_f32, grammar):
    """The reference's lazy loop, restated on the oracle (``oracle.grammar_choices``)."""
    return [VerifiedToken(t, k) for t, k in oracle.grammar_choices(draft, rows_f32, grammar)]


def make_round(rng, vocab, k, grammar, p_accept=0.85, eos_boost=False):
    """Target rows and a draft that follows the target's own choices until a seeded mismatch."""
    rows = rng.standard_normal((k + 1, vocab), dtype=np.float32) * np.float32(3)
    if eos_boost:
        rows[:, 0] += np.float32(6)
    fork = grammar.fork()
    draft = []
    for i in range(k):
        if fork.is_terminated():
            break
        mask = fork.packed_mask_np()[None, :]
        tok = int(oracle.reduce_rows(rows[i:i + 1], mask)[0][0])
        if tok < 0:
            break
        if rng.random() > p_accept:
            allowed = np.asarray(fork.allowed_token_ids())
            others = allowed[allowed != tok]
            tok = int(rng.choice(others)) if others.size else int(rng.integers(vocab))
        draft.append(tok)
        if not fork.accept_token(tok):
            break
    return rows[: len(draft) + 1], draft


def test_fork_masks_follow_the_draft_and_blank_unreachable_rows():
    vocab = 4096
    g = wl.SyntheticDFAGrammar(vocab, states=16, seed=3)
    rng = np.random.default_rng(0)
    for _ in range(20):
        fork = g.fork()
        draft, expect = [], [fork.packed_mask_np().copy()]
        for _ in range(6):
            allowed = fork.allowed_token_ids()
            tok = int(rng.choice(allowed)) if allowed and rng.random() < 0.9 else int(rng.integers(vocab))
            draft.append(tok)
            ok = fork.accept_token(tok) and not fork.is_terminated()
            expect.append(fork.packed_mask_np().copy() if ok else np.zeros_like(expect[0]))
            if not ok:
                while len(expect) < 7:
                    draft.append(int(rng.integers(vocab)))
                    expect.append(np.zeros_like(expect[0]))
                break
        out = np.full((8, (vocab + 31) // 32), 7, dtype=np.int32)
        rows = fork_masks(g, draft, vocab, out)
        assert rows == len(draft) + 1
        assert np.array_equal(out[:rows], np.stack(expect[:rows]))
        assert g.state == 0 and not g.is_terminated()  # the committed state is untouched


def test_fork_masks_of_a_generic_grammar_from_allowed_ids():
    class Ids:
        vocab_size = 100

        def __init__(self, allowed=(3, 64, 99)):
            self.allowed = allowed

        def fork(self):
            return Ids(self.allowed)

        def is_terminated(self):
            return False

        def allowed_token_ids(self):
            return self.allowed

        def accept_token(self, t):
            return t in self.allowed

    out = np.zeros((2, 4), dtype=np.int32)
    fork_masks(Ids(), [64], 100, out)
    words = out[0].view(np.uint32)
    assert words[0] == 1 << 3 and words[2] == 1 << 0 and words[3] == 1 << 3


@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [8320, 248320])
def test_batched_grammar_verification_equals_the_lazy_reference_loop(cuda_module, vocab):
    torch = pytest.importorskip("torch")
    from bitmask_speculation_b200.grammar_verification import DraftForkMasks, verify_with_grammar
    rng = np.random.default_rng(vocab)
    buf = DraftForkMasks(vocab, 9, torch.device("cuda"))
    for trial in range(24):
        g_ref = wl.SyntheticDFAGrammar(vocab, states=64, seed=trial)
        g_gpu = g_ref.fork()
        for rnd in range(3):
            k = int(rng.integers(0, 9))
            rows, draft = make_round(rng, vocab, k, g_ref, eos_boost=(trial % 4 == 0))
            bits = wl.to_bf16_bits(rows)
            rows_bf = oracle.widen(bits, "bfloat16")
            want = reference_choices(draft, rows_bf, g_ref)
            logits = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
            got = list(verify_with_grammar(draft, logits, g_gpu, buffer=buf))
            assert got == want, (trial, rnd, draft)
            assert (g_gpu.state, g_gpu.is_terminated()) == (g_ref.state, g_ref.is_terminated())
            if g_ref.is_terminated():
                break


@pytest.mark.gpu
def test_batch_of_sequences_in_one_round_equals_per_sequence_loops(cuda_module):
    torch = pytest.importorskip("torch")
    from bitmask_speculation_b200.grammar_verification import DraftForkMasks, verify_with_grammars
    vocab, seqs, k = 151936, 48, 8
    rng = np.random.default_rng(17)
    refs = [wl.SyntheticDFAGrammar(vocab, states=64, seed=s % 5) for s in range(seqs)]
    gpus = [g.fork() for g in refs]
    buf = DraftForkMasks(vocab, seqs * (k + 1), torch.device("cuda"))
    for rnd in range(3):
        block = np.zeros((seqs * (k + 1), vocab), dtype=np.uint16)
        drafts, wants = [], []
        for s in range(seqs):
            if refs[s].is_terminated():
                drafts.append(())
                wants.append([])
                continue
            rows, draft = make_round(rng, vocab, int(rng.integers(0, k + 1)), refs[s], eos_boost=(s % 7 == 0))
            bits = wl.to_bf16_bits(rows)
            block[s * (k + 1): s * (k + 1) + len(draft) + 1] = bits
            drafts.append(draft)
            wants.append(reference_choices(draft, oracle.widen(bits, "bfloat16"), refs[s]))
        logits = torch.from_numpy(block.view(np.int16)).view(torch.bfloat16).cuda()
        its = verify_with_grammars(drafts, logits, gpus, k=k, buffer=buf)
        for s in range(seqs):
            assert list(its[s]) == wants[s], (rnd, s)
            assert (gpus[s].state, gpus[s].is_terminated()) == (refs[s].state, refs[s].is_terminated())


def test_grammar_round_synthesis_on_cpu():
    """The bench's round synthesis: fork-mask rows agree with fork_masks, drafts follow grammars."""
    torch = pytest.importorskip("torch")
    from bitmask_speculation_b200.grammar_verification import fork_masks

    def select(rows, masks):
        bits = rows.view(torch.int16).numpy().view(np.uint16)
        tok, _, st = oracle.reduce_rows(bits, masks, dtype="bfloat16")
        return tok, st

    vocab, seqs, k = 8320, 12, 8
    logits, masks, prop, lens, grammars, drafts = wl.grammar_round_torch(seqs, select, vocab=vocab, device="cpu")
    assert logits.shape == (seqs * (k + 1), vocab) and masks.shape == (seqs * (k + 1), (vocab + 31) // 32)
    buf = np.zeros((k + 1, masks.shape[1]), np.int32)
    for s in range(seqs):
        assert lens[s].item() == len(drafts[s]) and prop[s, : len(drafts[s])].tolist() == list(drafts[s])
        rows = fork_masks(grammars[s], drafts[s], vocab, buf)
        assert np.array_equal(buf[:rows], masks.numpy()[s * (k + 1): s * (k + 1) + rows])


def test_fork_state_indices_match_fork_masks():
    from bitmask_speculation_b200.grammar_verification import fork_state_indices
    vocab = 4096
    g = wl.SyntheticDFAGrammar(vocab, states=16, seed=5)
    table = np.vstack([g.mask_table(), np.zeros((1, g.mask_table().shape[1]), np.int32)])
    rng = np.random.default_rng(1)
    for _ in range(30):
        draft = [int(rng.choice(g.allowed_ids_np())) if rng.random() < 0.9 else int(rng.integers(vocab))
                 for _ in range(int(rng.integers(0, 9)))]
        masks = np.zeros((9, table.shape[1]), np.int32)
        idx = np.full(9, -5, np.int32)
        rows = fork_masks(g, draft, vocab, masks)
        assert fork_state_indices(g, draft, idx, g.mask_table().shape[0]) == rows
        assert np.array_equal(table[idx[:rows]], masks[:rows])


@pytest.mark.gpu
def test_device_mask_table_round_equals_uploaded_masks(cuda_module):
    """Table indices instead of mask words: same events, same grammar states; an index outside
    the table fails its row with status 8."""
    torch = pytest.importorskip("torch")
    from bitmask_speculation_b200.grammar_verification import (DeviceMaskTable, DraftForkMasks,
                                                               verify_with_grammars)
    from bitmask_speculation_b200.verification import verify_batch
    vocab, seqs, k = 248320, 32, 8
    rng = np.random.default_rng(23)
    base = wl.SyntheticDFAGrammar(vocab, states=64, seed=2)
    a = [base.fork() for _ in range(seqs)]
    for g in a:
        for _ in range(int(rng.integers(0, 4))):
            ids = g.allowed_ids_np()
            g.accept_token(int(rng.choice(ids[ids != 0])) if (ids != 0).any() else 0)
    b = [g.fork() for g in a]
    buf = DraftForkMasks(vocab, seqs * (k + 1), torch.device("cuda"))
    table = DeviceMaskTable.for_grammar(base, seqs * (k + 1), torch.device("cuda"))
    for rnd in range(2):
        block = np.zeros((seqs * (k + 1), vocab), dtype=np.uint16)
        drafts = []
        for s in range(seqs):
            if a[s].is_terminated():
                drafts.append(())
                continue
            rows, draft = make_round(rng, vocab, int(rng.integers(0, k + 1)), a[s].fork())
            block[s * (k + 1): s * (k + 1) + len(draft) + 1] = wl.to_bf16_bits(rows)
            drafts.append(draft)
        logits = torch.from_numpy(block.view(np.int16)).view(torch.bfloat16).cuda()
        want = [list(it) for it in verify_with_grammars(drafts, logits, a, k=k, buffer=buf)]
        got = [list(it) for it in verify_with_grammars(drafts, logits, b, k=k, table=table)]
        assert got == want, rnd
        assert [(g.state, g.is_terminated()) for g in a] == [(g.state, g.is_terminated()) for g in b]
    # out-of-range table indices fail exactly those rows
    rows = seqs * (k + 1)
    idx = torch.zeros(rows, dtype=torch.int32, device="cuda")
    idx[3] = 65
    idx[4] = -1
    res = verify_batch(logits, table.table, torch.zeros((seqs, k), dtype=torch.int64, device="cuda"),
                       torch.zeros(seqs, dtype=torch.int32, device="cuda"), mask_rows=idx).to_host()
    assert res.row_status[3] == 8 and res.row_status[4] == 8
    assert all(s != 8 for i, s in enumerate(res.row_status) if i not in (3, 4))
