"""Batched verification on the GPU vs the oracle's verify_prefix restatement."""

import math

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import _native
from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.scheduling import DensityPolicy, LinearDensityPolicy
from helpers import to_device

torch = pytest.importorskip("torch")
from bitmask_speculation_b200.verification import VerifiedToken, verify_batch, verify_rows  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _reset_override():
    yield
    _native.set_launch_override(0, 0)


def oracle_round(bits, masks, proposals, lengths, dtype, policy):
    tokens, counts, status = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)
    accept, token, kind, seq_status = oracle.verify(tokens, status, proposals, lengths)
    kind_code = 0 if isinstance(policy, DensityPolicy) else 1
    _, budgets = oracle.budget_rows(counts, bits.shape[1], kind=kind_code, low=policy.low_density,
                                    high=policy.high_density, min_budget=policy.min_budget,
                                    max_budget=policy.max_budget)
    return dict(row_tokens=tokens, row_counts=counts, row_status=status, row_budget=budgets,
                accept_len=accept, token=token, kind=kind, seq_status=seq_status)


def run_round(bits, masks, proposals, lengths, dtype, policy):
    out = verify_batch(to_device(bits, dtype), torch.from_numpy(masks).cuda(),
                       torch.from_numpy(np.ascontiguousarray(proposals, np.int64)).cuda(),
                       torch.from_numpy(np.ascontiguousarray(lengths, np.int32)).cuda(), policy=policy)
    return out.to_host()


@pytest.mark.parametrize("policy", [DensityPolicy(), LinearDensityPolicy()])
def test_verify_config_matches_oracle(cuda_module, policy):
    bits, masks, proposals, lengths = wl.verify_config_np(seed=3, seqs=4)
    host = run_round(bits, masks, proposals, lengths, "bfloat16", policy)
    expect = oracle_round(bits, masks, proposals, lengths, "bfloat16", policy)
    for key, value in expect.items():
        assert getattr(host, key) == value.tolist(), key


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_random_rounds_with_ragged_lengths_and_failures(cuda_module, dtype):
    rng = np.random.default_rng(11)
    seqs, k, vocab = 40, 5, 4224
    rows = seqs * (k + 1)
    values = rng.standard_normal((rows, vocab), dtype=np.float32)
    valid = rng.random((rows, vocab)) < rng.choice([0.001, 0.05, 0.6], size=(rows, 1))
    valid[:, 0] |= rng.random(rows) < 0.5
    # NaN and empty rows sprinkled in: they fail a sequence only when consumed.
    for r in rng.choice(rows, 12, replace=False):
        values[r, rng.integers(vocab)] = np.nan
    for r in rng.choice(rows, 12, replace=False):
        valid[r] = False
    masks = wl.pack_bits_np(valid)
    bits = values if dtype == "float32" else (wl.to_bf16_bits(values) if dtype == "bfloat16" else wl.to_f16_bits(values))
    tok, _, st = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)
    proposals = np.zeros((seqs, k), np.int64)
    for s in range(seqs):
        for i in range(k):
            row = s * (k + 1) + i
            proposals[s, i] = tok[row] if (rng.random() < 0.8 and tok[row] >= 0) else rng.integers(vocab)
    lengths = rng.integers(0, k + 1, size=seqs).astype(np.int32)
    policy = DensityPolicy()
    host = run_round(bits, masks, proposals, lengths, dtype, policy)
    expect = oracle_round(bits, masks, proposals, lengths, dtype, policy)
    for key, value in expect.items():
        assert getattr(host, key) == value.tolist(), key
    assert any(host.seq_status) and not all(host.seq_status)


def test_nan_after_mismatch_is_ignored_but_consumed_nan_fails(cuda_module):
    vocab, k = 64, 3
    logits = torch.zeros((k + 1, vocab), device="cuda")
    for i, choice in enumerate([5, 9, 0, 0]):
        logits[i, choice] = 10.0
    masks = torch.full((k + 1, 2), -1, dtype=torch.int32, device="cuda")
    logits[2:] = math.nan  # rows after the first mismatch
    events = list(verify_rows([5, 4, 7], logits, masks))
    assert events == [VerifiedToken(5, "accepted"), VerifiedToken(9, "correction")]
    logits[0] = math.nan
    stream = verify_rows([5, 4, 7], logits, masks)
    with pytest.raises(ValueError, match="NaN"):
        next(stream)


def test_bonus_and_fallback_kinds(cuda_module):
    vocab = 64
    logits = torch.zeros((3, vocab), device="cuda")
    logits[0, 1] = logits[1, 2] = logits[2, 3] = 5.0
    masks = torch.full((3, 2), -1, dtype=torch.int32, device="cuda")
    assert [(e.token_id, e.kind) for e in verify_rows([1, 2], logits, masks)] == [
        (1, "accepted"), (2, "accepted"), (3, "bonus")]
    assert [(e.token_id, e.kind) for e in verify_rows([], logits[:1].contiguous(), masks[:1].contiguous())] == [
        (1, "fallback")]


def test_golden_verification_event_sequences(cuda_module, golden):
    """Every golden verify_prefix case, replayed as one-hot target rows on the GPU."""
    for case in golden["verification"]:
        vocab, draft, targets = case["vocab"], case["draft"], case["targets"]
        rows = len(draft) + 1
        logits = torch.zeros((rows, vocab), device="cuda")
        for i, t in enumerate(targets[:rows]):
            logits[i, t] = 1.0
        masks = torch.full((rows, 1), -1, dtype=torch.int32, device="cuda")
        events = [(e.token_id, e.kind) for e in verify_rows(draft, logits, masks)]
        assert events == [tuple(e) for e in case["events"]], case


def test_bad_lengths_are_flagged_per_sequence(cuda_module):
    vocab, k = 32, 2
    logits = torch.zeros((2 * (k + 1), vocab), device="cuda")
    masks = torch.full((2 * (k + 1), 1), -1, dtype=torch.int32, device="cuda")
    proposals = torch.zeros((2, k), dtype=torch.int64, device="cuda")
    lengths = torch.tensor([3, 2], dtype=torch.int32, device="cuda")
    host = verify_batch(logits, masks, proposals, lengths).to_host()
    assert host.seq_status == [6, 0]
    assert host.accept_len[1] == 2 and host.kind[1] == 1


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_indexed_selection_into_caller_buffers(cuda_module, dtype):
    """``select_indexed_into`` (one-row verification rounds through a device table index, no
    workspace): every row's token and status equal the oracle's on its table row, an index past the
    table fails its row with status 8, an all-zero table row with status 1; replayed from a CUDA
    graph it gives the same results."""
    rng = np.random.default_rng(31)
    vocab, rows = 151936, 7
    table = wl.pack_bits_np(rng.random((5, vocab)) < rng.choice([0.5, 0.01, 1e-4], size=(5, 1)))
    table[4] = 0
    index = np.array([0, 1, 2, 3, 4, 5, 2], dtype=np.int32)  # 4: empty row, 5: past the table
    values = rng.standard_normal((rows, vocab), dtype=np.float32)
    from helpers import as_dtype_bits
    bits = as_dtype_bits(values, dtype)
    dt = None if dtype == "float32" else dtype
    want_tok, _, want_st = oracle.reduce_rows(bits, table[index.clip(0, 4)], dtype=dt)
    want_st[5], want_tok[5] = 8, -1
    logits, dtable = to_device(bits, dtype), torch.from_numpy(table).cuda()
    didx = torch.from_numpy(index).cuda()
    tokens = torch.full((rows,), -7, dtype=torch.int64, device="cuda")
    status = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(6 * rows, dtype=torch.int32, device="cuda")
    cuda_module.select_indexed_into(logits, dtable, didx, tokens, status, scratch)
    assert status.cpu().tolist() == want_st.tolist()
    assert tokens.cpu().tolist() == want_tok.tolist()
    tokens.fill_(-7)
    status.fill_(-7)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="relaxed"):
        cuda_module.select_indexed_into(logits, dtable, didx, tokens, status, scratch)
    graph.replay()
    torch.cuda.synchronize()
    assert status.cpu().tolist() == want_st.tolist()
    assert tokens.cpu().tolist() == want_tok.tolist()
