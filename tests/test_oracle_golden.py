"""Pin the CPU oracle to outputs of the reference implementation itself.

The golden fixtures were produced by ``tests/golden/make_golden.py`` from the
reference's own ``torch_reduce``, ``masked_argmax``, ``packed_mask_count``,
``masked_sample_reference``, ``verify_prefix`` and ``DensityPolicy``.
"""

import math

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl

from conftest import GOLDEN


@pytest.fixture(scope="module")
def reduce_small():
    return np.load(GOLDEN / "reduce_small.npz")


def test_reduce_small_cases_match_reference(golden, reduce_small):
    for i, meta in enumerate(golden["reduce_small"]):
        values = reduce_small[f"c{i}_values"]
        masks = reduce_small[f"c{i}_masks"]
        dtype = meta["dtype"]
        tokens, counts, status = oracle.reduce_rows(values, masks, dtype=dtype if dtype != "float32" else None)
        assert tokens.tolist() == reduce_small[f"c{i}_tokens"].tolist(), meta
        assert counts.tolist() == reduce_small[f"c{i}_counts"].tolist(), meta
        assert status.tolist() == reduce_small[f"c{i}_status"].tolist(), meta


def test_argmax_config_matches_reference(golden):
    values, masks = wl.argmax_config_np(seed=1)
    tokens, counts, status = oracle.reduce_rows(values, masks)
    expect = golden["reduce_configs"]["argmax_config_seed1"]
    assert [tokens.tolist(), counts.tolist(), status.tolist()] == expect
    assert counts.tolist()[2:] == [4, 16, counts[4], 1]


def test_verify_config_reduce_and_counts_match_reference(golden):
    bits, masks, proposals, lengths = wl.verify_config_np(seed=3, seqs=4)
    tokens, counts, status = oracle.reduce_rows(bits, masks, dtype="bfloat16")
    assert [tokens.tolist(), counts.tolist(), status.tolist()] == golden["reduce_configs"][
        "verify_config_seed3_seqs4_reduce"]
    assert counts.tolist() == golden["reduce_configs"]["verify_config_seed3_seqs4_counts_ref"]


def test_counts_match_packed_mask_count(golden):
    masks = np.load(GOLDEN / "count_masks.npz")
    for i, case in enumerate(golden["counts"]):
        vocab, fill = case["vocab"], case["fill"]
        if fill == "random":
            mask = masks[f"m{i}"]
        else:
            mask = np.full(wl.words_for(vocab), fill, np.int32)
        assert oracle.mask_count(mask, vocab) == case["count"], case
    for word, vocab, count in golden["signed_words"]:
        assert oracle.mask_count(np.array([word], np.int32), vocab) == count


def _sample(values, mask, temperature, uniform):
    v = np.asarray([values], np.float32)
    m = np.asarray([mask], np.int64).astype(np.int32)
    return oracle.sample_rows(v, m, temperature, [uniform])


ERRORS = {1: "no valid", 2: "NaN", 3: "uniform", 4: "finite probability", 5: "positive infinity"}


def test_sampling_known_answers(golden):
    for case in golden["sampling_known"]:
        tokens, status = _sample(case["values"], case["mask"], case["temperature"], case["uniform"])
        if case["error"]:
            assert status[0] != 0 and ERRORS[int(status[0])] in case["error"], case
        else:
            assert status[0] == 0 and tokens[0] == case["token"], case


def test_sampling_random_rows(golden):
    for row in golden["sampling_rows"]:
        for temperature, uniform, token, error in row["results"]:
            tokens, status = _sample(row["values"], row["mask"], temperature, uniform)
            assert not error and status[0] == 0 and tokens[0] == token, (row["vocab"], temperature, uniform)


def test_sampling_config_fp16(golden):
    bits, masks, uniforms, temperature = wl.sample_config_np(seed=2)
    for r, results in enumerate(golden["sampling_config_seed2"]):
        us = [u for u, _, _ in results]
        tokens, status = oracle.sample_rows(np.repeat(bits[r:r + 1], len(us), 0),
                                            np.repeat(masks[r:r + 1], len(us), 0),
                                            temperature, us, dtype="float16")
        assert status.tolist() == [0] * len(us)
        assert tokens.tolist() == [t for _, t, _ in results], r


def test_fsum_matches_math_fsum():
    rng = np.random.default_rng(3)
    for n in [0, 1, 2, 10, 1000, 100000]:
        x = rng.random(n) * np.exp(rng.uniform(-40, 40, n))
        assert oracle.fsum(x) == math.fsum(x.tolist())
    assert oracle.fsum([1e16, 1.0, 1e-16]) == math.fsum([1e16, 1.0, 1e-16])
    assert oracle.fsum([0.1] * 10) == 1.0


def test_policy_budgets(golden):
    for density, k in golden["policy"]["default"]:
        assert oracle.budget(density) == k, density
    for density, k in golden["policy"]["custom_0.1_0.8_2_7"]:
        assert oracle.budget(density, low=.1, high=.8, min_budget=2, max_budget=7) == k
    for density, k in golden["policy"]["constant_0_1_3_3"]:
        assert oracle.budget(density, low=0, high=1, min_budget=3, max_budget=3) == k
    for count, k in golden["policy"]["counts_at_248320"]:
        _, budget = oracle.budget_rows([count], 248320)
        assert budget[0] == k, count


def test_linear_policy_endpoints():
    assert oracle.budget(0.0, kind=1, low=1e-3, high=0.1) == 8
    assert oracle.budget(math.nextafter(1e-3, 0), kind=1, low=1e-3, high=0.1) == 8
    assert oracle.budget(1e-3, kind=1, low=1e-3, high=0.1) == 8
    assert oracle.budget(0.1, kind=1, low=1e-3, high=0.1) == 1
    assert oracle.budget(0.5, kind=1, low=1e-3, high=0.1) == 1
    mids = [oracle.budget(d, kind=1, low=1e-3, high=0.1) for d in np.linspace(1e-3, 0.1, 50)]
    assert mids == sorted(mids, reverse=True)


def test_verification_events(golden):
    kinds = {0: "correction", 1: "bonus", 2: "fallback"}
    for case in golden["verification"]:
        draft, targets = case["draft"], case["targets"]
        k = len(draft)
        row_tokens = np.asarray(targets, np.int64)[None, :]
        status = np.zeros_like(row_tokens, dtype=np.int32)
        proposals = np.asarray([draft], np.int64).reshape(1, k)
        accept, token, kind, seq_status = oracle.verify(row_tokens, status, proposals, [k])
        events = case["events"]
        assert seq_status[0] == 0
        assert accept[0] == len(events) - 1
        assert [list(e) for e in events[:-1]] == [[t, "accepted"] for t in draft[:accept[0]]]
        assert [int(token[0]), kinds[int(kind[0])]] == list(events[-1])
        # Rows the reference never requested are the ones the oracle never inspected.
        assert case["calls"] == list(range(len(events)))


def test_verification_ignores_failed_rows_after_mismatch():
    # Row 2 (after a mismatch at row 1) is NaN: no error; row 0 NaN: error.
    tokens = np.array([[5, 3, -1, -1]])
    status = np.array([[0, 0, 2, 2]], np.int32)
    accept, token, kind, seq_status = oracle.verify(tokens, status, [[5, 4, 9]], [3])
    assert (accept[0], token[0], kind[0], seq_status[0]) == (1, 3, 0, 0)
    status = np.array([[2, 0, 0, 0]], np.int32)
    accept, token, kind, seq_status = oracle.verify(tokens, status, [[5, 4, 9]], [3])
    assert (token[0], seq_status[0]) == (-1, 2)
