"""Popcount, density and draft budgets on the GPU (tests/gpu/test_popcount.py of the reference)."""

import math

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.scheduling import DensityPolicy, LinearDensityPolicy, device_budgets

torch = pytest.importorskip("torch")
from bitmask_speculation_b200.kernels.cuda import mask_count, mask_density  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("vocab", [1, 31, 32, 33, 255, 256, 257, 248320, 248321])
@pytest.mark.parametrize("fill", [0, -1, -2147483648])
def test_signed_and_tail_counts_match_cpu(cuda_module, vocab, fill):
    cpu = np.full(((vocab + 31) // 32,), fill, dtype=np.int32)
    mask = torch.from_numpy(cpu).cuda()
    expected = oracle.mask_count(cpu, vocab)
    output = mask_count(mask, vocab)
    assert output.shape == () and output.dtype == torch.int64 and output.is_cuda
    assert output.item() == expected
    assert mask_density(mask, vocab).item() == pytest.approx(expected / vocab, rel=1e-15, abs=0)
    assert np.array_equal(mask.cpu().numpy(), cpu)


def test_repeated_calls_own_their_outputs(cuda_module):
    mask = torch.tensor([-1, -1], dtype=torch.int32, device="cuda")
    first = mask_count(mask, 33)
    second = mask_count(mask, 64)
    empty = mask_count(torch.zeros_like(mask), 64)
    assert (first.item(), second.item(), empty.item()) == (33, 64, 0)
    assert len({first.data_ptr(), second.data_ptr(), empty.data_ptr()}) == 3


def test_golden_counts(cuda_module, golden):
    from conftest import GOLDEN
    masks = np.load(GOLDEN / "count_masks.npz")
    for i, case in enumerate(golden["counts"]):
        vocab, fill = case["vocab"], case["fill"]
        mask = masks[f"m{i}"] if fill == "random" else np.full(wl.words_for(vocab), fill, np.int32)
        assert mask_count(torch.from_numpy(mask).cuda(), vocab).item() == case["count"], case


@pytest.mark.parametrize("policy", [DensityPolicy(), DensityPolicy(.1, .8, 2, 7), DensityPolicy(0, 1, 3, 3),
                                    LinearDensityPolicy(), LinearDensityPolicy(1e-4, 0.5, 2, 16)])
def test_device_budgets_match_policy_exactly(cuda_module, policy):
    rng = np.random.default_rng(3)
    vocab = 248320
    rows = 512
    counts = np.concatenate([
        np.array([0, 1, 2, 1240, 1241, 1242, 4966, 4967, 4968, 248, 249, 24832, 24833, vocab]),
        rng.integers(0, vocab + 1, rows - 14)])
    masks = np.zeros((rows, wl.words_for(vocab)), np.int32)
    valid = np.zeros((rows, vocab), bool)
    for r, c in enumerate(counts):
        valid[r, rng.choice(vocab, size=int(c), replace=False)] = True
    masks = wl.pack_bits_np(valid)
    got_c, got_d, got_k = device_budgets(torch.from_numpy(masks).cuda(), vocab, policy)
    assert got_c.tolist() == counts.tolist()
    assert got_d.tolist() == [int(c) / vocab for c in counts]
    assert got_k.tolist() == [policy.budget(int(c) / vocab) for c in counts]
    kind = 0 if isinstance(policy, DensityPolicy) else 1
    _, ok = oracle.budget_rows(counts, vocab, kind=kind, low=policy.low_density, high=policy.high_density,
                               min_budget=policy.min_budget, max_budget=policy.max_budget)
    assert got_k.tolist() == ok.tolist()


def test_budget_band_edges_at_the_reference_boundaries(cuda_module, golden):
    policy = DensityPolicy()
    for density, k in golden["policy"]["default"]:
        assert policy.budget(density) == k
    # counts whose density straddles 0.005 and 0.02 at V = 248,320
    for count, k in golden["policy"]["counts_at_248320"]:
        mask = wl.pack_bits_np(wl.exact_count_mask(np.random.default_rng(count), 248320, count)[None])
        _, _, got = device_budgets(torch.from_numpy(mask).cuda(), 248320, policy)
        assert got.item() == k, count
    assert math.nextafter(0.005, 0) < 0.005
