"""Fused masked argmax + count on the GPU vs the reference's tests, golden vectors and the oracle.

Mirrors tests/gpu/test_argmax.py, test_cuda_batch.py and test_random_masks.py of
the reference, then compares every dtype and launch shape with the CPU oracle
bit for bit (token, count, status).
"""

import math

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import _native
from bitmask_speculation_b200 import workloads as wl
from conftest import GOLDEN
from helpers import as_dtype_bits, to_device

torch = pytest.importorskip("torch")
from bitmask_speculation_b200.kernels import cuda  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _reset_override():
    yield
    _native.set_launch_override(0, 0)


# ---------------------------------------------------------------- reference tests
@pytest.mark.parametrize("vocab", [1, 31, 32, 33, 255, 256, 257, 8193])
@pytest.mark.parametrize("value", [0.0, float("-inf"), float("inf")])
def test_ties_choose_first_valid_across_lanes_and_warps(cuda_module, vocab, value):
    logits = torch.full((vocab,), value, dtype=torch.float32, device="cuda")
    mask = torch.full(((vocab + 31) // 32,), -1, dtype=torch.int32, device="cuda")
    assert cuda.masked_argmax(logits, mask).item() == 0


def test_sparse_support_excludes_higher_invalid_logit(cuda_module):
    logits = torch.zeros(257, device="cuda")
    logits[0] = 999
    logits[31] = logits[256] = 10
    mask = torch.zeros(9, dtype=torch.int32, device="cuda")
    mask[0] = -2147483648
    mask[-1] = -1  # Dirty tail must not create out-of-vocabulary candidates.
    before = logits.clone()
    assert cuda.masked_argmax(logits, mask).item() == 31
    assert torch.equal(logits, before)


def test_empty_support_and_nan_are_explicit_errors(cuda_module):
    logits = torch.zeros(33, device="cuda")
    mask = torch.zeros(2, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="no valid"):
        cuda.masked_argmax(logits, mask)
    mask[0] = 1
    logits[32] = float("nan")  # NaN at an invalid position must still fail.
    with pytest.raises(ValueError, match="NaN"):
        cuda.masked_argmax(logits, mask)


def reference_rows(logits, masks):
    vocab = logits.shape[1]
    ids = torch.arange(vocab, device=logits.device)
    tokens, counts = [], []
    for row in range(logits.shape[0]):
        allowed = ((masks[row, ids // 32].to(torch.int64) >> (ids % 32)) & 1).bool()
        valid = ids[allowed]
        tokens.append(valid[logits[row, valid].argmax()].item() if valid.numel() else -1)
        counts.append(int(allowed.sum()))
    return tokens, counts


@pytest.mark.parametrize("batch,vocab", [(0, 33), (1, 1), (1, 4095), (1, 4097), (3, 33),
                                         (6, 151936), (12, 248320)])
def test_batch_matches_reference_rows(cuda_module, batch, vocab):
    generator = torch.Generator(device="cuda").manual_seed(41)
    logits = torch.randn((batch, vocab), device="cuda", generator=generator)
    masks = torch.randint(-2147483648, 2147483647, (batch, (vocab + 31) // 32),
                          device="cuda", dtype=torch.int32, generator=generator)
    if batch:
        masks[:, 0] |= 1
    saved = logits.clone(), masks.clone()
    result = cuda.batched_masked_reduce(logits, masks).check()
    assert result.token_ids.shape == result.valid_counts.shape == result.status.shape == (batch,)
    tokens, counts = reference_rows(logits, masks)
    assert result.token_ids.tolist() == tokens and result.valid_counts.tolist() == counts
    for row in range(batch):
        assert cuda.masked_argmax(logits[row].contiguous(), masks[row].contiguous()).item() == tokens[row]
    assert torch.equal(logits, saved[0]) and torch.equal(masks, saved[1])


def test_batch_rows_fail_independently_and_ties_pick_lowest_id(cuda_module):
    logits = torch.zeros((4, 8193), device="cuda")
    masks = torch.full((4, 257), -1, device="cuda", dtype=torch.int32)
    masks[0] = 0
    logits[1, 8192] = math.nan
    logits[2, 4096] = logits[2, 8191] = 5.0  # equal maxima in different blocks
    result = cuda.batched_masked_reduce(logits, masks)
    assert result.status.tolist() == [1, 2, 0, 0]
    assert result.token_ids.tolist()[2:] == [4096, 0]
    assert result.valid_counts.tolist() == [0, 8193, 8193, 8193]


@pytest.mark.parametrize("vocab", [31, 32, 33, 255, 256, 257, 4097, 248321])
def test_random_words_and_logits_match_independent_references(cuda_module, vocab):
    from bitmask_speculation_b200.kernels.cuda import mask_count, masked_argmax
    generator = torch.Generator().manual_seed(vocab)
    for _ in range(4):
        mask = torch.randint(-(1 << 31), (1 << 31), ((vocab + 31) // 32,), dtype=torch.int32, generator=generator)
        mask[0] |= 1
        logits = torch.randn(vocab, generator=generator)
        cuda_mask, cuda_logits = mask.cuda(), logits.cuda()
        assert mask_count(cuda_mask, vocab).item() == oracle.mask_count(mask.numpy(), vocab)
        tok, _, _ = oracle.reduce_rows(logits.numpy()[None], mask.numpy()[None])
        assert masked_argmax(cuda_logits, cuda_mask).item() == tok[0]
        assert torch.equal(cuda_mask.cpu(), mask) and torch.equal(cuda_logits.cpu(), logits)


# ---------------------------------------------------------------- golden vectors
def test_golden_small_cases_all_dtypes(cuda_module, golden):
    data = np.load(GOLDEN / "reduce_small.npz")
    for i, meta in enumerate(golden["reduce_small"]):
        values = to_device(data[f"c{i}_values"], meta["dtype"])
        masks = torch.from_numpy(data[f"c{i}_masks"]).cuda()
        tokens, counts, status = cuda_module.masked_reduce_batch(values, masks)
        assert tokens.tolist() == data[f"c{i}_tokens"].tolist(), meta
        assert counts.tolist() == data[f"c{i}_counts"].tolist(), meta
        assert status.tolist() == data[f"c{i}_status"].tolist(), meta


def test_golden_argmax_config(cuda_module, golden):
    values, masks = wl.argmax_config_np(seed=1)
    tokens, counts, status = cuda_module.masked_reduce_batch(to_device(values, "float32"),
                                                             torch.from_numpy(masks).cuda())
    assert [tokens.tolist(), counts.tolist(), status.tolist()] == golden["reduce_configs"]["argmax_config_seed1"]


def test_golden_verify_config_rows_bf16(cuda_module, golden):
    bits, masks, _, _ = wl.verify_config_np(seed=3, seqs=4)
    tokens, counts, status = cuda_module.masked_reduce_batch(to_device(bits, "bfloat16"),
                                                             torch.from_numpy(masks).cuda())
    assert [tokens.tolist(), counts.tolist(), status.tolist()] == golden["reduce_configs"][
        "verify_config_seed3_seqs4_reduce"]


# ---------------------------------------------------------------- oracle, every launch shape
def random_batch(rng, rows, vocab, dtype, style="plain"):
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(3)
    if style == "ties":
        values = np.round(values)
    masks = rng.integers(-(1 << 31), 1 << 31, size=(rows, wl.words_for(vocab)), dtype=np.int64).astype(np.int32)
    if style == "sparse":
        masks &= rng.integers(-(1 << 31), 1 << 31, size=masks.shape, dtype=np.int64).astype(np.int32)
        masks &= rng.integers(-(1 << 31), 1 << 31, size=masks.shape, dtype=np.int64).astype(np.int32)
        masks[:, rng.random(masks.shape[1]) < 0.9] = 0
    if rows >= 3:
        masks[1] = 0                                        # empty row
        values[2, rng.integers(vocab)] = np.nan             # NaN row
    return as_dtype_bits(values, dtype), masks


def compare_with_oracle(cuda_module, values, masks, dtype):
    expect = oracle.reduce_rows(values, masks, dtype=None if dtype == "float32" else dtype)
    got = cuda_module.masked_reduce_batch(to_device(values, dtype), torch.from_numpy(masks).cuda())
    for g, e, name in zip(got, expect, ("tokens", "counts", "status")):
        assert np.array_equal(g.cpu().numpy(), e), name


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("cluster", [0, 1, 2, 4, 8, 16])
def test_oracle_parity_every_cluster_size(cuda_module, dtype, cluster):
    rng = np.random.default_rng(100 + cluster)
    _native.set_launch_override(cluster, 0)
    for vocab in [248320, 151936, 4224, 8192, 248321, 50257]:
        for style in ["plain", "ties", "sparse"]:
            values, masks = random_batch(rng, 5, vocab, dtype, style)
            compare_with_oracle(cuda_module, values, masks, dtype)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_persistent_clusters_loop_over_many_rows(cuda_module, dtype):
    """Few clusters, many rows: every cluster streams several rows through its ring."""
    rng = np.random.default_rng(7)
    values, masks = random_batch(rng, 37, 248320, dtype)
    for cluster, clusters in [(1, 3), (2, 5), (4, 2), (16, 1)]:
        _native.set_launch_override(cluster, clusters)
        compare_with_oracle(cuda_module, values, masks, dtype)


def test_more_rows_than_the_reference_grid_limit(cuda_module):
    rng = np.random.default_rng(8)
    rows, vocab = 70000, 64
    values = rng.standard_normal((rows, vocab), dtype=np.float32)
    masks = rng.integers(-(1 << 31), 1 << 31, size=(rows, 2), dtype=np.int64).astype(np.int32)
    compare_with_oracle(cuda_module, values, masks, "float32")


def test_unaligned_rows_use_the_plain_load_path(cuda_module):
    """Odd vocabularies (rows not 16-byte aligned) and views offset by one element."""
    rng = np.random.default_rng(9)
    for vocab in [1, 2, 3, 7, 33, 1025, 4097, 50257]:
        values, masks = random_batch(rng, 4, vocab, "bfloat16")
        compare_with_oracle(cuda_module, values, masks, "bfloat16")
    base = torch.randn(1 + 8192, device="cuda")
    row = base[1:]  # 4-byte aligned, not 16-byte aligned
    mask = torch.full((256,), -1, dtype=torch.int32, device="cuda")
    tok, _, _ = oracle.reduce_rows(row.cpu().numpy()[None], mask.cpu().numpy()[None])
    assert cuda.masked_argmax(row, mask).item() == tok[0]


def test_signed_words(cuda_module):
    for word, vocab, token, count in [(-2147483648, 32, 31, 1), (-1, 31, 0, 31), (2147483647, 32, 0, 31),
                                      (-2147483647, 32, 0, 2)]:
        logits = torch.zeros((1, vocab), device="cuda")
        mask = torch.tensor([[word]], dtype=torch.int32, device="cuda")
        tokens, counts, status = cuda_module.masked_reduce_batch(logits, mask)
        assert (tokens.item(), counts.item(), status.item()) == (token, count, 0)


def test_negative_zero_ties_with_positive_zero(cuda_module):
    logits = torch.tensor([[-0.0, 0.0, -1.0], [0.0, -0.0, -1.0]], device="cuda")
    mask = torch.tensor([[7], [7]], dtype=torch.int32, device="cuda")
    tokens, _, _ = cuda_module.masked_reduce_batch(logits, mask)
    assert tokens.tolist() == [0, 0]
