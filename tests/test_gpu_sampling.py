"""Masked sampling on the GPU: reference tests, golden vectors, oracle parity, chi-square.

Tolerance (stated here, as the parity contract requires): a sampled index must
equal the reference's for the same uniform u, except when u lies within 1e-6
(in normalised CDF units) of a CDF boundary of the GPU's token.
"""

import math

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import _native
from bitmask_speculation_b200 import workloads as wl
from helpers import as_dtype_bits, sample_matches, to_device, widened

torch = pytest.importorskip("torch")
from bitmask_speculation_b200.kernels.cuda import (_checked_selection, batched_masked_sample,  # noqa: E402
                                                   masked_argmax, masked_sample)

pytestmark = pytest.mark.gpu
TOL = 1e-6


@pytest.fixture(autouse=True)
def _reset_override():
    yield
    _native.set_launch_override(0, 0)


def _ref(values, mask, temperature, uniform):
    tokens, status = oracle.sample_rows(np.asarray([values], np.float32), np.asarray([mask], np.int32),
                                        temperature, [uniform])
    return int(tokens[0]), int(status[0])


# ---------------------------------------------------------------- reference tests
@pytest.mark.parametrize("temperature", [0.0, 1e-320, .1, 1.0, 100.0])
@pytest.mark.parametrize("uniform", [0.0, .13, .51, .999999999])
def test_native_sampling_matches_explicit_uniform_reference(cuda_module, temperature, uniform):
    values = [1000., -math.inf, -2., 1., .5]
    expected, _ = _ref(values, [-2], temperature, uniform)
    result = _checked_selection(cuda_module.masked_sample(
        torch.tensor(values, device="cuda"), torch.tensor([-2], dtype=torch.int32, device="cuda"), temperature,
        torch.tensor(uniform, dtype=torch.float64, device="cuda")))
    assert result.item() == expected


def test_seed_replay_and_greedy_consumes_no_rng(cuda_module):
    logits = torch.zeros(3, device="cuda")
    mask = torch.tensor([7], dtype=torch.int32, device="cuda")
    generator = torch.Generator(device=logits.device).manual_seed(37)
    state = generator.get_state().clone()
    greedy = masked_sample(logits, mask, temperature=0, generator=generator)
    assert torch.equal(state, generator.get_state())
    assert greedy.item() == masked_argmax(logits, mask).item()
    first = [masked_sample(logits, mask, generator=generator).item() for _ in range(32)]
    assert not torch.equal(state, generator.get_state())
    generator.set_state(state)
    assert first == [masked_sample(logits, mask, generator=generator).item() for _ in range(32)]


def test_empirical_probabilities_match_masked_softmax(cuda_module):
    logits = torch.tensor([999., 0., math.log(3.)], device="cuda")
    mask = torch.tensor([6], dtype=torch.int32, device="cuda")
    generator = torch.Generator(device=logits.device).manual_seed(123)
    tokens = [masked_sample(logits, mask, generator=generator).item() for _ in range(4096)]
    assert set(tokens) <= {1, 2}
    assert abs(tokens.count(1) / len(tokens) - .25) < .05


@pytest.mark.parametrize("values,word,match", [
    ([0.], 0, "no valid"), ([-math.inf], 1, "finite probability"),
    ([math.inf], 1, "positive infinity"), ([0., math.nan], 1, "NaN"),
])
def test_sampling_value_errors(cuda_module, values, word, match):
    with pytest.raises(ValueError, match=match):
        masked_sample(torch.tensor(values, device="cuda"), torch.tensor([word], dtype=torch.int32, device="cuda"))


def test_invalid_uniform_native_status(cuda_module):
    for uniform in [-.1, 1., math.nan]:
        with pytest.raises(ValueError, match="uniform"):
            _checked_selection(cuda_module.masked_sample(
                torch.zeros(1, device="cuda"), torch.ones(1, dtype=torch.int32, device="cuda"), 1.,
                torch.tensor(uniform, dtype=torch.float64, device="cuda")))


@pytest.mark.parametrize("vocab", [4097, 151936])
def test_large_vocabulary_sampling_matches_reference(cuda_module, vocab):
    generator = torch.Generator(device="cuda").manual_seed(7)
    logits = torch.randn(vocab, device="cuda", generator=generator) * 3
    mask = torch.randint(-2147483648, 2147483647, ((vocab + 31) // 32,), device="cuda",
                         dtype=torch.int32, generator=generator)
    mask[0] |= 1
    row, mrow = logits.cpu().numpy(), mask.cpu().numpy()
    for temperature in (0.5, 1.0, 4.0):
        for uniform in (0.0, 0.17, 0.5, 0.83, 0.999):
            expected, _ = _ref(row, mrow, temperature, uniform)
            actual = _checked_selection(cuda_module.masked_sample(
                logits, mask, temperature, torch.tensor(uniform, dtype=torch.float64, device="cuda"))).item()
            assert sample_matches(row, mrow, temperature, uniform, actual, expected, TOL)


# ---------------------------------------------------------------- golden vectors
def test_golden_known_answers(cuda_module, golden):
    for case in golden["sampling_known"]:
        values = torch.tensor(case["values"], dtype=torch.float32, device="cuda")
        mask = torch.tensor(case["mask"], dtype=torch.int32, device="cuda")
        u = torch.tensor(case["uniform"], dtype=torch.float64, device="cuda")
        token, status = cuda_module.masked_sample(values, mask, case["temperature"], u)
        if case["error"]:
            assert status.item() != 0, case
        else:
            assert status.item() == 0 and token.item() == case["token"], case


def test_golden_random_rows(cuda_module, golden):
    for row in golden["sampling_rows"]:
        values = np.asarray(row["values"], np.float32)
        mask = np.asarray(row["mask"], np.int32)
        for temperature, uniform, token, _ in row["results"]:
            got = cuda_module.masked_sample(torch.from_numpy(values).cuda(), torch.from_numpy(mask).cuda(),
                                            temperature, torch.tensor(uniform, dtype=torch.float64, device="cuda"))
            assert got[1].item() == 0
            assert sample_matches(values, mask, temperature, uniform, got[0].item(), token, TOL)


def test_golden_sampling_config_fp16_batched(cuda_module, golden):
    bits, masks, uniforms, temperature = wl.sample_config_np(seed=2)
    rows = []
    us = []
    for r, results in enumerate(golden["sampling_config_seed2"]):
        for u, _, _ in results:
            rows.append(r)
            us.append(u)
    logits = to_device(bits[rows], "float16")
    m = torch.from_numpy(masks[rows]).cuda()
    u = torch.tensor(us, dtype=torch.float64, device="cuda")
    tokens, counts, status = cuda_module.masked_sample_batch(logits, m, temperature, u)
    assert status.tolist() == [0] * len(rows)
    expect = [t for results in golden["sampling_config_seed2"] for _, t, _ in results]
    f32 = widened(bits, "float16")
    for i, r in enumerate(rows):
        assert sample_matches(f32[r], masks[r], temperature, us[i], tokens[i].item(), expect[i], TOL), (r, us[i])
    assert counts.tolist() == [oracle.mask_count(masks[r], wl.VOCAB) for r in rows]


# ---------------------------------------------------------------- oracle parity, all shapes
@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("cluster", [0, 1, 4, 16])
def test_batched_sampler_matches_oracle(cuda_module, dtype, cluster):
    rng = np.random.default_rng(200 + cluster)
    _native.set_launch_override(cluster, 0)
    for vocab in [248320, 151936, 8320, 50257]:
        rows = 6
        values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(2.5)
        dens = [1.0, 0.5, 0.01, 0.3, 1e-4, 0.9]
        valid = np.stack([rng.random(vocab) < d for d in dens])
        valid[:, 0] = True
        values[3, rng.random(vocab) < 0.1] = -np.inf   # zero-mass valid tokens
        masks = wl.pack_bits_np(valid)
        bits = as_dtype_bits(values, dtype)
        f32 = widened(bits, dtype)
        for temperature in (0.7, 1.0, 3.0):
            u = rng.random(rows)
            exp_tok, exp_st = oracle.sample_rows(bits, masks, temperature, u,
                                                 dtype=None if dtype == "float32" else dtype)
            tokens, _, status = cuda_module.masked_sample_batch(
                to_device(bits, dtype), torch.from_numpy(masks).cuda(), temperature,
                torch.from_numpy(u).cuda())
            assert status.tolist() == exp_st.tolist()
            for r in range(rows):
                assert sample_matches(f32[r], masks[r], temperature, u[r], tokens[r].item(), exp_tok[r], TOL), (
                    vocab, temperature, r)


def test_batched_sampler_row_errors_are_independent(cuda_module):
    vocab = 8192
    logits = torch.zeros((6, vocab), device="cuda")
    masks = torch.full((6, vocab // 32), -1, dtype=torch.int32, device="cuda")
    masks[0] = 0
    logits[1, 5] = math.nan
    logits[2, 7] = math.inf
    logits[3] = -math.inf
    u = torch.tensor([.5, .5, .5, .5, 1.0, .25], dtype=torch.float64, device="cuda")
    tokens, counts, status = cuda_module.masked_sample_batch(logits, masks, 1.0, u)
    assert status.tolist() == [1, 2, 5, 4, 3, 0]
    assert tokens.tolist()[:5] == [-1] * 5
    assert 0 <= tokens[5].item() < vocab


def test_chi_square_on_row_zero(cuda_module):
    """10^6 draws of configuration-2 row 0 against oracle fp64 probabilities."""
    scipy_stats = pytest.importorskip("scipy.stats")
    bits, masks, _, temperature = wl.sample_config_np(seed=2)
    x = widened(bits[0], "float16").astype(np.float64)
    mw = masks[0].view(np.uint32)
    t = np.arange(wl.VOCAB)
    valid = ((mw[t >> 5] >> (t & 31).astype(np.uint32)) & 1).astype(bool)
    w = np.where(valid, np.exp((x - x[valid].max()) / temperature), 0.0)
    p = w / w.sum()
    copies = 1000
    logits = to_device(np.repeat(bits[:1], copies, 0), "float16")
    m = torch.from_numpy(np.repeat(masks[:1], copies, 0)).cuda()
    g = torch.Generator(device="cuda").manual_seed(2024)
    hist = torch.zeros(wl.VOCAB, dtype=torch.int64, device="cuda")
    for _ in range(1000):
        u = torch.rand(copies, dtype=torch.float64, device="cuda", generator=g)
        tokens, _, status = cuda_module.masked_sample_batch(logits, m, temperature, u)
        hist += torch.bincount(tokens, minlength=wl.VOCAB)
    counts = hist.cpu().numpy()
    n = counts.sum()
    assert n == 10**6
    # Bins of tokens in descending probability, each with expected count >= 5.
    order = np.argsort(-p)
    exp_sorted = p[order] * n
    obs_sorted = counts[order]
    edges, acc = [], 0.0
    for i, e in enumerate(exp_sorted):
        acc += e
        if acc >= 5:
            edges.append(i + 1)
            acc = 0.0
    if edges[-1] != len(order):
        edges[-1] = len(order)
    starts = [0] + edges[:-1]
    f_exp = np.array([exp_sorted[a:b].sum() for a, b in zip(starts, edges)])
    f_obs = np.array([obs_sorted[a:b].sum() for a, b in zip(starts, edges)])
    f_exp *= f_obs.sum() / f_exp.sum()
    stat, pvalue = scipy_stats.chisquare(f_obs, f_exp)
    assert pvalue > 1e-3, (stat, pvalue, len(f_exp))


@pytest.mark.parametrize("temperature", [1e-320, 1e-40, 1e-3, 0.05, 7.0, 1e30, 1e300])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_extreme_temperatures_and_magnitudes_on_the_bulk_path(cuda_module, temperature, dtype):
    """Huge logits, ties at the maximum, -inf valid tokens, tiny and huge temperatures (V = 8,192)."""
    rng = np.random.default_rng(31)
    vocab, rows = 8192, 6
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(4)
    values[0, :10] = 3e38          # huge logits (x - max must not overflow)
    values[0, 10:20] = -3e38
    values[1, 100] = values[1, 4000] = values[1].max() + 1  # tied maxima
    values[2, rng.random(vocab) < 0.5] = -np.inf
    values[3] = np.round(values[3])  # many ties everywhere
    valid = rng.random((rows, vocab)) < 0.7
    valid[:, 0] = True
    valid[1, [100, 4000]] = True
    masks = wl.pack_bits_np(valid)
    bits = as_dtype_bits(values, dtype)
    f32 = widened(bits, dtype)
    u = np.array([0.0, 0.3, 0.5, 0.999, 0.77, 0.123456])
    exp_tok, exp_st = oracle.sample_rows(bits, masks, temperature, u, dtype=None if dtype == "float32" else dtype)
    tokens, _, status = cuda_module.masked_sample_batch(to_device(bits, dtype), torch.from_numpy(masks).cuda(),
                                                        temperature, torch.from_numpy(u).cuda())
    assert status.tolist() == exp_st.tolist()
    for r in range(rows):
        assert sample_matches(f32[r], masks[r], temperature, u[r], tokens[r].item(), exp_tok[r], TOL), (r, temperature)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("cluster", [0, 1, 4])
def test_rising_maxima_and_large_offsets(cuda_module, dtype, cluster):
    """Running maxima that rise chunk after chunk, jumps just below and above 2^20 in weight,
    and logits far from zero (|max log2(e) / T| beyond 2^11), against the oracle."""
    rng = np.random.default_rng(77 + cluster)
    _native.set_launch_override(cluster, 0)
    vocab, rows = 151936, 8
    values = rng.standard_normal((rows, vocab), dtype=np.float32)
    values[0] = np.linspace(-50, 50, vocab, dtype=np.float32)           # rises in every chunk
    values[1] = np.linspace(50, -50, vocab, dtype=np.float32)           # first chunk holds the max
    values[2, -3000:] += 9.0                                            # late jump, 2^13 in weight
    values[3, -3000:] += 16.0                                           # late jump, 2^23 in weight
    values[4, 70000:70010] = 40.0                                       # isolated spike mid-row
    if dtype == "float32":
        values[5] = values[5] * 3 + 3000.0                              # m log2(e) / T ~ 4.3e3
        values[6] = values[6] * 2 + 1e6                                 # ~1.4e6
        values[7] = values[7] * 500 + 1e9                               # ~1.4e7 at T = 100
    else:
        values[5] = values[5] * 3 + 3000.0
        values[6] = values[6] * 64 + 1e5
        values[7] = values[7] * 2048 + 1e7
    valid = rng.random((rows, vocab)) < 0.6
    valid[:, -1] = True
    masks = wl.pack_bits_np(valid)
    bits = as_dtype_bits(values, dtype)
    f32 = widened(bits, dtype)
    for temperature in (0.5, 1.0, 100.0):
        for trial in range(3):
            u = rng.random(rows)
            exp_tok, exp_st = oracle.sample_rows(bits, masks, temperature, u,
                                                 dtype=None if dtype == "float32" else dtype)
            tokens, _, status = cuda_module.masked_sample_batch(
                to_device(bits, dtype), torch.from_numpy(masks).cuda(), temperature, torch.from_numpy(u).cuda())
            assert status.tolist() == exp_st.tolist()
            for r in range(rows):
                assert sample_matches(f32[r], masks[r], temperature, u[r], tokens[r].item(), exp_tok[r], TOL), (
                    r, temperature, trial)
