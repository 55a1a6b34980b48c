"""The dynamic schedule: ticketed rows, rows split across CTAs and merged through the workspace,
workspace reuse across calls and CUDA-graph replays, against the oracle.

Capping the number of CTAs (1, 3, 37) forces every row of the last group to be split into
blocks of chunks, so pieces of one row are produced by different CTAs (or by one CTA, in turn)
and merged by whichever completes the row.  Sampler tolerance: a token must equal the oracle's
for the same uniform unless u lies within 1e-6 (normalised CDF units) of a boundary.
"""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import _native
from bitmask_speculation_b200 import workloads as wl
from helpers import as_dtype_bits, sample_matches, to_device, widened

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu
TOL = 1e-6
SHAPES = [(1, 248320), (5, 151936), (64, 50257), (300, 8320), (7, 100), (40, 262144)]


@pytest.fixture(autouse=True)
def _reset_override():
    yield
    _native.set_launch_override(0, 0)


def _inputs(rng, rows, vocab, dtype):
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(3)
    dens = rng.choice([1.0, 0.5, 0.05, 1e-3], size=rows)
    valid = rng.random((rows, vocab)) < dens[:, None]
    valid[:, -1] = True
    if rows > 2:
        values[1, :] = np.float32(1.5)           # ties everywhere: lowest valid index wins
        values[2, vocab // 3] = np.float32(40)   # one spike inside a middle piece
        valid[2, vocab // 3] = True
    masks = wl.pack_bits_np(valid)
    return as_dtype_bits(values, dtype), masks


@pytest.mark.parametrize("ctas", [0, 1, 3, 37])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_dynamic_argmax_matches_oracle(cuda_module, dtype, ctas):
    _native.set_launch_override(0, ctas)
    rng = np.random.default_rng(11 + ctas)
    for rows, vocab in SHAPES:
        bits, masks = _inputs(rng, rows, vocab, dtype)
        exp = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)
        got = cuda_module.masked_reduce_batch(to_device(bits, dtype), torch.from_numpy(masks).cuda())
        for g, e in zip(got, exp):
            assert np.array_equal(g.cpu().numpy(), e), (rows, vocab)


@pytest.mark.parametrize("ctas", [0, 1, 3, 37])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_dynamic_sampler_matches_oracle(cuda_module, dtype, ctas):
    _native.set_launch_override(0, ctas)
    rng = np.random.default_rng(23 + ctas)
    for rows, vocab in SHAPES:
        bits, masks = _inputs(rng, rows, vocab, dtype)
        f32 = widened(bits, dtype)
        for temperature in (0.7, 2.0):
            u = rng.random(rows)
            exp_tok, exp_st = oracle.sample_rows(bits, masks, temperature, u,
                                                 dtype=None if dtype == "float32" else dtype)
            tokens, counts, status = cuda_module.masked_sample_batch(
                to_device(bits, dtype), torch.from_numpy(masks).cuda(), temperature, torch.from_numpy(u).cuda())
            assert status.tolist() == exp_st.tolist()
            exp_counts = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)[1]
            assert counts.tolist() == exp_counts.tolist()
            for r in range(rows):
                assert sample_matches(f32[r], masks[r], temperature, u[r], tokens[r].item(), exp_tok[r], TOL), (
                    rows, vocab, temperature, r)


def test_row_errors_stay_independent_when_rows_are_split(cuda_module):
    _native.set_launch_override(0, 3)
    vocab = 151936
    logits = torch.zeros((6, vocab), device="cuda")
    masks = torch.full((6, vocab // 32), -1, dtype=torch.int32, device="cuda")
    masks[0] = 0
    logits[1, 100000] = float("nan")
    logits[2, 70000] = float("inf")
    logits[3] = -float("inf")
    u = torch.tensor([.5, .5, .5, .5, 1.0, .25], dtype=torch.float64, device="cuda")
    tokens, counts, status = cuda_module.masked_sample_batch(logits, masks, 1.0, u)
    assert status.tolist() == [1, 2, 5, 4, 3, 0]
    assert tokens.tolist()[:5] == [-1] * 5
    assert counts.tolist() == [0] + [vocab] * 5
    t, c, s = cuda_module.masked_reduce_batch(logits, masks)
    assert s.tolist() == [1, 2, 0, 0, 0, 0]
    assert t.tolist()[2] == 70000 and t.tolist()[3] == 0


def test_workspace_is_reused_across_calls_and_shapes(cuda_module):
    """Each call tags its pieces with a new epoch and leaves the counters at zero."""
    rng = np.random.default_rng(5)
    _native.set_launch_override(0, 5)
    cases = [(50, 248320, "bfloat16"), (3, 8320, "float32"), (50, 248320, "bfloat16"), (11, 151936, "float16")]
    for rows, vocab, dtype in cases * 2:
        bits, masks = _inputs(rng, rows, vocab, dtype)
        exp = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)
        got = cuda_module.masked_reduce_batch(to_device(bits, dtype), torch.from_numpy(masks).cuda())
        for g, e in zip(got, exp):
            assert np.array_equal(g.cpu().numpy(), e)


def test_graph_replays_reuse_the_workspace(cuda_module):
    """Replays of one captured launch share its epoch; the kernel's own counter resets make
    every replay start clean."""
    rng = np.random.default_rng(9)
    rows, vocab, dtype = 48, 151936, "bfloat16"
    _native.set_launch_override(0, 7)
    datasets = [_inputs(rng, rows, vocab, dtype) for _ in range(3)]
    logits = to_device(datasets[0][0], dtype)
    masks = torch.from_numpy(datasets[0][1]).cuda()
    u = torch.from_numpy(rng.random(rows)).cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        cuda_module.masked_reduce_batch(logits, masks)  # allocates this stream's workspace
        cuda_module.masked_sample_batch(logits, masks, 0.7, u)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = cuda_module.masked_reduce_batch(logits, masks)
        sout = cuda_module.masked_sample_batch(logits, masks, 0.7, u)
    for bits, m in datasets * 2:
        logits.copy_(to_device(bits, dtype))
        masks.copy_(torch.from_numpy(m).cuda())
        g.replay()
        torch.cuda.synchronize()
        exp = oracle.reduce_rows(bits, m, dtype=dtype)
        for got, e in zip(out, exp):
            assert np.array_equal(got.cpu().numpy(), e)
        uh = u.cpu().numpy()
        exp_tok, exp_st = oracle.sample_rows(bits, m, 0.7, uh, dtype=dtype)
        f32 = widened(bits, dtype)
        assert sout[2].tolist() == exp_st.tolist()
        for r in range(rows):
            assert sample_matches(f32[r], m[r], 0.7, uh[r], sout[0][r].item(), exp_tok[r], TOL)


def test_fixed_schedule_without_workspace_matches(cuda_module):
    rng = np.random.default_rng(3)
    bits, masks = _inputs(rng, 33, 248320, "bfloat16")
    exp = oracle.reduce_rows(bits, masks, dtype="bfloat16")
    cuda_module.use_workspace = False
    try:
        got = cuda_module.masked_reduce_batch(to_device(bits, "bfloat16"), torch.from_numpy(masks).cuda())
    finally:
        cuda_module.use_workspace = True
    for g, e in zip(got, exp):
        assert np.array_equal(g.cpu().numpy(), e)
