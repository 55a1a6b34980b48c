"""The flat sampler schedule (a workspace given, fewer than 1.5 rows per resident CTA): the batch's
chunks stream as blocks taken by every CTA, each consumer warp stores one granule record per chunk
to the workspace, and a second launch merges every row.  Batches from one row to the top of the
range, 16-bit and fp32 chunking, rows of one chunk and of a ragged last chunk, and every failing
row kind must give the oracle's statuses and counts exactly and its tokens within the 1e-6
CDF-boundary rule -- and the same results as the fixed schedule (no workspace)."""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl
from helpers import as_dtype_bits, sample_matches, to_device

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture
def module(cuda_module):
    saved = cuda_module.use_workspace
    yield cuda_module
    cuda_module.use_workspace = saved


def _batch(rows, vocab, dtype, seed):
    """Mixed densities with every failing row kind the sampler reports (where the batch has room)."""
    rng = np.random.default_rng(seed)
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(2.0)
    dens = rng.choice([1.0, 0.5, 0.1, 0.01, 1e-4], size=rows)
    valid = rng.random((rows, vocab)) < dens[:, None]
    valid[:, 0] = True
    special = {}
    if rows > 6:
        values[1, rng.integers(vocab)] = np.nan                 # NaN anywhere: status 2
        valid[2, :] = False                                     # no valid token: status 1
        values[3, :] = -np.inf                                  # no finite mass: status 4
        values[4, 7] = np.inf                                   # valid +inf: status 5
        valid[4, 7] = True
        valid[5, :] = False                                     # one valid token, in the last chunk
        valid[5, vocab - 1] = True
        values[6, vocab // 2] = np.float32(60.0)                # one dominant token mid-row
        special = {1: 2, 2: 1, 3: 4, 4: 5}
    bits = as_dtype_bits(values, dtype)
    return bits, wl.pack_bits_np(valid), special


def _sample(module, bits, masks, dtype, temperature, uniforms, use_workspace):
    module.use_workspace = use_workspace
    out = module.masked_sample_batch(to_device(bits, dtype), torch.from_numpy(masks).cuda(), temperature,
                                     torch.from_numpy(uniforms).cuda())
    return [t.cpu().numpy() for t in out]


def _check(bits, masks, dtype, temperature, uniforms, got):
    tokens, counts, status = got
    dt = None if dtype == "float32" else dtype
    et, es = oracle.sample_rows(bits, masks, temperature, uniforms, dtype=dt)
    _, ec, _ = oracle.reduce_rows(bits, masks, dtype=dt)
    assert np.array_equal(status, es)
    assert np.array_equal(counts, ec)
    for r in np.flatnonzero(tokens != et):
        row = oracle.widen(bits[r], dtype) if dt else bits[r]
        assert sample_matches(row, masks[r], temperature, uniforms[r], int(tokens[r]), int(et[r])), (r, tokens[r], et[r])
    return es


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("rows,vocab", [(1, 248320), (3, 8192), (8, 248320), (16, 131072), (64, 151936),
                                        (100, 248320), (200, 32000), (480, 128256)])
def test_flat_schedule_matches_oracle_and_fixed(module, dtype, rows, vocab):
    bits, masks, special = _batch(rows, vocab, dtype, 7 * rows + vocab)
    temperature = 0.7
    uniforms = np.random.default_rng(rows + 1).random(rows)
    got = _sample(module, bits, masks, dtype, temperature, uniforms, True)
    es = _check(bits, masks, dtype, temperature, uniforms, got)
    for r, code in special.items():
        assert es[r] == code
    fixed = _sample(module, bits, masks, dtype, temperature, uniforms, False)
    assert np.array_equal(fixed[1], got[1]) and np.array_equal(fixed[2], got[2])
    _check(bits, masks, dtype, temperature, uniforms, fixed)


@pytest.mark.parametrize("temperature", [1e-3, 5.0])
def test_flat_schedule_temperatures_and_edge_uniforms(module, temperature):
    """Sharp and flat distributions, uniforms at 0, just below 1, and out of range (status 3)."""
    rows, vocab, dtype = 48, 248320, "float16"
    bits, masks, _ = _batch(rows, vocab, dtype, 11)
    uniforms = np.random.default_rng(3).random(rows)
    uniforms[10], uniforms[11], uniforms[12], uniforms[13] = 0.0, np.nextafter(1.0, 0.0), 1.0, -0.25
    got = _sample(module, bits, masks, dtype, temperature, uniforms, True)
    es = _check(bits, masks, dtype, temperature, uniforms, got)
    assert es[12] == 3 and es[13] == 3


def test_flat_schedule_back_to_back_launches(module):
    """Launches of different sizes in one stream reuse the workspace records and counters."""
    vocab, dtype, temperature = 151936, "bfloat16", 0.9
    module.use_workspace = True
    for i, rows in enumerate((120, 7, 300, 7, 64, 665)):
        bits, masks, _ = _batch(rows, vocab, dtype, 100 + i)
        uniforms = np.random.default_rng(200 + i).random(rows)
        got = _sample(module, bits, masks, dtype, temperature, uniforms, True)
        _check(bits, masks, dtype, temperature, uniforms, got)


def test_flat_schedule_replayed_from_a_cuda_graph(module):
    """The flat schedule's launch pair captured once and replayed with new uniforms each time (the
    workspace's ticket counter and records are left ready by every launch): each replay equals a
    direct call with the same inputs."""
    rows, vocab, dtype, temperature = 64, 248320, "float16", 0.7
    bits, masks, _ = _batch(rows, vocab, dtype, 5)
    module.use_workspace = True
    logits, dmasks = to_device(bits, dtype), torch.from_numpy(masks).cuda()
    u = torch.empty(rows, dtype=torch.float64, device="cuda")
    u.copy_(torch.from_numpy(np.random.default_rng(0).random(rows)))
    module.masked_sample_batch(logits, dmasks, temperature, u)  # workspace and kernels set up
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="relaxed"):
        out = module.masked_sample_batch(logits, dmasks, temperature, u)
    for seed in range(1, 5):
        fresh = np.random.default_rng(seed).random(rows)
        u.copy_(torch.from_numpy(fresh))
        graph.replay()
        got = [t.cpu().numpy() for t in out]
        want = [t.cpu().numpy() for t in module.masked_sample_batch(logits, dmasks, temperature, u)]
        for g, w in zip(got, want):
            assert np.array_equal(g, w), seed
        _check(bits, masks, dtype, temperature, fresh, got)
