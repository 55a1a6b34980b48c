"""The benchmark configurations at their own sizes against the oracle.

* Configuration 3 (256 sequences x 9 rows = 2,304 bf16 rows at V = 248,320): every output of one
  ``bms_verify_batch`` round -- per-row token, count, status and draft budget, per-sequence
  accepted length, token, kind and status -- on the dynamic schedule (workspace) and on the fixed
  one, equal to ``oracle.reduce_rows`` -> ``oracle.verify`` -> ``oracle.budget_rows``
  (benchmarks/reductions.py:9-17, decoding/verification.py:18-48, decoding/scheduling.py:40-46).
* Configuration 5 (65,536 bf16 rows, log-uniform mask densities): one launch over all rows (beyond
  the reference's 65,535-row grid limit), every row's token, count and status equal to the oracle,
  compared in slices of 4,096 rows; and the sampler over the same rows at T = 0.7, every token equal
  to the oracle's for the same uniform unless u lies within 1e-6 of a CDF boundary of the GPU's token.
* Configurations 1 and 2 at full vocabulary: bit-exact argmax / counts and sampler tokens within
  the same tolerance.
"""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.scheduling import DensityPolicy
from helpers import sample_matches, to_device

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SLICE = 4096


def _bf16_host(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture
def schedule(cuda_module):
    """Runs a test on the dynamic (workspace) and fixed schedules of the batched kernels."""
    saved = cuda_module.use_workspace
    yield cuda_module
    cuda_module.use_workspace = saved


@pytest.mark.parametrize("dynamic", [True, False], ids=["dynamic", "fixed"])
def test_configuration_3_full_round_matches_oracle(schedule, dynamic):
    from bitmask_speculation_b200.verification import verify_batch
    schedule.use_workspace = dynamic
    logits, masks, proposals, lengths = wl.verify_batch_torch(256, seed=3, device="cuda")
    policy = DensityPolicy()
    host = verify_batch(logits, masks, proposals, lengths, policy=policy).to_host()

    bits, m = _bf16_host(logits), masks.cpu().numpy()
    props, lens = proposals.cpu().numpy(), lengths.cpu().numpy()
    tokens, counts, status = oracle.reduce_rows(bits, m, dtype="bfloat16")
    accept, token, kind, seq_status = oracle.verify(tokens, status, props, lens)
    _, budgets = oracle.budget_rows(counts, wl.VOCAB, low=policy.low_density, high=policy.high_density,
                                    min_budget=policy.min_budget, max_budget=policy.max_budget)
    expect = dict(row_tokens=tokens, row_counts=counts, row_status=status, row_budget=budgets,
                  accept_len=accept, token=token, kind=kind, seq_status=seq_status)
    assert len(host.row_tokens) == 2304 and len(host.accept_len) == 256
    for key, value in expect.items():
        got = np.asarray(getattr(host, key))
        bad = np.flatnonzero(got != value)
        assert bad.size == 0, (key, bad[:8], got[bad[:8]], value[bad[:8]])
    # The workload is the configuration's: every sequence checks all 8 drafts, the acceptance
    # follows the seeded geometric draw, and the three mask kinds give all three budgets.
    assert set(np.unique(budgets)) <= {1, 4, 8} and len(set(np.unique(budgets))) >= 2
    assert 0 < accept.mean() < 8


@pytest.fixture(scope="module")
def configuration_5(cuda_module):
    logits, masks = wl.scale_rows_torch(65536, seed=5, device="cuda")
    yield logits, masks
    del logits, masks
    torch.cuda.empty_cache()


def test_configuration_5_all_rows_match_oracle(configuration_5, cuda_module):
    logits, masks = configuration_5
    tokens, counts, status = cuda_module.masked_reduce_batch(logits, masks)
    tokens, counts, status = tokens.cpu().numpy(), counts.cpu().numpy(), status.cpu().numpy()
    assert tokens.shape == (65536,)
    for r0 in range(0, 65536, SLICE):
        r1 = r0 + SLICE
        et, ec, es = oracle.reduce_rows(_bf16_host(logits[r0:r1]), masks[r0:r1].cpu().numpy(), dtype="bfloat16")
        for name, got, want in (("tokens", tokens[r0:r1], et), ("counts", counts[r0:r1], ec),
                                ("status", status[r0:r1], es)):
            bad = np.flatnonzero(got != want)
            assert bad.size == 0, (name, r0 + bad[:8], got[bad[:8]], want[bad[:8]])
    assert (status == 0).all()


def test_configuration_5_sampler_matches_oracle(configuration_5, cuda_module):
    logits, masks = configuration_5
    temperature = wl.SAMPLE_TEMPERATURE
    uniforms = np.random.default_rng(55).random(65536)
    tokens, counts, status = cuda_module.masked_sample_batch(logits, masks, temperature,
                                                             torch.from_numpy(uniforms).cuda())
    tokens, counts, status = tokens.cpu().numpy(), counts.cpu().numpy(), status.cpu().numpy()
    mismatched = 0
    for r0 in range(0, 65536, SLICE):
        r1 = r0 + SLICE
        bits, m = _bf16_host(logits[r0:r1]), masks[r0:r1].cpu().numpy()
        et, es = oracle.sample_rows(bits, m, temperature, uniforms[r0:r1], dtype="bfloat16")
        assert np.array_equal(status[r0:r1], es)
        for r in np.flatnonzero(tokens[r0:r1] != et):
            widened = oracle.widen(bits[r], "bfloat16")
            assert sample_matches(widened, m[r], temperature, uniforms[r0 + r], int(tokens[r0 + r]), int(et[r])), \
                (r0 + r, tokens[r0 + r], et[r])
            mismatched += 1
    # Every differing row passed the tolerance rule above.  How many differ depends on how many
    # boundaries lie near u: with n positive-weight tokens in a row, u falls within d of some
    # boundary with probability 2 d n, and rows here hold ~27,000 valid tokens on average, so a few
    # rows in 65,536 (d ~ 1e-9 of fp32 partial sums) are expected; a systematic error would show in
    # a large fraction of the rows.
    assert mismatched <= 65536 // 1000, mismatched


def test_configuration_1_exact(cuda_module):
    values, masks = wl.argmax_config_np(seed=1)
    got = cuda_module.masked_reduce_batch(torch.from_numpy(values).cuda(), torch.from_numpy(masks).cuda())
    for g, e in zip(got, oracle.reduce_rows(values, masks)):
        assert np.array_equal(g.cpu().numpy(), e)


def test_configuration_2_full_vocabulary(cuda_module):
    bits, masks, uniforms, temperature = wl.sample_config_np(seed=2)
    tokens, counts, status = cuda_module.masked_sample_batch(
        to_device(bits, "float16"), torch.from_numpy(masks).cuda(), temperature, torch.from_numpy(uniforms).cuda())
    et, es = oracle.sample_rows(bits, masks, temperature, uniforms, dtype="float16")
    assert status.tolist() == es.tolist()
    for r, (g, e) in enumerate(zip(tokens.tolist(), et.tolist())):
        assert sample_matches(oracle.widen(bits[r], "float16"), masks[r], temperature, uniforms[r], g, e), r
    _, ec, _ = oracle.reduce_rows(bits, masks, dtype="float16")
    assert np.array_equal(counts.cpu().numpy(), ec)
