"""Mid-sized batches (one row per SM up to 1.5 rows per resident CTA) on every schedule they can
take: the fixed one (no workspace), and with a workspace either the fixed one or -- for the sampler
-- the flat schedule (the batch's chunks streamed as blocks taken as tickets by every CTA, then a
merge launch per row).  Results must equal the oracle (argmax, counts, statuses bit-exact; sampled
tokens within the 1e-6 CDF-boundary rule) across dtypes, vocabularies (bulk-copy and plain-load
rows, 16-bit and fp32 chunking), failing rows and mask tables."""

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
    rng = np.random.default_rng(seed)
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(2.5)
    dens = rng.choice([1.0, 0.6, 0.1, 0.01, 1e-4, 0.0], size=rows, p=[0.2, 0.2, 0.2, 0.2, 0.15, 0.05])
    valid = rng.random((rows, vocab)) < dens[:, None]
    values[3, :] = np.float32(0.75)                       # ties: the lowest valid index wins
    values[7, rng.integers(vocab)] = np.nan               # NaN anywhere fails the row
    values[11, :] = -np.inf                               # no finite mass for the sampler
    valid[11, :5] = True
    bits = as_dtype_bits(values, dtype)
    return bits, wl.pack_bits_np(valid)


def _host(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("rows,vocab", [(148, 248320), (256, 248320), (444, 151936), (600, 50257), (665, 128256)])
def test_argmax_matches_oracle_and_fixed_schedule(module, dtype, rows, vocab):
    bits, masks = _batch(rows, vocab, dtype, rows + vocab)
    logits, dmasks = to_device(bits, dtype), torch.from_numpy(masks).cuda()
    module.use_workspace = True
    got = [_host(t) for t in module.masked_reduce_batch(logits, dmasks)]
    again = [_host(t) for t in module.masked_reduce_batch(logits, dmasks)]  # the workspace is reusable
    module.use_workspace = False
    fixed = [_host(t) for t in module.masked_reduce_batch(logits, dmasks)]
    want = oracle.reduce_rows(bits, masks, dtype=None if dtype == "float32" else dtype)
    for g, a, f, w in zip(got, again, fixed, want):
        assert np.array_equal(g, w)
        assert np.array_equal(a, w)
        assert np.array_equal(f, w)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("rows,vocab,temperature", [(256, 248320, 0.7), (480, 248320, 0.7), (600, 151936, 1.3),
                                                    (520, 50257, 0.05), (665, 128256, 1.0)])
def test_sampler_matches_oracle(module, dtype, rows, vocab, temperature):
    bits, masks = _batch(rows, vocab, dtype, 3 * rows + vocab)
    uniforms = np.random.default_rng(rows).random(rows)
    module.use_workspace = True
    tokens, counts, status = module.masked_sample_batch(to_device(bits, dtype), torch.from_numpy(masks).cuda(),
                                                        temperature, torch.from_numpy(uniforms).cuda())
    dt = None if dtype == "float32" else dtype
    et, es = oracle.sample_rows(bits, masks, temperature, uniforms, dtype=dt)
    _, ec, _ = oracle.reduce_rows(bits, masks, dtype=dt)
    assert np.array_equal(_host(status), es)
    assert np.array_equal(_host(counts), ec)
    got = _host(tokens)
    for r in np.flatnonzero(got != et):
        row = oracle.widen(bits[r], dtype) if dt else bits[r]
        assert sample_matches(row, masks[r], temperature, uniforms[r], int(got[r]), int(et[r])), (r, got[r], et[r])
    assert (es == 2).any() and (es == 4).any() and (es == 1).any() and (es == 0).sum() > rows // 2


def test_verification_round_with_a_mask_table(module):
    """32 sequences x 9 rows (288 rows) with device-resident table masks, one index out of range."""
    from bitmask_speculation_b200.verification import verify_batch
    rng = np.random.default_rng(5)
    seqs, k, vocab = 32, 8, 248320
    rows = seqs * (k + 1)
    table_valid = rng.random((12, vocab)) < rng.choice([0.6, 0.05, 1e-4], size=(12, 1))
    table = wl.pack_bits_np(table_valid)
    mask_rows = rng.integers(0, 12, size=rows).astype(np.int32)
    mask_rows[40] = 12  # outside the table: status 8 for that row
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(3)
    bits = wl.to_bf16_bits(values)
    full = table[mask_rows.clip(0, 11)]
    tok, _, _ = oracle.reduce_rows(bits, full, dtype="bfloat16")
    proposals = np.where(rng.random((seqs, k)) < 0.85, tok.reshape(seqs, k + 1)[:, :k],
                         rng.integers(vocab, size=(seqs, k))).astype(np.int64)
    lengths = rng.integers(0, k + 1, size=seqs).astype(np.int32)
    module.use_workspace = True
    out = verify_batch(to_device(bits, "bfloat16"), torch.from_numpy(table).cuda(), torch.from_numpy(proposals).cuda(),
                       torch.from_numpy(lengths).cuda(), mask_rows=torch.from_numpy(mask_rows).cuda()).to_host()
    et, ec, es = oracle.reduce_rows(bits, full, dtype="bfloat16")
    es[40], et[40] = 8, -1
    acc, token, kind, sst = oracle.verify(et, es, proposals, lengths)
    assert out.row_status == es.tolist() and out.row_tokens == et.tolist()
    assert out.row_counts[:40] == ec[:40].tolist() and out.row_counts[41:] == ec[41:].tolist()
    assert out.accept_len == acc.tolist() and out.token == token.tolist() and out.kind == kind.tolist()
    assert out.seq_status == sst.tolist()
