"""Vocabulary shards on one GPU: partials + merge equal the single-GPU cluster merge bit for bit.

A single-GPU launch with cluster size N covers the same token slices as N vocabulary shards
(``shard_bounds``), so the sharded path must reproduce its tokens, counts and statuses exactly --
for the sampler too, since both run the same rank merge and owner walk.  The NCCL all-gather is
replaced here by stacking the N partial tensors.
"""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import _native
from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.sharding import NativeShardBackend, shard_bounds
from helpers import as_dtype_bits, sample_matches, to_device, widened

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _reset_override():
    yield
    _native.set_launch_override(0, 0)


def emulate_shards(logits, masks, world, temperature, uniforms):
    backend = NativeShardBackend()
    vocab = logits.shape[1]
    bounds = shard_bounds(vocab, world)
    parts, aux = [], []
    for off, size in bounds:
        sl = logits[:, off:off + size].contiguous()
        pr, ax = backend.partials(sl, masks, off, temperature)
        parts.append(pr)
        aux.append((sl, ax))
    gathered = torch.stack(parts)
    outs = []
    for r, (off, size) in enumerate(bounds):
        sl, ax = aux[r]
        outs.append(backend.merge(gathered, r, temperature, uniforms, sl, masks, off, ax))
    tokens = torch.stack([o[0] for o in outs]).max(0).values
    status = torch.stack([o[2] for o in outs]).max(0).values
    for o in outs[1:]:
        assert torch.equal(o[1], outs[0][1])  # counts identical on every rank
    if temperature == 0:
        for o in outs[1:]:
            assert torch.equal(o[0], outs[0][0]) and torch.equal(o[2], outs[0][2])
    return tokens, outs[0][1], status


def make_rows(seed, rows, vocab, dtype):
    rng = np.random.default_rng(seed)
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(3)
    dens = rng.choice([1.0, 0.6, 0.05, 1e-4], size=rows)
    valid = rng.random((rows, vocab)) < dens[:, None]
    valid[:, rng.integers(vocab)] = True
    if rows > 3:
        valid[1] = False                       # empty row
        values[2, rng.integers(vocab)] = np.nan  # NaN row
        values[3, valid[3]] = -np.inf          # no finite mass (sampler) / -inf ties (argmax)
    return as_dtype_bits(values, dtype), wl.pack_bits_np(valid)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_argmax_shards_equal_cluster_merge_and_oracle(cuda_module, world, dtype):
    vals, masks = make_rows(5 + world, 12, wl.VOCAB, dtype)
    logits = to_device(vals, dtype)
    m = torch.from_numpy(masks).cuda()
    _native.set_launch_override(world, 0)
    ref = cuda_module.masked_reduce_batch(logits, m)
    got = emulate_shards(logits, m, world, 0.0, None)
    for g, r in zip(got, ref):
        assert torch.equal(g, r)
    exp = oracle.reduce_rows(vals, masks, dtype=None if dtype == "float32" else dtype)
    for g, e in zip(got, exp):
        assert np.array_equal(g.cpu().numpy(), e)


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_sampler_shards_bit_exact_to_cluster_merge(cuda_module, world, dtype):
    vals, masks = make_rows(50 + world, 16, wl.VOCAB, dtype)
    logits = to_device(vals, dtype)
    m = torch.from_numpy(masks).cuda()
    u = torch.from_numpy(np.random.default_rng(world).random(16)).cuda()
    _native.set_launch_override(world, 0)
    ref_tok, ref_cnt, ref_st = cuda_module.masked_sample_batch(logits, m, 0.8, u)
    tok, cnt, st = emulate_shards(logits, m, world, 0.8, u)
    assert torch.equal(tok, ref_tok) and torch.equal(cnt, ref_cnt) and torch.equal(st, ref_st)
    exp_tok, exp_st = oracle.sample_rows(vals, masks, 0.8, u.cpu().numpy(), dtype=dtype)
    assert st.tolist() == exp_st.tolist()
    f32 = widened(vals, dtype)
    for r in range(16):
        assert sample_matches(f32[r], masks[r], 0.8, float(u[r]), int(tok[r]), int(exp_tok[r]))


def test_shard_bounds_match_cluster_segments():
    assert shard_bounds(248320, 8) == [(31040 * r, 31040) for r in range(8)]
    assert shard_bounds(248320, 2) == [(0, 124160), (124160, 124160)]
    b = shard_bounds(151936, 8)
    assert all(off % 32 == 0 for off, _ in b) and sum(s for _, s in b) == 151936


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_partials_through_a_mask_table_equal_gathered_masks(temperature, dtype):
    """``bms_shard_partials_indexed`` reads row r's mask from ``masks[mask_rows[r]]``: its partials
    (and sampler granules) must equal those of the gathered mask rows bit for bit, and an index
    outside the table must fail its row with status 8."""
    rng = np.random.default_rng(9)
    rows, table_rows, vocab = 96, 40, 20_000
    _, masks = make_rows(5, table_rows, vocab, dtype)
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(3)
    logits = to_device(as_dtype_bits(values, dtype), dtype)
    table = rng.integers(0, table_rows, size=rows).astype(np.int32)
    backend = NativeShardBackend()
    gathered = torch.from_numpy(masks[table]).cuda()
    dev_masks = torch.from_numpy(masks).cuda()
    pa, (ga, _) = backend.partials(logits, gathered, 0, temperature)
    pb, (gb, _) = backend.partials(logits, dev_masks, 0, temperature, mask_rows=torch.from_numpy(table).cuda())
    assert torch.equal(pa, pb)
    if temperature:
        assert torch.equal(ga, gb)
    bad = table.copy()
    bad[7], bad[50] = table_rows, -1
    pc, ax = backend.partials(logits, dev_masks, 0, 0.0, mask_rows=torch.from_numpy(bad).cuda())
    _, _, status = backend.merge(pc[None], 0, 0.0, None, logits, gathered, 0, ax)
    st = status.cpu().numpy()
    assert st[7] == 8 and st[50] == 8
    ok = np.ones(rows, dtype=bool)
    ok[[7, 50]] = False
    _, _, want = backend.merge(pa[None] if temperature == 0 else backend.partials(logits, gathered, 0, 0.0)[0][None],
                               0, 0.0, None, logits, gathered, 0, ax)
    assert np.array_equal(st[ok], want.cpu().numpy()[ok])
