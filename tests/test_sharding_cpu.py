"""Host logic of the multi-GPU paths on CPU: shard bounds, row shards, and the vocabulary-sharded
collective sequence (all-gather of 32-byte partials, merge, max all-reduce) with two gloo ranks.

The CUDA kernels cannot run here, so the ranks plug in a CPU backend built on the oracle; the
product path (``NativeShardBackend``) only differs in where partials and merges are computed.
"""

import math
import os
import struct

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bitmask_speculation_b200 import workloads as wl
from bitmask_speculation_b200.sharding import row_shard, shard_bounds, vocab_sharded_select


def test_row_shards_cover_every_row_once():
    for rows in [0, 1, 7, 2304, 65536]:
        for world in [1, 2, 3, 8]:
            parts = [row_shard(rows, world, r) for r in range(world)]
            covered = [i for sl in parts for i in range(rows)[sl]]
            assert covered == list(range(rows))
            sizes = [sl.stop - sl.start for sl in parts]
            assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_are_word_aligned_and_complete():
    for vocab in [64, 1000, 50257, 151936, 248320]:
        for world in [1, 2, 4, 8]:
            if vocab < 32 * world:
                continue
            b = shard_bounds(vocab, world)
            assert all(off % 32 == 0 for off, _ in b)
            assert [off for off, _ in b] == sorted(off for off, _ in b)
            assert sum(size for _, size in b) == vocab and b[0][0] == 0


def _ordered(v: float) -> int:
    u = struct.unpack("<I", struct.pack("<f", v + 0.0))[0]
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


class OracleShardBackend:
    """CPU stand-in for the kernels (test only): same record format and merge rules."""

    def partials(self, logits, masks, offset, temperature):
        vals = logits.numpy()
        rows, size = vals.shape
        words = masks.numpy().view(np.uint32)
        t = np.arange(offset, offset + size)
        bits = ((words[:, t >> 5] >> (t & 31).astype(np.uint32)) & 1).astype(bool)
        rec = np.zeros((rows, 32), np.uint8)
        for r in range(rows):
            v, b = vals[r], bits[r]
            nan = bool(np.isnan(v).any())
            cnt = int(b.sum())
            ok = b & ~np.isnan(v)
            if temperature == 0:
                if ok.any():
                    idx = np.flatnonzero(ok)
                    best = idx[np.argmax(v[idx])]
                    hi, lo = _ordered(float(v[best])), 0xFFFFFFFF - (offset + int(best))
                else:
                    hi, lo = 0, 0
                rec[r, :16] = np.frombuffer(struct.pack("<IIII", hi, lo, cnt, int(nan)), np.uint8)
            else:
                m = float(v[ok].max()) if ok.any() else -math.inf
                fin = ok & np.isfinite(v)
                s = math.fsum(math.exp((float(x) - m) / temperature) for x in v[fin]) if math.isfinite(m) else 0.0
                rec[r, :16] = np.frombuffer(struct.pack("<fIII", m, cnt, int(nan), 0), np.uint8)
                rec[r, 16:24] = np.frombuffer(struct.pack("<d", s), np.uint8)
        return torch.from_numpy(rec), (offset, vals, bits)

    def merge(self, gathered, shard, temperature, uniforms, logits, masks, offset, aux):
        g = gathered.numpy()
        shards, rows, _ = g.shape
        tokens = np.full(rows, -1, np.int64)
        counts = np.zeros(rows, np.int64)
        status = np.zeros(rows, np.int32)
        for r in range(rows):
            recs = [g[q, r] for q in range(shards)]
            if temperature == 0:
                keys = [struct.unpack("<IIII", bytes(x[:16])) for x in recs]
                hi = max(k[0] for k in keys)
                lo = max(k[1] for k in keys if k[0] == hi)
                total = sum(k[2] for k in keys)
                nan = any(k[3] for k in keys)
                status[r] = 2 if nan else (1 if total == 0 else 0)
                tokens[r] = 0xFFFFFFFF - lo if status[r] == 0 else -1
                counts[r] = total
            else:
                parts = [struct.unpack("<fIII", bytes(x[:16])) + struct.unpack("<d", bytes(x[16:24])) for x in recs]
                M = max(p[0] for p in parts)
                total = sum(p[1] for p in parts)
                nan = any(p[2] for p in parts)
                counts[r] = total
                status[r] = 2 if nan else 5 if M == math.inf else 1 if total == 0 else 4 if M == -math.inf else 0
                if status[r]:
                    continue
                masses = [p[4] * math.exp((p[0] - M) / temperature) if p[4] > 0 else 0.0 for p in parts]
                cutoff = float(uniforms[r]) * sum(masses)
                run, owner, prefix = 0.0, -1, 0.0
                for q, m in enumerate(masses):
                    if m > 0 and owner < 0 and cutoff < run + m:
                        owner, prefix = q, run
                    run += m
                if owner != shard:
                    continue
                off, vals, bits = aux
                acc = prefix
                for t in range(vals.shape[1]):
                    x = float(vals[r, t])
                    if not bits[r, t] or not math.isfinite(x):
                        continue
                    w = math.exp((x - M) / temperature)
                    if w == 0:
                        continue
                    acc += w
                    tokens[r] = off + t
                    if cutoff < acc:
                        break
        return torch.from_numpy(tokens), torch.from_numpy(counts), torch.from_numpy(status)


def _worker(rank, world, port, vocab, rows, temperature, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        rng = np.random.default_rng(9)
        vals = rng.standard_normal((rows, vocab), dtype=np.float32) * 2
        valid = rng.random((rows, vocab)) < 0.3
        valid[:, 0] = True
        valid[1] = False
        vals[2, 5] = np.nan
        masks = wl.pack_bits_np(valid)
        uniforms = rng.random(rows)
        off, size = shard_bounds(vocab, world)[rank]
        out = vocab_sharded_select(torch.from_numpy(np.ascontiguousarray(vals[:, off:off + size])),
                                   torch.from_numpy(masks), vocab, temperature=temperature,
                                   uniforms=torch.from_numpy(uniforms), backend=OracleShardBackend())
        queue.put((rank, [o.tolist() for o in out]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("temperature", [0.0, 0.9])
def test_vocab_sharded_collectives_two_gloo_ranks(temperature):
    world, vocab, rows = 2, 1000, 6
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29500 + int(temperature * 10) + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, vocab, rows, temperature, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1]  # identical on every rank
    rng = np.random.default_rng(9)
    vals = rng.standard_normal((rows, vocab), dtype=np.float32) * 2
    valid = rng.random((rows, vocab)) < 0.3
    valid[:, 0] = True
    valid[1] = False
    vals[2, 5] = np.nan
    masks = wl.pack_bits_np(valid)
    uniforms = rng.random(rows)
    tokens, counts, status = results[0]
    if temperature == 0:
        exp = oracle.reduce_rows(vals, masks)
        assert [tokens, counts, status] == [e.tolist() for e in exp]
    else:
        exp_tok, exp_st = oracle.sample_rows(vals, masks, temperature, uniforms)
        assert status == exp_st.tolist()
        assert tokens == exp_tok.tolist()
