"""Peer-memory exchange of vocabulary-shard partials (``bms_shard_partials_exchange`` /
``bms_shard_merge_exchange``, ``sharding.PeerExchange``).

On one GPU, N ranks are emulated with N exchange areas on the device: each step launches every
rank's selection (which stores its partials into all areas and publishes its epoch), then every
rank's merge, so no kernel ever waits on another running kernel.  The merged argmax must equal a
single launch over the full rows bit for bit, over several steps (both slot parities and the
consumed-epoch wait).  A merge whose step was never published gives up after its bounded wait and
reports status 7.  With two or more GPUs the same exchange runs between two processes over NVLink.
"""

import os

import numpy as np
import pytest

from bitmask_speculation_b200 import workloads as wl

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

STATUS_TIMEOUT = 7


def _reference(native, logits, masks):
    tokens, counts, status = native.masked_reduce_batch(logits, masks)
    return tokens.cpu(), counts.cpu(), status.cpu()


@pytest.mark.parametrize("ranks", [1, 2, 3, 8])
def test_emulated_ranks_match_a_single_launch(cuda_module, ranks):
    from bitmask_speculation_b200.sharding import PeerExchange, shard_bounds
    dev = torch.device("cuda", 0)
    rows, cap = 37, 64
    areas = [PeerExchange.create(dev, ranks, cap)[0] for _ in range(ranks)]
    try:
        ex = [PeerExchange(cap, areas=areas, rank=q, device=dev) for q in range(ranks)]
        bounds = shard_bounds(wl.VOCAB, ranks)
        for step in range(1, 6):
            logits, masks = wl.scale_rows_torch(rows - (step % 2), seed=50 + step, device=dev)
            n = logits.shape[0]
            if step == 3:  # NaN in one shard, an empty mask in another row
                logits[5, bounds[-1][0] + 7] = float("nan")
                masks[9].zero_()
            want = _reference(cuda_module, logits, masks)
            for q, (off, size) in enumerate(bounds):
                ex[q].partials(logits[:, off:off + size].contiguous(), masks, off, step)
            for q in range(ranks):
                got = [t.cpu() for t in ex[q].merge(n, step)]
                for g, w in zip(got, want):
                    assert torch.equal(g, w), (ranks, step, q)
            if step == 3:
                assert int(want[2][5]) == 2 and int(want[2][9]) == 1
    finally:
        torch.cuda.synchronize(dev)
        for a in areas:
            PeerExchange.destroy(dev, a)


def test_unpublished_step_times_out_then_recovers(cuda_module):
    from bitmask_speculation_b200.sharding import PeerExchange, shard_bounds
    dev = torch.device("cuda", 0)
    areas = [PeerExchange.create(dev, 2, 16)[0] for _ in range(2)]
    try:
        ex = [PeerExchange(16, areas=areas, rank=q, device=dev) for q in range(2)]
        # Step 1: nobody selected -- both merges wait about one second and give up.
        for q in range(2):
            tokens, counts, status = ex[q].merge(5, 1)
            assert torch.all(status.cpu() == STATUS_TIMEOUT) and torch.all(tokens.cpu() == -1)
        # Step 2 runs normally.
        logits, masks = wl.scale_rows_torch(5, seed=61, device=dev)
        want = _reference(cuda_module, logits, masks)
        for q, (off, size) in enumerate(shard_bounds(wl.VOCAB, 2)):
            ex[q].partials(logits[:, off:off + size].contiguous(), masks, off, 2)
        for q in range(2):
            for g, w in zip(ex[q].merge(5, 2), want):
                assert torch.equal(g.cpu(), w)
    finally:
        torch.cuda.synchronize(dev)
        for a in areas:
            PeerExchange.destroy(dev, a)


def test_rows_a_peer_did_not_publish_fail_with_status_7(cuda_module):
    """Ranks must pass the same rows.  If one rank's step has fewer rows, the slots past its batch
    still hold partials of the step two earlier (same slot parity); their epoch tag fails those
    rows with status 7 instead of merging stale partials, and ``check_statuses`` raises."""
    from bitmask_speculation_b200.sharding import PeerExchange, shard_bounds
    dev = torch.device("cuda", 0)
    areas = [PeerExchange.create(dev, 2, 64)[0] for _ in range(2)]
    bounds = shard_bounds(wl.VOCAB, 2)
    try:
        ex = [PeerExchange(64, areas=areas, rank=q, device=dev) for q in range(2)]
        for step, rows1 in ((1, 40), (2, 40), (3, 30)):
            logits, masks = wl.scale_rows_torch(40, seed=80 + step, device=dev)
            want = _reference(cuda_module, logits, masks)
            for q, (off, size) in enumerate(bounds):
                n = 40 if q == 0 else rows1
                ex[q].partials(logits[:n, off:off + size].contiguous(), masks[:n].contiguous(), off, step)
            tokens, counts, status = (t.cpu() for t in ex[0].merge(40, step))
            if step < 3:
                assert torch.equal(tokens, want[0]) and torch.equal(status, want[2])
                ex[1].merge(40, step)
                continue
            assert torch.equal(tokens[:30], want[0][:30]) and torch.equal(counts[:30], want[1][:30])
            assert torch.all(status[30:] == STATUS_TIMEOUT) and torch.all(tokens[30:] == -1)
            with pytest.raises(RuntimeError, match="did not arrive"):
                PeerExchange.check_statuses(status)
            ex[1].merge(30, step)
    finally:
        torch.cuda.synchronize(dev)
        for a in areas:
            PeerExchange.destroy(dev, a)


def test_exchange_rejects_bad_arguments(cuda_module):
    from bitmask_speculation_b200 import _native
    from bitmask_speculation_b200.sharding import PeerExchange
    dev = torch.device("cuda", 0)
    own, _ = PeerExchange.create(dev, 2, 8)
    try:
        ex = PeerExchange(8, areas=[own, own], rank=0, device=dev)
        logits, masks = wl.scale_rows_torch(9, seed=3, device=dev)
        with pytest.raises(ValueError, match="rows_cap"):
            ex.select(logits[:, :1024].contiguous(), masks, 0)
        with pytest.raises(_native.NativeError, match="epoch"):
            ex.merge(4, 0)
        assert _native.library().bms_exchange_bytes(9, 8) == -1
    finally:
        torch.cuda.synchronize(dev)
        PeerExchange.destroy(dev, own)


def _two_gpu_worker(rank, port, out):
    import torch.distributed as dist
    from bitmask_speculation_b200.kernels._extension import load_extension
    from bitmask_speculation_b200.sharding import PeerExchange, shard_bounds, vocab_sharded_select
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        native = load_extension()
        ex = PeerExchange(300, device=dev)
        off, size = shard_bounds(wl.VOCAB, 2)[rank]
        ok = True
        for step in range(4):
            logits, masks = wl.scale_rows_torch(300 - step, seed=70 + step, device=dev)
            want = [t.cpu() for t in native.masked_reduce_batch(logits, masks)]
            shard = logits[:, off:off + size].contiguous()
            got = [t.cpu() for t in vocab_sharded_select(shard, masks, wl.VOCAB, exchange=ex)]
            nccl = [t.cpu() for t in vocab_sharded_select(shard, masks, wl.VOCAB)]
            ok = ok and all(torch.equal(g, w) for g, w in zip(got, want))
            ok = ok and all(torch.equal(g, w) for g, w in zip(nccl, want))
        torch.cuda.synchronize(dev)
        dist.barrier()
        ex.close()
        out.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_exchange_matches_nccl_and_single_launch(cuda_module):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29600 + int(np.random.default_rng().integers(0, 300))
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    results = dict(out.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)
