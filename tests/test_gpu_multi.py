"""Multi-GPU paths on real GPUs (skipped with fewer than two devices).

Vocabulary-sharded selection over NCCL must equal the single-GPU cluster merge covering the same
slices, bit for bit (argmax and sampling); row sharding needs no collective at all.
"""

import datetime
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _inputs(rows, vocab):
    from bitmask_speculation_b200 import workloads as wl
    rng = np.random.default_rng(77)
    vals = wl.to_bf16_bits(rng.standard_normal((rows, vocab), dtype=np.float32) * 3)
    valid = rng.random((rows, vocab)) < rng.choice([1.0, 0.3, 1e-3], size=(rows, 1))
    valid[:, 7] = True
    return vals, wl.pack_bits_np(valid), rng.random(rows)


def _worker(rank, world, port, rows, vocab, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import torch.distributed as dist
    from bitmask_speculation_b200.sharding import shard_bounds, vocab_sharded_select
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        vals, masks, uniforms = _inputs(rows, vocab)
        off, size = shard_bounds(vocab, world)[rank]
        shard = torch.from_numpy(np.ascontiguousarray(vals[:, off:off + size]).view(np.int16)).view(torch.bfloat16).cuda()
        m = torch.from_numpy(masks).cuda()
        u = torch.from_numpy(uniforms).cuda()
        arg = vocab_sharded_select(shard, m, vocab)
        smp = vocab_sharded_select(shard, m, vocab, temperature=0.8, uniforms=u)
        torch.cuda.synchronize()
        queue.put((rank, [t.cpu().tolist() for t in arg], [t.cpu().tolist() for t in smp]))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_vocab_sharded_nccl_equals_single_gpu_cluster_merge(cuda_module, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"{world} CUDA devices required")
    import torch.multiprocessing as mp
    from bitmask_speculation_b200 import _native
    rows, vocab = 64, 248320
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29650 + os.getpid() % 500
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, vocab, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, arg, smp = queue.get(timeout=300)
        results[r] = (arg, smp)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(results[r] == results[0] for r in results)
    vals, masks, uniforms = _inputs(rows, vocab)
    logits = torch.from_numpy(vals.view(np.int16)).view(torch.bfloat16).cuda()
    m = torch.from_numpy(masks).cuda()
    _native.set_launch_override(world, 0)
    try:
        ref_arg = [t.cpu().tolist() for t in cuda_module.masked_reduce_batch(logits, m)]
        ref_smp = [t.cpu().tolist() for t in cuda_module.masked_sample_batch(logits, m, 0.8,
                                                                             torch.from_numpy(uniforms).cuda())]
    finally:
        _native.set_launch_override(0, 0)
    assert results[0][0] == ref_arg
    assert results[0][1] == ref_smp
