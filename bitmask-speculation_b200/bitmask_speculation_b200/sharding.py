"""Multi-GPU selection: row sharding (no collective) and vocabulary sharding (NCCL merge).

Rows are independent, so large batches shard by row: every rank selects its own contiguous
slice of rows with the single-GPU kernels and no collective is needed (``row_shard``).

A row can also be split by vocabulary: rank r holds tokens ``[offset_r, offset_r + size_r)`` of
every row (``shard_bounds``; offsets are multiples of 32 so each shard starts on a mask word) and
the full mask rows.  Each rank computes one 32-byte partial per row (``bms_shard_partials``), the
partials are all-gathered over NCCL in rank order, and every rank merges them
(``bms_shard_merge``) with the same arithmetic as the single-GPU kernel's cluster merge.  For
sampling, the rank holding the crossing walks its shard and a max all-reduce shares the token.
Argmax, counts and status are identical on every rank; a single-GPU run whose cluster ranks cover
the same slices (cluster size = world size) gives bit-identical results.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _native

PARTIAL_BYTES = 32


def shard_bounds(vocab: int, world: int) -> list[tuple[int, int]]:
    """(token_offset, size) of each rank's vocabulary slice; offsets are multiples of 32."""
    if world < 1:
        raise ValueError("world size must be positive")
    seg = ((vocab + world - 1) // world + 31) // 32 * 32
    out = []
    for r in range(world):
        start = min(r * seg, vocab)
        out.append((start, max(0, min(seg, vocab - start))))
    if any(size == 0 for _, size in out):
        raise ValueError("vocabulary too small for this many shards")
    return out


def row_shard(rows: int, world: int, rank: int) -> slice:
    """Contiguous, remainder-balanced slice of rows for one rank (row sharding, no collective)."""
    q, r = divmod(rows, world)
    start = rank * q + min(rank, r)
    return slice(start, start + q + (1 if rank < r else 0))


@dataclass
class NativeShardBackend:
    """The CUDA kernels behind ``vocab_sharded_select`` (the only product backend)."""

    def partials(self, logits, masks, token_offset, temperature):
        import torch
        rows, vocab_shard = logits.shape
        dev = logits.device
        lib = _native.library()
        dtype = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[logits.dtype]
        partials = torch.empty((rows, PARTIAL_BYTES), dtype=torch.uint8, device=dev)
        granules, stride = None, 0
        if temperature != 0:
            stride = int(lib.bms_shard_granule_bytes(dtype, vocab_shard))
            stride = (stride + 15) // 16 * 16
            granules = torch.empty((rows, stride), dtype=torch.uint8, device=dev)
        _native.check(lib.bms_shard_partials(
            logits.data_ptr(), dtype, masks.data_ptr(), masks.shape[1], rows, vocab_shard, token_offset,
            float(temperature), partials.data_ptr(), granules.data_ptr() if granules is not None else None,
            stride, dev.index, torch.cuda.current_stream(dev).cuda_stream))
        return partials, (granules, stride)

    def merge(self, gathered, shard, temperature, uniforms, logits, masks, token_offset, aux):
        import torch
        shards, rows, _ = gathered.shape
        dev = gathered.device
        lib = _native.library()
        dtype = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[logits.dtype]
        granules, stride = aux
        tokens = torch.empty(rows, dtype=torch.int64, device=dev)
        counts = torch.empty(rows, dtype=torch.int64, device=dev)
        status = torch.empty(rows, dtype=torch.int32, device=dev)
        _native.check(lib.bms_shard_merge(
            gathered.data_ptr(), shards, shard, rows, float(temperature),
            uniforms.data_ptr() if uniforms is not None else None, logits.data_ptr(), dtype, masks.data_ptr(),
            masks.shape[1], logits.shape[1], token_offset,
            granules.data_ptr() if granules is not None else None, stride, tokens.data_ptr(), counts.data_ptr(),
            status.data_ptr(), dev.index, torch.cuda.current_stream(dev).cuda_stream))
        return tokens, counts, status


def vocab_sharded_select(logits_shard, masks, vocab: int, *, temperature: float = 0.0, uniforms=None,
                         group=None, backend=None):
    """Masked argmax (temperature 0) or sample of rows whose vocabulary is split across ranks.

    ``logits_shard`` is this rank's [rows, size] slice (``shard_bounds(vocab, world)[rank]``),
    ``masks`` the full [rows, ceil(vocab / 32)] mask rows, ``uniforms`` float64 [rows] (sampling;
    the same values on every rank).  Returns (tokens, counts, status), identical on every rank.
    One all-gather of 32-byte partials (plus one max all-reduce when sampling).
    """
    import torch
    import torch.distributed as dist
    backend = backend or NativeShardBackend()
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    offset, size = shard_bounds(vocab, world)[rank]
    rows = logits_shard.shape[0]
    if logits_shard.shape[1] != size:
        raise ValueError(f"rank {rank} must hold {size} tokens of every row, got {logits_shard.shape[1]}")
    if masks.shape != (rows, (vocab + 31) // 32):
        raise ValueError("masks must be the full [rows, ceil(vocab / 32)] rows")
    if temperature != 0 and (uniforms is None or uniforms.shape != (rows,)):
        raise ValueError("sampling needs one float64 uniform per row")
    partials, aux = backend.partials(logits_shard, masks, offset, temperature)
    flat = torch.empty((world * rows, PARTIAL_BYTES), dtype=partials.dtype, device=partials.device)
    dist.all_gather_into_tensor(flat, partials, group=group)
    gathered = flat.view(world, rows, PARTIAL_BYTES)
    tokens, counts, status = backend.merge(gathered, rank, temperature, uniforms, logits_shard, masks, offset, aux)
    if temperature != 0:
        # Only the owning rank knows the sampled token; status can differ only there.
        packed = torch.stack([tokens, status.to(torch.int64)])
        dist.all_reduce(packed, op=dist.ReduceOp.MAX, group=group)
        tokens, status = packed[0].contiguous(), packed[1].to(torch.int32)
    return tokens, counts, status
