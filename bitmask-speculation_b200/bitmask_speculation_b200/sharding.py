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

``PeerExchange`` replaces the all-gather for argmax steps (at most 8 ranks, one GPU each): every
rank maps every other rank's exchange area (CUDA IPC over NVLink), the selection kernel stores
each row's partial into all areas while it streams, and the merge waits on epoch flags in its
own area -- no collective call on the data path.
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

    def partials(self, logits, masks, token_offset, temperature, mask_rows=None):
        """Per-row partials of ``logits`` under ``masks`` (row r's mask is ``masks[mask_rows[r]]``
        when the int32 device table ``mask_rows`` is given: ``bms_shard_partials_indexed``)."""
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
        _native.check(lib.bms_shard_partials_indexed(
            logits.data_ptr(), dtype, masks.data_ptr(), masks.shape[1],
            mask_rows.data_ptr() if mask_rows is not None else None, masks.shape[0], rows, vocab_shard,
            token_offset, float(temperature), partials.data_ptr(),
            granules.data_ptr() if granules is not None else None, stride, dev.index,
            torch.cuda.current_stream(dev).cuda_stream))
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


class PeerExchange:
    """Exchange areas of a vocabulary-sharded group (``bms_exchange_*``): this rank's own area and
    the peers' mapped areas in rank order, for batches of at most ``rows_cap`` rows.  ``areas`` may
    be given directly (ranks emulated in one process on one device); otherwise the areas are
    created and exported on every rank of ``group`` and the handles all-gathered once.  Every rank
    runs the same steps in the same order; ``step`` is the epoch of the last one."""

    def __init__(self, rows_cap: int, *, group=None, device=None, areas=None, rank=None):
        import torch
        self.rows_cap = int(rows_cap)
        self._lib = _native.library()
        self._owned = []
        self._opened = []
        self.step = 0
        device = torch.device("cuda") if device is None else torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        if areas is not None:
            self.ranks, self.rank = len(areas), int(rank)
            self.areas = list(areas)
        else:
            import torch.distributed as dist
            self.rank, self.ranks = dist.get_rank(group), dist.get_world_size(group)
            own, handle = self.create(self.device, self.ranks, self.rows_cap)
            self._owned.append(own)
            mine = torch.tensor(bytearray(bytes(handle.bytes)), dtype=torch.uint8, device=self.device)
            allh = torch.empty((self.ranks, 64), dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(allh, mine, group=group)
            allh = allh.cpu().numpy()
            self.areas = []
            for q in range(self.ranks):
                if q == self.rank:
                    self.areas.append(own)
                    continue
                h = _native.IpcHandle()
                ctypes.memmove(h.bytes, bytes(allh[q]), 64)
                ptr = ctypes.c_void_p()
                _native.check(self._lib.bms_exchange_open(self.device.index, ctypes.byref(h), ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                self.areas.append(ptr.value)
            dist.barrier(group=group)  # every peer mapped before any step stores into it
        self._areas_c = (ctypes.c_void_p * self.ranks)(*self.areas)

    @staticmethod
    def create(device, ranks: int, rows_cap: int):
        """Allocate one zeroed exchange area on ``device``: (device pointer, IPC handle)."""
        lib = _native.library()
        ptr, handle = ctypes.c_void_p(), _native.IpcHandle()
        _native.check(lib.bms_exchange_create(device.index, ranks, rows_cap, ctypes.byref(ptr), ctypes.byref(handle)))
        return ptr.value, handle

    @staticmethod
    def destroy(device, area):
        _native.check(_native.library().bms_exchange_destroy(device.index, area))

    def close(self):
        """Unmap the peers' areas and free this rank's own (call on every rank, after its last step
        and a barrier, so that no peer still stores into it)."""
        for a in self._opened:
            _native.check(self._lib.bms_exchange_close(self.device.index, a))
        for a in self._owned:
            self.destroy(self.device, a)
        self._opened, self._owned = [], []

    def partials(self, logits_shard, masks, token_offset: int, step: int):
        import torch
        rows, vocab_shard = logits_shard.shape
        dtype = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[logits_shard.dtype]
        _native.check(self._lib.bms_shard_partials_exchange(
            logits_shard.data_ptr(), dtype, masks.data_ptr(), masks.shape[1], rows, vocab_shard, token_offset,
            self._areas_c, self.ranks, self.rank, self.rows_cap, step, self.device.index,
            torch.cuda.current_stream(self.device).cuda_stream))

    def merge(self, rows: int, step: int):
        import torch
        tokens = torch.empty(rows, dtype=torch.int64, device=self.device)
        counts = torch.empty(rows, dtype=torch.int64, device=self.device)
        status = torch.empty(rows, dtype=torch.int32, device=self.device)
        _native.check(self._lib.bms_shard_merge_exchange(
            self._areas_c, self.ranks, self.rank, self.rows_cap, step, rows, tokens.data_ptr(), counts.data_ptr(),
            status.data_ptr(), self.device.index, torch.cuda.current_stream(self.device).cuda_stream))
        return tokens, counts, status

    def select(self, logits_shard, masks, token_offset: int, *, check: bool = True):
        """One argmax step: this rank's partials into every area, then the merge of the step.

        Every rank must pass the same rows.  Status 7 marks rows whose partials did not arrive from
        every rank -- a peer that stalled past the one-second device wait, or a peer whose step had
        fewer rows.  With ``check`` (the default) that raises ``RuntimeError`` after the merge (one
        device-to-host read of the statuses); with ``check=False`` the caller inspects the
        statuses itself (``check_statuses``), e.g. once after many steps."""
        if logits_shard.shape[0] > self.rows_cap:
            raise ValueError(f"{logits_shard.shape[0]} rows exceed the exchange's rows_cap {self.rows_cap}")
        self.step += 1
        self.partials(logits_shard, masks, token_offset, self.step)
        out = self.merge(logits_shard.shape[0], self.step)
        if check:
            self.check_statuses(out[2])
        return out

    @staticmethod
    def check_statuses(status) -> None:
        """Raise ``RuntimeError`` if any row of a merged exchange step reports status 7."""
        bad = (status == 7).nonzero().flatten()
        if bad.numel():
            raise RuntimeError(f"peer-memory exchange: partials of {bad.numel()} rows did not arrive from every "
                               f"rank (status 7; first row {int(bad[0])}): a peer stalled or passed other rows")


def vocab_sharded_select(logits_shard, masks, vocab: int, *, temperature: float = 0.0, uniforms=None,
                         group=None, backend=None, exchange: PeerExchange | None = None,
                         check_exchange: bool = True):
    """Masked argmax (temperature 0) or sample of rows whose vocabulary is split across ranks.

    ``logits_shard`` is this rank's [rows, size] slice (``shard_bounds(vocab, world)[rank]``),
    ``masks`` the full [rows, ceil(vocab / 32)] mask rows, ``uniforms`` float64 [rows] (sampling;
    the same values on every rank).  Returns (tokens, counts, status), identical on every rank.
    One all-gather of 32-byte partials (plus one max all-reduce when sampling); with ``exchange``
    (argmax only) the partials travel through peer memory instead and no collective is called
    (``check_exchange``: raise on rows whose partials did not arrive, see ``PeerExchange.select``).
    """
    import torch
    import torch.distributed as dist
    backend = backend or NativeShardBackend()
    if exchange is not None:
        rank, world = exchange.rank, exchange.ranks
    else:
        rank, world = dist.get_rank(group), dist.get_world_size(group)
    offset, size = shard_bounds(vocab, world)[rank]
    rows = logits_shard.shape[0]
    if logits_shard.shape[1] != size:
        raise ValueError(f"rank {rank} must hold {size} tokens of every row, got {logits_shard.shape[1]}")
    if masks.shape != (rows, (vocab + 31) // 32):
        raise ValueError("masks must be the full [rows, ceil(vocab / 32)] rows")
    if temperature != 0 and (uniforms is None or uniforms.shape != (rows,)):
        raise ValueError("sampling needs one float64 uniform per row")
    if exchange is not None:
        if temperature != 0:
            raise ValueError("the peer-memory exchange carries argmax partials only (temperature 0)")
        return exchange.select(logits_shard, masks, offset, check=check_exchange)
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
