"""Stochastic speculative acceptance (speculative sampling) on the batched sampler's normalisers.

The reference decodes greedily; stochastic acceptance is outside its correctness contract
(docs/design.md:5-11), so this is an extension with no reference counterpart.  The rule is the
standard one for drafts sampled from the draft model's distribution: with p_i the target's and q_i
the draft's masked softmax at temperature T for position i, draft d_i is accepted with probability
min(1, p_i(d_i) / q_i(d_i)); at the first rejection j a replacement is drawn from
max(0, p_j - q_j) normalised, and if all L drafts are accepted a bonus token is drawn from p_L.
Every emitted token is then distributed exactly as target sampling would give it.

Device work per round: the selection kernel's sampler partials (row max and mass, one streaming
pass) for the target rows and the draft rows -- the draft rows read the round's mask rows through
a table (``bms_shard_partials_indexed``), no gathered copy -- then ``bms_speculative_accept`` (a
cluster of 1-8 CTAs per sequence: the acceptance tests, then an inverse-CDF pass over the one row
that is sampled).  ``lazy=True`` instead lets that one launch stream, position by position, the
target and draft rows to their normalisers and test each draft, stopping at the first rejection.
"""

from __future__ import annotations

from dataclasses import dataclass

from . import _native
from .kernels._validation import temperature_input
from .verification import KINDS, VerifiedToken

_DRAFT_MASK_ROWS: dict = {}  # (seqs, K, device) -> int32 table: draft row s*K + i -> mask row s*(K+1) + i


def _draft_mask_rows(seqs: int, k: int, device):
    import torch
    key = (seqs, k, str(device))
    table = _DRAFT_MASK_ROWS.get(key)
    if table is None:
        r = torch.arange(seqs * k, dtype=torch.int64, device=device)
        table = ((r // k) * (k + 1) + r % k).to(torch.int32)
        if len(_DRAFT_MASK_ROWS) >= 16:
            _DRAFT_MASK_ROWS.clear()
        _DRAFT_MASK_ROWS[key] = table
    return table


_ERRORS = {1: "mask has no valid token", 2: "logits contain NaN", 4: "valid logits have no finite probability mass",
           5: "positive infinity is unsupported for stochastic sampling", 6: "proposal count outside [0, K]",
           7: "device wait timed out"}


@dataclass(frozen=True, slots=True)
class SpeculativeAcceptance:
    """Device tensors of one round: per sequence the accepted length, the drawn token, its kind
    (0 replacement, 1 bonus, 2 fallback) and a status."""

    accept_len: object
    token: object
    kind: object
    status: object

    def events(self, seq: int, proposals) -> list[VerifiedToken]:
        """The round of sequence ``seq`` as events (one device-to-host read per call): accepted
        drafts, then the replacement ("correction"), bonus or fallback token.  A failed status
        raises ``ValueError``."""
        a, t, k, st = (int(x[seq]) for x in (self.accept_len, self.token, self.kind, self.status))
        if st:
            raise ValueError(_ERRORS.get(st, f"speculative acceptance status {st}"))
        return [VerifiedToken(int(p), "accepted") for p in list(proposals)[:a]] + [VerifiedToken(t, KINDS[k])]


def speculative_accept(target_logits, draft_logits, masks, proposals, lengths, *, temperature: float,
                       accept_uniforms=None, resample_uniforms=None, generator=None,
                       lazy: bool = False) -> SpeculativeAcceptance:
    """One stochastic verification round for S sequences of up to K drafts.

    ``target_logits`` [S*(K+1), V] (row s*(K+1)+i scores position i of sequence s), ``draft_logits``
    [S*K, V] (the draft model's scores the drafts were sampled from), same dtype (float32, bfloat16 or
    float16) and device; ``masks`` [S*(K+1), ceil(V/32)] int32, mask row s*(K+1)+i constraining both
    models at position i; ``proposals`` int64 [S, K]; ``lengths`` int32 [S].  Uniforms float64
    ``accept_uniforms`` [S, K] and ``resample_uniforms`` [S] are drawn from ``generator`` when not
    given.  No host synchronization.

    By default the sampler partials of every target and draft row come first (two selection
    launches), then the acceptance kernel.  ``lazy=True`` (rows and mask rows 16-byte aligned, rows a
    multiple of 16 bytes, mask rows a multiple of 4 words): one launch computes the normalisers of
    only the positions it consumes, stopping at the first rejection -- fewer bytes, but each
    sequence's positions run one after another, so it pays when accepted runs are short.  Both
    follow the same rule; they can differ only where a uniform sits within rounding of a decision.
    """
    import torch
    temperature = temperature_input(temperature)
    if temperature == 0:
        raise ValueError("stochastic acceptance needs a positive temperature (temperature 0 is verify_batch)")
    from .sharding import NativeShardBackend
    rows, vocab = target_logits.shape
    seqs, k = proposals.shape
    dev = target_logits.device
    if rows != seqs * (k + 1) or tuple(draft_logits.shape) != (seqs * k, vocab):
        raise ValueError("target_logits must be [S*(K+1), V] and draft_logits [S*K, V]")
    if draft_logits.dtype != target_logits.dtype or draft_logits.device != dev:
        raise ValueError("draft and target logits must share dtype and device")
    words = (vocab + 31) // 32
    if masks.dtype != torch.int32 or tuple(masks.shape) != (rows, words) or not masks.is_contiguous():
        raise ValueError("masks must be a contiguous int32 [S*(K+1), ceil(V/32)] tensor")
    if proposals.dtype != torch.int64 or lengths.dtype != torch.int32 or tuple(lengths.shape) != (seqs,):
        raise ValueError("proposals must be int64 [S, K] and lengths int32 [S]")
    target_logits, draft_logits = target_logits.contiguous(), draft_logits.contiguous()
    tensors = (target_logits, masks) + ((draft_logits,) if draft_logits.numel() else ())
    streamable = ((vocab * target_logits.element_size()) % 16 == 0 and words % 4 == 0
                  and all(t.data_ptr() % 16 == 0 for t in tensors))
    if lazy and not streamable:
        raise ValueError("lazy acceptance needs 16-byte aligned rows of a multiple of 16 bytes and mask rows "
                         "of a multiple of 4 words")
    tpart = qpart = None
    if not lazy:
        backend = NativeShardBackend()
        tpart, _ = backend.partials(target_logits, masks, 0, temperature)
        if seqs * k:
            qpart, _ = backend.partials(draft_logits, masks, 0, temperature, mask_rows=_draft_mask_rows(seqs, k, dev))
    if accept_uniforms is None:
        accept_uniforms = torch.rand((seqs, k), dtype=torch.float64, device=dev, generator=generator)
    if resample_uniforms is None:
        resample_uniforms = torch.rand(seqs, dtype=torch.float64, device=dev, generator=generator)
    for u, shape in ((accept_uniforms, (seqs, k)), (resample_uniforms, (seqs,))):
        if u.dtype != torch.float64 or tuple(u.shape) != shape or u.device != dev or not u.is_contiguous():
            raise ValueError("uniforms must be contiguous float64 tensors on the logits' device")
    out = SpeculativeAcceptance(torch.empty(seqs, dtype=torch.int32, device=dev),
                                torch.empty(seqs, dtype=torch.int64, device=dev),
                                torch.empty(seqs, dtype=torch.int32, device=dev),
                                torch.empty(seqs, dtype=torch.int32, device=dev))
    if seqs == 0:
        return out
    dtype = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[target_logits.dtype]
    ptr = (lambda t: None if t is None or t.numel() == 0 else t.data_ptr())
    _native.check(_native.library().bms_speculative_accept(
        target_logits.data_ptr(), ptr(draft_logits), dtype, masks.data_ptr(), seqs, k + 1, vocab, ptr(proposals),
        lengths.data_ptr(), ptr(tpart), ptr(qpart), temperature, ptr(accept_uniforms),
        resample_uniforms.data_ptr(), out.accept_len.data_ptr(), out.token.data_ptr(), out.kind.data_ptr(),
        out.status.data_ptr(), dev.index, torch.cuda.current_stream(dev).cuda_stream))
    return out


class AcceptancePolicy:
    """Chooses ``speculative_accept``'s mode from the rounds seen so far: the lazy round reads only
    the positions up to the first rejection but runs each sequence's positions one after another,
    so it pays when accepted runs are short.  Measured on B200 (256 sequences x K = 8, V = 248,320
    bf16), lazy against full partials: 0.27 / 0.48 ms with a mean accepted run of 0.36 drafts,
    0.39 / 0.48 with 1.05, 0.51 / 0.48 with 1.93, 0.54 / 0.48 with 2.6.  ``observe(accept_len)`` takes a round's accepted lengths (host values, the
    ones an engine reads anyway); ``lazy`` is the mode for the next round: lazy while the moving
    average of the mean accepted run stays below ``threshold``.  Rounds that cannot stream (see
    ``speculative_accept``) must pass ``lazy=False`` whatever this says."""

    def __init__(self, threshold: float = 1.5, decay: float = 0.8, initial: float | None = None):
        if not 0.0 <= decay < 1.0:
            raise ValueError("decay must be in [0, 1)")
        self.threshold = float(threshold)
        self.decay = float(decay)
        self.mean_run = initial

    def observe(self, accept_len) -> None:
        values = [int(a) for a in accept_len]
        if not values:
            return
        run = sum(values) / len(values)
        self.mean_run = run if self.mean_run is None else self.decay * self.mean_run + (1.0 - self.decay) * run

    @property
    def lazy(self) -> bool:
        return self.mean_run is not None and self.mean_run < self.threshold


__all__ = ["AcceptancePolicy", "SpeculativeAcceptance", "speculative_accept"]
