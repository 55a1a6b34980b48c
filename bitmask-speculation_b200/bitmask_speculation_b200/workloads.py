"""Seeded synthetic workloads for the masked-selection path at V = 248,320.

No public dataset is involved in the reference's kernel benchmarks; these
generators reproduce the shapes, dtypes and value/mask distributions of the
five benchmark configurations:

1. masked argmax + count: 6 rows fp32 N(0, 3^2); masks Bernoulli(0.5) x2,
   exactly 4 and 16 valid tokens, Bernoulli(0.02), a single valid bit;
2. masked sampling: 8 rows fp16 N(0, 2^2), T = 0.7, Bernoulli masks with
   densities {1, .5, .1, .01, 1e-4 (>= 1 valid), .9, .3, .05}, per-row uniform;
3. verification round: S sequences x (K+1) = 9 rows bf16 N(0, 3^2); masks 40%
   enum-like (2-32 valid), 30% Bernoulli(0.05), 30% Bernoulli(0.6); drafts match
   the target argmax until a geometric mismatch (acceptance 0.88 per position);
5. scale-out: rows bf16 N(0, 3^2), Bernoulli masks at log-uniform densities in
   [1e-4, 1].

The numpy generators (``*_np``) are bit-reproducible across machines and feed
the golden fixtures and parity tests; the torch generators (``*_torch``) build
benchmark-sized inputs directly on the device.  Masks are packed little-endian
per 32-bit word (token t is bit t % 32 of word t // 32) into signed int32, with
every bit at or beyond the vocabulary cleared.
"""

from __future__ import annotations

import numpy as np

VOCAB = 248_320
SAMPLE_DENSITIES = (1.0, 0.5, 0.1, 0.01, 1e-4, 0.9, 0.3, 0.05)
SAMPLE_TEMPERATURE = 0.7
DRAFT_K = 8
ACCEPT_PROB = 0.88


def words_for(vocab: int) -> int:
    return (vocab + 31) // 32


# ---------------------------------------------------------------- numpy side
def pack_bits_np(valid: np.ndarray) -> np.ndarray:
    """[R, V] bool -> [R, ceil(V/32)] int32 packed words, tail bits zero."""
    valid = np.asarray(valid, dtype=bool)
    rows, vocab = valid.shape
    words = words_for(vocab)
    padded = np.zeros((rows, words * 32), dtype=bool)
    padded[:, :vocab] = valid
    packed = np.packbits(padded.reshape(rows, words, 32), axis=2, bitorder="little")
    return np.ascontiguousarray(packed).view("<u4").reshape(rows, words).astype(np.uint32).view(np.int32)


def unpack_bits_np(masks: np.ndarray, vocab: int) -> np.ndarray:
    m = np.ascontiguousarray(masks, dtype=np.int32).view(np.uint32)
    rows = m.shape[0]
    bits = np.unpackbits(m.view(np.uint8).reshape(rows, -1), axis=1, bitorder="little")
    return bits[:, :vocab].astype(bool)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (round to nearest even; NaN kept quiet)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded[nan] = 0x7FC0
    return rounded


def to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def exact_count_mask(rng: np.random.Generator, vocab: int, count: int) -> np.ndarray:
    valid = np.zeros(vocab, dtype=bool)
    valid[rng.choice(vocab, size=count, replace=False)] = True
    return valid


def argmax_config_np(seed: int = 1, vocab: int = VOCAB):
    """Configuration 1: (logits f32 [6, V], masks int32 [6, W])."""
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((6, vocab), dtype=np.float32) * np.float32(3.0))
    valid = np.zeros((6, vocab), dtype=bool)
    valid[0] = rng.random(vocab) < 0.5
    valid[1] = rng.random(vocab) < 0.5
    valid[2] = exact_count_mask(rng, vocab, 4)
    valid[3] = exact_count_mask(rng, vocab, 16)
    valid[4] = rng.random(vocab) < 0.02
    valid[5] = exact_count_mask(rng, vocab, 1)
    return logits, pack_bits_np(valid)


def sample_config_np(seed: int = 2, vocab: int = VOCAB, densities=SAMPLE_DENSITIES):
    """Configuration 2: (fp16 bits [8, V], masks [8, W], uniforms [8], T)."""
    rng = np.random.default_rng(seed)
    logits = to_f16_bits(rng.standard_normal((len(densities), vocab), dtype=np.float32) * np.float32(2.0))
    valid = np.zeros((len(densities), vocab), dtype=bool)
    for r, p in enumerate(densities):
        valid[r] = rng.random(vocab) < p
        if not valid[r].any():
            valid[r, rng.integers(vocab)] = True
    uniforms = rng.random(len(densities))
    return logits, pack_bits_np(valid), uniforms, SAMPLE_TEMPERATURE


def verify_masks_np(rng: np.random.Generator, rows: int, vocab: int) -> np.ndarray:
    valid = np.zeros((rows, vocab), dtype=bool)
    kinds = rng.random(rows)
    for r in range(rows):
        if kinds[r] < 0.4:
            valid[r] = exact_count_mask(rng, vocab, int(rng.integers(2, 33)))
        elif kinds[r] < 0.7:
            valid[r] = rng.random(vocab) < 0.05
        else:
            valid[r] = rng.random(vocab) < 0.6
        if not valid[r].any():
            valid[r, rng.integers(vocab)] = True
    return valid


def masked_argmax_np(values: np.ndarray, valid: np.ndarray) -> np.ndarray:
    """Lowest-index masked argmax per row (input synthesis only; rows are NaN-free)."""
    masked = np.where(valid, values, -np.inf)
    return masked.argmax(axis=1)


def draft_proposals_np(rng: np.random.Generator, targets: np.ndarray, valid: np.ndarray,
                       seqs: int, k: int, accept: float = ACCEPT_PROB):
    """Drafts equal to the target argmax up to a geometric first mismatch."""
    proposals = np.zeros((seqs, k), dtype=np.int64)
    for s in range(seqs):
        mismatch = int(rng.geometric(1.0 - accept)) - 1  # accepted positions before the miss
        for i in range(k):
            row = s * (k + 1) + i
            if i < mismatch:
                proposals[s, i] = targets[row]
            else:
                choices = np.flatnonzero(valid[row])
                other = choices[choices != targets[row]]
                pool = other if other.size else np.arange(valid.shape[1])[
                    np.arange(valid.shape[1]) != targets[row]]
                proposals[s, i] = int(rng.choice(pool))
                # Positions after the first mismatch are never compared.
                for j in range(i + 1, k):
                    proposals[s, j] = int(rng.integers(valid.shape[1]))
                break
    return proposals


def verify_config_np(seed: int = 3, seqs: int = 4, vocab: int = VOCAB, k: int = DRAFT_K):
    """Configuration 3 at a parity-test size.

    Returns (bf16 bits [S*(K+1), V], masks, proposals [S, K], lengths [S]).
    """
    rng = np.random.default_rng(seed)
    rows = seqs * (k + 1)
    values = rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(3.0)
    bits = to_bf16_bits(values)
    valid = verify_masks_np(rng, rows, vocab)
    widened = (bits.astype(np.uint32) << 16).view(np.float32)
    targets = masked_argmax_np(widened, valid)
    proposals = draft_proposals_np(rng, targets, valid, seqs, k)
    lengths = np.full(seqs, k, dtype=np.int32)
    return bits, pack_bits_np(valid), proposals, lengths


# ---------------------------------------------------------------- torch side
def pack_bits_torch(valid):
    """[R, V] bool (device) -> [R, W] int32 packed words, tail bits zero."""
    import torch
    rows, vocab = valid.shape
    words = words_for(vocab)
    padded = torch.nn.functional.pad(valid, (0, words * 32 - vocab))
    weights = (torch.ones(32, dtype=torch.int64, device=valid.device) << torch.arange(
        32, device=valid.device))
    packed = (padded.view(rows, words, 32).to(torch.int64) * weights).sum(2)
    return torch.where(packed >= 2**31, packed - 2**32, packed).to(torch.int32).contiguous()


def bernoulli_masks_torch(rows: int, vocab: int, densities, generator, device):
    """Per-row Bernoulli masks (density tensor [rows]), at least one valid bit per row."""
    import torch
    valid = torch.rand((rows, vocab), generator=generator, device=device) < densities[:, None]
    empty = ~valid.any(1)
    if bool(empty.any()):
        idx = torch.randint(vocab, (rows,), generator=generator, device=device)
        valid[empty, idx[empty]] = True
    return valid


def enum_masks_torch(rows: int, vocab: int, generator, device, lo: int = 2, hi: int = 32):
    import torch
    counts = torch.randint(lo, hi + 1, (rows,), generator=generator, device=device)
    keys = torch.rand((rows, vocab), generator=generator, device=device)
    # The `count` smallest keys of each row are its valid tokens.
    kth = torch.sort(keys, dim=1).values.gather(1, (counts - 1)[:, None])
    return keys <= kth


def verify_batch_torch(seqs: int, vocab: int = VOCAB, k: int = DRAFT_K, seed: int = 3,
                       device="cuda", chunk_rows: int = 256):
    """Configuration 3 at benchmark size, built on the device.

    Returns (logits bf16 [S*(K+1), V], masks int32 [S*(K+1), W], proposals
    int64 [S, K], lengths int32 [S]).
    """
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    rows = seqs * (k + 1)
    logits = torch.empty((rows, vocab), dtype=torch.bfloat16, device=device)
    masks = torch.empty((rows, words_for(vocab)), dtype=torch.int32, device=device)
    targets = torch.empty(rows, dtype=torch.int64, device=device)
    alt = torch.empty(rows, dtype=torch.int64, device=device)
    kinds = torch.rand(rows, generator=g, device=device)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        n = r1 - r0
        vals = (torch.randn((n, vocab), generator=g, device=device) * 3.0).to(torch.bfloat16)
        kind = kinds[r0:r1]
        dens = torch.where(kind < 0.7, 0.05, 0.6).to(torch.float32)
        valid = bernoulli_masks_torch(n, vocab, dens, g, device)
        enum = enum_masks_torch(n, vocab, g, device)
        valid = torch.where((kind < 0.4)[:, None], enum, valid)
        logits[r0:r1] = vals
        masks[r0:r1] = pack_bits_torch(valid)
        masked = vals.float().masked_fill(~valid, float("-inf"))
        targets[r0:r1] = masked.argmax(1)
        # A second valid token per row, for the first mismatching draft.
        second = masked.masked_fill(
            torch.nn.functional.one_hot(targets[r0:r1], vocab).bool(), float("-inf")).argmax(1)
        alt[r0:r1] = second
    geo = torch.empty(seqs, device=device).geometric_(1.0 - ACCEPT_PROB, generator=g).long() - 1
    t = targets.view(seqs, k + 1)[:, :k]
    a = alt.view(seqs, k + 1)[:, :k]
    pos = torch.arange(k, device=device)[None, :]
    proposals = torch.where(pos < geo[:, None], t, a)
    lengths = torch.full((seqs,), k, dtype=torch.int32, device=device)
    return logits, masks, proposals.contiguous(), lengths


def scale_rows_torch(rows: int, vocab: int = VOCAB, seed: int = 5, device="cuda",
                     chunk_rows: int = 512):
    """Configuration 5: bf16 N(0, 3^2) rows with log-uniform mask densities."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    logits = torch.empty((rows, vocab), dtype=torch.bfloat16, device=device)
    masks = torch.empty((rows, words_for(vocab)), dtype=torch.int32, device=device)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        n = r1 - r0
        logits[r0:r1] = (torch.randn((n, vocab), generator=g, device=device) * 3.0).to(torch.bfloat16)
        dens = torch.exp(torch.empty(n, device=device).uniform_(np.log(1e-4), 0.0, generator=g))
        masks[r0:r1] = pack_bits_torch(bernoulli_masks_torch(n, vocab, dens, g, device))
    return logits, masks


# ---------------------------------------------------------------- synthetic grammar
class SyntheticDFAGrammar:
    """Token-level DFA grammar of the end-to-end configuration's shape: ``states`` states, each
    allowing either an enumerated set of 1-8 token IDs or a Bernoulli(``free_density``) free-text
    set; accepting token t in state q moves to ``(q * 31 + t * 7 + 1) % states``.  Accepting an
    EOS token (``eos`` IDs, allowed in the free-text states) terminates it.

    Implements the reference's ``ForkableGrammarState`` protocol (grammar/state.py:13-44) plus
    ``packed_mask`` (an owned CPU int32 row, grammar/xgrammar.py:63-70) and ``mask_density``.
    Masks are precomputed per state and shared by forks (read-only).
    """

    def __init__(self, vocab: int, *, states: int = 64, seed: int = 7, free_density: float = 0.3,
                 eos=(0,), _tables=None, _state: int = 0, _terminated: bool = False):
        self._vocab = int(vocab)
        if _tables is None:
            rng = np.random.default_rng(seed)
            valid = np.zeros((states, self._vocab), dtype=bool)
            free = rng.random(states) < 0.5
            for q in range(states):
                if free[q]:
                    valid[q] = rng.random(self._vocab) < free_density
                    valid[q, list(eos)] = True
                else:
                    ids = rng.choice(np.arange(len(eos), self._vocab), size=int(rng.integers(1, 9)), replace=False)
                    valid[q, ids] = True
            _tables = (pack_bits_np(valid), [np.flatnonzero(v) for v in valid], frozenset(int(e) for e in eos),
                       valid.sum(axis=1))
        self._tables = _tables
        self._state = _state
        self._terminated = _terminated

    @property
    def vocab_size(self) -> int:
        return self._vocab

    @property
    def state(self) -> int:
        return self._state

    def is_terminated(self) -> bool:
        return self._terminated

    def allowed_token_ids(self):
        return () if self._terminated else tuple(int(t) for t in self._tables[1][self._state])

    def allowed_ids_np(self) -> np.ndarray:
        """Allowed token IDs of the current state as a numpy array (read-only)."""
        return np.zeros(0, dtype=np.int64) if self._terminated else self._tables[1][self._state]

    def packed_mask(self):
        import torch
        words = self._tables[0][self._state]
        return torch.from_numpy(np.zeros_like(words) if self._terminated else words.copy())

    def packed_mask_np(self) -> np.ndarray:
        """The current state's mask row (read-only view; zeros once terminated)."""
        return np.zeros_like(self._tables[0][0]) if self._terminated else self._tables[0][self._state]

    def mask_density(self) -> float:
        return 0.0 if self._terminated else float(self._tables[3][self._state]) / self._vocab

    def mask_table(self) -> np.ndarray:
        """Packed masks of every state, [states, W] int32 (shared by forks, read-only)."""
        return self._tables[0]

    def state_index(self) -> int:
        """Row of ``mask_table()`` holding the current state's mask; -1 once terminated."""
        return -1 if self._terminated else self._state

    def device_advance(self, state, token):
        """``accept_token`` on the device for a token the state allows: int64 tensors ``state`` and
        ``token`` of one shape give (next state, whether the token is an EOS, which terminates)."""
        import torch
        nxt = torch.remainder(state * 31 + token * 7 + 1, len(self._tables[1]))
        eos = torch.zeros_like(token, dtype=torch.bool)
        for e in sorted(self._tables[2]):
            eos = eos | (token == e)
        return nxt, eos

    def accept_token(self, token: int) -> bool:
        token = int(token)
        if self._terminated or not (0 <= token < self._vocab):
            return False
        words = self._tables[0][self._state]
        if not (int(words[token >> 5]) >> (token & 31)) & 1:
            return False
        if token in self._tables[2]:
            self._terminated = True
        else:
            self._state = (self._state * 31 + token * 7 + 1) % len(self._tables[1])
        return True

    def fork(self) -> "SyntheticDFAGrammar":
        return SyntheticDFAGrammar(self._vocab, _tables=self._tables, _state=self._state,
                                   _terminated=self._terminated)


def grammar_round_torch(seqs: int, select, vocab: int = VOCAB, k: int = DRAFT_K, seed: int = 11, device="cuda",
                        p_accept: float = 0.88):
    """One grammar-constrained verification round of ``seqs`` sequences (input synthesis).

    Each sequence gets a ``SyntheticDFAGrammar`` (shared 64-state tables) advanced by a few random
    non-terminating tokens, target rows bf16 N(0, 3^2) [seqs*(k+1), vocab] on the device, and a
    draft that takes the target's own masked choice (``select(rows, masks) -> (tokens, status)``
    numpy arrays, for device rows [seqs, vocab] and int32 mask rows) with probability ``p_accept``
    per position and another allowed token otherwise.  Returns
    (logits, fork masks [seqs*(k+1), W] on the device, proposals int64 [seqs, k], lengths int32
    [seqs], the sequences' committed grammars, the drafts).
    """
    import torch
    rng = np.random.default_rng(seed)
    base = SyntheticDFAGrammar(vocab, states=64, seed=seed)
    eos = base._tables[2]
    grammars = []
    for _ in range(seqs):
        g = base.fork()
        for _ in range(int(rng.integers(0, 6))):
            ids = g.allowed_ids_np()
            ids = ids[~np.isin(ids, list(eos))]
            if ids.size:
                g.accept_token(int(rng.choice(ids)))
        grammars.append(g)
    gen = torch.Generator(device=device).manual_seed(seed)
    logits = (torch.randn(seqs * (k + 1), vocab, generator=gen, device=device) * 3).to(torch.bfloat16)
    words = words_for(vocab)
    masks = np.zeros((seqs * (k + 1), words), dtype=np.int32)
    forks = [g.fork() for g in grammars]
    live = [not f.is_terminated() for f in forks]
    drafts = [[] for _ in range(seqs)]
    for i in range(k + 1):
        for s in range(seqs):
            masks[s * (k + 1) + i] = forks[s].packed_mask_np() if live[s] else 0
        if i == k:
            break
        rows = torch.arange(seqs, device=device) * (k + 1) + i
        tok, st = select(logits[rows].contiguous(), masks[i::k + 1].copy())
        for s in range(seqs):
            if not live[s]:
                continue
            if st[s] != 0:
                live[s] = False
                continue
            t = int(tok[s])
            if rng.random() > p_accept:
                ids = forks[s].allowed_ids_np()
                ids = ids[ids != t]
                if ids.size:
                    t = int(rng.choice(ids))
            drafts[s].append(t)
            if not forks[s].accept_token(t) or forks[s].is_terminated():
                live[s] = False
    proposals = np.zeros((seqs, k), dtype=np.int64)
    lengths = np.zeros(seqs, dtype=np.int32)
    for s, d in enumerate(drafts):
        proposals[s, : len(d)] = d
        lengths[s] = len(d)
    return (logits, torch.from_numpy(masks).to(device), torch.from_numpy(proposals).to(device),
            torch.from_numpy(lengths).to(device), grammars, [tuple(d) for d in drafts])
