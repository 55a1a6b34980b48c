"""CPU oracle for the masked-selection path -- TEST INFRASTRUCTURE ONLY.

A plain-C restatement (``oracle.c``) of the reference's own CPU/PyTorch
implementation of the path, wrapped with ctypes and numpy.  Only the tests,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it, and
only as the checker or the timed CPU baseline: the shipped library never calls
it and has no CPU fallback.

Reference functions restated (file:line in karthikeyansura/bitmask-speculation):

* ``mask_count``    -- grammar/density.py:23-48 ``packed_mask_count``
* ``reduce_rows``   -- benchmarks/reductions.py:9-17 ``torch_reduce`` with the
  native token/status convention of csrc/argmax.cu:77-98
* ``sample_rows``   -- kernels/reference.py:10-52 ``masked_sample_reference``
  (status codes of csrc/sample.cu:24-25)
* ``fsum``          -- CPython ``math.fsum`` used by reference.py:42
* ``budget``        -- decoding/scheduling.py:40-46 ``DensityPolicy.budget``
* ``verify``        -- decoding/verification.py:18-48 ``verify_prefix`` over
  per-row targets (models/transformers.py:181-201)

The oracle is pinned against golden vectors produced by the reference itself
(``tests/golden/``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "oracle.c"
LIBRARY = HERE / "_build" / "liboracle.so"

DTYPE_CODES = {"float32": 0, "bfloat16": 1, "float16": 2}
_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> Path:
    """Compile ``oracle.c`` with gcc + OpenMP into ``oracle/_build``."""
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < SOURCE.stat().st_mtime:
        tmp = LIBRARY.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11",
                        "-fno-fast-math", "-ffp-contract=off", "-o", str(tmp), str(SOURCE), "-lm"],
                       check=True)
        os.replace(tmp, LIBRARY)
    return LIBRARY


def _load():
    global _lib
    with _lock:
        if _lib is None:
            lib = ctypes.CDLL(str(build()))
            p, i64, i32, f64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_double
            lib.orc_mask_count.argtypes = [p, i64]
            lib.orc_mask_count.restype = i64
            lib.orc_reduce_rows.argtypes = [p, ctypes.c_int, p, i64, i64, p, p, p, ctypes.c_int]
            lib.orc_sample_rows.argtypes = [p, ctypes.c_int, p, i64, i64, f64, p, p, p, ctypes.c_int]
            lib.orc_fsum.argtypes = [p, i64]
            lib.orc_fsum.restype = f64
            lib.orc_budget.argtypes = [i32, f64, f64, i32, i32, f64]
            lib.orc_budget.restype = i32
            lib.orc_budget_rows.argtypes = [i32, f64, f64, i32, i32, p, i64, i64, p, p]
            lib.orc_verify.argtypes = [p, p, i64, i64, p, p, p, p, p, p]
            lib.orc_widen.argtypes = [p, ctypes.c_int, i64, p]
            lib.orc_max_threads.restype = ctypes.c_int
            _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _logit_array(logits, dtype: str | None):
    """Accept a numpy array (float32, or uint16 bit patterns with ``dtype``)."""
    a = np.ascontiguousarray(logits)
    if dtype is None:
        if a.dtype != np.float32:
            raise TypeError("pass float32 logits, or uint16 bit patterns with dtype=")
        dtype = "float32"
    elif dtype != "float32" and a.dtype != np.uint16:
        raise TypeError("bfloat16/float16 logits are passed as uint16 bit patterns")
    return a, DTYPE_CODES[dtype]


def max_threads() -> int:
    return int(_load().orc_max_threads())


def mask_count(mask: np.ndarray, vocab: int) -> int:
    m = np.ascontiguousarray(mask, dtype=np.int32)
    if m.ndim != 1 or m.size != (vocab + 31) // 32:
        raise ValueError("mask must hold ceil(vocab / 32) words")
    return int(_load().orc_mask_count(_ptr(m), vocab))


def reduce_rows(logits, masks, *, dtype: str | None = None, threads: int = 0):
    """Masked argmax + valid count + status per row: (tokens, counts, status)."""
    a, code = _logit_array(logits, dtype)
    m = np.ascontiguousarray(masks, dtype=np.int32)
    rows, vocab = a.shape
    if m.shape != (rows, (vocab + 31) // 32):
        raise ValueError("mask shape must be [rows, ceil(vocab / 32)]")
    tokens = np.empty(rows, np.int64)
    counts = np.empty(rows, np.int64)
    status = np.empty(rows, np.int32)
    if rows:
        _load().orc_reduce_rows(_ptr(a), code, _ptr(m), rows, vocab, _ptr(tokens), _ptr(counts),
                                _ptr(status), threads)
    return tokens, counts, status


def sample_rows(logits, masks, temperature: float, uniforms, *, dtype: str | None = None,
                threads: int = 0):
    """Inverse-CDF masked softmax sample per row with explicit uniforms: (tokens, status)."""
    a, code = _logit_array(logits, dtype)
    m = np.ascontiguousarray(masks, dtype=np.int32)
    rows, vocab = a.shape
    u = np.ascontiguousarray(uniforms, dtype=np.float64).reshape(rows)
    tokens = np.empty(rows, np.int64)
    status = np.empty(rows, np.int32)
    if rows:
        _load().orc_sample_rows(_ptr(a), code, _ptr(m), rows, vocab, float(temperature), _ptr(u),
                                _ptr(tokens), _ptr(status), threads)
    return tokens, status


def fsum(values) -> float:
    v = np.ascontiguousarray(values, dtype=np.float64)
    return float(_load().orc_fsum(_ptr(v), v.size))


def budget(density: float, *, kind: int = 0, low: float = 0.005, high: float = 0.02,
           min_budget: int = 1, max_budget: int = 8) -> int:
    return int(_load().orc_budget(kind, low, high, min_budget, max_budget, density))


def budget_rows(counts, vocab: int, *, kind: int = 0, low: float = 0.005, high: float = 0.02,
                min_budget: int = 1, max_budget: int = 8):
    c = np.ascontiguousarray(counts, dtype=np.int64)
    density = np.empty(c.size, np.float64)
    k = np.empty(c.size, np.int32)
    _load().orc_budget_rows(kind, low, high, min_budget, max_budget, _ptr(c), c.size, vocab,
                            _ptr(density), _ptr(k))
    return density, k


def verify(row_tokens, row_status, proposals, lengths):
    """Longest-prefix acceptance per sequence.

    ``row_tokens``/``row_status`` are [S*(K+1)] per-row targets and statuses,
    ``proposals`` is [S, K] and ``lengths`` [S].  Returns (accept_len, token,
    kind, seq_status) with kind 0 correction, 1 bonus, 2 fallback.
    """
    p = np.ascontiguousarray(proposals, dtype=np.int64)
    seqs, k = p.shape
    t = np.ascontiguousarray(row_tokens, dtype=np.int64).reshape(seqs * (k + 1))
    s = np.ascontiguousarray(row_status, dtype=np.int32).reshape(seqs * (k + 1))
    ln = np.ascontiguousarray(lengths, dtype=np.int32).reshape(seqs)
    accept = np.empty(seqs, np.int32)
    token = np.empty(seqs, np.int64)
    kind = np.empty(seqs, np.int32)
    seq_status = np.empty(seqs, np.int32)
    _load().orc_verify(_ptr(t), _ptr(s), seqs, k + 1, _ptr(p), _ptr(ln), _ptr(accept),
                       _ptr(token), _ptr(kind), _ptr(seq_status))
    return accept, token, kind, seq_status


def widen(logits, dtype: str) -> np.ndarray:
    """Exact float32 widening of float32 / bfloat16 / float16 bit patterns."""
    a, code = _logit_array(logits, dtype)
    out = np.empty(a.shape, np.float32)
    _load().orc_widen(_ptr(a), code, a.size, _ptr(out))
    return out


def cdf_interval(row_f32: np.ndarray, mask_row: np.ndarray, temperature: float, token: int):
    """Normalised CDF interval [F(token-), F(token)] of the reference sampler's weights
    exp((x - max) / T) over the valid finite logits of one float32 row (fp64, exact sums)."""
    import math
    vocab = row_f32.size
    words = np.ascontiguousarray(mask_row, dtype=np.int32).view(np.uint32)
    t = np.arange(vocab)
    valid = ((words[t >> 5] >> (t & 31).astype(np.uint32)) & 1).astype(bool)
    x = row_f32.astype(np.float64)
    finite = valid & np.isfinite(x)
    m = x[valid].max()
    w = np.zeros(vocab)
    with np.errstate(over="ignore", invalid="ignore"):
        w[finite] = np.exp((x[finite] - m) / temperature)
    total = math.fsum(w[valid])
    cum = np.cumsum(w)
    hi = cum[token] / total
    lo = (cum[token] - w[token]) / total
    return lo, hi


def sample_matches(row_f32, mask_row, temperature, uniform, gpu_token, ref_token, tol=1e-6) -> bool:
    """The sampler's parity rule: the GPU's token equals the reference's for the same uniform, or
    u lies within ``tol`` (normalised CDF) of a boundary of the GPU's token's interval."""
    if gpu_token == ref_token:
        return True
    if gpu_token < 0:
        return False
    lo, hi = cdf_interval(row_f32, mask_row, temperature, gpu_token)
    if hi <= lo:  # a token of zero weight is never drawn
        return False
    dist = 0.0 if lo <= uniform < hi else min(abs(uniform - lo), abs(uniform - hi))
    return dist <= tol


def masked_softmax(row_f32, mask_row, temperature: float) -> np.ndarray:
    """fp64 probabilities exp((x - max) / T) / sum over the valid finite logits of one row (zero
    elsewhere)."""
    vocab = row_f32.size
    words = np.ascontiguousarray(mask_row, dtype=np.int32).view(np.uint32)
    t = np.arange(vocab)
    valid = ((words[t >> 5] >> (t & 31).astype(np.uint32)) & 1).astype(bool) & np.isfinite(row_f32)
    x = row_f32.astype(np.float64)
    w = np.zeros(vocab)
    w[valid] = np.exp((x[valid] - x[valid].max()) / temperature)
    return w / w.sum()


def speculative_accept(target_f32, draft_f32, masks, proposals, lengths, temperature, u_accept, u_resample):
    """The speculative-sampling rule, restated in fp64 as the checker of this library's stochastic
    acceptance (an extension: the reference has no stochastic acceptance, so parity is unpinned).
    Draft i is accepted iff u_i q_i(d_i) < p_i(d_i); at the first rejection j the token is drawn by
    inverse CDF from max(0, p_j - q_j) normalised, after L acceptances from p_L.  Rows are the
    target's [S*(K+1), V] and the draft's [S*K, V] float32 values; every row is assumed sampleable.
    Returns per sequence (accept_len, token, kind, the margin min |u q - p| / p over its tests, the
    sampled distribution)."""
    seqs, k = np.asarray(proposals).shape
    out = []
    for s in range(seqs):
        L = int(lengths[s])
        j, margin = L, np.inf
        for i in range(L):
            r = s * (k + 1) + i
            p = masked_softmax(target_f32[r], masks[r], temperature)
            q = masked_softmax(draft_f32[s * k + i], masks[r], temperature)
            d = int(proposals[s, i])
            if p[d] > 0:
                margin = min(margin, abs(u_accept[s, i] * q[d] - p[d]) / p[d])
            if not (q[d] > 0 and u_accept[s, i] * q[d] < p[d]):
                j = i
                break
        r = s * (k + 1) + j
        p = masked_softmax(target_f32[r], masks[r], temperature)
        dist = p
        if j < L:
            res = np.maximum(0.0, p - masked_softmax(draft_f32[s * k + j], masks[r], temperature))
            if res.sum() > 0:
                dist = res / res.sum()
        cum = np.cumsum(dist)
        cut = u_resample[s] * cum[-1]
        token = int(np.searchsorted(cum, cut, side="right"))
        token = min(token, int(np.flatnonzero(dist > 0)[-1]))
        out.append((j, token, 0 if j < L else (1 if L > 0 else 2), margin, dist))
    return out


def grammar_choices(draft, rows, grammar, *, dtype: str | None = None):
    """The reference's grammar-constrained verification loop (models/transformers.py:181-201:
    ``_choices`` + ``constrained_choices`` over decoding/verification.py:18-48 ``verify_prefix``),
    restated on the oracle: row i is selected by the masked argmax under the committed grammar's
    packed mask, which is then advanced; stop at the first mismatch, after the bonus, or once the
    grammar terminates.  ``rows`` are the K+1 target rows (float32 values, or bit patterns of
    ``dtype``).  Returns a list of (token, kind); a failed row raises ``ValueError`` when reached.
    """
    def select(i):
        tok, _, st = reduce_rows(rows[i:i + 1], np.asarray(grammar.packed_mask_np())[None, :], dtype=dtype,
                                 threads=1)
        if st[0] == 1:
            raise ValueError("mask has no valid token")
        if st[0] == 2:
            raise ValueError("next-token logits contain NaN")
        if not grammar.accept_token(int(tok[0])):
            raise ValueError("grammar rejected its selected token")
        return int(tok[0])

    def choices():
        for i, p in enumerate(draft):
            t = select(i)
            if t != p:
                yield (t, "correction")
                return
            yield (p, "accepted")
        yield (select(len(draft)), "bonus" if draft else "fallback")

    out = []
    gen = choices()
    while not grammar.is_terminated():
        ev = next(gen, None)
        if ev is None:
            break
        out.append(ev)
    return out
