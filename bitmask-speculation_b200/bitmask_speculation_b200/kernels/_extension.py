"""The native module: the reference's pybind surface on top of the C ABI.

``load_extension()`` returns an object with the five functions the reference's
JIT-built module exported (csrc/bindings.cpp:10-17) -- ``runtime_version``,
``mask_count``, ``masked_argmax``, ``masked_reduce_batch`` and ``masked_sample``
-- with the same arguments, return values, stream/device behaviour and error
type (``RuntimeError`` for contract violations, as TORCH_CHECK raised; device
status codes for data errors), plus the batched entry points that have no
reference counterpart.  Tensor metadata is checked here (csrc/checks.h:8-40);
the C library re-checks every pointer before it launches anything.

Differences from the reference module, by design: float16 and bfloat16 logits
are accepted without a widening copy, and batches are not limited to 65,535
rows.
"""

from __future__ import annotations

from functools import lru_cache

from .. import _native

_INT32_MAX = 2147483647


def _torch():
    import torch
    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    codes = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
    if t.dtype not in codes:
        raise RuntimeError("logits must be float32, bfloat16 or float16")
    return codes[t.dtype]


def _stream(device):
    return _torch().cuda.current_stream(device).cuda_stream


def _check_mask(mask, vocab: int) -> None:
    torch = _torch()
    if not (0 < vocab <= _INT32_MAX):
        raise RuntimeError("invalid vocabulary size")
    if not mask.is_cuda:
        raise RuntimeError("mask must be CUDA")
    if mask.layout != torch.strided or mask.dim() != 1 or not mask.is_contiguous():
        raise RuntimeError("mask must be a contiguous strided row")
    if mask.dtype != torch.int32:
        raise RuntimeError("mask must be int32")
    if mask.numel() != (vocab + 31) // 32:
        raise RuntimeError("incorrect mask word count")


def _check_selection(logits, mask) -> int:
    torch = _torch()
    if not logits.is_cuda:
        raise RuntimeError("logits must be CUDA")
    if logits.layout != torch.strided or logits.dim() != 1 or not logits.is_contiguous():
        raise RuntimeError("logits must be a contiguous strided row")
    _dtype_code(logits)
    _check_mask(mask, logits.numel())
    if logits.device != mask.device:
        raise RuntimeError("logits and mask devices differ")
    return logits.numel()


def _check_batch(logits, masks, table: bool = False):
    torch = _torch()
    if not (logits.is_cuda and masks.is_cuda):
        raise RuntimeError("batch inputs must be CUDA")
    if logits.device != masks.device:
        raise RuntimeError("logits and mask devices differ")
    if logits.layout != torch.strided or logits.dim() != 2 or not logits.is_contiguous():
        raise RuntimeError("logits must be a contiguous [B, V] tensor")
    if masks.layout != torch.strided or masks.dim() != 2 or not masks.is_contiguous():
        raise RuntimeError("masks must be a contiguous [B, ceil(V / 32)] tensor")
    _dtype_code(logits)
    if masks.dtype != torch.int32:
        raise RuntimeError("masks must be int32")
    rows, vocab = logits.shape
    if not (0 < vocab <= _INT32_MAX):
        raise RuntimeError("invalid vocabulary size")
    if (masks.shape[0] < 1 if table else masks.shape[0] != rows) or masks.shape[1] != (vocab + 31) // 32:
        raise RuntimeError("incorrect mask shape")
    return rows, vocab


def _check_uniform(uniform, device, rows=None):
    torch = _torch()
    if not uniform.is_cuda or uniform.device != device:
        raise RuntimeError("uniform device differs")
    if uniform.dtype != torch.float64 or uniform.layout != torch.strided or not uniform.is_contiguous():
        raise RuntimeError("uniform must be a float64 tensor")
    if rows is None and uniform.dim() != 0:
        raise RuntimeError("uniform must be a float64 scalar")
    if rows is not None and (uniform.dim() != 1 or uniform.numel() != rows):
        raise RuntimeError("uniforms must be a float64 [B] tensor")


def _temperature(value) -> float:
    import math
    t = float(value)
    if not math.isfinite(t) or t < 0:
        raise RuntimeError("invalid temperature")
    return t


class NativeModule:
    """Torch-tensor front end of ``libbms_b200.so`` with the reference's names."""

    def __init__(self):
        self._lib = _native.library()
        self._workspaces = {}
        #: pass a workspace to the batched kernels (dynamic schedule); False selects the fixed one
        self.use_workspace = True

    def workspace(self, device):
        """The zeroed workspace of (device, current stream), allocated on first use.

        A workspace serves one stream: calls on one stream never overlap, and each call leaves
        it ready for the next.  Returns (pointer, bytes), or (None, 0) when disabled.
        """
        if not self.use_workspace:
            return None, 0
        key = (device.index, _stream(device))
        ws = self._workspaces.get(key)
        if ws is None:
            nbytes = int(self._lib.bms_workspace_bytes(device.index))
            if nbytes <= 0:
                raise RuntimeError(f"no workspace size for device {device}")
            ws = _torch().zeros(nbytes, dtype=_torch().uint8, device=device)
            self._workspaces[key] = ws
        return ws.data_ptr(), ws.numel()

    # -- reference surface ---------------------------------------------------
    def runtime_version(self) -> int:
        import ctypes
        v = ctypes.c_int32(0)
        _native.check(self._lib.bms_runtime_version(ctypes.byref(v)))
        return int(v.value)

    def mask_count(self, mask, vocab: int):
        torch = _torch()
        vocab = int(vocab)
        _check_mask(mask, vocab)
        out = torch.empty((), dtype=torch.int64, device=mask.device)
        _native.check(self._lib.bms_mask_count(mask.data_ptr(), vocab, out.data_ptr(),
                                               mask.device.index, _stream(mask.device)))
        return out

    def masked_argmax(self, logits, mask):
        torch = _torch()
        vocab = _check_selection(logits, mask)
        dev = logits.device
        token = torch.empty((), dtype=torch.int64, device=dev)
        status = torch.empty((), dtype=torch.int32, device=dev)
        _native.check(self._lib.bms_masked_argmax(
            logits.data_ptr(), _dtype_code(logits), mask.data_ptr(), vocab, token.data_ptr(),
            status.data_ptr(), dev.index, _stream(dev)))
        return [token, status]

    def masked_reduce_batch(self, logits, masks):
        torch = _torch()
        rows, vocab = _check_batch(logits, masks)
        dev = logits.device
        tokens = torch.empty(rows, dtype=torch.int64, device=dev)
        counts = torch.empty(rows, dtype=torch.int64, device=dev)
        status = torch.empty(rows, dtype=torch.int32, device=dev)
        if rows:
            ws, nbytes = self.workspace(dev)
            _native.check(self._lib.bms_masked_reduce_batch(
                logits.data_ptr(), _dtype_code(logits), masks.data_ptr(), rows, vocab,
                tokens.data_ptr(), counts.data_ptr(), status.data_ptr(), ws, nbytes, dev.index, _stream(dev)))
        return [tokens, counts, status]

    def masked_sample(self, logits, mask, temperature, uniform):
        vocab = _check_selection(logits, mask)
        temperature = _temperature(temperature)
        if temperature == 0:  # csrc/sample.cu:120
            return self.masked_argmax(logits, mask)
        torch = _torch()
        dev = logits.device
        _check_uniform(uniform, dev)
        token = torch.empty((), dtype=torch.int64, device=dev)
        status = torch.empty((), dtype=torch.int32, device=dev)
        _native.check(self._lib.bms_masked_sample(
            logits.data_ptr(), _dtype_code(logits), mask.data_ptr(), vocab, temperature,
            uniform.data_ptr(), token.data_ptr(), status.data_ptr(), dev.index, _stream(dev)))
        return [token, status]

    # -- batched entry points (no reference counterpart) ------------------------
    def masked_sample_batch(self, logits, masks, temperature, uniforms):
        torch = _torch()
        rows, vocab = _check_batch(logits, masks)
        temperature = _temperature(temperature)
        dev = logits.device
        tokens = torch.empty(rows, dtype=torch.int64, device=dev)
        counts = torch.empty(rows, dtype=torch.int64, device=dev)
        status = torch.empty(rows, dtype=torch.int32, device=dev)
        if temperature != 0:
            _check_uniform(uniforms, dev, rows)
        if rows:
            ws, nbytes = self.workspace(dev)
            _native.check(self._lib.bms_masked_sample_batch(
                logits.data_ptr(), _dtype_code(logits), masks.data_ptr(), rows, vocab, temperature,
                uniforms.data_ptr() if temperature != 0 else None, tokens.data_ptr(),
                counts.data_ptr(), status.data_ptr(), ws, nbytes, dev.index, _stream(dev)))
        return [tokens, counts, status]

    def mask_budget(self, masks, vocab: int, policy):
        torch = _torch()
        vocab = int(vocab)
        if not masks.is_cuda or masks.dtype != torch.int32 or masks.dim() != 2 or not masks.is_contiguous():
            raise RuntimeError("masks must be a contiguous CUDA int32 [B, ceil(V / 32)] tensor")
        if not (0 < vocab <= _INT32_MAX) or masks.shape[1] != (vocab + 31) // 32:
            raise RuntimeError("incorrect mask shape")
        rows = masks.shape[0]
        dev = masks.device
        counts = torch.empty(rows, dtype=torch.int64, device=dev)
        density = torch.empty(rows, dtype=torch.float64, device=dev)
        budget = torch.empty(rows, dtype=torch.int32, device=dev)
        if rows:
            import ctypes
            _native.check(self._lib.bms_mask_budget(
                masks.data_ptr(), rows, vocab, ctypes.byref(policy), counts.data_ptr(),
                density.data_ptr(), budget.data_ptr(), dev.index, _stream(dev)))
        return [counts, density, budget]

    def verify_batch(self, logits, masks, proposals, lengths, policy, mask_rows=None):
        """Batched verification round; see ``bms_verify_batch``.  With ``mask_rows`` (int32 [rows]),
        ``masks`` is a table of mask rows on the device and row r uses row mask_rows[r]."""
        import ctypes
        torch = _torch()
        rows, vocab = _check_batch(logits, masks, table=mask_rows is not None)
        if mask_rows is not None and (mask_rows.dtype != torch.int32 or mask_rows.shape != (rows,)
                                      or not mask_rows.is_contiguous() or mask_rows.device != logits.device):
            raise RuntimeError("mask_rows must be a contiguous int32 [rows] tensor on the logits' device")
        if proposals.dtype != torch.int64 or proposals.dim() != 2 or not proposals.is_contiguous():
            raise RuntimeError("proposals must be a contiguous int64 [S, K] tensor")
        seqs, k = proposals.shape
        if rows != seqs * (k + 1):
            raise RuntimeError("logits must hold S * (K + 1) rows")
        if lengths.dtype != torch.int32 or lengths.shape != (seqs,) or not lengths.is_contiguous():
            raise RuntimeError("lengths must be a contiguous int32 [S] tensor")
        dev = logits.device
        for t in (proposals, lengths):
            if t.device != dev:
                raise RuntimeError("verification inputs must share one CUDA device")
        out = dict(
            row_tokens=torch.empty(rows, dtype=torch.int64, device=dev),
            row_counts=torch.empty(rows, dtype=torch.int64, device=dev),
            row_status=torch.empty(rows, dtype=torch.int32, device=dev),
            row_budget=torch.empty(rows, dtype=torch.int32, device=dev),
            accept_len=torch.empty(seqs, dtype=torch.int32, device=dev),
            token=torch.empty(seqs, dtype=torch.int64, device=dev),
            kind=torch.empty(seqs, dtype=torch.int32, device=dev),
            seq_status=torch.empty(seqs, dtype=torch.int32, device=dev),
        )
        if seqs:
            ws, nbytes = self.workspace(dev)
            _native.check(self._lib.bms_verify_batch(
                logits.data_ptr(), _dtype_code(logits), masks.data_ptr(), seqs, k + 1, vocab,
                proposals.data_ptr() if k else None, lengths.data_ptr(), ctypes.byref(policy),
                out["row_tokens"].data_ptr(), out["row_counts"].data_ptr(),
                out["row_status"].data_ptr(), out["row_budget"].data_ptr(),
                out["accept_len"].data_ptr(), out["token"].data_ptr(), out["kind"].data_ptr(),
                out["seq_status"].data_ptr(), None if mask_rows is None else mask_rows.data_ptr(),
                0 if mask_rows is None else masks.shape[0], ws, nbytes, dev.index, _stream(dev)))
        return out


    def select_indexed_into(self, logits, table, mask_rows, tokens, status, scratch):
        """Masked argmax of each row of ``logits`` [R, V] under table row ``mask_rows[r]`` of
        ``table`` (an index outside the table fails the row with status 8), written into
        ``tokens`` (int64 [R]) and ``status`` (int32 [R]); ``scratch`` is an int32 device tensor of
        at least 6 * R elements (zeroed lengths and per-sequence outputs).  One ``bms_verify_batch``
        launch pair of one-row sequences on the current stream, no workspace, no allocation and
        no host synchronization: the call a device-side decoding loop makes per step."""
        rows, vocab = logits.shape
        dev = logits.device
        if scratch.numel() < 6 * rows:
            raise RuntimeError("scratch must hold 6 int32 values per row")
        s = scratch.data_ptr()
        _native.check(self._lib.bms_verify_batch(
            logits.data_ptr(), _dtype_code(logits), table.data_ptr(), rows, 1, vocab, None, s, None,
            tokens.data_ptr(), None, status.data_ptr(), None, s + 4 * rows, s + 8 * rows, s + 16 * rows,
            s + 20 * rows, mask_rows.data_ptr(), table.shape[0], None, 0, dev.index, _stream(dev)))


@lru_cache(maxsize=1)
def load_extension() -> NativeModule:
    """Load the prebuilt sm_100a library; never substitute CPU code for a CUDA call."""
    torch = _torch()
    if torch.version.cuda is None or not torch.cuda.is_available():
        raise RuntimeError("a CUDA-enabled PyTorch build and visible NVIDIA GPU are required")
    return NativeModule()
