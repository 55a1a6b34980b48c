"""End-to-end constrained decoding harness (the end-to-end measurement configuration).

Random-init Qwen-style decoders in plain PyTorch stand in for the reference's Transformers models
(models/transformers.py), and the reference's request loops are restated over this library's
kernels:

* ``constrained_greedy`` -- decoding/greedy.py:51-92 ``greedy_decode`` with a grammar: one target
  forward and one masked argmax per token, the grammar advanced by each choice;
* ``speculative_c4`` -- decoding/speculative.py:96-208 ``speculative_decode`` with
  ``constrain_draft=True`` and a ``DensityPolicy`` (the reference's c4 mode): per round the density
  of the committed grammar sets K, the draft model proposes up to K tokens greedily on a grammar
  fork (decoding/speculative.py:63-95), one target forward scores prefix + draft, and the whole
  round is verified by ``grammar_verification.verify_with_grammar`` (one launch pair, one sync)
  instead of the reference's per-row loop.

Speculative decoding with greedy verification reproduces target-only greedy decoding token for
token; ``tests/test_gpu_decode.py`` checks that, and ``bench.py --workload decode`` measures it.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .grammar_verification import DeviceMaskTable, DraftForkMasks, verify_with_grammar, verify_with_grammars
from .scheduling import DensityPolicy


def _torch():
    import torch
    return torch


# ---------------------------------------------------------------- model
def build_decoder(vocab: int, *, layers: int, dim: int, heads: int, kv_heads: int | None = None,
                  ffn: int | None = None, dtype=None, device="cuda", seed: int = 0):
    """A random-init Qwen-style decoder: token embedding, ``layers`` blocks of RMSNorm ->
    grouped-query causal attention with rotary positions -> RMSNorm -> SwiGLU MLP, final RMSNorm and
    an untied LM head.  Weights are N(0, 0.02^2) from ``seed``."""
    torch = _torch()
    nn = torch.nn
    dtype = torch.bfloat16 if dtype is None else dtype
    kv_heads = kv_heads or max(1, heads // 4)
    ffn = ffn or 3 * dim
    head_dim = dim // heads

    class RMSNorm(nn.Module):
        def __init__(self):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(dim))

        def forward(self, x):
            v = x.float()
            v = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6)
            return (v * self.weight.float()).to(x.dtype)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.n1, self.n2 = RMSNorm(), RMSNorm()
            self.q = nn.Linear(dim, heads * head_dim, bias=False)
            self.kv = nn.Linear(dim, 2 * kv_heads * head_dim, bias=False)
            self.o = nn.Linear(heads * head_dim, dim, bias=False)
            self.up = nn.Linear(dim, 2 * ffn, bias=False)
            self.down = nn.Linear(ffn, dim, bias=False)

        def forward(self, x, cos, sin):
            t = x.shape[0]
            h = self.n1(x)
            q = self.q(h).view(t, heads, head_dim).transpose(0, 1)
            k, v = self.kv(h).view(t, 2, kv_heads, head_dim).unbind(1)
            k, v = k.transpose(0, 1), v.transpose(0, 1)
            q, k = _rotate(q, cos, sin), _rotate(k, cos, sin)
            k = k.repeat_interleave(heads // kv_heads, 0)
            v = v.repeat_interleave(heads // kv_heads, 0)
            a = torch.nn.functional.scaled_dot_product_attention(q[None], k[None], v[None], is_causal=True)[0]
            x = x + self.o(a.transpose(0, 1).reshape(t, heads * head_dim))
            g, u = self.up(self.n2(x)).chunk(2, -1)
            return x + self.down(torch.nn.functional.silu(g) * u)

    class Decoder(nn.Module):
        def __init__(self):
            super().__init__()
            self.vocab_size = vocab
            self.embed = nn.Embedding(vocab, dim)
            self.blocks = nn.ModuleList(Block() for _ in range(layers))
            self.norm = RMSNorm()
            self.head = nn.Linear(dim, vocab, bias=False)
            inv = 1.0 / (1e6 ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
            self.register_buffer("inv_freq", inv.float(), persistent=False)
            self._graphs = None  # padded length -> (CUDA graph, token buffer, trunk output, rotary tables)
            self._pool = None

        def _rope(self, length: int):
            pos = torch.arange(length, device=self.inv_freq.device, dtype=torch.float32)
            ang = pos[:, None] * self.inv_freq[None, :]
            return ang.cos().to(self.head.weight.dtype), ang.sin().to(self.head.weight.dtype)

        def _trunk(self, ids, cos, sin):
            x = self.embed(ids)
            for b in self.blocks:
                x = b(x, cos, sin)
            return x

        def enable_graphs(self):
            """Replay the embedding and the blocks from one CUDA graph per padded length (captured
            on first use), so that a forward costs a handful of launches: the token copy, the graph
            and the final norm and LM head of the requested rows.  The graph holds the same
            kernels as the eager forward."""
            if self._graphs is None:
                self._graphs = {}
                self._pool = torch.cuda.graph_pool_handle()
            return self

        def _captured(self, length: int):
            entry = self._graphs.get(length)
            if entry is None:
                ids = torch.zeros(length, dtype=torch.long, device=self.head.weight.device)
                cos, sin = self._rope(length)
                side = torch.cuda.Stream(device=ids.device)
                side.wait_stream(torch.cuda.current_stream(ids.device))
                with torch.cuda.stream(side):
                    for _ in range(2):  # library handles and workspaces exist before capture
                        self._trunk(ids, cos, sin)
                torch.cuda.current_stream(ids.device).wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, pool=self._pool):
                    out = self._trunk(ids, cos, sin)
                entry = self._graphs[length] = (graph, ids, out, cos, sin)
            return entry

        @torch.inference_mode()
        def logits(self, tokens, first: int, rows: int):
            """Logits of positions [first, first + rows) after one forward over ``tokens``.  The
            sequence is padded at the end to a multiple of 64 tokens (causal attention: padding
            never reaches earlier positions) so that kernel shapes repeat across calls."""
            n = len(tokens)
            padded = list(tokens) + [0] * (-n % 64)
            host = torch.tensor(padded, dtype=torch.long)
            if self._graphs is not None:
                graph, ids, out, _, _ = self._captured(len(padded))
                ids.copy_(host, non_blocking=True)
                graph.replay()
                x = out
            else:
                ids = host.to(self.head.weight.device, non_blocking=True)
                x = self._trunk(ids, *self._rope(ids.shape[0]))
            return self.head(self.norm(x[first:first + rows])).contiguous()

    gen = torch.Generator().manual_seed(seed)
    model = Decoder()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "weight" in name and p.dim() == 2:
                p.copy_(torch.randn(p.shape, generator=gen) * 0.02)
    return model.to(device=device, dtype=dtype).eval()


def _rotate(x, cos, sin):
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    return _torch().cat((a * cos - b * sin, a * sin + b * cos), -1)


# ---------------------------------------------------------------- selection
class _Selector:
    """Masked argmax of one row under a grammar's current mask (the reference's _select_token,
    models/transformers.py:131-145: ``dispatch.select_token`` without advancing, then advance; NaN or
    an empty mask raise).  With ``table`` the state masks are read on the device.  ``seconds``
    accumulates the host time spent selecting (a synchronizing call, so it covers the device work)."""

    seconds = 0.0

    def __init__(self, vocab: int, device, table: DeviceMaskTable | None = None):
        self.table = table

    def __call__(self, row, grammar) -> int:
        import time
        from .dispatch import select_token
        t0 = time.perf_counter()
        token = select_token(row, grammar, "cuda", table=self.table)
        self.seconds += time.perf_counter() - t0
        if not grammar.accept_token(token):
            raise ValueError("grammar rejected its selected token")
        return token


class _DraftStep:
    """One greedy constrained draft step on the device, over static buffers so that it can be
    replayed from a CUDA graph: the draft forward over ``ids`` (the round's padded length), norm and
    LM head of row ``ctl[0]`` (the context's last position), the masked argmax of that row under
    table row ``ctl[2] ? empty : ctl[1]`` (the state; ``select_indexed_into``), the token recorded
    in ``rec[:, ctl[3]]`` (token, status, terminated before it) and written at ``ids[ctl[0] + 1]``,
    and the grammar's transition (``device_advance``).  ``ctl`` = [position, state, terminated,
    step] int64."""

    def __init__(self, model, padded: int, table: DeviceMaskTable, grammar, max_steps: int):
        torch = _torch()
        from .kernels._extension import load_extension
        self.native = load_extension()
        dev = model.head.weight.device
        self.model, self.table, self.grammar = model, table, grammar
        self.ids = torch.zeros(padded, dtype=torch.long, device=dev)
        self.cos, self.sin = model._rope(padded)
        self.ctl = torch.zeros(4, dtype=torch.long, device=dev)
        self.empty = torch.full((1,), table.empty, dtype=torch.long, device=dev)
        self.idx = torch.empty(1, dtype=torch.int32, device=dev)
        self.token = torch.empty(1, dtype=torch.long, device=dev)
        self.status = torch.empty(1, dtype=torch.int32, device=dev)
        self.scratch = torch.zeros(6, dtype=torch.int32, device=dev)
        self.rec = torch.zeros((3, max_steps), dtype=torch.long, device=dev)
        self.graph = None

    def run(self):
        torch = _torch()
        m, ctl = self.model, self.ctl
        pos, state, term, step = ctl[0:1], ctl[1:2], ctl[2:3], ctl[3:4]
        x = m._trunk(self.ids, self.cos, self.sin)
        row = m.head(m.norm(x.index_select(0, pos)))
        self.idx.copy_(torch.where(term != 0, self.empty, state))
        self.native.select_indexed_into(row, self.table.table, self.idx, self.token, self.status, self.scratch)
        self.rec[0].index_copy_(0, step, self.token)
        self.rec[1].index_copy_(0, step, self.status.long())
        self.rec[2].index_copy_(0, step, term)
        # A failed row (status != 0, token -1) is discarded by the host; the steps after it still
        # need a valid token ID to embed.
        token = self.token.clamp(min=0)
        self.ids.index_copy_(0, pos + 1, token)
        nxt, is_eos = self.grammar.device_advance(state, token)
        ctl.copy_(torch.cat((pos + 1, nxt, term | is_eos.long(), step + 1)))

    def capture(self, pool):
        """Replay the step from a CUDA graph (after two eager runs on a side stream set up every
        library handle and launch configuration)."""
        torch = _torch()
        dev = self.ids.device
        side = torch.cuda.Stream(device=dev)
        # The warm-up runs start from position 0, state 0, step 0 (a step object reused from eager
        # rounds holds its last round's position and step, which the runs would carry past the
        # buffers); every round uploads its own ids and control values.
        self.ids.zero_()
        self.ctl.zero_()
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                self.run()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        # relaxed: the selection's C entry point queries pointer attributes while it is captured
        with torch.cuda.graph(graph, pool=pool, capture_error_mode="relaxed"):
            self.run()
        self.ids.zero_()
        self.ctl.zero_()
        self.graph = graph
        return self

    def step(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.run()


def _device_draft(model, prefix, steps: int, grammar, table: DeviceMaskTable, eos) -> tuple[list[int], float]:
    """Greedy constrained drafting of up to ``steps`` tokens after ``prefix`` with the grammar's
    states on the device (the draft loop of decoding/speculative.py:63-95, for grammars with a
    finite state set and ``device_advance``).  Every step (``_DraftStep``: one CUDA-graph replay
    when the model replays graphs) runs the draft forward over the round's padded length (the last
    step's context rounded up to 64 tokens), the masked argmax of the context's last row under its
    state's table row and the grammar's transition, all on the device; the host reads the round
    back once and keeps the tokens up to where the per-step loop stops: a terminated fork, or before
    a draft EOS.  A failed selection raises ``ValueError`` as the per-step loop does.  Returns the
    proposals and the host time from the first step's launch to the read-back."""
    torch = _torch()
    from .dispatch import _STATUS_MESSAGES
    import time
    if steps <= 0:
        return [], 0.0
    n = len(prefix)
    padded = n + steps + (-(n + steps) % 64)
    key = (padded, id(table), id(getattr(grammar, "_tables", grammar)))
    cache = model.__dict__.setdefault("_draft_steps", {})
    ds = cache.get(key)
    if ds is None or ds.rec.shape[1] < steps:
        ds = cache[key] = _DraftStep(model, padded, table, grammar, max(steps, 16))
    if model._graphs is not None and ds.graph is None:
        ds.capture(model._pool)
    host = torch.zeros(padded + 4, dtype=torch.long)
    host[:n] = torch.tensor(prefix, dtype=torch.long)
    host[padded:] = torch.tensor([n - 1, grammar.state_index(), 0, 0], dtype=torch.long)
    host = host.pin_memory()
    ds.ids.copy_(host[:padded], non_blocking=True)
    ds.ctl.copy_(host[padded:], non_blocking=True)
    t0 = time.perf_counter()
    for _ in range(steps):
        ds.step()
    got = ds.rec[:, :steps].cpu().tolist()
    seconds = time.perf_counter() - t0
    proposals: list[int] = []
    for token, code, was_terminated in zip(*got):
        if was_terminated:
            break
        if code:
            raise ValueError(_STATUS_MESSAGES.get(code, f"native selection status {code}"))
        if token in eos:
            break
        proposals.append(int(token))
    return proposals, seconds


@dataclass(frozen=True, slots=True)
class DecodeResult:
    token_ids: tuple
    stop_reason: str
    eos_token_id: int | None = None
    rounds: int = 0
    proposed: int = 0
    accepted: int = 0
    select_seconds: float = field(default=0.0, compare=False)  # host time in selection and verification calls
    draft_seconds: float = field(default=0.0, compare=False)  # host time in device-drafted rounds (launch to read-back)


# ---------------------------------------------------------------- request loops
def constrained_greedy(target, prompt, grammar, *, max_new_tokens: int, eos=(), selector=None,
                       table: DeviceMaskTable | None = None) -> DecodeResult:
    """Target-only constrained greedy decoding (decoding/greedy.py:51-92)."""
    prompt = tuple(int(t) for t in prompt)
    eos = frozenset(int(t) for t in eos)
    sel = selector or _Selector(target.vocab_size, target.head.weight.device, table)
    out: list[int] = []

    def finish(reason, token=None):
        return DecodeResult(tuple(out), reason, token, select_seconds=sel.seconds)

    for _ in range(max_new_tokens):
        if grammar.is_terminated():
            return finish("grammar")
        seq = prompt + tuple(out)
        token = sel(target.logits(seq, len(seq) - 1, 1)[0], grammar)
        if token in eos:
            return finish("eos", token)
        out.append(token)
        if grammar.is_terminated():
            return finish("grammar")
    return finish("length")


def _lazy_rounds(draft, rows, grammar, sel):
    """The reference's per-row verification (models/transformers.py:181-201 ``_choices`` over
    decoding/verification.py:18-48): row i selected under the committed grammar when the event
    is requested, stopping at the first mismatch or at termination."""
    from .verification import VerifiedToken

    def choices():
        for i, p in enumerate(draft):
            t = sel(rows[i], grammar)
            if t != p:
                yield VerifiedToken(t, "correction")
                return
            yield VerifiedToken(p, "accepted")
        yield VerifiedToken(sel(rows[len(draft)], grammar), "bonus" if draft else "fallback")

    gen = choices()
    while not grammar.is_terminated():
        event = next(gen, None)
        if event is None:
            return
        yield event


def speculative_c4(target, draft, prompt, grammar, *, max_new_tokens: int, eos=(), policy=None,
                   selector=None, buffer=None, verify: str = "batched",
                   table: DeviceMaskTable | None = None) -> DecodeResult:
    """Density-scheduled constrained speculative decoding (decoding/speculative.py:96-208 with
    constrain_draft=True and a DensityPolicy).  ``verify="batched"`` verifies each round with
    ``verify_with_grammar`` (one launch pair, one sync); ``"lazy"`` with the reference's per-row
    loop (one masked argmax and one sync per consumed row) on the same target rows.  With ``table``
    (the grammar's state masks resident on the device) selections read their masks from it and
    batched rounds upload table indices instead of mask words; a grammar that also advances on the
    device (``device_advance``) drafts each round on the device with one read-back
    (``_device_draft``) instead of one synchronizing selection per draft token."""
    prompt = tuple(int(t) for t in prompt)
    eos = frozenset(int(t) for t in eos)
    policy = DensityPolicy() if policy is None else policy
    device = target.head.weight.device
    sel = selector or _Selector(target.vocab_size, device, table)
    device_draft = table is not None and selector is None and hasattr(grammar, "device_advance")
    buf = buffer or (None if table is not None else DraftForkMasks(target.vocab_size, policy.max_budget + 1, device))
    out: list[int] = []
    rounds = proposed = accepted = 0

    verify_seconds = draft_seconds = 0.0

    def finish(reason, token=None):
        return DecodeResult(tuple(out), reason, token, rounds, proposed, accepted, sel.seconds + verify_seconds,
                            draft_seconds)

    while len(out) < max_new_tokens:
        if grammar.is_terminated():
            return finish("grammar")
        prefix = prompt + tuple(out)
        budget = min(policy.budget(grammar.mask_density()), max_new_tokens - len(out))
        # Draft on a fork (decoding/speculative.py:63-95): stop before a draft EOS or at the fork's
        # termination; the fork is discarded before verification.
        if device_draft:
            proposals, secs = _device_draft(draft, prefix, budget, grammar, table, eos)
            draft_seconds += secs
        else:
            branch = grammar.fork()
            proposals = []
            for _ in range(budget):
                if branch.is_terminated():
                    break
                ctx = prefix + tuple(proposals)
                token = sel(draft.logits(ctx, len(ctx) - 1, 1)[0], branch)
                if token in eos:
                    break
                proposals.append(token)
        proposed += len(proposals)
        rounds += 1
        seq = prefix + tuple(proposals)
        rows = target.logits(seq, len(prefix) - 1, len(proposals) + 1)
        before = len(out)
        if verify == "batched":
            import time
            t0 = time.perf_counter()
            if table is not None:
                events = verify_with_grammars([proposals], rows, [grammar], k=len(proposals), table=table,
                                              policy=policy)[0]
            else:
                events = verify_with_grammar(proposals, rows, grammar, buffer=buf, policy=policy)
            verify_seconds += time.perf_counter() - t0
        else:
            events = _lazy_rounds(tuple(proposals), rows, grammar, sel)
        for event in events:
            accepted += event.kind == "accepted"
            if event.token_id in eos:
                return finish("eos", event.token_id)
            out.append(event.token_id)
            if grammar.is_terminated():
                return finish("grammar")
            if len(out) == max_new_tokens:
                return finish("length")
        if len(out) == before:
            raise RuntimeError("target verification made no progress")
    return finish("length")


def random_prompts(n: int, length: int, vocab: int, seed: int = 0) -> list[tuple[int, ...]]:
    rng = np.random.default_rng(seed)
    return [tuple(int(t) for t in rng.integers(1, vocab, size=length)) for _ in range(n)]


def config_models(vocab: int, device="cuda", dtype=None, seed: int = 0):
    """The end-to-end configuration's target (4 layers, d=1024, 16 heads) and draft (1 layer,
    d=512), random-init, bf16 by default."""
    target = build_decoder(vocab, layers=4, dim=1024, heads=16, dtype=dtype, device=device, seed=seed)
    draft = build_decoder(vocab, layers=1, dim=512, heads=8, dtype=dtype, device=device, seed=seed + 1)
    return target, draft


__all__ = ["build_decoder", "config_models", "constrained_greedy", "speculative_c4", "random_prompts",
           "DecodeResult"]
