"""Stochastic speculative acceptance (``stochastic.speculative_accept``; an extension: the reference
decodes greedily, docs/design.md:5-11, so there is no reference output to pin it to).  The proof is
distributional: with drafts drawn from the draft model's masked softmax q, the first emitted token
must follow the target's masked softmax p (chi-square), and the acceptance rate must be
sum_x min(p(x), q(x)).  At full vocabulary the GPU must also agree with the rule restated in fp64
(``oracle.speculative_accept``) except where a uniform sits within rounding of a decision: 1e-5
relative for the acceptance tests, and 1e-5 of a CDF boundary for the drawn token (fp32 weights, and
the replacement distribution p - q cancels leading digits where p and q are close)."""

import numpy as np
import pytest

import oracle
from bitmask_speculation_b200 import workloads as wl

torch = pytest.importorskip("torch")
scipy_stats = pytest.importorskip("scipy.stats")
pytestmark = pytest.mark.gpu


def _bf16(values):
    return torch.from_numpy(wl.to_bf16_bits(values).view(np.int16)).view(torch.bfloat16)


def _widen(t):
    return (t.cpu().view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_first_token_follows_the_target_distribution():
    from bitmask_speculation_b200.stochastic import speculative_accept
    rng = np.random.default_rng(4)
    vocab, n, temp = 1024, 200_000, 0.9
    valid = rng.random(vocab) < 0.3
    mask = wl.pack_bits_np(valid[None, :])
    tvals = _bf16(rng.standard_normal((2, vocab), dtype=np.float32) * np.float32(1.2))
    dvals = _bf16(rng.standard_normal((1, vocab), dtype=np.float32) * np.float32(1.2))
    p = oracle.masked_softmax(_widen(tvals[0]), mask[0], temp)
    q = oracle.masked_softmax(_widen(dvals[0]), mask[0], temp)
    drafts = rng.choice(vocab, size=n, p=q)  # the draft model's samples
    dev = torch.device("cuda")
    target = tvals.to(dev).repeat(n, 1)                     # [2n, V]: position 0 and the bonus row
    draft = dvals.to(dev).repeat(n, 1)                      # [n, V]
    masks = torch.from_numpy(mask).to(dev).repeat(2 * n, 1)
    out = speculative_accept(target, draft, masks, torch.from_numpy(drafts[:, None]).to(dev),
                             torch.ones(n, dtype=torch.int32, device=dev), temperature=temp,
                             generator=torch.Generator(device=dev).manual_seed(1))
    acc, tok, st = out.accept_len.cpu().numpy(), out.token.cpu().numpy(), out.status.cpu().numpy()
    assert (st == 0).all()
    first = np.where(acc >= 1, drafts, tok)
    # acceptance rate: sum_x min(p, q)
    rate = np.minimum(p, q).sum()
    assert abs(acc.mean() - rate) < 4 * np.sqrt(rate * (1 - rate) / n)
    # chi-square of the first emitted token against p (bins with expected count >= 5)
    counts = np.bincount(first, minlength=vocab)
    expected = p * n
    big = expected >= 5
    obs = np.append(counts[big], counts[~big].sum())
    exp = np.append(expected[big], expected[~big].sum())
    keep = exp > 0
    assert counts[~valid].sum() == 0
    assert scipy_stats.chisquare(obs[keep], exp[keep] * obs.sum() / exp[keep].sum()).pvalue > 1e-4


def test_fallback_token_without_drafts_follows_the_target_distribution():
    from bitmask_speculation_b200.stochastic import speculative_accept
    rng = np.random.default_rng(8)
    vocab, n, temp = 512, 100_000, 0.7
    valid = rng.random(vocab) < 0.5
    mask = torch.from_numpy(wl.pack_bits_np(valid[None, :])).cuda()
    row = _bf16(rng.standard_normal((1, vocab), dtype=np.float32))
    p = oracle.masked_softmax(_widen(row[0]), mask.cpu().numpy()[0], temp)
    out = speculative_accept(row.cuda().repeat(n, 1), torch.empty((0, vocab), dtype=torch.bfloat16, device="cuda"),
                             mask.repeat(n, 1), torch.zeros((n, 0), dtype=torch.int64, device="cuda"),
                             torch.zeros(n, dtype=torch.int32, device="cuda"), temperature=temp)
    tok = out.token.cpu().numpy()
    assert (out.kind.cpu().numpy() == 2).all() and (out.accept_len.cpu().numpy() == 0).all()
    counts = np.bincount(tok, minlength=vocab)
    big = p * n >= 5
    obs = np.append(counts[big], counts[~big].sum())
    exp = np.append(p[big] * n, p[~big].sum() * n)
    assert scipy_stats.chisquare(obs, exp * obs.sum() / exp.sum()).pvalue > 1e-4


def test_full_vocabulary_rounds_agree_with_the_restated_rule():
    from bitmask_speculation_b200.stochastic import speculative_accept
    rng = np.random.default_rng(12)
    seqs, k, vocab, temp = 48, 8, wl.VOCAB, 0.8
    rows = seqs * (k + 1)
    valid = wl.verify_masks_np(rng, rows, vocab)
    masks = wl.pack_bits_np(valid)
    tvals = _bf16(rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(2))
    dvals_np = _widen(tvals).reshape(seqs, k + 1, vocab)[:, :k].reshape(seqs * k, vocab).copy()
    dvals_np += rng.standard_normal(dvals_np.shape, dtype=np.float32) * np.float32(0.7)  # a similar draft model
    dvals = _bf16(dvals_np)
    tf, df = _widen(tvals), _widen(dvals)
    proposals = np.zeros((seqs, k), dtype=np.int64)
    lengths = rng.integers(0, k + 1, size=seqs).astype(np.int32)
    for s in range(seqs):
        for i in range(lengths[s]):
            r = s * (k + 1) + i
            proposals[s, i] = rng.choice(vocab, p=oracle.masked_softmax(df[s * k + i], masks[r], temp))
    ua = rng.random((seqs, k))
    ur = rng.random(seqs)
    out = speculative_accept(tvals.cuda(), dvals.cuda(), torch.from_numpy(masks).cuda(), torch.from_numpy(proposals).cuda(),
                             torch.from_numpy(lengths).cuda(), temperature=temp,
                             accept_uniforms=torch.from_numpy(ua).cuda(), resample_uniforms=torch.from_numpy(ur).cuda())
    acc, tok, kind, st = (t.cpu().numpy() for t in (out.accept_len, out.token, out.kind, out.status))
    assert (st == 0).all()
    want = oracle.speculative_accept(tf, df, masks, proposals, lengths, temp, ua, ur)
    checked = 0
    for s, (j, t, kd, margin, dist) in enumerate(want):
        if margin < 1e-5:
            continue  # a uniform within rounding of an acceptance threshold
        assert acc[s] == j and kind[s] == kd, s
        if tok[s] != t:
            cum = np.cumsum(dist)
            lo, hi = cum[tok[s]] - dist[tok[s]], cum[tok[s]]
            assert dist[tok[s]] > 0 and min(abs(ur[s] - lo), abs(ur[s] - hi)) <= 1e-5, (s, tok[s], t)
        checked += 1
    assert checked >= seqs - 2 and (acc > 0).any() and (acc < lengths).any()


@pytest.mark.parametrize("lazy", [False, True])
def test_failed_and_invalid_rows_report_statuses(lazy):
    from bitmask_speculation_b200.stochastic import speculative_accept
    vocab, k = 256, 2
    tvals = torch.zeros((3 * (k + 1), vocab), device="cuda")
    dvals = torch.zeros((3 * k, vocab), device="cuda")
    masks = torch.full((3 * (k + 1), vocab // 32), -1, dtype=torch.int32, device="cuda")
    tvals[0, 5] = float("nan")          # sequence 0: its first target row is consumed -> NaN
    masks[3 * 1 + 0].zero_()            # sequence 1: the first row has no valid token
    lengths = torch.tensor([2, 1, 3], dtype=torch.int32, device="cuda")  # sequence 2: L > K
    out = speculative_accept(tvals, dvals, masks, torch.zeros((3, k), dtype=torch.int64, device="cuda"), lengths,
                             temperature=1.0, lazy=lazy)
    assert out.status.cpu().tolist() == [2, 1, 6]
    with pytest.raises(ValueError, match="NaN"):
        out.events(0, [0, 0])


@pytest.mark.parametrize("lazy", [True, False])
@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_results_do_not_depend_on_how_many_ctas_share_a_sequence(dtype, lazy):
    """The kernel splits each sequence's row over 8, 4, 2 or 1 CTAs (one cluster) by the batch size:
    8 sequences take 8 CTAs each, 40 take 4, 100 take 2 and 300 take one (a grid-stride loop).  The
    first 8 sequences, embedded in each batch, must give the same results every time, and those of
    the restated rule."""
    from bitmask_speculation_b200.kernels._extension import load_extension
    from bitmask_speculation_b200.stochastic import speculative_accept
    dev = torch.device("cuda")
    temp, k, vocab, seqs = 0.8, wl.DRAFT_K, wl.VOCAB, 300
    logits, masks, _, _ = wl.verify_batch_torch(seqs, seed=21, device=dev)
    words = masks.shape[1]
    g = torch.Generator(device=dev).manual_seed(5)
    first_k = logits.view(seqs, k + 1, vocab)[:, :k].reshape(seqs * k, vocab)
    draft = (first_k.float() + 0.7 * torch.randn(first_k.shape, generator=g, device=dev)).to(torch.bfloat16)
    dmasks = masks.view(seqs, k + 1, words)[:, :k].reshape(seqs * k, words).contiguous()
    u = torch.rand(seqs * k, dtype=torch.float64, generator=g, device=dev)
    proposals = load_extension().masked_sample_batch(draft, dmasks, temp, u)[0].view(seqs, k).contiguous()
    lengths = torch.randint(0, k + 1, (seqs,), generator=g, device=dev).to(torch.int32)
    ua = torch.rand((seqs, k), dtype=torch.float64, generator=g, device=dev)
    ur = torch.rand(seqs, dtype=torch.float64, generator=g, device=dev)
    if dtype == "float32":
        logits, draft = logits.float(), draft.float()
    results = []
    for n in (8, 40, 100, 300):
        out = speculative_accept(logits[: n * (k + 1)], draft[: n * k], masks[: n * (k + 1)], proposals[:n],
                                 lengths[:n], temperature=temp, accept_uniforms=ua[:n], resample_uniforms=ur[:n],
                                 lazy=lazy)
        assert (out.status == 0).all()
        results.append([t[:8].cpu() for t in (out.accept_len, out.token, out.kind)])
    for other in results[1:]:
        for a, b in zip(results[0], other):
            assert torch.equal(a, b)
    n_chk = 6
    tf = _widen(logits[: n_chk * (k + 1)].to(torch.bfloat16))
    df = _widen(draft[: n_chk * k].to(torch.bfloat16))
    want = oracle.speculative_accept(tf, df, masks[: n_chk * (k + 1)].cpu().numpy(), proposals[:n_chk].cpu().numpy(),
                                     lengths[:n_chk].cpu().numpy(), temp, ua[:n_chk].cpu().numpy(),
                                     ur[:n_chk].cpu().numpy())
    acc, tok, kind = (t.numpy() for t in results[0])
    for s, (j, t, kd, margin, dist) in enumerate(want):
        if margin < 1e-5:
            continue
        assert acc[s] == j and kind[s] == kd, s
        if tok[s] != t:
            cum = np.cumsum(dist)
            lo, hi = cum[tok[s]] - dist[tok[s]], cum[tok[s]]
            assert min(abs(ur[s].item() - lo), abs(ur[s].item() - hi)) <= 1e-5, (s, tok[s], t)


@pytest.mark.parametrize("vocab,lazy", [(1001, False), (4104, False), (4096, False), (3968, False), (4096, True),
                                        (3968, True)])
def test_rows_that_cannot_be_bulk_copied_agree_with_the_restated_rule(vocab, lazy):
    """Rows stream through shared memory by 16-byte bulk copies only when a row is a multiple of 16
    bytes and a mask row a multiple of 4 words; V = 1001 (2002-byte rows) and V = 4104 (129 mask
    words) take the register path instead, V = 4096 and V = 3968 (a last 256-token tile of 128
    tokens) stream, in both modes.  All must follow the rule."""
    from bitmask_speculation_b200.stochastic import speculative_accept
    rng = np.random.default_rng(vocab)
    seqs, k, temp = 24, 4, 0.9
    rows = seqs * (k + 1)
    valid = rng.random((rows, vocab)) < 0.6
    masks = wl.pack_bits_np(valid)
    tvals = _bf16(rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(1.5))
    dvals_np = _widen(tvals).reshape(seqs, k + 1, vocab)[:, :k].reshape(seqs * k, vocab).copy()
    dvals_np += rng.standard_normal(dvals_np.shape, dtype=np.float32) * np.float32(0.5)
    dvals = _bf16(dvals_np)
    tf, df = _widen(tvals), _widen(dvals)
    proposals = np.zeros((seqs, k), dtype=np.int64)
    lengths = rng.integers(0, k + 1, size=seqs).astype(np.int32)
    for s in range(seqs):
        for i in range(lengths[s]):
            proposals[s, i] = rng.choice(vocab, p=oracle.masked_softmax(df[s * k + i], masks[s * (k + 1) + i], temp))
    ua, ur = rng.random((seqs, k)), rng.random(seqs)
    out = speculative_accept(tvals.cuda(), dvals.cuda(), torch.from_numpy(masks).cuda(), torch.from_numpy(proposals).cuda(),
                             torch.from_numpy(lengths).cuda(), temperature=temp,
                             accept_uniforms=torch.from_numpy(ua).cuda(), resample_uniforms=torch.from_numpy(ur).cuda(),
                             lazy=lazy)
    acc, tok, kind, st = (t.cpu().numpy() for t in (out.accept_len, out.token, out.kind, out.status))
    assert (st == 0).all()
    want = oracle.speculative_accept(tf, df, masks, proposals, lengths, temp, ua, ur)
    checked = 0
    for s, (j, t, kd, margin, dist) in enumerate(want):
        if margin < 1e-5:
            continue
        assert acc[s] == j and kind[s] == kd, s
        if tok[s] != t:
            cum = np.cumsum(dist)
            lo, hi = cum[tok[s]] - dist[tok[s]], cum[tok[s]]
            assert dist[tok[s]] > 0 and min(abs(ur[s] - lo), abs(ur[s] - hi)) <= 1e-5, (s, tok[s], t)
        checked += 1
    assert checked >= seqs - 2


@pytest.mark.parametrize("vocab", [4096, 4104])
def test_long_draft_windows_in_half_precision_agree_with_the_restated_rule(vocab):
    """K = 40 drafts take two 32-lane ballot passes of the acceptance tests; fp16 logits; V = 4096
    streams through shared memory, V = 4104 (129 mask words) takes the register path.  A close
    draft model keeps many sequences accepting past position 32."""
    from bitmask_speculation_b200.stochastic import speculative_accept
    rng = np.random.default_rng(vocab + 40)
    seqs, k, temp = 12, 40, 1.0
    rows = seqs * (k + 1)
    valid = rng.random((rows, vocab)) < 0.7
    masks = wl.pack_bits_np(valid)
    tvals = (rng.standard_normal((rows, vocab), dtype=np.float32) * np.float32(0.3)).astype(np.float16)
    dvals = (tvals.astype(np.float32).reshape(seqs, k + 1, vocab)[:, :k].reshape(seqs * k, vocab)
             + rng.standard_normal((seqs * k, vocab), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    tf, df = tvals.astype(np.float32), dvals.astype(np.float32)
    proposals = np.zeros((seqs, k), dtype=np.int64)
    lengths = rng.integers(30, k + 1, size=seqs).astype(np.int32)
    for s in range(seqs):
        for i in range(lengths[s]):
            proposals[s, i] = rng.choice(vocab, p=oracle.masked_softmax(df[s * k + i], masks[s * (k + 1) + i], temp))
    ua, ur = rng.random((seqs, k)), rng.random(seqs)
    out = speculative_accept(torch.from_numpy(tvals).cuda(), torch.from_numpy(dvals).cuda(),
                             torch.from_numpy(masks).cuda(), torch.from_numpy(proposals).cuda(),
                             torch.from_numpy(lengths).cuda(), temperature=temp,
                             accept_uniforms=torch.from_numpy(ua).cuda(), resample_uniforms=torch.from_numpy(ur).cuda())
    acc, tok, kind, st = (t.cpu().numpy() for t in (out.accept_len, out.token, out.kind, out.status))
    assert (st == 0).all()
    want = oracle.speculative_accept(tf, df, masks, proposals, lengths, temp, ua, ur)
    checked = 0
    for s, (j, t, kd, margin, dist) in enumerate(want):
        if margin < 1e-5:
            continue
        assert acc[s] == j and kind[s] == kd, s
        if tok[s] != t:
            cum = np.cumsum(dist)
            lo, hi = cum[tok[s]] - dist[tok[s]], cum[tok[s]]
            assert dist[tok[s]] > 0 and min(abs(ur[s] - lo), abs(ur[s] - hi)) <= 1e-5, (s, tok[s], t)
        checked += 1
    assert checked >= seqs - 2 and (acc > 32).any()


def test_lazy_normalisers_agree_with_full_partials():
    """The lazy round (normalisers computed by the acceptance kernel for the consumed positions only)
    and the round on every row's sampler partials follow the same rule: at full vocabulary they
    agree on every sequence except where a uniform sits within rounding of a decision."""
    from bitmask_speculation_b200.kernels._extension import load_extension
    from bitmask_speculation_b200.stochastic import speculative_accept
    dev = torch.device("cuda")
    temp, k, vocab, seqs = 0.8, wl.DRAFT_K, wl.VOCAB, 160
    logits, masks, _, _ = wl.verify_batch_torch(seqs, seed=33, device=dev)
    words = masks.shape[1]
    g = torch.Generator(device=dev).manual_seed(8)
    first_k = logits.view(seqs, k + 1, vocab)[:, :k].reshape(seqs * k, vocab)
    draft = (first_k.float() + 0.3 * torch.randn(first_k.shape, generator=g, device=dev)).to(torch.bfloat16)
    dmasks = masks.view(seqs, k + 1, words)[:, :k].reshape(seqs * k, words).contiguous()
    u = torch.rand(seqs * k, dtype=torch.float64, generator=g, device=dev)
    proposals = load_extension().masked_sample_batch(draft, dmasks, temp, u)[0].view(seqs, k).contiguous()
    lengths = torch.randint(0, k + 1, (seqs,), generator=g, device=dev).to(torch.int32)
    ua = torch.rand((seqs, k), dtype=torch.float64, generator=g, device=dev)
    ur = torch.rand(seqs, dtype=torch.float64, generator=g, device=dev)
    outs = [speculative_accept(logits, draft, masks, proposals, lengths, temperature=temp, accept_uniforms=ua,
                               resample_uniforms=ur, lazy=lazy) for lazy in (True, False)]
    for o in outs:
        assert (o.status == 0).all()
    same = (outs[0].accept_len == outs[1].accept_len) & (outs[0].token == outs[1].token) & (outs[0].kind == outs[1].kind)
    assert int(same.sum()) >= seqs - 2
    assert (outs[0].accept_len > 0).any() and (outs[0].accept_len < lengths).any()


def test_lazy_clusters_looping_over_sequences_that_fail_early():
    """600 sequences, so every cluster loops over several; every third fails on its first target row
    (NaN) and so ends without a sampling pass, one in seven has a length outside [0, K].  The lazy
    round must report what the full-partials round reports for every sequence."""
    from bitmask_speculation_b200.stochastic import speculative_accept
    rng = np.random.default_rng(600)
    seqs, k, vocab, temp = 600, 4, 4096, 1.0
    rows = seqs * (k + 1)
    tvals = rng.standard_normal((rows, vocab), dtype=np.float32)
    tvals[np.arange(0, seqs, 3) * (k + 1), 7] = np.nan
    dvals = tvals.reshape(seqs, k + 1, vocab)[:, :k].reshape(seqs * k, vocab) * np.float32(0.9)
    masks = wl.pack_bits_np(rng.random((rows, vocab)) < 0.5)
    proposals = rng.integers(0, vocab, size=(seqs, k))
    lengths = rng.integers(0, k + 1, size=seqs).astype(np.int32)
    lengths[::7] = k + 1
    args = [_bf16(tvals).cuda(), _bf16(dvals).cuda(), torch.from_numpy(masks).cuda(),
            torch.from_numpy(proposals).cuda(), torch.from_numpy(lengths).cuda()]
    ua = torch.from_numpy(rng.random((seqs, k))).cuda()
    ur = torch.from_numpy(rng.random(seqs)).cuda()
    lazy, full = (speculative_accept(*args, temperature=temp, accept_uniforms=ua, resample_uniforms=ur, lazy=z)
                  for z in (True, False))
    st = lazy.status.cpu().numpy()
    assert np.array_equal(st, full.status.cpu().numpy())
    assert (st[::7] == 6).all() and (st[3::21] == 2).all() and (st == 0).sum() > seqs // 3
    ok = st == 0
    for a, b in ((lazy.accept_len, full.accept_len), (lazy.token, full.token), (lazy.kind, full.kind)):
        assert np.array_equal(a.cpu().numpy()[ok], b.cpu().numpy()[ok])
