"""End-to-end constrained decoding: density-scheduled speculative decoding (the reference's c4 mode,
decoding/speculative.py:96-208) verified in one batched round per step reproduces target-only
constrained greedy decoding (decoding/greedy.py:51-92) token for token, stop reason included.

fp32 models keep the target's logits independent of the forward length to well below the gap
between the best and second-best valid logit, so greedy and speculative runs see the same choices.
"""

import json
from pathlib import Path

import pytest

from bitmask_speculation_b200 import workloads as wl

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def models(cuda_module):
    from bitmask_speculation_b200.decode import build_decoder
    vocab = 8320
    target = build_decoder(vocab, layers=2, dim=256, heads=4, dtype=torch.float32, seed=1)
    draft = build_decoder(vocab, layers=1, dim=128, heads=2, dtype=torch.float32, seed=2)
    return vocab, target, draft


@pytest.mark.parametrize("same_draft", [False, True])
def test_speculative_c4_equals_constrained_greedy(models, same_draft):
    from bitmask_speculation_b200.decode import constrained_greedy, random_prompts, speculative_c4
    vocab, target, draft = models
    draft = target if same_draft else draft
    for i, prompt in enumerate(random_prompts(6, 16, vocab, seed=3)):
        g_ref = wl.SyntheticDFAGrammar(vocab, states=64, seed=10 + i)
        g_spec = g_ref.fork()
        want = constrained_greedy(target, prompt, g_ref, max_new_tokens=48, eos=(0,))
        got = speculative_c4(target, draft, prompt, g_spec, max_new_tokens=48, eos=(0,))
        assert got.token_ids == want.token_ids, (i, got, want)
        assert (got.stop_reason, got.eos_token_id) == (want.stop_reason, want.eos_token_id)
        assert g_spec.state == g_ref.state and g_spec.is_terminated() == g_ref.is_terminated()
        if same_draft:
            assert got.accepted == got.proposed  # the target drafting for itself is always accepted


def test_batched_and_lazy_verification_agree_in_bf16(cuda_module):
    """bf16 config-shaped models (smaller): the batched round and the reference's per-row loop see
    the same target rows and must choose the same tokens."""
    from bitmask_speculation_b200.decode import build_decoder, random_prompts, speculative_c4
    vocab = 151936
    target = build_decoder(vocab, layers=2, dim=512, heads=8, seed=5)
    draft = build_decoder(vocab, layers=1, dim=256, heads=4, seed=6)
    for i, prompt in enumerate(random_prompts(4, 32, vocab, seed=7)):
        g0 = wl.SyntheticDFAGrammar(vocab, states=64, seed=20 + i)
        a = speculative_c4(target, draft, prompt, g0.fork(), max_new_tokens=40, eos=(0,))
        b = speculative_c4(target, draft, prompt, g0.fork(), max_new_tokens=40, eos=(0,), verify="lazy")
        assert a == b, i


def test_device_mask_table_decoding_equals_uploaded_masks(models):
    """Selections and rounds reading the grammar's state masks from a device table choose exactly
    what the uploaded-mask path chooses."""
    from bitmask_speculation_b200.decode import random_prompts, speculative_c4
    from bitmask_speculation_b200.grammar_verification import DeviceMaskTable
    vocab, target, draft = models
    for i, prompt in enumerate(random_prompts(4, 16, vocab, seed=9)):
        g0 = wl.SyntheticDFAGrammar(vocab, states=64, seed=30 + i)
        table = DeviceMaskTable.for_grammar(g0, 16, torch.device("cuda"))
        a = speculative_c4(target, draft, prompt, g0.fork(), max_new_tokens=40, eos=(0,))
        b = speculative_c4(target, draft, prompt, g0.fork(), max_new_tokens=40, eos=(0,), table=table)
        c = speculative_c4(target, draft, prompt, g0.fork(), max_new_tokens=40, eos=(0,), table=table,
                           verify="lazy")
        assert a == b == c, i


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_graph_replayed_trunk_matches_eager_forward(cuda_module, dtype):
    """The CUDA-graph forward (one graph per padded length) holds the eager forward's kernels: the
    logits of every requested slice are bit-identical, across lengths that reuse a graph."""
    from bitmask_speculation_b200.decode import build_decoder, random_prompts
    vocab = 8320
    eager = build_decoder(vocab, layers=2, dim=256, heads=4, dtype=getattr(torch, dtype), seed=11)
    graphed = build_decoder(vocab, layers=2, dim=256, heads=4, dtype=getattr(torch, dtype), seed=11).enable_graphs()
    for prompt in random_prompts(3, 50, vocab, seed=12):
        for n in (1, 14, 64, 65, 100):  # 64-token padded lengths 64, 128 and 64 again
            seq = (prompt * 3)[:n]
            for first, rows in ((n - 1, 1), (max(0, n - 9), min(9, n))):
                a = eager.logits(seq, first, rows)
                b = graphed.logits(seq, first, rows)
                assert torch.equal(a, b), (dtype, n, first, rows)
    assert sorted(graphed._graphs) == [64, 128]


def test_speculative_c4_with_graphs_equals_eager(models):
    from bitmask_speculation_b200.decode import build_decoder, constrained_greedy, random_prompts, speculative_c4
    vocab, target, draft = models
    g_target = build_decoder(vocab, layers=2, dim=256, heads=4, dtype=torch.float32, seed=1).enable_graphs()
    g_draft = build_decoder(vocab, layers=1, dim=128, heads=2, dtype=torch.float32, seed=2).enable_graphs()
    for i, prompt in enumerate(random_prompts(3, 16, vocab, seed=13)):
        g0 = wl.SyntheticDFAGrammar(vocab, states=64, seed=40 + i)
        a = speculative_c4(target, draft, prompt, g0.fork(), max_new_tokens=48, eos=(0,))
        b = speculative_c4(g_target, g_draft, prompt, g0.fork(), max_new_tokens=48, eos=(0,))
        c = constrained_greedy(g_target, prompt, g0.fork(), max_new_tokens=48, eos=(0,))
        assert a == b, i
        assert b.token_ids == c.token_ids, i


def _decode_golden():
    return json.loads((Path(__file__).resolve().parent / "golden" / "decode_golden.json").read_text())["sets"]


@pytest.mark.parametrize("name", ["small", "tiny_eos", "tiny_grammar_stop", "config4_fp32"])
def test_decodes_match_the_reference_engine(cuda_module, name):
    """Token streams, stop reasons and proposal accounting of the reference's own DecodingEngine
    (``target_constrained`` = greedy_decode, ``c4`` = speculative_decode with DensityPolicy budgets;
    decoding/greedy.py:46-92, decoding/speculative.py:98-210), recorded on CPU in fp32 by
    tests/golden/make_decode_golden.py, reproduced by this library's constrained_greedy and
    speculative_c4 on the same fp32 models and grammars on the GPU."""
    from bitmask_speculation_b200.decode import build_decoder, constrained_greedy, speculative_c4
    spec = next(s for s in _decode_golden() if s["name"] == name)
    vocab, new, eos = spec["vocab"], spec["new_tokens"], tuple(spec["eos"])
    target = build_decoder(vocab, dtype=torch.float32, **spec["target"])
    draft = build_decoder(vocab, dtype=torch.float32, **spec["draft"])
    for i, req in enumerate(spec["requests"]):
        base = wl.SyntheticDFAGrammar(vocab, states=64, seed=req["grammar_seed"])
        prompt = tuple(req["prompt"])
        greedy = constrained_greedy(target, prompt, base.fork(), max_new_tokens=new, eos=eos)
        want = req["target_constrained"]
        assert (list(greedy.token_ids), greedy.stop_reason, greedy.eos_token_id) == (
            want["token_ids"], want["stop_reason"], want["eos_token_id"]), (name, i, "greedy")
        c4 = speculative_c4(target, draft, prompt, base.fork(), max_new_tokens=new, eos=eos)
        want = req["c4"]
        assert (list(c4.token_ids), c4.stop_reason, c4.eos_token_id) == (
            want["token_ids"], want["stop_reason"], want["eos_token_id"]), (name, i, "c4")
        assert (c4.rounds, c4.proposed, c4.accepted) == (want["rounds"], want["proposed"], want["accepted"]), \
            (name, i, "accounting")


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_device_drafting_with_graphs_equals_eager(cuda_module, dtype):
    """Rounds drafted on the device (state masks in a DeviceMaskTable, the DFA advanced on the
    device, one read-back per round) give the same decode whether the trunks replay CUDA graphs or
    run eagerly, with batched and lazy verification; in fp32 they also equal target-only greedy."""
    from bitmask_speculation_b200.decode import build_decoder, constrained_greedy, random_prompts, speculative_c4
    from bitmask_speculation_b200.grammar_verification import DeviceMaskTable
    vocab = 8320
    dt = getattr(torch, dtype)
    target = build_decoder(vocab, layers=2, dim=256, heads=4, dtype=dt, seed=21)
    draft = build_decoder(vocab, layers=1, dim=128, heads=2, dtype=dt, seed=22)
    g_target = build_decoder(vocab, layers=2, dim=256, heads=4, dtype=dt, seed=21).enable_graphs()
    g_draft = build_decoder(vocab, layers=1, dim=128, heads=2, dtype=dt, seed=22).enable_graphs()
    for i, prompt in enumerate(random_prompts(3, 16, vocab, seed=23)):
        g0 = wl.SyntheticDFAGrammar(vocab, states=64, seed=50 + i)
        table = DeviceMaskTable.for_grammar(g0, 16, torch.device("cuda"))
        a = speculative_c4(target, draft, prompt, g0.fork(), max_new_tokens=48, eos=(0,), table=table)
        b = speculative_c4(g_target, g_draft, prompt, g0.fork(), max_new_tokens=48, eos=(0,), table=table)
        c = speculative_c4(g_target, g_draft, prompt, g0.fork(), max_new_tokens=48, eos=(0,), table=table,
                           verify="lazy")
        assert a == b == c, i
        assert a.proposed > 0
        if dtype == "float32":
            want = constrained_greedy(target, prompt, g0.fork(), max_new_tokens=48, eos=(0,))
            assert a.token_ids == want.token_ids and a.stop_reason == want.stop_reason, i
