"""Golden decodes from the reference's own engine, for the end-to-end (c4) configuration.

Run in a checkout that has the reference package importable (CPU is enough), e.g.

    PYTHONPATH=/root/reference/src python tests/golden/make_decode_golden.py

It runs karthikeyansura/bitmask-speculation's ``DecodingEngine.generate`` -- its ``greedy_decode``
(mode ``target_constrained``) and ``speculative_decode`` (mode ``c4``: constrained drafts, budgets
from the reference's ``DensityPolicy``) over its ``TransformersGreedyModel`` adapter with the CPU
``reference`` selection backend -- on this repository's random-init fp32 decoders (wrapped as
Transformers-style causal models) and ``workloads.SyntheticDFAGrammar``, and records each request's
tokens, stop reason, EOS token and proposal accounting in ``decode_golden.json``.  The GPU tests
rebuild the same models (same seeds, fp32) and grammars on the device and compare this library's
``constrained_greedy`` and ``speculative_c4`` with these records.  The tests never import the
reference.

Model sets: the small models of ``tests/test_gpu_decode.py`` (V = 8,320); two V = 96 sets whose
grammars reach EOS, with and without EOS as a stop token (stop reasons "eos" and "grammar"); and
the end-to-end configuration's architecture (target 4 layers d=1024 16 heads, draft 1 layer d=512,
V = 248,320) in fp32 on fewer prompts and tokens, which the CPU forward time bounds.
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path
from types import SimpleNamespace

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "bitmask-speculation_b200"))

import torch  # noqa: E402

from bitmask_speculation.decoding.scheduling import DensityPolicy  # noqa: E402
from bitmask_speculation.engine import DecodingEngine  # noqa: E402
from bitmask_speculation.models.transformers import TransformersGreedyModel  # noqa: E402

from bitmask_speculation_b200 import workloads as wl  # noqa: E402
from bitmask_speculation_b200.decode import build_decoder, random_prompts  # noqa: E402

# (name, vocab, target spec, draft spec, prompts, prompt length, new tokens, grammar seed base, EOS ids)
# The V = 96 sets reach the grammar's EOS (token 0, allowed in its free-text states) within the run:
# with EOS as a stop token the request ends with "eos", without it the grammar terminates ("grammar").
SETS = [
    ("small", 8320, dict(layers=2, dim=256, heads=4, seed=1), dict(layers=1, dim=128, heads=2, seed=2),
     6, 16, 48, 10, (0,)),
    ("tiny_eos", 96, dict(layers=2, dim=64, heads=2, seed=3), dict(layers=1, dim=32, heads=1, seed=4),
     8, 8, 48, 60, (0,)),
    ("tiny_grammar_stop", 96, dict(layers=2, dim=64, heads=2, seed=3), dict(layers=1, dim=32, heads=1, seed=4),
     8, 8, 48, 60, ()),
    ("config4_fp32", wl.VOCAB, dict(layers=4, dim=1024, heads=16, seed=0), dict(layers=1, dim=512, heads=8, seed=1),
     2, 64, 48, 4, (0,)),
]


class CausalLM(torch.nn.Module):
    """A Transformers-style causal LM around the harness decoder: ``forward(input_ids)`` returns
    logits for every position ([1, L, V]), as the reference's adapter expects."""

    def __init__(self, decoder):
        super().__init__()
        self.decoder = decoder
        self.config = SimpleNamespace(vocab_size=decoder.vocab_size, is_encoder_decoder=False)

    def forward(self, input_ids, **kwargs):
        ids = [int(t) for t in input_ids[0]]
        return SimpleNamespace(logits=self.decoder.logits(ids, 0, len(ids))[None])


def main() -> None:
    torch.set_num_threads(max(1, torch.get_num_threads()))
    out = {"note": "reference DecodingEngine on CPU, fp32, DensityPolicy() defaults", "sets": []}
    for name, vocab, tspec, dspec, n, plen, new, gseed, eos in SETS:
        t0 = time.time()
        target = CausalLM(build_decoder(vocab, dtype=torch.float32, device="cpu", **tspec)).eval()
        draft = CausalLM(build_decoder(vocab, dtype=torch.float32, device="cpu", **dspec)).eval()
        engine = DecodingEngine(TransformersGreedyModel(target, backend="reference"),
                                TransformersGreedyModel(draft, backend="reference", draft_cache=False))
        prompts = random_prompts(n, plen, vocab, seed=3)
        requests = []
        for i, prompt in enumerate(prompts):
            base = wl.SyntheticDFAGrammar(vocab, states=64, seed=gseed + i)
            rec = {"prompt": list(prompt), "grammar_seed": gseed + i}
            for mode in ("target_constrained", "c4"):
                kw = dict(mode=mode, max_new_tokens=new, eos_token_ids=eos, grammar_factory=base.fork)
                if mode == "c4":
                    kw["draft_policy"] = DensityPolicy()
                r = engine.generate(prompt, **kw)
                entry = {"token_ids": list(r.token_ids), "stop_reason": r.stop_reason, "eos_token_id": r.eos_token_id}
                if r.accounting is not None:
                    a = r.accounting
                    entry.update(proposed=a.proposed, verified=a.verified, accepted=a.accepted, rounds=a.rounds,
                                 budgets=[s.effective_budget for s in r.schedule])
                rec[mode] = entry
            requests.append(rec)
            print(name, i, len(rec["c4"]["token_ids"]), rec["c4"]["stop_reason"], f"{time.time() - t0:.1f}s",
                  flush=True)
        out["sets"].append({"name": name, "vocab": vocab, "target": tspec, "draft": dspec, "new_tokens": new,
                            "eos": list(eos), "requests": requests})
    (HERE / "decode_golden.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
