"""Regenerate the golden fixtures from the reference implementation itself.

Run in a checkout that has the reference package importable, e.g.

    PYTHONPATH=/root/reference/src python tests/golden/make_golden.py

It imports karthikeyansura/bitmask-speculation's own CPU/PyTorch functions
(``torch_reduce``, ``masked_argmax``, ``packed_mask_count``,
``masked_sample_reference``, ``verify_prefix``, ``DensityPolicy``), runs them on
seeded inputs from ``bitmask_speculation_b200.workloads`` and the reference's own
test cases, and writes their outputs next to this script.  Large inputs are not
stored: the fixture keeps the generator seed and shape and the tests rebuild the
identical arrays with numpy.  The fixtures travel with the repository; the tests
never import the reference.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "bitmask-speculation_b200"))

import torch  # noqa: E402

from bitmask_speculation.benchmarks.reductions import torch_reduce  # noqa: E402
from bitmask_speculation.decoding.scheduling import DensityPolicy  # noqa: E402
from bitmask_speculation.decoding.verification import verify_prefix  # noqa: E402
from bitmask_speculation.grammar.density import packed_mask_count  # noqa: E402
from bitmask_speculation.grammar.selection import masked_argmax  # noqa: E402
from bitmask_speculation.kernels.reference import masked_sample_reference  # noqa: E402

from bitmask_speculation_b200 import workloads as wl  # noqa: E402

TORCH_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def as_torch(values: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "float32":
        return torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32))
    bits = torch.from_numpy(np.ascontiguousarray(values, dtype=np.uint16).view(np.int16))
    return bits.view(TORCH_DTYPES[dtype])


def native_tokens(tokens: torch.Tensor, status: torch.Tensor) -> np.ndarray:
    """torch_reduce reports V for failed rows; the native API reports -1."""
    return np.where(status.numpy() == 0, tokens.numpy(), -1).astype(np.int64)


def reduce_case(values, masks, dtype):
    tokens, counts, status = torch_reduce(as_torch(values, dtype), torch.from_numpy(masks))
    return native_tokens(tokens, status), counts.numpy().astype(np.int64), status.numpy().astype(np.int32)


def random_reduce_inputs(rng, rows, vocab, dtype, style):
    values = rng.standard_normal((rows, vocab), dtype=np.float32)
    if style == "ties":
        values = np.round(values * 2) / 2  # many exact ties, including +-0.0
        values[values == 0] = np.where(rng.random((values == 0).sum()) < 0.5, -0.0, 0.0)
    if style == "inf":
        pick = rng.random((rows, vocab))
        values[pick < 0.05] = -np.inf
        values[(pick > 0.97)] = np.inf
    if style == "allneg":
        values[:] = -np.inf
    masks = rng.integers(-(1 << 31), 1 << 31, size=(rows, wl.words_for(vocab)), dtype=np.int64).astype(np.int32)
    masks[:, 0] |= 1
    if style == "nan":
        values[0, rng.integers(vocab)] = np.nan  # anywhere: fails the row
    if style == "empty":
        masks[-1] = 0
    if style == "dirty":
        masks[:, -1] = -1  # tail bits beyond V must be ignored
    if dtype == "bfloat16":
        values = wl.to_bf16_bits(values)
    elif dtype == "float16":
        values = wl.to_f16_bits(values)
    return values, masks


def make_reduce():
    rng = np.random.default_rng(20240601)
    small = []
    styles = ["plain", "ties", "inf", "allneg", "nan", "empty", "dirty"]
    for vocab in [1, 2, 31, 32, 33, 63, 64, 65, 255, 256, 257, 1024, 4097, 4224]:
        for dtype in ["float32", "bfloat16", "float16"]:
            for style in styles if vocab <= 1024 else ["plain", "ties", "nan", "dirty"]:
                values, masks = random_reduce_inputs(rng, 3, vocab, dtype, style)
                tokens, counts, status = reduce_case(values, masks, dtype)
                small.append(dict(vocab=vocab, dtype=dtype, style=style, values=values,
                                  masks=masks, tokens=tokens, counts=counts, status=status))
    arrays = {}
    meta = []
    for i, case in enumerate(small):
        for key in ("values", "masks", "tokens", "counts", "status"):
            arrays[f"c{i}_{key}"] = case[key]
        meta.append({k: case[k] for k in ("vocab", "dtype", "style")})

    # Known answers from the reference's own tests.
    # tests/integration/test_reduction_baseline.py:7-20
    ka = []
    scores = np.full((2, 33), -np.inf, np.float32)
    masks = np.array([[-2147483648, 1], [0, -1]], np.int32)
    ka.append(("baseline_signed_tail_neginf", scores, masks))
    scores = np.zeros((2, 3), np.float32)
    scores[0, 2] = np.nan
    ka.append(("baseline_masked_nan_and_empty", scores, np.array([[1], [0]], np.int32)))
    # tests/gpu/test_cuda_batch.py:42-51
    scores = np.zeros((4, 8193), np.float32)
    masks = np.full((4, 257), -1, np.int32)
    masks[0] = 0
    scores[1, 8192] = np.nan
    scores[2, 4096] = scores[2, 8191] = 5.0
    ka.append(("batch_rows_fail_independently", scores, masks))
    # tests/gpu/test_argmax.py:17-26
    scores = np.zeros((1, 257), np.float32)
    scores[0, 0] = 999
    scores[0, 31] = scores[0, 256] = 10
    masks = np.zeros((1, 9), np.int32)
    masks[0, 0] = -2147483648
    masks[0, -1] = -1
    ka.append(("argmax_sparse_dirty_tail", scores, masks))
    for name, scores, masks in ka:
        tokens, counts, status = reduce_case(scores, masks, "float32")
        i = len(meta)
        arrays[f"c{i}_values"] = scores
        arrays[f"c{i}_masks"] = masks
        arrays[f"c{i}_tokens"] = tokens
        arrays[f"c{i}_counts"] = counts
        arrays[f"c{i}_status"] = status
        meta.append(dict(vocab=scores.shape[1], dtype="float32", style=name))

    # Cross-check torch_reduce against the per-row reference selection on the small cases.
    for i, m in enumerate(meta):
        values = as_torch(arrays[f"c{i}_values"], m["dtype"])
        masks = arrays[f"c{i}_masks"]
        for r in range(values.shape[0]):
            allowed = [t for t in range(m["vocab"]) if (int(masks[r, t // 32]) >> (t % 32)) & 1]
            try:
                expect = masked_argmax(values[r], allowed)
            except ValueError:
                expect = -1
            assert expect == arrays[f"c{i}_tokens"][r], (m, r)
    np.savez_compressed(HERE / "reduce_small.npz", **arrays)
    return meta


def make_reduce_configs():
    """Outputs only; the tests regenerate inputs from the workload seeds."""
    out = {}
    values, masks = wl.argmax_config_np(seed=1)
    out["argmax_config_seed1"] = [a.tolist() for a in reduce_case(values, masks, "float32")]
    bits, masks, proposals, lengths = wl.verify_config_np(seed=3, seqs=4)
    out["verify_config_seed3_seqs4_reduce"] = [a.tolist() for a in reduce_case(bits, masks, "bfloat16")]
    out["verify_config_seed3_seqs4_counts_ref"] = [
        packed_mask_count(torch.from_numpy(masks[r]), wl.VOCAB) for r in range(masks.shape[0])]
    return out


def make_counts():
    rng = np.random.default_rng(7)
    cases = []
    for vocab in [1, 2, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256, 257, 248320, 248321]:
        for fill in [0, -1, -2147483648, "random"]:
            words = wl.words_for(vocab)
            if fill == "random":
                mask = rng.integers(-(1 << 31), 1 << 31, size=words, dtype=np.int64).astype(np.int32)
                seed = None
            else:
                mask = np.full(words, fill, np.int32)
            count = packed_mask_count(torch.from_numpy(mask), vocab)
            entry = dict(vocab=vocab, fill=fill, count=count)
            if fill == "random":
                entry["words"] = mask.tolist() if words <= 16 else None
                entry["seed_index"] = len(cases)
            cases.append((entry, mask))
    arrays = {f"m{i}": mask for i, (_, mask) in enumerate(cases) if _["fill"] == "random"}
    np.savez_compressed(HERE / "count_masks.npz", **arrays)
    # tests/unit/test_signed_words.py:7-11
    signed = [(-2147483648, 32), (-2147483648, 31), (-1, 32), (-1, 31), (2147483647, 32)]
    signed_out = [[w, v, packed_mask_count(torch.tensor([w], dtype=torch.int32), v)] for w, v in signed]
    return [c for c, _ in cases], signed_out


def sample_case(values, mask, temperature, uniform):
    try:
        return masked_sample_reference(values, mask, temperature=temperature, uniform=uniform), ""
    except ValueError as exc:
        return -1, str(exc)


def make_sampling():
    cases = []
    # tests/unit/test_sampling_reference.py and tests/gpu/test_sampling.py known answers.
    known = [
        ([999.0, 0.0, math.log(3.0)], [6], 1.0, [0, .249, .251, .999999]),
        ([-math.inf, 0.0, 0.0], [-1], 1.0, [0, .5]),
        ([1000., -math.inf, -2., 1., .5], [-2], None, [0.0, .13, .51, .999999999]),
        ([-3e38, 3e38, -math.inf], [-1], None, [.999]),
        ([math.inf, 2.], [-2], 1.0, [0]),
        ([0.0], [0], 1.0, [.5]),
        ([-math.inf], [1], 1.0, [.5]),
        ([math.inf], [1], 1.0, [.5]),
        ([0.0, math.nan], [1], 1.0, [.5]),
    ]
    temps_grid = {2: [0.0, 1e-320, .1, 1.0, 100.0], 3: [1e-320, 1e-10, 1.0, 1e300]}
    for k, (vals, mask, temp, us) in enumerate(known):
        temps = temps_grid.get(k, [temp])
        for t in temps:
            for u in us:
                v = torch.tensor(vals, dtype=torch.float32)
                token, err = sample_case(v, torch.tensor(mask, dtype=torch.int32), t, u)
                cases.append(dict(values=vals, mask=mask, temperature=t, uniform=u,
                                  token=token, error=err))
    # Random rows at small vocabularies (inputs stored).
    rng = np.random.default_rng(11)
    rows = []
    for vocab in [5, 33, 257, 4097]:
        values = (rng.standard_normal(vocab, dtype=np.float32) * 3).astype(np.float32)
        mask = rng.integers(-(1 << 31), 1 << 31, size=wl.words_for(vocab), dtype=np.int64).astype(np.int32)
        mask[0] |= 1
        results = []
        for t in [0.5, 1.0, 4.0]:
            for u in [0.0, 0.17, 0.5, 0.83, 0.999]:
                token, err = sample_case(torch.from_numpy(values), torch.from_numpy(mask), t, u)
                results.append([t, u, token, err])
        rows.append(dict(vocab=vocab, values=values.tolist(), mask=mask.tolist(), results=results))
    # Configuration 2 (fp16 widened exactly to fp32, as the reference requires fp32).
    bits, masks, uniforms, temp = wl.sample_config_np(seed=2)
    config = []
    widened = (torch.from_numpy(bits.view(np.int16)).view(torch.float16)).float()
    extra_u = [0.0, 0.25, 0.5, 0.75, 0.999]
    for r in range(bits.shape[0]):
        row = []
        for u in [float(uniforms[r])] + extra_u:
            token, err = sample_case(widened[r].contiguous(), torch.from_numpy(masks[r]), temp, u)
            row.append([u, token, err])
        config.append(row)
    return cases, rows, config


def make_verification():
    rng = np.random.default_rng(5)
    cases = []
    for _ in range(400):
        vocab = int(rng.integers(2, 9))
        k = int(rng.integers(0, 6))
        targets = rng.integers(0, vocab, size=k + 1).tolist()
        draft = [t if rng.random() < 0.7 else int(rng.integers(0, vocab)) for t in targets[:k]]
        calls = []

        def select(i, targets=targets, calls=calls):
            calls.append(i)
            return targets[i]

        events = [(e.token_id, e.kind) for e in verify_prefix(draft, select, vocab_size=vocab)]
        cases.append(dict(vocab=vocab, draft=draft, targets=targets, events=events, calls=calls))
    # tests/unit/test_verification.py:9-28
    for draft, target in [([1, 2, 3], [0]), ([1, 2, 3], [1, 0]), ([1, 2, 3], [1, 2, 0]),
                          ([1, 2], [1, 2, 3]), ([], [2])]:
        calls = []
        padded = target + [0] * (len(draft) + 1 - len(target))

        def select(i, padded=padded, calls=calls):
            calls.append(i)
            return padded[i]

        events = [(e.token_id, e.kind) for e in verify_prefix(draft, select, vocab_size=4)]
        cases.append(dict(vocab=4, draft=draft, targets=padded, events=events, calls=calls))
    return cases


def make_policy():
    d = DensityPolicy()
    points = [0.0, math.nextafter(.005, 0), .005, math.nextafter(.005, 1), .01,
              math.nextafter(.02, 0), .02, math.nextafter(.02, 1), .5, 1.0, 1e-300, 5e-324]
    rng = np.random.default_rng(9)
    points += rng.random(200).tolist() + (rng.random(200) * 0.03).tolist()
    out = {"default": [[p, d.budget(p)] for p in points]}
    custom = DensityPolicy(.1, .8, 2, 7)
    out["custom_0.1_0.8_2_7"] = [[p, custom.budget(p)] for p in [0, .1, .8, 1] + points]
    const = DensityPolicy(0, 1, 3, 3)
    out["constant_0_1_3_3"] = [[p, const.budget(p)] for p in [0, .3, 1]]
    # Densities as the engine computes them: packed_mask_count / V at V = 248,320.
    vocab = 248320
    counts = [0, 1, 2, 1240, 1241, 1242, 4966, 4967, 4968, 100000, vocab]
    out["counts_at_248320"] = [[c, d.budget(c / vocab)] for c in counts]
    return out


def main():
    reduce_meta = make_reduce()
    reduce_configs = make_reduce_configs()
    counts, signed = make_counts()
    sampling_known, sampling_rows, sampling_config = make_sampling()
    verification = make_verification()
    policy = make_policy()
    doc = {
        "generator": "tests/golden/make_golden.py (reference: karthikeyansura/bitmask-speculation)",
        "torch": torch.__version__,
        "numpy": np.__version__,
        "reduce_small": reduce_meta,
        "reduce_configs": reduce_configs,
        "counts": counts,
        "signed_words": signed,
        "sampling_known": sampling_known,
        "sampling_rows": sampling_rows,
        "sampling_config_seed2": sampling_config,
        "verification": verification,
        "policy": policy,
    }
    (HERE / "golden.json").write_text(json.dumps(doc, indent=None, separators=(",", ":")))
    print("wrote", HERE / "golden.json", HERE / "reduce_small.npz", HERE / "count_masks.npz")


if __name__ == "__main__":
    main()
