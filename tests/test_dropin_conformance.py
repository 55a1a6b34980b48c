"""Drop-in conformance with the reference's own call sites (CPU; no GPU needed).

The reference is swapped in by making its ``kernels._extension.load_extension`` return this
library's ``NativeModule``.  The reference's sources are present only on the host where the
library is built, not on the GPU machines, so this test reads them where they are present and
skips elsewhere.  It checks, call site by call site, that ``NativeModule`` serves every call the
reference makes on its native module -- in kernels/cuda.py, kernels/dispatch.py,
benchmarks/reductions.py and its GPU tests -- with a method of that name that binds the same
arguments and returns a sequence the site can unpack; that the status messages its callers match
on are the same; and that the rebuilt ``dispatch.select_token`` binds the reference's signature.
The results of those calls are checked on the GPU by the parity tests against the oracle.
"""

import ast
import inspect
import os
from pathlib import Path

import pytest

REF = Path(os.environ.get("BMS_REFERENCE_SRC", "/root/reference/src")) / "bitmask_speculation"
REF_TESTS = REF.parents[1] / "tests" / "gpu"

pytestmark = pytest.mark.skipif(not (REF / "kernels" / "cuda.py").exists(),
                                reason="the reference's sources are not on this machine")

# Methods whose result the reference unpacks, and how many values it expects:
#   kernels/cuda.py:19-21 ``output, status = result`` (masked_argmax, masked_sample),
#   kernels/cuda.py:68 ``tokens, counts, status = ...masked_reduce_batch(...)``.
UNPACKED = {"masked_argmax": 2, "masked_sample": 2, "masked_reduce_batch": 3}


def _native_calls(path: Path):
    """(method, positional args, keyword names) of every call on the native module in a file: calls
    on ``load_extension()`` directly, or on a name bound to it (``native``, ``cuda_module``)."""
    tree = ast.parse(path.read_text())
    bound = {"cuda_module"}
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and isinstance(node.value, ast.Call) and \
                getattr(node.value.func, "id", None) == "load_extension":
            bound.update(t.id for t in node.targets if isinstance(t, ast.Name))
    calls = []
    for node in ast.walk(tree):
        if not (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)):
            continue
        owner = node.func.value
        direct = isinstance(owner, ast.Call) and getattr(owner.func, "id", None) == "load_extension"
        if direct or (isinstance(owner, ast.Name) and owner.id in bound):
            calls.append((node.func.attr, len(node.args), [k.arg for k in node.keywords]))
    return calls


def _sites():
    files = [REF / "kernels" / "cuda.py", REF / "kernels" / "dispatch.py", REF / "benchmarks" / "reductions.py"]
    files += sorted(REF_TESTS.glob("test_*.py"))
    out = []
    for f in files:
        if f.exists():
            out += [(f.name, *c) for c in _native_calls(f)]
    return out


def test_every_native_call_of_the_reference_binds_to_native_module():
    from bitmask_speculation_b200.kernels._extension import NativeModule
    sites = _sites()
    names = {name for _, name, _, _ in sites}
    # The five exports of csrc/bindings.cpp:10-17 are all used somewhere.
    assert {"runtime_version", "mask_count", "masked_argmax", "masked_reduce_batch", "masked_sample"} <= names
    for fname, name, nargs, kwargs in sites:
        method = getattr(NativeModule, name, None)
        assert callable(method), f"{fname}: NativeModule has no {name}"
        inspect.signature(method).bind(object(), *([None] * nargs), **{k: None for k in kwargs})


def test_results_unpack_as_the_reference_expects():
    """Return statements of NativeModule's methods build lists of the arity the reference's sites
    unpack (read from this library's source, since calling them needs a GPU)."""
    from bitmask_speculation_b200.kernels import _extension
    tree = ast.parse(inspect.getsource(_extension))
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "NativeModule")
    arity = {}
    for fn in cls.body:
        if isinstance(fn, ast.FunctionDef):
            for node in ast.walk(fn):
                if isinstance(node, ast.Return) and isinstance(node.value, ast.List):
                    arity.setdefault(fn.name, set()).add(len(node.value.elts))
    for name, n in UNPACKED.items():
        assert n in arity.get(name, set()), (name, arity.get(name))
    # masked_sample at temperature 0 returns masked_argmax's result (csrc/sample.cu:120).
    src = inspect.getsource(_extension.NativeModule.masked_sample)
    assert "return self.masked_argmax(logits, mask)" in src


def _status_messages(path: Path) -> dict:
    """``code == N: raise ValueError("...")`` pairs of a status check."""
    out = {}
    for node in ast.walk(ast.parse(path.read_text())):
        if isinstance(node, ast.If) and isinstance(node.test, ast.Compare) and \
                isinstance(node.test.comparators[0], ast.Constant) and node.body and \
                isinstance(node.body[0], ast.Raise) and isinstance(node.body[0].exc, ast.Call):
            args = node.body[0].exc.args
            if args and isinstance(args[0], ast.Constant):
                out[node.test.comparators[0].value] = args[0].value
    return out


def test_status_messages_are_the_reference_callers_messages():
    from bitmask_speculation_b200.kernels import cuda
    ref = _status_messages(REF / "kernels" / "cuda.py")
    assert set(ref) == {1, 2, 3, 4, 5}
    for code, message in ref.items():
        assert cuda._MESSAGES[code] == message, code


def test_validation_messages_match_except_the_two_documented_relaxations():
    from bitmask_speculation_b200.kernels import _validation

    def messages(tree):
        return {n.exc.args[0].value for n in ast.walk(tree) if isinstance(n, ast.Raise) and
                isinstance(n.exc, ast.Call) and n.exc.args and isinstance(n.exc.args[0], ast.Constant)}
    ref = messages(ast.parse((REF / "kernels" / "_validation.py").read_text()))
    ours = messages(ast.parse(inspect.getsource(_validation)))
    relaxed = {"logits must be a float32 tensor",                  # float16 / bfloat16 accepted
               "batch size exceeds the CUDA grid-y limit of 65535"}  # no row limit
    assert ref - relaxed <= ours, ref - relaxed - ours
    assert "logits must be a float32, bfloat16 or float16 tensor" in ours


def test_select_token_binds_the_reference_signature():
    from bitmask_speculation_b200 import dispatch
    tree = ast.parse((REF / "kernels" / "dispatch.py").read_text())
    ref = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "select_token")
    ours = inspect.signature(dispatch.select_token)
    ref_positional = [a.arg for a in ref.args.args]
    assert list(ours.parameters)[:len(ref_positional)] == ref_positional
    assert {a.arg for a in ref.args.kwonlyargs} <= set(ours.parameters)
    assert ours.parameters["backend"].default == "cuda"
    # The reference's dtype rejection test matches "float32" in the TypeError message.
    assert "float32" in inspect.getsource(dispatch.select_token)
