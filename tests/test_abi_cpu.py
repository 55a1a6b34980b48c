"""The C-ABI library: loads, exports every declared symbol, rejects bad calls (no GPU)."""

import ctypes
import re
from pathlib import Path

import pytest

from bitmask_speculation_b200 import _native
from bitmask_speculation_b200.build import LIBRARY, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "bms_b200.h"


@pytest.fixture(scope="module")
def lib():
    build()
    return _native.library()


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"BMS_API\s+[\w\s\*]*?\b(bms_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_symbols()
    assert set(_native.EXPORTS) == set(names)
    # Each entry point names the reference interface it replaces (or says it is new).
    text = HEADER.read_text()
    for ref in ["csrc/runtime.cu", "csrc/popcount.cu", "csrc/argmax.cu:117", "csrc/argmax.cu:127",
                "csrc/sample.cu:116", "decoding/verification.py", "decoding/scheduling.py"]:
        assert ref in text


def test_library_exports_every_declared_symbol(lib):
    assert LIBRARY.exists()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_library_is_sm100a_only_and_links_no_torch():
    import subprocess
    deps = subprocess.run(["ldd", str(LIBRARY)], capture_output=True, text=True).stdout
    assert "libtorch" not in deps and "libc10" not in deps
    assert "libcudart.so" not in deps  # runtime linked statically


def test_runtime_version_without_gpu(lib):
    v = ctypes.c_int32(0)
    assert lib.bms_runtime_version(ctypes.byref(v)) == 0
    assert v.value >= 12000


def test_invalid_arguments_fail_before_any_launch(lib):
    null = None
    # Unknown dtype
    rc = lib.bms_masked_reduce_batch(null, 7, null, 1, 32, null, null, null, null, 0, 0, null)
    assert rc == _native.ERROR_INVALID_ARGUMENT
    assert b"float32" in lib.bms_last_error()
    # Invalid vocabulary
    rc = lib.bms_masked_reduce_batch(null, 0, null, 1, 0, null, null, null, null, 0, 0, null)
    assert rc == _native.ERROR_INVALID_ARGUMENT and b"vocabulary" in lib.bms_last_error()
    rc = lib.bms_masked_argmax(null, 0, null, 2**31, null, null, 0, null)
    assert rc == _native.ERROR_INVALID_ARGUMENT
    # Negative rows
    rc = lib.bms_masked_reduce_batch(null, 0, null, -1, 32, null, null, null, null, 0, 0, null)
    assert rc == _native.ERROR_INVALID_ARGUMENT
    # Temperature contract
    for t in (-1.0, float("nan"), float("inf")):
        rc = lib.bms_masked_sample(null, 0, null, 32, t, null, null, null, 0, null)
        assert rc == _native.ERROR_INVALID_ARGUMENT and b"temperature" in lib.bms_last_error()
    # Launch override contract
    assert lib.bms_set_launch_override(3, 0) == _native.ERROR_INVALID_ARGUMENT
    assert lib.bms_set_launch_override(0, -1) == _native.ERROR_INVALID_ARGUMENT
    assert lib.bms_set_launch_override(0, 0) == 0
    # Policy contract
    bad = _native.Policy(5, 1, 8, 0, 0.005, 0.02)
    rc = lib.bms_mask_budget(null, 1, 32, ctypes.byref(bad), null, null, ctypes.c_void_p(16), 0, null)
    assert rc == _native.ERROR_INVALID_ARGUMENT and b"policy" in lib.bms_last_error()
    bad = _native.Policy(0, 1, 8, 0, 0.02, 0.005)
    rc = lib.bms_mask_budget(null, 1, 32, ctypes.byref(bad), null, null, ctypes.c_void_p(16), 0, null)
    assert rc == _native.ERROR_INVALID_ARGUMENT
    # Verification shape contract
    rc = lib.bms_verify_batch(null, 0, null, 1, 0, 32, null, null, null, null, null, null, null,
                              null, null, null, null, null, 0, null, 0, 0, null)
    assert rc == _native.ERROR_INVALID_ARGUMENT and b"rows_per_seq" in lib.bms_last_error()


def test_error_message_is_thread_local(lib):
    import threading
    lib.bms_masked_reduce_batch(None, 9, None, 1, 32, None, None, None, None, 0, 0, None)
    seen = []

    def other():
        seen.append(lib.bms_last_error())

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen == [b""]
    assert b"float32" in lib.bms_last_error()


def test_python_api_fails_loudly_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    from bitmask_speculation_b200.kernels._extension import load_extension
    load_extension.cache_clear()
    with pytest.raises(RuntimeError, match="GPU"):
        load_extension()
