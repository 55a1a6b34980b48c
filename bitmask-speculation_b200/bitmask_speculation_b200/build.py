"""Build the sm_100a shared library in-tree with nvcc.

The library (``_lib/libbms_b200.so``) exports the C ABI of ``include/bms_b200.h``;
it is compiled ahead of time for ``sm_100a`` only (no JIT, no other targets) and
links the CUDA runtime statically, so it depends on the driver alone.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
SOURCE_ROOT = PACKAGE.parent / "csrc"
INCLUDE = PACKAGE.parents[1] / "include"
LIBRARY = PACKAGE / "_lib" / "libbms_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def sources() -> list[Path]:
    return sorted(p for p in SOURCE_ROOT.iterdir() if p.suffix in {".cu", ".cuh", ".h"}) + [
        INCLUDE / "bms_b200.h"]


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build the library")
    return found


def stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(p.stat().st_mtime > built for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``csrc/bms_abi.cu`` into ``_lib/libbms_b200.so`` if stale."""
    if not force and not stale():
        return LIBRARY
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIBRARY.with_suffix(f".{os.getpid()}.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp),
           str(SOURCE_ROOT / "bms_abi.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force=True, verbose=True))
