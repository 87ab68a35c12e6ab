"""Build recipe for the in-tree CUDA library ``fast_infer_b200/libfast_infer_b200.so``.

Compiles every ``csrc/*.cu`` for sm_100a with nvcc (one process per file, in
parallel) and links them into one shared library exposing the C ABI declared in
``include/fast_infer_b200.h``. The library links the CUDA runtime statically and
reaches the driver API (tensor-map encoding) through cudaGetDriverEntryPoint, so
it has no link-time dependency on libcuda or on torch.

    python -m fast_infer_b200.build            # or __graft_entry__.build()
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_NAME = "libfast_infer_b200.so"
LIB_PATH = PKG / LIB_NAME
BUILD_DIR = ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build fast_infer_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(objs: list[Path]) -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    deps.append(Path(__file__))
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library if any source is newer than it. Returns its path."""
    srcs = sources()
    BUILD_DIR.mkdir(exist_ok=True)
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    if not force and not _stale(objs):
        return LIB_PATH
    nvcc = _nvcc()

    def compile_one(src_obj):
        src, obj = src_obj
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-Xptxas", "-v", "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        logs = list(ex.map(compile_one, zip(srcs, objs)))
    if verbose:
        for s, log in zip(srcs, logs):
            print(f"--- {s.name}\n{log}")
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
