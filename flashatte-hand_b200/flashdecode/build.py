"""Build the sm_100a shared library ``libflashdecode_sm100.so`` in-tree.

``python -m flashdecode.build`` (with ``flashatte-hand_b200`` on sys.path) or
``build()`` compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` and links
them into ``flashdecode/libflashdecode_sm100.so``.  nvcc cross-compiles, so
this runs on a machine without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT_DIR = PKG_DIR.parent  # flashatte-hand_b200/
CSRC = ROOT_DIR / "csrc"
INCLUDE = ROOT_DIR.parent / "include"
BUILD_DIR = ROOT_DIR / "_build"
LIB_NAME = "libflashdecode_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr"]


def nvcc_path() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                  + list(INCLUDE.glob("*.h")))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    lib_m = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= lib_m for p in _deps())


def _compile(nvcc: str, src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose), srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
