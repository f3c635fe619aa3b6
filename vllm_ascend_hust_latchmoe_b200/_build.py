"""Build liblatchmoe_b200.so in-tree with nvcc for sm_100a (B200).

The library is a plain C-ABI shared object (no torch types cross its boundary); the
package loads it with ctypes. It is built next to this file so that it travels with the
source tree; nothing is installed into site-packages.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_NAME = "liblatchmoe_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

NVCC_FLAGS = (
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-shared",
    "-Xcompiler",
    "-fPIC",
)


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs_mtime() -> float:
    paths = _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    return max(p.stat().st_mtime for p in paths)


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return str(cand)
    raise RuntimeError("nvcc not found: set NVCC or put /usr/local/cuda/bin on PATH")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ into one shared library (skipped when up to date)."""
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= _inputs_mtime():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{INCLUDE}", "-o", str(tmp), *map(str, _sources())]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
