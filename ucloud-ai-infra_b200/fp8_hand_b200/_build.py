"""Builds libbs_fp8_sm100.so in-tree with nvcc for sm_100a.

The reference compiles generated PTX with ptxas at install time (patches/fp8_hand_sm89.py:596-611);
here the whole C-ABI library is one nvcc translation unit, built once, never on the request path.

    python -m fp8_hand_b200._build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT_DIR = PKG_DIR.parent                      # ucloud-ai-infra_b200/
CSRC = ROOT_DIR / "csrc"
INCLUDE = ROOT_DIR.parent / "include"
LIB_NAME = "libbs_fp8_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME
MAIN_SOURCE = CSRC / "bs_capi.cu"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library when it is missing or older than a source; returns its path."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(MAIN_SOURCE)]
    proc = subprocess.run(cmd, cwd=str(CSRC), capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    (PKG_DIR / "build.log").write_text(" ".join(cmd) + "\n" + log)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{log[-4000:]}")
    if verbose:
        print(log)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
