"""Installs this path's three hooks into an SGLang tree, as the reference's installer does for its sm_89
module (patches/apply_sglang_fp8_hand_gemm.py:68-114).

    python -m fp8_hand_b200.install_sglang [--root /path/to/site-packages/sglang] [--no-build]

The same three call sites are edited, each only if its original text occurs exactly once:

  kernels/ops/gemm/fp8_kernel.py   w8a8_block_fp8_matmul_triton tries `matmul` first, after C is allocated
                                   (reference hook :26-33, import :34-38)
  srt/models/qwen2_moe.py          the MLP forward takes the fused gate_up + SiLU*up + quant front half
                                   (reference :39-56)
  srt/model_loader/loader.py       the loader moves FP8 weights to tile-first storage after loading
                                   (reference :59-65)

Differences from the reference installer: the hooks import this package (`fp8_hand_b200`, which must be
importable by SGLang's python, e.g. through PYTHONPATH) under the reference's module name `fp8_hand_sm89`,
instead of a module file copied into the SGLang tree; and the build step compiles the sm_100a library
(`precompile()`) instead of running ptxas on generated PTX. A file that already names the module is
reported and left alone, so running the installer twice changes nothing.
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from dataclasses import dataclass
from pathlib import Path

MODULE_IMPORT = "from fp8_hand_b200 import fp8_hand_sm100 as fp8_hand_sm89\n"
MARK = "fp8_hand_b200"


@dataclass(frozen=True)
class Edit:
    old: str
    new: str


# SGLang 0.5.22 source lines at each site (the text the reference's installer matches) and their hooked form.
GEMM_FILE = "kernels/ops/gemm/fp8_kernel.py"
GEMM_EDITS = (
    Edit("    M, N, K, C = prepare_block_fp8_matmul_inputs(A, B, As, Bs, block_size, output_dtype)\n"
         "\n"
         "    block_n, block_k = block_size\n",
         "    M, N, K, C = prepare_block_fp8_matmul_inputs(A, B, As, Bs, block_size, output_dtype)\n"
         "\n"
         "    if fp8_hand_sm89.matmul(A, B, C, As, Bs, M, N, K, block_size):\n"
         "        return C\n"
         "\n"
         "    block_n, block_k = block_size\n"),
    Edit("from sglang.srt.layers import deep_gemm_wrapper\n",
         MODULE_IMPORT + "from sglang.srt.layers import deep_gemm_wrapper\n"),
)
MLP_FILE = "srt/models/qwen2_moe.py"
MLP_EDITS = (
    Edit("        x,\n"
         "    ):\n"
         "        gate_up, _ = self.gate_up_proj(x)\n"
         "        if self._enable_silu_fp4_quant_fusion and not isinstance(gate_up, tuple):\n",
         "        x,\n"
         "    ):\n"
         "        " + MODULE_IMPORT +
         "\n"
         "        fused = fp8_hand_sm89.fused_gate_up(self.gate_up_proj, x)\n"
         "        if fused is not None:\n"
         "            x, _ = self.down_proj(fused)\n"
         "            return x\n"
         "        gate_up, _ = self.gate_up_proj(x)\n"
         "        if self._enable_silu_fp4_quant_fusion and not isinstance(gate_up, tuple):\n"),
)
LOADER_FILE = "srt/model_loader/loader.py"
LOADER_EDITS = (
    Edit("        maybe_quantize_lm_head(model)\n",
         "        maybe_quantize_lm_head(model)\n"
         "        " + MODULE_IMPORT +
         "\n"
         "        fp8_hand_sm89.relayout(model)\n"),
)
SITES = ((GEMM_FILE, GEMM_EDITS), (MLP_FILE, MLP_EDITS), (LOADER_FILE, LOADER_EDITS))


class InstallError(RuntimeError):
    """An SGLang file whose text does not match the site the hook belongs at."""


def sglang_root() -> Path:
    spec = importlib.util.find_spec("sglang")
    if spec is None or spec.origin is None:
        raise InstallError("sglang is not importable by this python; pass --root")
    return Path(spec.origin).parent


def patch_file(path: Path, edits: tuple[Edit, ...]) -> str:
    """Applies every edit to `path` (each original text must occur exactly once). Returns "patched" or
    "already patched"; raises InstallError and leaves the file untouched when a site does not match."""
    text = path.read_text()
    if MARK in text:
        return "already patched"
    for e in edits:
        n = text.count(e.old)
        if n != 1:
            raise InstallError(f"{path}: expected one match of the hook site, found {n}")
    for e in edits:
        text = text.replace(e.old, e.new)
    path.write_text(text)
    return "patched"


def install(root: Path, build: bool = True, log=print) -> dict[str, str]:
    """Patches the three sites under `root` (the `sglang` package directory) and, with build=True,
    compiles the library. Every site is checked before any file is written."""
    root = Path(root)
    for rel, edits in SITES:
        path = root / rel
        if not path.exists():
            raise InstallError(f"{path} does not exist")
        text = path.read_text()
        if MARK not in text:
            for e in edits:
                if text.count(e.old) != 1:
                    raise InstallError(f"{path}: expected one match of the hook site, found {text.count(e.old)}")
    result = {}
    for rel, edits in SITES:
        result[rel] = patch_file(root / rel, edits)
        log(f"{result[rel]}: {root / rel}")
    if build:
        from . import fp8_hand_sm100
        log(f"precompiled: {fp8_hand_sm100.precompile()}")
    return result


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--root", type=Path, default=None, help="the sglang package directory (default: import it)")
    ap.add_argument("--no-build", action="store_true", help="skip compiling the sm_100a library")
    a = ap.parse_args(argv)
    try:
        install(a.root if a.root is not None else sglang_root(), build=not a.no_build)
    except InstallError as e:
        print(str(e), file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
