"""Generates the golden fixtures that pin the CPU oracle to the reference's own code.

Runs only where the reference checkout exists (this build container); the GPU box and the tests
read the committed outputs, never the reference. Usage:

    python tests/golden/make_golden.py [--ref /path/to/reference]

What it executes from the reference (lexing-2026/ucloud-ai-infra), unmodified:
  * patches/fp8_hand_sm89.py, imported as a module (it needs only torch): `relayout` on a small
    CPU model with the sm_89 capability check answered "yes", and `select`;
  * `quant` from scripts/fp8_gemm_factor_check.py:22-27, `quant_block` from
    scripts/fp8_gemm_variants.py:121-128 and `ref_matmul` from
    logs/artifacts/20261030_48g/C/infer/bench_gemm.py:19-24. Those scripts import SGLang at module
    level (not installed here), so each function's own source is lifted out with `ast` and
    executed on its own with the globals it reads (torch, FP8_MAX, FP8).
Outputs: golden.npz (arrays) and golden.json (metadata, hashes, the reference select table).
"""
from __future__ import annotations

import argparse
import os
import ast
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
FP8_MAX = 448.0


def lift_function(path: Path, name: str, globs: dict):
    """Executes only the `def name(...)` of a reference source file and returns the function."""
    tree = ast.parse(path.read_text(), filename=str(path))
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            mod = ast.Module(body=[node], type_ignores=[])
            ns = dict(globs)
            exec(compile(mod, str(path), "exec"), ns)
            return ns[name]
    raise KeyError(f"{name} not found in {path}")


def import_hand_module(ref: Path):
    spec = importlib.util.spec_from_file_location("fp8_hand_sm89_reference", ref / "patches/fp8_hand_sm89.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def seeded_bf16(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BS_FP8_REFERENCE_TREE"),
                    help="checkout of lexing-2026/ucloud-ai-infra (default: $BS_FP8_REFERENCE_TREE)")
    a = ap.parse_args()
    if not a.ref:
        print("pass --ref (or set BS_FP8_REFERENCE_TREE) to the reference checkout", file=sys.stderr)
        return 1
    ref = Path(a.ref)
    if not (ref / "patches/fp8_hand_sm89.py").exists():
        print(f"reference not found at {ref}", file=sys.stderr)
        return 1

    quant = lift_function(ref / "scripts/fp8_gemm_factor_check.py", "quant", {"torch": torch, "FP8_MAX": FP8_MAX})
    quant_block = lift_function(ref / "scripts/fp8_gemm_variants.py", "quant_block",
                                {"torch": torch, "FP8_MAX": FP8_MAX, "FP8": torch.float8_e4m3fn})
    ref_matmul = lift_function(ref / "logs/artifacts/20261030_48g/C/infer/bench_gemm.py", "ref_matmul",
                               {"torch": torch})

    out: dict[str, np.ndarray] = {}
    meta: dict = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__}

    # ---- activation quant (1 x 128) incl. edge rows: zeros, x50 outliers, tiny, large
    M, K, N = 6, 512, 256
    x = seeded_bf16((M, K), 11)
    x[1] = 0
    x[2] *= 50
    x[3] *= 1e-30
    x[4, :128] = 3.0e4
    x[5, 5] = -448.0
    xf = x.float()
    A, As = quant(xf, 1, 128)
    A2, As2 = quant_block(xf, 1, 128)
    assert torch.equal(A.view(torch.uint8), A2.view(torch.uint8)) and torch.equal(As, As2)
    out["act_x_bf16_bits"] = x.view(torch.int16).numpy()
    out["act_q_bits"] = A.view(torch.uint8).numpy()
    out["act_scale"] = As.numpy()

    # ---- weight quant (128 x 128) of N(0, 0.02)
    w = seeded_bf16((N, K), 12, std=0.02)
    B, Bs = quant(w.float(), 128, 128)
    B2, Bs2 = quant_block(w.float(), 128, 128)
    assert torch.equal(B.view(torch.uint8), B2.view(torch.uint8)) and torch.equal(Bs, Bs2)
    out["w_bf16_bits"] = w.view(torch.int16).numpy()
    out["w_q_bits"] = B.view(torch.uint8).numpy()
    out["w_scale"] = Bs.numpy()

    # ---- the reference's torch GEMM oracle on those operands (rows 1..5 only: row 0 regular)
    C = ref_matmul(A, B, As, Bs)
    out["gemm_ref_out"] = C.numpy()

    # ---- tile-first relayout by the reference module itself
    H = import_hand_module(ref)
    H.ENABLED = True
    H.torch.cuda.get_device_capability = lambda *args, **kw: (8, 9)
    H.torch.cuda.empty_cache = lambda: None

    class Lin(torch.nn.Module):
        def __init__(self, n, k, seed):
            super().__init__()
            rng = np.random.default_rng(seed)
            raw = torch.from_numpy(rng.integers(0, 256, size=(n, k), dtype=np.uint8))
            self.weight = torch.nn.Parameter(raw.view(torch.float8_e4m3fn), requires_grad=False)
            self.weight_scale_inv = torch.nn.Parameter(torch.ones(n // 128, k // 128), requires_grad=False)

    model = torch.nn.Module()
    model.proj = Lin(256, 5120, 21)          # eligible in the reference (K = 5120)
    model.small_k = Lin(256, 512, 22)        # K not in the reference's KS: left alone there
    model.lm_head = Lin(256, 5120, 23)       # lm_head: always left alone
    raw = {n: m.weight.detach().view(torch.uint8).clone() for n, m in model.named_children()}
    H.relayout(model)
    meta["relayout"] = {}
    for name, mod in model.named_children():
        tiles = getattr(mod.weight, "tiles", None)
        entry = {"shape": list(raw[name].shape), "seed": {"proj": 21, "small_k": 22, "lm_head": 23}[name],
                 "moved": tiles is not None}
        if tiles is not None:
            t = tiles.contiguous().numpy()
            entry["tiles_shape"] = list(t.shape)
            entry["tiles_sha256"] = hashlib.sha256(t.tobytes()).hexdigest()
            entry["weight_device"] = str(mod.weight.device)
            out[f"relayout_{name}_first_tile"] = t[0, 0]
            out[f"relayout_{name}_last_tile"] = t[-1, -1]
        meta["relayout"][name] = entry

    # ---- the reference's sm_89 tile table (informational; the B200 tiles differ by design)
    meta["select_sm89"] = {f"{n}x{m}": H.select(n, m) for n in (5120, 10240, 34816) for m in (1, 8, 16, 32, 112, 128, 129, 8192)}
    meta["env_defaults_sm89"] = {"ENABLED": "0", "FUSED": "1", "FUSED_MIN_M": str(H.FUSED_MIN_M)}

    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "golden.npz", HERE / "golden.json")
    return 0


if __name__ == "__main__":
    sys.exit(main())
