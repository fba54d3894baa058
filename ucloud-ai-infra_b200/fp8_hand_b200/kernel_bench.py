"""Per-kernel timing of the block-FP8 path (the B200 counterpart of the reference's
logs/artifacts/20261031_hand/bench_hand.py). Also the command that ncu captures run, so each
case launches only the kernels it names after its warm-up.

    python -m fp8_hand_b200.kernel_bench --case fused --M 8192 [--N 34816] [--K 5120] [--iters 20]
    python -m fp8_hand_b200.kernel_bench --case gemm  --M 8192 --N 5120 --K 17408
    python -m fp8_hand_b200.kernel_bench --case quant --M 8192 --K 5120
    python -m fp8_hand_b200.kernel_bench --case all          # the config tables, one JSON line each

Weights are larger than L2 for every config shape, so repeated launches stream them from HBM.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch

from . import ops

HBM_DEFAULT = 6558.4


def _weights(N, K, device, seed=0):
    g = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn(N, K, device=device, generator=g) * 0.02).to(torch.bfloat16).float()
    s = w.abs().reshape(N // 128, 128, K // 128, 128).amax(dim=(1, 3)) / 448.0
    s = s.clamp_min(1e-12)
    q = (w / s.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(torch.float8_e4m3fn)
    return ops.pack_tiles(q), s.contiguous()


def _acts(M, K, device, seed=1):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
    return ops.group_quant(x)


def _time(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def run_case(case, M, N, K, warmup, iters, device, hbm):
    if case == "quant":
        g = torch.Generator(device=device).manual_seed(3)
        x = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
        ms = _time(lambda: ops.group_quant(x), warmup, iters)
        nbytes = M * K * 3 + M * K / 128 * 4
        return dict(case=case, M=M, K=K, ms=round(ms, 5), GBs=round(nbytes / ms / 1e6, 1),
                    frac_hbm=round(nbytes / ms / 1e6 / hbm, 3))
    tiles, s = _weights(N, K, device)
    A, As = _acts(M, K, device)
    if case == "fused":
        fn = lambda: ops.gemm_silu_quant(A, tiles, As, s, b_tiled=True)  # noqa: E731
        out_bytes = M * N / 2 + 4 * M * N / 256
    else:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=device)
        fn = lambda: ops.gemm(A, tiles, As, s, b_tiled=True, out=out)  # noqa: E731
        out_bytes = 2 * M * N
    ms = _time(fn, warmup, iters)
    flops = 2.0 * M * N * K
    nbytes = M * K + N * K + 4 * M * K / 128 + 4 * (N / 128) * (K / 128) + out_bytes
    return dict(case=case, M=M, N=N, K=K, ms=round(ms, 5), TFLOPs=round(flops / ms / 1e9, 1),
                GBs=round(nbytes / ms / 1e6, 1), frac_hbm=round(nbytes / ms / 1e6 / hbm, 3))


ALL = (
    [("gemm", 128, 6144, 5120)]                                                   # config 1
    + [("fused", m, 34816, 5120) for m in (1, 8, 14, 56, 112)]                    # config 2
    + [("fused", m, 34816, 5120) for m in (1024, 4096, 8192)]                     # config 3
    + [("gemm", m, 5120, 17408) for m in (1, 112, 1024, 4096, 8192)]              # down_proj
    + [("gemm", 8192, 10240, 5120), ("gemm", 8192, 5120, 6144), ("gemm", 8192, 34816, 5120)]  # config 4
    + [("gemm", m, 248320, 5120) for m in (1, 112)]                               # lm_head
    + [("quant", m, 0, 5120) for m in (112, 8192)]
)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=("fused", "gemm", "quant", "all"), default="fused")
    ap.add_argument("--M", type=int, default=8192)
    ap.add_argument("--N", type=int, default=34816)
    ap.add_argument("--K", type=int, default=5120)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--hbm", type=float, default=HBM_DEFAULT)
    a = ap.parse_args(argv)
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cases = ALL if a.case == "all" else [(a.case, a.M, a.N, a.K)]
    for case, M, N, K in cases:
        print(json.dumps(run_case(case, M, N, K, a.warmup, a.iters, device, a.hbm)), flush=True)
        torch.cuda.empty_cache()
    return 0


if __name__ == "__main__":
    sys.exit(main())
