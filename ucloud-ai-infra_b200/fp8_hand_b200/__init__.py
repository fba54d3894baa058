"""B200-native (sm_100a) block-scaled FP8 linear path: a drop-in for the reference's
patches/fp8_hand_sm89.py behind SGLang's w8a8_block_fp8_matmul / Fp8LinearMethod entry.

    import fp8_hand_b200 as fp8_hand_sm89     # same functions and env switches

Modules:
  fp8_hand_sm100   the drop-in surface (relayout, matmul, fused_gate_up, select, precompile)
  ops              tensor-level kernels (group quant, pack, GEMM, fused gate_up)
  sglang_compat    stand-ins for the SGLang call sites the hooks live in
  tp               tensor-parallel MLP over NCCL
"""
from .fp8_hand_sm100 import (  # noqa: F401
    BK, ENABLED, FUSED_ENABLED, FUSED_MIN_M, fused_gate_up, matmul, precompile, relayout, select, status)
