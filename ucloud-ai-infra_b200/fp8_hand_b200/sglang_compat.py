"""Stand-ins for the SGLang call sites the reference hooks into (SGLang 0.5.22 is not part of this
repository). They reproduce the three hook points of patches/apply_sglang_fp8_hand_gemm.py so the
drop-in module is exercised exactly as SGLang would call it:

  w8a8_block_fp8_matmul(A, B, As, Bs, block_size, output_dtype)   GEMM entry; the reference's hook
      `if fp8_hand_sm89.matmul(A, B, C, As, Bs, M, N, K, block_size): return C` sits after C is
      allocated (:26-33). Weights that were not relayouted run this library's row-major kernel
      where SGLang would run Triton.
  Fp8BlockLinear.forward(x)                                       Fp8LinearMethod.apply: activation
      quant then the GEMM entry; a pre-quantised (q, scale) tuple skips the quant, which is how
      the fused output reaches down_proj (:50-53).
  GatedMLP.forward(x)                                             the patched MLP forward (:45-56).
  post_load(model)                                                the loader hook (:59-65).
"""
from __future__ import annotations

import torch
from torch import nn

from . import fp8_hand_sm100 as fp8_hand
from . import ops

BLOCK = 128


def per_token_group_quant_fp8(x: torch.Tensor, group_size: int = BLOCK):
    """SGLang's activation quant entry (called at H:690-693): (A e4m3, As fp32 [..., K/128])."""
    return ops.group_quant(x, group_size)


def w8a8_block_fp8_matmul(A, B, As, Bs, block_size, output_dtype=torch.bfloat16):
    """SGLang's block-FP8 GEMM entry with the reference's hook in place."""
    N, K = B.shape
    M = A.numel() // A.shape[-1]
    C = torch.empty((*A.shape[:-1], N), dtype=output_dtype, device=A.device)
    if fp8_hand.matmul(A, B, C, As, Bs, M, N, K, block_size):
        return C
    if list(block_size) != [BLOCK, BLOCK]:
        raise ValueError(f"block_size {block_size}: only [128, 128] weight blocks exist on this path")
    return ops.gemm(A, B, As, Bs, b_tiled=False, out=C, out_dtype=output_dtype)


class Fp8BlockLinear(nn.Module):
    """Linear layer with block-FP8 weights, the shape of SGLang's Fp8LinearMethod-backed linear:
    weight e4m3 [N, K], weight_scale_inv fp32 [N/128, K/128]; forward returns (out, bias)."""

    def __init__(self, weight: torch.Tensor, weight_scale_inv: torch.Tensor, bias: torch.Tensor | None = None):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.weight_scale_inv = nn.Parameter(weight_scale_inv, requires_grad=False)
        self.bias = bias

    def forward(self, x):
        if isinstance(x, tuple):
            q, s = x
            out_dtype = torch.bfloat16
        else:
            q, s = per_token_group_quant_fp8(x.view(-1, x.shape[-1]), BLOCK)
            out_dtype = x.dtype
        out = w8a8_block_fp8_matmul(q, self.weight, s, self.weight_scale_inv, [BLOCK, BLOCK], out_dtype)
        if not isinstance(x, tuple):
            out = out.view(*x.shape[:-1], -1)
        return out, self.bias


def silu_and_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """The unfused chain's activation (SGLang silu_and_mul): only reached when the fused kernel is
    switched off (SGLANG_FP8_HAND_FUSED=0) or ineligible. Runs the library's kernel (bs_fp8_silu_mul)."""
    from . import ops
    return ops.silu_mul(gate_up)


class GatedMLP(nn.Module):
    """gate_up_proj -> SiLU(gate) * up -> down_proj with the reference's patched forward."""

    def __init__(self, gate_up_proj: Fp8BlockLinear, down_proj: Fp8BlockLinear):
        super().__init__()
        self.gate_up_proj = gate_up_proj
        self.down_proj = down_proj

    def forward(self, x):
        fused = fp8_hand.fused_gate_up(self.gate_up_proj, x)
        if fused is not None:
            x, _ = self.down_proj(fused)
            return x
        gate_up, _ = self.gate_up_proj(x)
        x, _ = self.down_proj(silu_and_mul(gate_up))
        return x


def post_load(model: nn.Module, cache=None) -> None:
    """Loader post-hook (apply_sglang_fp8_hand_gemm.py:59-65): tile-first pre-pack, read from the
    tile-pack file `cache` when it exists (written there otherwise)."""
    fp8_hand.relayout(model, cache=cache)
