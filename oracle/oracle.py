"""CPU oracle for the block-scaled FP8 linear path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module, and
only as the checker or the timed CPU reference, never as the product path.

It restates, in torch-CPU / numpy code, the reference's own CPU-runnable arithmetic of the path
(lexing-2026/ucloud-ai-infra; "H" = patches/fp8_hand_sm89.py):

  quant_block        scripts/fp8_gemm_factor_check.py:22-27 (same as scripts/fp8_gemm_variants.py:121-128
                     and the lm_head quantiser, patches/apply_sglang_fp8_lm_head.py:66-75)
  ref_matmul         logs/artifacts/20261030_48g/C/infer/bench_gemm.py:19-24 (dequantise, fp32 matmul)
  blockwise_matmul   the hand kernel's arithmetic, H:189-199 and H:275-280: one fp32 partial per
                     128-K block, S = fp32(a_s * b_s), C = fma(partial, S, C)
  silu_quant         the fused epilogue, H:532-579: y = silu(g) * u, scale = max(amax, 1e-10) / 448,
                     inv = 1 / scale, q = sat_e4m3(y * inv)
  relayout_tiles     the tile-first pre-pack, H:667
  rmsnorm_group_quant  RMSNorm fused with the group quant, as the reference fuses it into its GDN output
                     norm (patches/apply_sglang_gdn_prefill.py:538-591), with the bf16 rounding of the
                     unfused norm output and the library kernel's summation order
  make_*             the seeded input generators of the north-star configs (weights N(0, 0.02)
                     quantised per 128x128 block, activations N(0, 1) quantised per 1x128 group,
                     optionally 1% of rows scaled x50), following scripts/fp8_gemm_factor_check.py:53-61

Parity pin: tests/golden/make_golden.py runs the reference's own functions (quant,
quant_block, ref_matmul, relayout) in this container and commits their outputs; tests check this
module against them. The fused epilogue exists in the reference only as sm_89 PTX, so it is
pinned by restatement (H:532-579) and by the reference's torch pieces it is built from.
"""
from __future__ import annotations

import numpy as np
import torch

FP8_MAX = 448.0
BLOCK = 128
E4M3 = torch.float8_e4m3fn


# ----------------------------------------------------------------------------- quantisers
def quant_block(x: torch.Tensor, rows: int, cols: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Max-abs e4m3 quant per (rows x cols) block in fp32: s = max(amax / 448, 1e-12),
    q = e4m3(x / s). rows=1, cols=128 is the per-token-group activation quant."""
    x = x.float()
    R, C = x.shape
    s = x.abs().reshape(R // rows, rows, C // cols, cols).amax(dim=(1, 3)) / FP8_MAX
    s = s.clamp_min(1e-12)
    full = s.repeat_interleave(rows, 0).repeat_interleave(cols, 1)
    return (x / full).to(E4M3), s


def group_quant(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Activation quant, 1 x 128 groups."""
    return quant_block(x, 1, BLOCK)


def rmsnorm_group_quant(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """RMSNorm then the per-token-group quant, with the rounding points of the unfused pair (the bf16 norm
    output, then quant_block) and the library kernel's fixed fp32 summation order for sum(h^2), which
    depends on K only. A row belongs to 256 threads (eight warps); thread t holds the 16-byte chunks
    c = t + 256 j and keeps two partial sums, of its even and of its odd elements: for its chunks in
    increasing c and e = 0..3, even += h[8c + 2e]^2 and odd += h[8c + 2e + 1]^2 (each square rounded, then
    each add); its total is even + odd; each 32-thread warp combines its threads in a butterfly (xor 16, 8, 4,
    2, 1); the row's sum is the eight warp totals added in warp order.
    rs = 1 / sqrt(ss / K + eps) in IEEE fp32; y = bf16((h * rs) * w).
    With residual: h = bf16(x + residual), which is also returned (the fused add writes it back).
    Returns (A, As, h_bf16 or None)."""
    xf = x.float()
    h = (xf + residual.float()).to(torch.bfloat16).float() if residual is not None else xf
    M, K = h.shape
    nch = K // 8
    W = 8
    T = 32 * W
    hn = h.numpy().astype(np.float32)
    sq = (hn * hn).astype(np.float32)  # fp32 products, rounded once
    even = np.zeros((M, T), dtype=np.float32)
    odd = np.zeros((M, T), dtype=np.float32)
    tid = np.arange(T)
    for j in range((nch + T - 1) // T):
        c = T * j + tid
        live = c < nch
        for e in range(4):
            ce = np.where(live, c * 8 + 2 * e, 0)
            even = np.where(live[None, :], even + sq[:, ce], even).astype(np.float32)
            odd = np.where(live[None, :], odd + sq[:, ce + 1], odd).astype(np.float32)
    threads = (even + odd).astype(np.float32)
    warps = threads.reshape(M, W, 32)
    lane = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        warps = (warps + warps[:, :, lane ^ o]).astype(np.float32)
    ss = warps[:, 0, 0]
    for i in range(1, W):
        ss = (ss + warps[:, i, 0]).astype(np.float32)
    rs = np.float32(1) / np.sqrt((ss / np.float32(K) + np.float32(eps)).astype(np.float32))
    rs_t = torch.from_numpy(rs.astype(np.float32))
    y = ((h * rs_t[:, None]) * weight.float()[None, :]).to(torch.bfloat16)
    A, As = quant_block(y.float(), 1, BLOCK)
    return A, As, (h.to(torch.bfloat16) if residual is not None else None)


def weight_quant(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Weight quant, 128 x 128 blocks."""
    return quant_block(w, BLOCK, BLOCK)


# ----------------------------------------------------------------------------- GEMMs
def dequant(A: torch.Tensor, As: torch.Tensor, rows: int) -> torch.Tensor:
    """e4m3 [R, K] with per (rows x 128) scales -> fp32."""
    R, K = A.shape
    full = As.float().repeat_interleave(rows, 0)[:R].repeat_interleave(BLOCK, 1)
    return A.float() * full


def ref_matmul(A: torch.Tensor, B: torch.Tensor, As: torch.Tensor, Bs: torch.Tensor) -> torch.Tensor:
    """The reference's torch oracle: dequantise both operands, fp32 matmul."""
    M, K = A.shape
    N = B.shape[0]
    Ad = (A.float().view(M, K // BLOCK, BLOCK) * As[..., None]).reshape(M, K)
    Bd = (B.float().view(N // BLOCK, BLOCK, K // BLOCK, BLOCK) * Bs[:, None, :, None]).reshape(N, K)
    return Ad @ Bd.T


def blockwise_matmul(A: torch.Tensor, B: torch.Tensor, As: torch.Tensor, Bs: torch.Tensor) -> torch.Tensor:
    """The hand kernel's per-block arithmetic in fp32: for each 128-K block the partial P is the exact
    dot product rounded once to fp32 (products of e4m3 values are exact, and the sum is taken in
    fp64), S = fp32(a_s * b_s), then C = fp32(P * S + C) with a single rounding (fma)."""
    M, K = A.shape
    N = B.shape[0]
    KB = K // BLOCK
    Ad = A.double().view(M, KB, BLOCK)
    Bd = B.double().view(N, KB, BLOCK)
    acc = torch.zeros(M, N, dtype=torch.float32)
    bs_full = Bs.float().repeat_interleave(BLOCK, 0)  # [N, KB]
    for kb in range(KB):
        P = (Ad[:, kb, :] @ Bd[:, kb, :].T).float()
        S = As[:, kb].float()[:, None] * bs_full[:, kb][None, :]  # fp32 product, rounded once
        acc = (P.double() * S.double() + acc.double()).float()
    return acc


# ----------------------------------------------------------------------------- fused epilogue
def to_e4m3_sat(v: torch.Tensor) -> torch.Tensor:
    """fp32 -> e4m3, round to nearest even, saturating to +-448 (cvt.rn.satfinite)."""
    return v.clamp(-FP8_MAX, FP8_MAX).to(E4M3)


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """y = (g * (1 / (1 + e^-g))) * u in fp32, each step rounded as the kernel does."""
    g = g.float().numpy()
    u = u.float().numpy()
    with np.errstate(over="ignore"):
        t = np.float32(1.0) / (np.float32(1.0) + np.exp(-g, dtype=np.float32))
    y = (g * t).astype(np.float32) * u
    return torch.from_numpy(y.astype(np.float32))


def silu_quant(g: torch.Tensor, u: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused epilogue on fp32 accumulators g, u [M, I]: returns (Q e4m3 [M, I], Qs fp32 [M, I/128], y)."""
    y = silu_mul(g, u)
    M, inter = y.shape
    yg = y.view(M, inter // BLOCK, BLOCK)
    amax = yg.abs().amax(dim=-1)
    scale = torch.clamp(amax, min=1e-10) / torch.tensor(FP8_MAX, dtype=torch.float32)
    inv = torch.tensor(1.0, dtype=torch.float32) / scale
    q = to_e4m3_sat(yg * inv[..., None]).view(M, inter)
    return q, scale, y


def fused_gate_up(A, B, As, Bs) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused MLP front half on the kernel's fp32 accumulators: B = [gate; up] (2I rows)."""
    acc = blockwise_matmul(A, B, As, Bs)
    inter = B.shape[0] // 2
    return silu_quant(acc[:, :inter], acc[:, inter:])


def chain_gate_up(A, B, As, Bs) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The unfused chain the fused kernel replaces (restated from
    logs/artifacts/20261031_hand/fused_test.py:30-34): bf16 GEMM output, silu(g)*u, then the
    per-token-group quant of that bf16 y."""
    c = ref_matmul(A, B, As, Bs).to(torch.bfloat16)
    inter = B.shape[0] // 2
    g, u = c[:, :inter].float(), c[:, inter:].float()
    y = (torch.nn.functional.silu(g) * u).to(torch.bfloat16)
    q, s = group_quant(y)
    return q, s, y


# ----------------------------------------------------------------------------- layouts
def relayout_tiles(w_bytes: torch.Tensor) -> torch.Tensor:
    """Tile-first pre-pack of an e4m3/uint8 weight [N, K] -> [N/128, K/128, 128, 128] bytes."""
    N, K = w_bytes.shape
    u8 = w_bytes.view(torch.uint8) if w_bytes.dtype != torch.uint8 else w_bytes
    return u8.reshape(N // BLOCK, BLOCK, K // BLOCK, BLOCK).permute(0, 2, 1, 3).contiguous()


# ----------------------------------------------------------------------------- seeded inputs
def make_weight(N: int, K: int, seed: int, std: float = 0.02) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 N(0, std) weight [N, K], quantised per 128x128 block -> (e4m3 [N, K], fp32 [N/128, K/128])."""
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * std).to(torch.bfloat16)
    return weight_quant(w)


def make_activation(M: int, K: int, seed: int, outlier_frac: float = 0.0,
                    outlier_scale: float = 50.0) -> torch.Tensor:
    """bf16 N(0, 1) activations [M, K]; a fraction of rows scaled by `outlier_scale`."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    n_out = int(round(outlier_frac * M))
    if n_out:
        rows = torch.randperm(M, generator=g)[:n_out]
        x[rows] *= outlier_scale
    return x.to(torch.bfloat16)


def make_gemm_case(M: int, N: int, K: int, seed: int = 0, outlier_frac: float = 0.0):
    """Seeded (A, B, As, Bs, x) for one block-FP8 GEMM."""
    B, Bs = make_weight(N, K, seed)
    x = make_activation(M, K, seed + 1, outlier_frac)
    A, As = group_quant(x)
    return A, B, As, Bs, x


# ----------------------------------------------------------------------------- comparisons
def max_rel_error(out: torch.Tensor, ref: torch.Tensor, floor_frac: float = 1e-3) -> float:
    """max |out - ref| / max(|ref|, floor_frac * max|ref|) (relative error with the floor of
    logs/artifacts/20261031_hand/bench_hand.py:75 scaled to the output's range)."""
    out = out.float()
    ref = ref.float()
    floor = floor_frac * ref.abs().max().clamp_min(1e-30)
    return ((out - ref).abs() / torch.maximum(ref.abs(), floor)).max().item()


def norm_rel_error(out: torch.Tensor, ref: torch.Tensor) -> float:
    out = out.float()
    ref = ref.float()
    return ((out - ref).norm() / ref.norm().clamp_min(1e-30)).item()


def e4m3_ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|ordinal(a) - ordinal(b)| over e4m3 bit patterns (sign-magnitude -> monotone ordinal)."""
    def ordinal(t):
        u = t.view(torch.uint8).to(torch.int32)
        mag = u & 0x7F
        return torch.where(u & 0x80 != 0, -mag, mag)
    return (ordinal(a) - ordinal(b)).abs()
