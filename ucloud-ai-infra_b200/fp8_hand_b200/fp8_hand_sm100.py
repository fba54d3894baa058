"""Drop-in B200 (sm_100a) counterpart of the reference's patches/fp8_hand_sm89.py.

Same surface, same meaning, so the three SGLang hooks installed by
patches/apply_sglang_fp8_hand_gemm.py (:26-33 GEMM entry, :45-56 MLP forward, :59-65 loader) can
import this module instead:

  ENABLED / FUSED_ENABLED / FUSED_MIN_M   env switches SGLANG_FP8_HAND_GEMM, SGLANG_FP8_HAND_FUSED,
                                          SGLANG_FP8_HAND_FUSED_MIN_M (H:41-43)
  select(N, M) -> dict                    tile choice of an M x N product (H:74-81)
  precompile() -> list[str]               build step, never on the request path (H:596-611)
  relayout(model, cache=None)             tile-first weight pre-pack after loading (H:652-672); with a
                                          cache file (tilepack.py) the packed tiles are read, not permuted
  fused_gate_up(proj, x) -> (Q, Qs)|None  fused MLP front half (H:675-701)
  matmul(A, B, C, As, Bs, M, N, K, block_size) -> bool   GEMM hook (H:704-719)

Differences that follow from the hardware, not from the API:
  * the capability gate is sm_100 (B200) instead of sm_89;
  * any K and N that are multiples of 128 are eligible (the reference compiled cubins for
    K in {5120, 6144, 17408} only, H:46 and H:664);
  * the fused kernel covers every M, so FUSED_MIN_M defaults to 1 (the reference defaults to
    1024 because its fused kernel lost to the 3-kernel chain below M=1024 on the 4090);
  * the activation quant that feeds the fused kernel is this library's CUDA kernel instead of
    SGLang's Triton per_token_group_quant_fp8 (H:690-693).
"""
from __future__ import annotations

import logging
import os

import torch
from torch.nn import Parameter

from . import _build, _native, ops, tilepack

logger = logging.getLogger(__name__)

ENABLED = os.getenv("SGLANG_FP8_HAND_GEMM", "0") == "1"
FUSED_ENABLED = ENABLED and os.getenv("SGLANG_FP8_HAND_FUSED", "1") == "1"
FUSED_MIN_M = int(os.getenv("SGLANG_FP8_HAND_FUSED_MIN_M", "1"))

BK = 128
CAPABILITY = (10, 0)
DECODE_MAX_M = 128           # M <= 128 runs the swap-AB split-K kernel


def select(N: int, M: int, K: int = 5120, fused: bool = False) -> dict:
    """The kernel an M x N product (K deep; fused: the gate_up front half, N = 2I) launches, read from the
    library's own launch plan (bs_fp8_launch_plan), so the values are the ones that run: the reference's
    select(N, M) reported its sm_89 tile the same way (H:74-81). Keys:
      kind       "decode" (M <= 128: swap-AB, the weights are the MMA's 128-row side, tokens its N side)
                 or "prefill" (persistent tcgen05 tiles)
      BM, BN, BK tile: decode 128 weight rows x NTP tokens; prefill 128 or 256 (CTA pairs) rows x 256 columns
      NTP        decode: tokens padded to a multiple of 16
      stages, threads, grid, cluster, tmem_cols, smem_bytes, warpgroups (promotion)
      split      decode: "tile" (one CTA per weight tile), "k<s>" (s equal K splits) or "stream-k"; prefill:
                 "tile" (whole output tiles) or "stream-k" (plain GEMMs whose tiles would fill the last wave
                 less than 90 %; it runs when the call has the workspace bs_fp8_workspace_bytes reports)
      group_m    prefill raster: M tiles per group (the group's activation rows stay in L2)
    """
    p = _native.launch_plan(M, N, K, fused)
    out = dict(BK=BK, stages=p["stages"], threads=p["threads"], grid=p["grid"], cluster=p["cluster"],
               tmem_cols=p["tmem_cols"], smem_bytes=p["smem_bytes"], warpgroups=p["warpgroups"])
    if p["kind"] == 1:
        split = {0: "tile", -1: "stream-k"}.get(p["split"], f"k{p['split']}")
        out.update(kind="decode", BM=p["tile_rows"], BN=p["tile_cols"], NTP=p["tile_cols"], split=split)
    else:
        out.update(kind="prefill", BM=p["tile_rows"], BN=p["tile_cols"], group_m=p["group_m"], tiles=p["tiles"],
                   split="stream-k" if p["split"] == -1 else "tile")
    return out


def precompile() -> list[str]:
    """Builds the sm_100a library (only when a source is newer than the build)."""
    return [str(_build.build())]


def _is_b200() -> bool:
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == CAPABILITY


def eligible(name: str, weight: torch.Tensor, scale: torch.Tensor | None) -> bool:
    """Weights this path takes over at relayout time: e4m3 [N, K] with a [N/128, K/128] fp32 block
    scale, N and K multiples of 128; lm_head stays where it is, as in H:661."""
    if scale is None or weight is None or weight.dtype != torch.float8_e4m3fn or "lm_head" in name:
        return False
    if weight.dim() != 2:
        return False
    N, K = weight.shape
    return N % BK == 0 and K % BK == 0 and tuple(scale.shape) == (N // BK, K // BK)


def relayout(model: torch.nn.Module, cache: str | os.PathLike | None = None) -> None:
    """Moves every eligible FP8 linear to tile-first storage. The parameter keeps its shape on the
    meta device, so nothing can read the old layout by accident (H:652-672).

    cache: a tile-pack file (tilepack.py). Entries it holds are read from it instead of being packed, so
    their row-major weights need not be loaded at all (a weight on the meta device is fine); their block
    scales must equal the module's weight_scale_inv. If the file does not exist, the packed weights are
    written to it."""
    if not ENABLED or not _is_b200():
        return
    stored = tilepack.read_header(cache)["entries"] if cache is not None and os.path.exists(cache) else None
    todo = []
    for name, module in model.named_modules():
        weight = getattr(module, "weight", None)
        scale = getattr(module, "weight_scale_inv", None)
        if weight is None or getattr(weight, "tiles", None) is not None:
            continue
        if not eligible(name, weight, scale):
            if isinstance(weight, torch.Tensor) and weight.dtype == torch.float8_e4m3fn:
                logger.info("FP8 hand: %s %s stays on the row-major path", name, tuple(weight.shape))
            continue
        todo.append((name, module))
    cached = {}
    if stored is not None:
        names = [name for name, module in todo
                 if name in stored and (stored[name]["N"], stored[name]["K"]) == tuple(module.weight.shape)]
        if names:
            cached = tilepack.load(cache, device=todo[0][1].weight_scale_inv.device, names=names)
    packed = {}
    for name, module in todo:
        N, K = module.weight.shape
        if name in cached:
            tiles, scale = cached.pop(name)
            if not torch.equal(scale, module.weight_scale_inv.data):
                raise tilepack.TilePackError(f"{name}: block scales in {cache} differ from the loaded weight_scale_inv")
        else:
            if module.weight.device.type == "meta":
                raise tilepack.TilePackError(f"{name}: weight not loaded and not in the tile cache {cache}")
            tiles = ops.pack_tiles(module.weight.data)
            packed[name] = (tiles, module.weight_scale_inv.data)
        module.weight = Parameter(torch.empty(N, K, dtype=torch.float8_e4m3fn, device="meta"), requires_grad=False)
        module.weight.tiles = tiles
    if cache is not None and stored is None and packed:
        tilepack.save(cache, packed)
    torch.cuda.empty_cache()
    logger.info("FP8 hand: %d linears tile first (%d from %s)", len(todo), len(todo) - len(packed), cache)


def fused_gate_up(proj, x):
    """Returns (q, scale) for down_proj, or None to run the separate kernels (H:675-701).

    x is the bf16 activation [M, K], or an already quantised (A e4m3 [M, K], As fp32 [M, K/128]) pair, e.g.
    from ops.rmsnorm_group_quant, in the (fp8, scale) tuple form the reference hands between its hooks
    (patches/apply_sglang_gdn_prefill.py:578-589)."""
    pre = isinstance(x, tuple)
    if pre:
        if len(x) != 2 or x[0].dtype != torch.float8_e4m3fn or x[0].ndim != 2:
            return None
        rows = x[0].shape[0]
    else:
        if x.dtype != torch.bfloat16 or x.ndim != 2:
            return None
        rows = x.shape[0]
    if not FUSED_ENABLED or rows < FUSED_MIN_M:
        return None
    weight = getattr(proj, "weight", None)
    scale = getattr(proj, "weight_scale_inv", None)
    tiles = getattr(weight, "tiles", None)
    if tiles is None or scale is None or scale.ndim != 2:
        return None
    N, K = weight.shape
    if K % BK or N % (2 * BK) or getattr(proj, "bias", None) is not None:
        return None
    A, As = x if pre else ops.group_quant(x, BK)
    return ops.gemm_silu_quant(A, tiles, As, scale, b_tiled=True)


def matmul(A, B, C, As, Bs, M, N, K, block_size) -> bool:
    """Launches C = A @ B^T and returns True, or returns False for a weight that was not
    relayouted (H:704-719). C may be bf16 (the reference's only output) or fp32."""
    tiles = getattr(B, "tiles", None)
    if tiles is None:
        return False
    if block_size is not None and list(block_size) != [BK, BK]:
        raise ValueError(f"block_size {block_size}: only [128, 128] weight blocks exist on this path")
    if tiles.shape[0] * BK != N or tiles.shape[1] * BK != K:
        raise ValueError(f"tiles {tuple(tiles.shape)} do not match N={N}, K={K}")
    ops.gemm(A, tiles, As, Bs, b_tiled=True, out=C, out_dtype=C.dtype)
    return True


def status(clear: bool = True) -> int:
    """Device status word (0 = no kernel reported a bounded-wait timeout); synchronises."""
    return _native.status(clear)
