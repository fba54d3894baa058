"""Tensor-level entry points over the C-ABI: activation quant, weight pre-pack, block-scaled FP8
GEMM and the fused gate_up + SiLU*up + quant front half.

All functions take CUDA tensors, launch on the current stream of the tensors' device, never
synchronise and never fall back: a tensor outside the contract raises ValueError, a library
failure raises RuntimeError.
"""
from __future__ import annotations

import torch

from . import _native

E4M3 = torch.float8_e4m3fn
BLOCK = 128


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        _need(t.is_cuda, "tensors must be on a CUDA device (this path has no CPU implementation)")
        _need(t.device == dev, "all tensors must be on the same device")
    return dev


def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def group_quant(x: torch.Tensor, group_size: int = BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    """x bf16 [..., K] -> (A e4m3 [..., K], As fp32 [..., K/128]); per 1x128 group
    As = max(amax/448, 1e-12), A = e4m3(x / As)."""
    _need(group_size == BLOCK, "only 128-wide groups are supported")
    _need(x.dtype == torch.bfloat16, "x must be bf16")
    dev = _cuda(x)
    K = x.shape[-1]
    _need(K % BLOCK == 0, "K must be a multiple of 128")
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    A = torch.empty((M, K), dtype=E4M3, device=dev)
    As = torch.empty((M, K // BLOCK), dtype=torch.float32, device=dev)
    with _native.device_guard(dev):
        _native.check(_native.lib().bs_fp8_group_quant(
            x2.data_ptr(), x2.stride(0), A.data_ptr(), As.data_ptr(), M, K, _native.stream_handle(dev)),
            "bs_fp8_group_quant")
    return A.view(*x.shape[:-1], K), As.view(*x.shape[:-1], K // BLOCK)


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """gate_up bf16 [..., 2I] -> bf16 [..., I]: silu(g) * u in fp32 with one rounding (SGLang's silu_and_mul,
    the unfused chain's activation)."""
    _need(gate_up.dtype == torch.bfloat16, "gate_up must be bf16")
    dev = _cuda(gate_up)
    n2 = gate_up.shape[-1]
    _need(n2 % 16 == 0, "gate_up width must be a multiple of 16")
    x2 = gate_up.reshape(-1, n2)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M, inter = x2.shape[0], n2 // 2
    y = torch.empty((M, inter), dtype=torch.bfloat16, device=dev)
    with _native.device_guard(dev):
        _native.check(_native.lib().bs_fp8_silu_mul(
            x2.data_ptr(), x2.stride(0), y.data_ptr(), inter, M, inter, _native.stream_handle(dev)),
            "bs_fp8_silu_mul")
    return y.view(*gate_up.shape[:-1], inter)


def rmsnorm_group_quant(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                        residual: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm fused with the per-token-group quant of its output (the next linear's activation quant):
    h = x, or h = bf16(x + residual) stored into `residual` in place (fused add); y = bf16(h * rsqrt(mean(h^2)
    + eps) * weight); returns group_quant(y) = (A e4m3 [..., K], As fp32 [..., K/128]) without storing y."""
    _need(x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16, "x and weight must be bf16")
    dev = _cuda(x, weight) if residual is None else _cuda(x, weight, residual)
    K = x.shape[-1]
    _need(K % BLOCK == 0, "K must be a multiple of 128")
    _need(weight.shape == (K,) and weight.is_contiguous(), "weight must be contiguous [K]")
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    r_ptr, ldr = None, K
    if residual is not None:
        _need(residual.dtype == torch.bfloat16 and residual.shape == x.shape, "residual must be bf16 like x")
        r2 = residual.view(-1, K)
        _need(r2.stride(-1) == 1 and r2.stride(0) % 8 == 0 and r2.data_ptr() % 16 == 0,
              "residual rows must be contiguous and 16-byte aligned (it is updated in place)")
        r_ptr, ldr = r2.data_ptr(), r2.stride(0)
    A = torch.empty((M, K), dtype=E4M3, device=dev)
    As = torch.empty((M, K // BLOCK), dtype=torch.float32, device=dev)
    with _native.device_guard(dev):
        _native.check(_native.lib().bs_fp8_rmsnorm_group_quant(
            x2.data_ptr(), x2.stride(0), r_ptr, ldr, weight.data_ptr(), float(eps), A.data_ptr(), As.data_ptr(),
            M, K, _native.stream_handle(dev)), "bs_fp8_rmsnorm_group_quant")
    return A.view(*x.shape[:-1], K), As.view(*x.shape[:-1], K // BLOCK)


def pack_tiles(weight: torch.Tensor) -> torch.Tensor:
    """e4m3 weight [N, K] -> tile-first bytes [N/128, K/128, 128, 128] (H:667 layout)."""
    _need(weight.dim() == 2 and weight.dtype in (E4M3, torch.uint8), "weight must be e4m3 [N, K]")
    dev = _cuda(weight)
    N, K = weight.shape
    _need(N % BLOCK == 0 and K % BLOCK == 0, "N and K must be multiples of 128")
    w = _as_bytes(weight.contiguous())
    tiles = torch.empty((N // BLOCK, K // BLOCK, BLOCK, BLOCK), dtype=torch.uint8, device=dev)
    with _native.device_guard(dev):
        _native.check(_native.lib().bs_fp8_pack_tiles(w.data_ptr(), tiles.data_ptr(), N, K,
                                                      _native.stream_handle(dev)), "bs_fp8_pack_tiles")
    return tiles


def _weight_geometry(B: torch.Tensor, b_tiled: bool) -> tuple[int, int]:
    if b_tiled:
        _need(B.dim() == 4 and tuple(B.shape[2:]) == (BLOCK, BLOCK) and B.dtype in (torch.uint8, E4M3),
              "tile-first weights must be [N/128, K/128, 128, 128] bytes")
        return B.shape[0] * BLOCK, B.shape[1] * BLOCK
    _need(B.dim() == 2 and B.dtype in (E4M3, torch.uint8), "row-major weights must be e4m3 [N, K]")
    return B.shape[0], B.shape[1]


def _check_operands(A, B, As, Bs, b_tiled):
    _need(A.dtype in (E4M3, torch.uint8), "A must be e4m3")
    dev = _cuda(A, B, As, Bs)
    N, K = _weight_geometry(B, b_tiled)
    _need(A.shape[-1] == K, f"A has K={A.shape[-1]}, weights have K={K}")
    A2 = A.reshape(-1, K)
    M = A2.shape[0]
    _need(As.dtype == torch.float32 and Bs.dtype == torch.float32, "scales must be fp32")
    _need(As.numel() == M * (K // BLOCK), "As must be [M, K/128]")
    _need(tuple(Bs.shape) == (N // BLOCK, K // BLOCK), "Bs must be [N/128, K/128]")
    _need(B.is_contiguous(), "weights must be contiguous")
    if not A2.is_contiguous():
        A2 = A2.contiguous()
    return dev, A2, As.reshape(M, K // BLOCK).contiguous(), Bs.contiguous(), M, N, K


def gemm(A: torch.Tensor, B: torch.Tensor, As: torch.Tensor, Bs: torch.Tensor, *, b_tiled: bool = False,
         out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """C[m, n] = sum_kb (A . B)[m, n, kb] * As[m, kb] * Bs[n/128, kb] -> out [..., N] (bf16 or fp32)."""
    dev, A2, As2, Bs2, M, N, K = _check_operands(A, B, As, Bs, b_tiled)
    if out is None:
        out = torch.empty((*A.shape[:-1], N), dtype=out_dtype, device=dev)
    _need(out.dtype in (torch.bfloat16, torch.float32), "output must be bf16 or fp32")
    _need(out.device == dev and out.shape[-1] == N and out.numel() == M * N, "output must be [..., N]")
    out2 = out.view(M, N)
    _need(out2.stride(-1) == 1, "output rows must be contiguous")
    ldc = out2.stride(0) if M > 1 else N
    lib = _native.lib()
    with _native.device_guard(dev):
        ws_bytes = lib.bs_fp8_workspace_bytes(M, N, K, 0)
        ws = _native.workspace(dev, ws_bytes)
        _native.check(lib.bs_fp8_gemm(
            A2.data_ptr(), _as_bytes(B).data_ptr(), out2.data_ptr(), As2.data_ptr(), Bs2.data_ptr(), M, N, K, ldc,
            int(b_tiled), 0 if out.dtype == torch.bfloat16 else 1, _native.ptr(ws),
            0 if ws is None else ws.numel(), _native.stream_handle(dev)), "bs_fp8_gemm")
    return out


def gemm_reduce_multicast(A: torch.Tensor, B: torch.Tensor, As: torch.Tensor, Bs: torch.Tensor, out: torch.Tensor,
                          out_multicast: int, *, b_tiled: bool = False) -> torch.Tensor:
    """Row-parallel GEMM fused with the tensor-parallel sum: this rank's bf16 product is added into every
    rank's copy of `out` through the NVSwitch multicast address `out_multicast` (the address of out[0, 0] in
    the group's multicast mapping). `out` is this rank's copy, bf16 [M, N]; every rank zeroes its copy and
    the group synchronises before the call, and again before `out` is read."""
    dev, A2, As2, Bs2, M, N, K = _check_operands(A, B, As, Bs, b_tiled)
    _need(out.dtype == torch.bfloat16, "output must be bf16 (the switch adds bf16 pairs)")
    _need(out.device == dev and out.dim() == 2 and tuple(out.shape) == (M, N), "output must be [M, N]")
    _need(out.stride(-1) == 1, "output rows must be contiguous")
    _need(isinstance(out_multicast, int) and out_multicast != 0, "a multicast address is required")
    ldc = out.stride(0) if M > 1 else N
    lib = _native.lib()
    with _native.device_guard(dev):
        ws_bytes = lib.bs_fp8_workspace_bytes(M, N, K, 0)
        ws = _native.workspace(dev, ws_bytes)
        _native.check(lib.bs_fp8_gemm_reduce_multicast(
            A2.data_ptr(), _as_bytes(B).data_ptr(), out_multicast, As2.data_ptr(), Bs2.data_ptr(), M, N, K, ldc,
            int(b_tiled), _native.ptr(ws), 0 if ws is None else ws.numel(), _native.stream_handle(dev)),
            "bs_fp8_gemm_reduce_multicast")
    return out


def tp_reduce_switch(data: torch.Tensor, data_multicast: int, flags: torch.Tensor, flags_multicast: int, rank: int,
                     world: int, epoch: int, limit_ns: int = 0) -> torch.Tensor:
    """In-place tensor-parallel sum of the ranks' bf16 partials through the NVSwitch. `data` is this rank's copy
    of a symmetric bf16 buffer (contiguous, holding its partial) and `data_multicast` the multicast address of
    data's first element; `flags` this rank's copy of a symmetric int32 buffer of flag_words(world) words zeroed
    before the first call, `flags_multicast` its multicast address. Every rank calls with the same epoch (1, 2,
    ... per call on these flags). On return every rank's `data` holds the same sums."""
    dev = _cuda(data, flags)
    _need(data.dtype == torch.bfloat16 and data.is_contiguous(), "data must be contiguous bf16")
    _need(flags.dtype == torch.int32 and flags.numel() >= tp_flag_words(world), "flags too small for this world")
    _need(data.numel() % 8 == 0, "data must hold a multiple of 8 elements")
    lib = _native.lib()
    with _native.device_guard(dev):
        _native.check(lib.bs_fp8_tp_reduce_switch(
            data_multicast, flags.data_ptr(), flags_multicast, data.numel(), rank, world, epoch, limit_ns,
            _native.stream_handle(dev)), "bs_fp8_tp_reduce_switch")
    return data


def tp_flag_words(world: int) -> int:
    """int32 words of the flag buffer tp_reduce_switch needs for `world` ranks."""
    return int(_native.lib().bs_fp8_tp_flag_words(world))


def gemm_silu_quant(A: torch.Tensor, B: torch.Tensor, As: torch.Tensor, Bs: torch.Tensor, *,
                    b_tiled: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """gate_up GEMM + SiLU(gate)*up + per-token-group quant: B holds [gate; up] (2I rows).
    Returns Q e4m3 [..., I] and Qs fp32 [..., I/128]."""
    dev, A2, As2, Bs2, M, N2, K = _check_operands(A, B, As, Bs, b_tiled)
    _need(N2 % (2 * BLOCK) == 0, "gate_up rows must be a multiple of 256")
    inter = N2 // 2
    Q = torch.empty((*A.shape[:-1], inter), dtype=E4M3, device=dev)
    Qs = torch.empty((*A.shape[:-1], inter // BLOCK), dtype=torch.float32, device=dev)
    lib = _native.lib()
    with _native.device_guard(dev):
        ws_bytes = lib.bs_fp8_workspace_bytes(M, N2, K, 1)
        ws = _native.workspace(dev, ws_bytes)
        _native.check(lib.bs_fp8_gemm_silu_quant(
            A2.data_ptr(), _as_bytes(B).data_ptr(), Q.data_ptr(), As2.data_ptr(), Bs2.data_ptr(), Qs.data_ptr(),
            M, N2, K, int(b_tiled), _native.ptr(ws), 0 if ws is None else ws.numel(),
            _native.stream_handle(dev)), "bs_fp8_gemm_silu_quant")
    return Q, Qs
