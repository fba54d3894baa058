"""ctypes binding of libbs_fp8_sm100.so (declared in include/bs_fp8.h).

The reference drives its cubins through libcuda with ctypes (patches/fp8_hand_sm89.py:614-649);
this module plays that role for the sm_100a library: it loads the in-tree .so, declares the
C signatures, turns non-zero status codes into RuntimeError (the reference raises RuntimeError
on driver failures, H:630, :634, :649) and launches on torch's current stream.

There is no fallback: if the library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

from . import _build

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

BS_OK = 0
BS_ERR_TIMEOUT_SELFTEST = 199

# (name, restype, argtypes) for every symbol of include/bs_fp8.h
_VP, _I, _SZ, _U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64
SIGNATURES = {
    "bs_fp8_gemm": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _VP, _SZ, _VP]),
    "bs_fp8_gemm_silu_quant": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP, _SZ, _VP]),
    "bs_fp8_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "bs_fp8_gemm_noalloc": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _VP]),
    "bs_fp8_gemm_reduce_multicast": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP, _SZ, _VP]),
    "bs_fp8_group_quant": (_I, [_VP, _I, _VP, _VP, _I, _I, _VP]),
    "bs_fp8_rmsnorm_group_quant": (_I, [_VP, _I, _VP, _I, _VP, ctypes.c_float, _VP, _VP, _I, _I, _VP]),
    "bs_fp8_pack_tiles": (_I, [_VP, _VP, _I, _I, _VP]),
    "bs_fp8_silu_mul": (_I, [_VP, _I, _VP, _I, _I, _I, _VP]),
    "bs_fp8_tp_reduce_switch": (_I, [_U64, _VP, _U64, ctypes.c_longlong, _I, _I, ctypes.c_uint, _U64, _VP]),
    "bs_fp8_tp_flag_words": (ctypes.c_longlong, [_I]),
    "bs_fp8_status": (_I, [ctypes.POINTER(_I), _I]),
    "bs_fp8_selftest_wait_timeout": (_I, [_U64, _VP]),
    "bs_fp8_launch_plan": (_I, [_I, _I, _I, _I, ctypes.POINTER(_I), _I]),
    "bs_fp8_num_sms": (_I, []),
    "bs_fp8_error_string": (ctypes.c_char_p, [_I]),
    "bs_fp8_abi_version": (_I, []),
    "bs_fp8_last_cuda_error": (ctypes.c_char_p, []),
}
ABI_VERSION = 1


def library_path() -> Path:
    return _build.LIB_PATH


def lib() -> ctypes.CDLL:
    """The loaded library. Raises when it has not been built (no silent fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = library_path()
            if not path.exists():
                raise RuntimeError(
                    f"{path} is missing; build it with `python -m fp8_hand_b200._build` "
                    "(or __graft_entry__.build()). There is no CPU or Triton fallback.")
            handle = ctypes.CDLL(str(path))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            if handle.bs_fp8_abi_version() != ABI_VERSION:
                raise RuntimeError(f"{path}: ABI version {handle.bs_fp8_abi_version()} != {ABI_VERSION}")
            _LIB = handle
    return _LIB


def error_string(code: int) -> str:
    return lib().bs_fp8_error_string(int(code)).decode()


def check(rc: int, what: str) -> None:
    if rc != BS_OK:
        detail = lib().bs_fp8_last_cuda_error().decode() if rc == 5 else ""
        raise RuntimeError(f"{what}: {error_string(rc)} (status {rc}){': ' + detail if detail else ''}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _DeviceGuard:
    """Makes `device` current for the C library (which launches on cudaGetDevice())."""

    def __init__(self, device: torch.device):
        self.index = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def device_guard(device: torch.device) -> _DeviceGuard:
    return _DeviceGuard(device)


# ------------------------------------------------------------------ workspace
# Decode kernels hand partial tiles between CTAs through a caller-owned workspace whose counter
# words must be zero before first use; the kernels leave them at zero. One buffer per
# (device, stream), grown on demand. Calls that overlap on different streams each get their own.
_WS: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    key = (device.index, stream_handle(device))
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def reset_workspaces() -> None:
    """Zero every cached workspace (needed only after a kernel reported a timeout)."""
    for buf in _WS.values():
        buf.zero_()


PLAN_FIELDS = ("kind", "tile_rows", "tile_cols", "stages", "threads", "grid", "cluster", "group_m", "reserved",
               "tmem_cols", "split", "warpgroups", "smem_bytes", "tiles")  # include/bs_fp8.h BS_PLAN_*


def launch_plan(M: int, N: int, K: int, fused: bool) -> dict:
    """What the library launches for an M x N x K GEMM (fused: the gate_up front half) on the current device."""
    buf = (ctypes.c_int * len(PLAN_FIELDS))()
    check(lib().bs_fp8_launch_plan(int(M), int(N), int(K), int(bool(fused)), buf, len(PLAN_FIELDS)),
          "bs_fp8_launch_plan")
    return dict(zip(PLAN_FIELDS, list(buf)))


def num_sms() -> int:
    return lib().bs_fp8_num_sms()


def status(clear: bool = True) -> int:
    """Device status word of the current device (synchronises)."""
    code = ctypes.c_int(0)
    check(lib().bs_fp8_status(ctypes.byref(code), int(clear)), "bs_fp8_status")
    return code.value
