"""CPU: the C-ABI library's surface and the host-side logic of the drop-in module (no GPU work)."""
import ctypes
import importlib
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "bs_fp8.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*[\w\s\*]+?\b(bs_fp8_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from fp8_hand_b200 import _build, _native
    _build.build()
    return _native.lib()


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    nm = subprocess.run(["nm", "-D", "--defined-only", str(lib._name)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (bs_fp8_\w+)", nm))
    assert set(names) <= exported


def test_binding_covers_header():
    from fp8_hand_b200 import _native
    assert set(declared_functions()) == set(_native.SIGNATURES)


def test_abi_version_and_error_strings(lib):
    assert lib.bs_fp8_abi_version() == 1
    for code in (0, 1, 2, 3, 4, 5, 6, 7, 101, 102, 103, 104, 105, 199):
        text = lib.bs_fp8_error_string(code).decode()
        assert text and text != "unknown status code"
    assert lib.bs_fp8_error_string(12345).decode() == "unknown status code"


def test_argument_validation_needs_no_gpu(lib):
    s = None
    # K not a multiple of 128, N not a multiple of 128, ldc < N, bad dtype code: all rejected up front
    assert lib.bs_fp8_gemm(None, None, None, None, None, 4, 256, 200, 256, 0, 0, None, 0, s) == 1
    assert lib.bs_fp8_gemm(None, None, None, None, None, 4, 200, 256, 256, 0, 0, None, 0, s) == 1
    assert lib.bs_fp8_gemm(None, None, None, None, None, 4, 256, 256, 128, 0, 0, None, 0, s) == 1
    assert lib.bs_fp8_gemm(None, None, None, None, None, 4, 256, 256, 256, 0, 7, None, 0, s) == 1
    assert lib.bs_fp8_gemm(None, None, None, None, None, 4, 256, 256, 256, 2, 0, None, 0, s) == 1
    assert lib.bs_fp8_gemm_silu_quant(None, None, None, None, None, None, 4, 384, 256, 0, None, 0, s) == 1
    # M == 0 is a no-op that touches nothing
    assert lib.bs_fp8_gemm(None, None, None, None, None, 0, 256, 256, 256, 0, 0, None, 0, s) == 0
    assert lib.bs_fp8_group_quant(None, 256, None, None, 0, 256, s) == 0
    assert lib.bs_fp8_group_quant(None, 256, None, None, 4, 200, s) == 1
    assert lib.bs_fp8_pack_tiles(None, None, 100, 128, s) == 1
    assert lib.bs_fp8_rmsnorm_group_quant(None, 256, None, 256, None, 1e-6, None, None, 0, 256, s) == 0
    assert lib.bs_fp8_rmsnorm_group_quant(None, 256, None, 256, None, 1e-6, None, None, 4, 200, s) == 1
    assert lib.bs_fp8_rmsnorm_group_quant(None, 256, None, 256, None, -1.0, None, None, 4, 256, s) == 1
    assert lib.bs_fp8_rmsnorm_group_quant(None, 256, None, 256, None, 1e-6, None, None, 4, 256, s) == 1
    assert lib.bs_fp8_rmsnorm_group_quant(None, 17408, None, 17408, None, 1e-6, None, None, 4, 17408, s) == 1
    # null pointers with a real shape
    assert lib.bs_fp8_gemm(None, None, None, None, None, 4, 256, 256, 256, 0, 0, None, 0, s) == 1
    # the unfused chain's SiLU*up: width a multiple of 8, strides covering the rows; M == 0 a no-op
    assert lib.bs_fp8_silu_mul(None, 16, None, 8, 0, 8, s) == 0
    assert lib.bs_fp8_silu_mul(None, 24, None, 12, 4, 12, s) == 1
    assert lib.bs_fp8_silu_mul(None, 8, None, 8, 4, 8, s) == 1
    assert lib.bs_fp8_silu_mul(None, 16, None, 8, 4, 8, s) == 1  # null pointers with a real shape
    # the switch reduction: at least two ranks, rank in range, a whole number of 16-byte vectors, both multicast
    # addresses and the flags, a nonzero epoch; then 16-byte / 4-byte alignment
    ok_args = dict(data_mc=1 << 20, flags=1 << 20, flags_mc=1 << 21, count=8, rank=0, world=2, epoch=1)

    def switch(**kw):
        a = {**ok_args, **kw}
        return lib.bs_fp8_tp_reduce_switch(a["data_mc"], a["flags"], a["flags_mc"], a["count"], a["rank"],
                                           a["world"], a["epoch"], 0, s)
    assert switch(world=1) == 1 and switch(rank=2) == 1 and switch(rank=-1) == 1 and switch(count=12) == 1
    assert switch(data_mc=0) == 1 and switch(flags=None) == 1 and switch(flags_mc=0) == 1 and switch(epoch=0) == 1
    assert switch(data_mc=(1 << 20) + 8) == 2 and switch(flags_mc=(1 << 21) + 2) == 2
    assert switch(flags=(1 << 20) + 4) == 2
    assert lib.bs_fp8_tp_flag_words(1) == 0 and lib.bs_fp8_tp_flag_words(8) == 2 * 256 * 8
    # the multicast-reduction GEMM: the same shape rules (bf16 output only), M == 0 a no-op
    assert lib.bs_fp8_gemm_reduce_multicast(None, None, None, None, None, 0, 256, 256, 256, 0, None, 0, s) == 0
    assert lib.bs_fp8_gemm_reduce_multicast(None, None, None, None, None, 4, 256, 200, 256, 0, None, 0, s) == 1
    assert lib.bs_fp8_gemm_reduce_multicast(None, None, None, None, None, 4, 256, 256, 128, 0, None, 0, s) == 1
    assert lib.bs_fp8_gemm_reduce_multicast(None, None, None, None, None, 4, 256, 256, 256, 3, None, 0, s) == 1
    assert lib.bs_fp8_gemm_reduce_multicast(None, None, None, None, None, 4, 256, 256, 256, 0, None, 0, s) == 1


def _decode_grid(sms, tiles, kb):
    """One CTA per tile when tiles nearly match the SMs (>= 90%); s equal K splits per tile when that fills
    >= 95% of the SMs; else one CTA per SM (stream-K)."""
    if tiles <= sms and 10 * tiles >= 9 * sms:
        return tiles
    if tiles < sms:
        s = sms // tiles
        if 2 <= s <= kb and 20 * tiles * s >= 19 * sms:
            return tiles * s
    return min(sms, tiles * kb)


def _decode_ws(M, N, K, fused, sms):
    """A fixed 64 KB prefix of per-tile counters (the same for every shape), then the partial tiles."""
    tiles = N // 256 if fused else N // 128
    ntp = (M + 15) // 16 * 16
    return 65536 + _decode_grid(sms, tiles, K // 128) * 2 * (2 if fused else 1) * ntp * 128 * 4


def test_workspace_size_formula(lib):
    # decode shapes need counters + G * 2 * nwg * ntp * 128 floats; prefill shapes need none
    assert lib.bs_fp8_workspace_bytes(129, 256, 256, 0) == 0
    assert lib.bs_fp8_workspace_bytes(0, 256, 256, 0) == 0
    sms = lib.bs_fp8_num_sms() or 148
    for M, N, K, fused in [(1, 34816, 5120, 1), (112, 34816, 5120, 1), (128, 6144, 5120, 0), (5, 384, 17408, 0),
                           (3, 128, 256, 0)]:
        assert lib.bs_fp8_workspace_bytes(M, N, K, fused) == _decode_ws(M, N, K, fused, sms), (M, N, K, fused)
    assert lib.bs_fp8_workspace_bytes(1, 34816, 5120, 1) < lib.bs_fp8_workspace_bytes(112, 34816, 5120, 1)


def _fresh_module(monkeypatch, **env):
    for k in ("SGLANG_FP8_HAND_GEMM", "SGLANG_FP8_HAND_FUSED", "SGLANG_FP8_HAND_FUSED_MIN_M"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    import fp8_hand_b200.fp8_hand_sm100 as m
    return importlib.reload(m)


def test_env_switch_semantics(monkeypatch):
    m = _fresh_module(monkeypatch)
    assert (m.ENABLED, m.FUSED_ENABLED, m.FUSED_MIN_M) == (False, False, 1)
    m = _fresh_module(monkeypatch, SGLANG_FP8_HAND_GEMM="1")
    assert (m.ENABLED, m.FUSED_ENABLED) == (True, True)
    m = _fresh_module(monkeypatch, SGLANG_FP8_HAND_GEMM="1", SGLANG_FP8_HAND_FUSED="0")
    assert (m.ENABLED, m.FUSED_ENABLED) == (True, False)
    m = _fresh_module(monkeypatch, SGLANG_FP8_HAND_GEMM="1", SGLANG_FP8_HAND_FUSED_MIN_M="1024")
    assert m.FUSED_MIN_M == 1024
    _fresh_module(monkeypatch)


def test_select_tiles(lib):
    """select() reports the library's launch plan: the kernel, block and grid that actually run."""
    from fp8_hand_b200 import select
    sms = lib.bs_fp8_num_sms() or 148
    d = select(34816, 1, fused=True)
    assert d["kind"] == "decode" and d["NTP"] == 16 and d["threads"] == 384 and d["warpgroups"] == 2
    assert d["split"] == "tile" and d["grid"] == 136  # 136 gate/up tile pairs: one CTA each
    assert select(34816, 112, fused=True)["NTP"] == 112
    assert select(34816, 56, fused=True)["threads"] == 640  # four promotion warpgroups at 48..80 tokens
    assert select(5120, 1, K=17408)["threads"] == 256 and select(5120, 56, K=17408)["threads"] == 384
    assert select(5120, 1, K=17408)["split"] == "stream-k" and select(5120, 1, K=17408)["grid"] == sms
    assert select(6144, 128)["kind"] == "decode"
    assert 2 <= select(6144, 128)["stages"] <= 12
    p = select(34816, 129)
    assert p["kind"] == "prefill" and (p["BM"], p["BN"]) == (128, 256) and p["cluster"] == 1
    f = select(34816, 8192, fused=True)  # CTA pairs from 1024 rows, every M tile in one raster group
    assert (f["BM"], f["cluster"], f["group_m"], f["tiles"]) == (256, 2, 32, 32 * 136)
    assert f["grid"] == 2 * min(sms // 2, f["tiles"]) and f["stages"] == 6 and f["tmem_cols"] == 512
    dn = select(5120, 8192, K=17408)  # activation panel 142.6 MB > L2: groups of 2048 rows
    assert (dn["group_m"], dn["BM"]) == (16, 128) and dn["split"] == "tile"  # 1280 tiles: 8.6 full waves
    # 160 tiles would leave the second wave 8 % full: stream-K, with a workspace of two partial tiles per CTA
    assert select(5120, 1024, K=17408)["split"] == "stream-k" and f["split"] == "tile"
    assert lib.bs_fp8_workspace_bytes(1024, 5120, 17408, 0) == 65536 + sms * 2 * 128 * 256 * 4
    assert lib.bs_fp8_workspace_bytes(8192, 5120, 17408, 0) == 0 and lib.bs_fp8_workspace_bytes(1024, 34816, 5120, 1) == 0
    big = select(248320, 8192, K=5120)  # activation panel fits in L2: one group
    assert big["group_m"] == 64
    with pytest.raises(RuntimeError):
        select(34816 + 128, 8192, fused=True)  # fused N2 must be a multiple of 256


class _Proj(torch.nn.Module):
    def __init__(self, n, k, tiles=True):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.empty(n, k, dtype=torch.float8_e4m3fn, device="meta"),
                                         requires_grad=False)
        if tiles:
            self.weight.tiles = torch.empty(n // 128, k // 128, 128, 128, dtype=torch.uint8)
        self.weight_scale_inv = torch.nn.Parameter(torch.ones(n // 128, k // 128), requires_grad=False)
        self.bias = None


def test_dropin_fallback_contract(monkeypatch):
    """matmul -> False without tiles; fused_gate_up -> None when disabled, too small or ineligible.
    None of these reach the GPU."""
    m = _fresh_module(monkeypatch, SGLANG_FP8_HAND_GEMM="1", SGLANG_FP8_HAND_FUSED_MIN_M="64")
    x = torch.zeros(8, 256, dtype=torch.bfloat16)
    assert m.fused_gate_up(_Proj(512, 256), x) is None                  # M < FUSED_MIN_M
    assert m.fused_gate_up(_Proj(512, 256, tiles=False), torch.zeros(64, 256, dtype=torch.bfloat16)) is None
    assert m.fused_gate_up(_Proj(384, 256), torch.zeros(64, 256, dtype=torch.bfloat16)) is None  # N % 256
    assert m.fused_gate_up(_Proj(512, 256), torch.zeros(64, 256)) is None  # not bf16
    q8 = torch.zeros(8, 256, dtype=torch.float8_e4m3fn)
    assert m.fused_gate_up(_Proj(512, 256), (q8, torch.ones(8, 2))) is None  # pre-quantised, M < FUSED_MIN_M
    assert m.fused_gate_up(_Proj(512, 256), (q8.view(torch.uint8), torch.ones(8, 2))) is None  # not e4m3
    w = torch.empty(256, 256, dtype=torch.float8_e4m3fn)
    assert m.matmul(None, w, None, None, None, 8, 256, 256, [128, 128]) is False
    m = _fresh_module(monkeypatch, SGLANG_FP8_HAND_GEMM="1", SGLANG_FP8_HAND_FUSED="0")
    assert m.fused_gate_up(_Proj(512, 256), torch.zeros(4096, 256, dtype=torch.bfloat16)) is None
    _fresh_module(monkeypatch)


def test_relayout_is_noop_off_b200(monkeypatch):
    m = _fresh_module(monkeypatch, SGLANG_FP8_HAND_GEMM="1")
    model = torch.nn.Module()
    model.proj = torch.nn.Linear(128, 128, bias=False)
    model.proj.weight = torch.nn.Parameter(torch.zeros(128, 128).to(torch.float8_e4m3fn), requires_grad=False)
    model.proj.weight_scale_inv = torch.nn.Parameter(torch.ones(1, 1), requires_grad=False)
    before = model.proj.weight
    m.relayout(model)   # no B200 here: nothing changes
    assert model.proj.weight is before and getattr(model.proj.weight, "tiles", None) is None
    _fresh_module(monkeypatch)


def test_eligibility_rules():
    from fp8_hand_b200 import fp8_hand_sm100 as m
    w = torch.empty(256, 384, dtype=torch.float8_e4m3fn)
    s = torch.ones(2, 3)
    assert m.eligible("layers.0.mlp.gate_up_proj", w, s)
    assert not m.eligible("lm_head", w, s)
    assert not m.eligible("x", w, torch.ones(2, 2))
    assert not m.eligible("x", torch.empty(256, 384, dtype=torch.bfloat16), s)
    assert not m.eligible("x", torch.empty(200, 384, dtype=torch.float8_e4m3fn), torch.ones(1, 3))


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: the product path rejects host tensors loudly."""
    from fp8_hand_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.group_quant(torch.zeros(4, 128, dtype=torch.bfloat16))
    A = torch.zeros(4, 128, dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gemm(A, torch.zeros(128, 128, dtype=torch.float8_e4m3fn), torch.ones(4, 1), torch.ones(1, 1))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from fp8_hand_b200 import _native
    monkeypatch.setattr(_native, "_LIB", None)
    monkeypatch.setattr(_native, "library_path", lambda: tmp_path / "absent.so")
    with pytest.raises(RuntimeError, match="no CPU or Triton fallback"):
        _native.lib()


def test_build_command_targets_sm100a():
    from fp8_hand_b200 import _build
    flags = " ".join(_build.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags and "-lineinfo" in flags
