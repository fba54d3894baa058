"""GPU: bs_fp8_gemm_noalloc, the GEMM entry point for callers that cannot call cudaMalloc.

Such callers (an engine that reserves all device memory at start-up and allows no allocation
afterwards, an embedding that may only use its own arena, a thread that must not block on the
driver's allocator) cannot hand the decode kernel a workspace. This entry point runs the same
kernels with the split-K scratch held in a fixed array inside the library. Its results must equal
those of the ordinary entry point (which takes a caller-allocated workspace), on two calls in a
row, since the second call reuses whatever the first left in the shared array.

Collected last (file name), so a run that stops at the first failure has run everything else.
"""
import ctypes

import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GEMM_MAX_REL = 1e-2  # the bf16 GEMM bar used by tests/test_gpu_kernels.py
BS_ERR_SCRATCH = 7


def _call_noalloc(lib, A, B, As, Bs, C, b_tiled=0):
    M, K = A.shape
    N = C.shape[1]
    return lib.bs_fp8_gemm_noalloc(A.data_ptr(), B.data_ptr(), C.data_ptr(), As.data_ptr(), Bs.data_ptr(), M, N, K,
                                   C.stride(0), b_tiled, 0, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,N,K", [(16, 1024, 2048), (5, 384, 17408), (1, 256, 512), (200, 512, 1024)])
def test_noalloc_matches_workspace_entry_point(M, N, K):
    from fp8_hand_b200 import _build, _native, ops
    _build.build()
    lib = _native.lib()
    A, B, As, Bs, _ = O.make_gemm_case(M, N, K, seed=M + N + K, outlier_frac=0.05)
    Ad, Bd, Asd, Bsd = (t.cuda() for t in (A, B, As, Bs))
    expected = ops.gemm(Ad, Bd, Asd, Bsd)  # ordinary entry point, caller-owned workspace
    for _ in range(2):
        C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _call_noalloc(lib, Ad, Bd, Asd, Bsd, C) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(C.float()).all()
        assert O.max_rel_error(C.cpu(), expected.cpu()) <= GEMM_MAX_REL
    ref = O.blockwise_matmul(A, B, As, Bs)
    assert O.max_rel_error(C.cpu(), ref) <= GEMM_MAX_REL


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from fp8_hand_b200 import _build, _native
    _build.build()
    lib = _native.lib()
    M, N, K = 128, 6144, 5120  # split-K scratch for this shape is far above the 4 MiB array
    A = torch.zeros(M, K, dtype=torch.float8_e4m3fn, device="cuda")
    B = torch.zeros(N, K, dtype=torch.float8_e4m3fn, device="cuda")
    As = torch.ones(M, K // 128, device="cuda")
    Bs = torch.ones(N // 128, K // 128, device="cuda")
    C = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    rc = _call_noalloc(lib, A, B, As, Bs, C)
    assert rc == BS_ERR_SCRATCH
    assert "4 MiB" in lib.bs_fp8_error_string(rc).decode()
    assert (C == 0).all()
