"""GPU parity of every kernel against the CPU oracle (seeded inputs, identical bytes on both sides).

Bars (the parity bars this path is held to):
  * byte kernels (group quant, tile pack): bit-exact;
  * bf16 GEMM outputs: max relative error <= 1e-2 against the fp32-accumulated oracle, with the
    relative floor 1e-3 * max|ref| (logs/artifacts/20261031_hand/bench_hand.py:75 style);
  * fused e4m3 outputs: at most 0.1% of elements differ, none by more than 1 e4m3 ulp;
    group scales within 1e-6 relative.
"""
import ctypes

import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GEMM_MAX_REL = 1e-2
Q_ULP = 1
Q_FRAC = 1e-3
SCALE_REL = 1e-6


def _ops():
    from fp8_hand_b200 import ops
    return ops


def _dev(*ts):
    return [t.cuda() for t in ts]


# --------------------------------------------------------------------------- byte kernels
@pytest.mark.parametrize("M,K", [(1, 128), (7, 512), (128, 5120), (301, 1024), (33, 17408)])
def test_group_quant_bit_exact(cuda_lib, M, K):
    x = O.make_activation(M, K, seed=M + K, outlier_frac=0.1)
    x[0, :128] = 0
    if M > 2:
        x[1, 3] = 3.0e4
        x[2] *= 1e-30
    A, As = _ops().group_quant(x.cuda())
    qr, sr = O.group_quant(x)
    assert torch.equal(A.cpu().view(torch.uint8), qr.view(torch.uint8))
    assert torch.equal(As.cpu(), sr)


@pytest.mark.parametrize("order", ["sorted", "shuffled"])
def test_group_quant_every_bf16_value(cuda_lib, order):
    """Every finite bf16 value quantised in 128-groups whose maximum is the group's own largest value or up to
    2^5 above it: bytes and scales equal the oracle's quantiser (IEEE division x / s; the kernel divides with
    a correctly rounded reciprocal and one correction step). Sorted groups hold values of similar magnitude,
    so their quotients cover the whole e4m3 range."""
    vals = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    finite = vals[torch.isfinite(vals.float())].float()
    g = torch.Generator().manual_seed(5)
    body = finite[finite.abs().argsort()] if order == "sorted" else finite[torch.randperm(len(finite), generator=g)]
    n = len(body) // 127 * 127
    body = body[:n].view(-1, 127)
    gmax = body.abs().amax(dim=1, keepdim=True)
    shift = torch.randint(0, 6, gmax.shape, generator=g).float()
    shift = torch.where(gmax > 1e36, torch.zeros_like(shift), shift)
    lead = gmax * torch.exp2(shift) * torch.where(torch.rand(gmax.shape, generator=g) < 0.5, -1.0, 1.0)
    x = torch.cat([lead, body], dim=1).to(torch.bfloat16)
    rows = x.shape[0] // 4 * 4
    x = x[:rows].reshape(rows // 4, 512)
    A, As = _ops().group_quant(x.cuda())
    qr, sr = O.group_quant(x)
    assert torch.equal(A.cpu().view(torch.uint8), qr.view(torch.uint8))
    assert torch.equal(As.cpu(), sr)


def test_group_quant_strided_rows(cuda_lib):
    x = O.make_activation(16, 1024, seed=5)
    big = torch.zeros(16, 1536, dtype=torch.bfloat16)
    big[:, :1024] = x
    A, As = _ops().group_quant(big.cuda()[:, :1024])
    qr, sr = O.group_quant(x)
    assert torch.equal(A.cpu().view(torch.uint8), qr.view(torch.uint8)) and torch.equal(As.cpu(), sr)


@pytest.mark.parametrize("M,inter,strided", [(1, 8, False), (300, 512, False), (37, 17408, True)])
def test_silu_mul_matches_oracle(cuda_lib, M, inter, strided):
    """The unfused chain's SiLU(g)*u kernel against the oracle's fp32 expression (torch silu on the CPU, one
    bf16 rounding). CUDA's expf and the CPU's exp may differ in the last fp32 bit, so at most 0.1 % of the
    outputs may differ, by one bf16 ulp. Zeros, tiny and large-magnitude gates are among the inputs."""
    g = torch.Generator().manual_seed(M + inter)
    gu = (torch.randn(M, 2 * inter, generator=g) * 4).to(torch.bfloat16)
    gu[0, : min(inter, 8)] = torch.tensor([0.0, -0.0, 80.0, -80.0, 1e-30, -1e-30, 3.0, -3.0])[: min(inter, 8)].to(
        torch.bfloat16)
    dev = gu.cuda()
    if strided:
        big = torch.zeros(M, 2 * inter + 64, dtype=torch.bfloat16, device="cuda")
        big[:, : 2 * inter] = dev
        dev = big[:, : 2 * inter]
    y = _ops().silu_mul(dev).cpu()
    ref = (torch.nn.functional.silu(gu[:, :inter].float()) * gu[:, inter:].float()).to(torch.bfloat16)
    assert y.shape == ref.shape and y.dtype == torch.bfloat16
    a, b = y.view(torch.int16).int(), ref.view(torch.int16).int()
    diff = (a - b).abs()
    assert int(diff.max()) <= 1, int(diff.max())
    assert (diff > 0).float().mean().item() <= 1e-3


@pytest.mark.parametrize("M,K,fused_add", [(1, 128, False), (7, 640, True), (300, 5120, False), (33, 5120, True),
                                            (64, 16384, True), (2049, 1024, True), (2048, 5120, False)])
def test_rmsnorm_group_quant_bit_exact(cuda_lib, M, K, fused_add):
    """Fused RMSNorm + group quant against the oracle restatement (same rounding points and summation
    order): e4m3 bytes, scales and the updated residual all bit-exact."""
    g = torch.Generator().manual_seed(M * 7 + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    x[0, :128] *= 40.0  # a group far above the row's rms
    w = (1 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16)
    r = torch.randn(M, K, generator=g).to(torch.bfloat16) if fused_add else None
    A_ref, As_ref, h_ref = O.rmsnorm_group_quant(x, w, 1e-6, r)
    rd = r.cuda() if fused_add else None
    A, As = _ops().rmsnorm_group_quant(x.cuda(), w.cuda(), 1e-6, residual=rd)
    torch.cuda.synchronize()
    assert torch.equal(A.cpu().view(torch.uint8), A_ref.view(torch.uint8))
    assert torch.equal(As.cpu(), As_ref)
    if fused_add:
        assert torch.equal(rd.cpu(), h_ref)


@pytest.mark.parametrize("fused", ["1", "0"])
def test_mlp_takes_fused_norm_output(cuda_lib, monkeypatch, fused):
    """Decoder-layer chain norm -> MLP through the drop-in API: GatedMLP takes the (A, As) pair of the fused
    norm kernel as its input, on the fused gate_up path and on the unfused fallback."""
    import importlib
    monkeypatch.setenv("SGLANG_FP8_HAND_GEMM", "1")
    monkeypatch.setenv("SGLANG_FP8_HAND_FUSED", fused)
    from fp8_hand_b200 import fp8_hand_sm100, sglang_compat
    importlib.reload(fp8_hand_sm100)
    try:
        M, H, inter = 200, 512, 1024
        gu, gus = O.make_weight(2 * inter, H, seed=21)
        dn, dns = O.make_weight(H, inter, seed=22)
        mlp = sglang_compat.GatedMLP(sglang_compat.Fp8BlockLinear(gu.cuda(), gus.cuda()),
                                     sglang_compat.Fp8BlockLinear(dn.cuda(), dns.cuda()))
        sglang_compat.post_load(mlp)
        g = torch.Generator().manual_seed(23)
        x = torch.randn(M, H, generator=g).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
        A, As = _ops().rmsnorm_group_quant(x.cuda(), w.cuda(), 1e-6)
        out = mlp((A, As)).cpu()
        A_ref, As_ref, _ = O.rmsnorm_group_quant(x, w, 1e-6)
        # the fallback rounds gate_up to bf16 before SiLU * up and the quant: the oracle's unfused chain
        front = O.fused_gate_up if fused == "1" else O.chain_gate_up
        Q_ref, Qs_ref, _ = front(A_ref, gu, As_ref, gus)
        ref = O.blockwise_matmul(Q_ref, dn, Qs_ref, dns)
        assert out.shape == (M, H) and out.dtype == torch.bfloat16
        assert O.norm_rel_error(out.float(), ref.float()) <= 1e-2
        if fused == "1":
            # the tuple goes straight into the fused kernel: same bytes as calling the ops by hand
            Q, Qs = _ops().gemm_silu_quant(A, mlp.gate_up_proj.weight.tiles, As, gus.cuda(), b_tiled=True)
            direct = _ops().gemm(Q, mlp.down_proj.weight.tiles, Qs, dns.cuda(), b_tiled=True)
            assert torch.equal(out, direct.cpu())
    finally:
        monkeypatch.delenv("SGLANG_FP8_HAND_FUSED")
        monkeypatch.delenv("SGLANG_FP8_HAND_GEMM")
        importlib.reload(fp8_hand_sm100)


def test_relayout_reads_tile_cache(cuda_lib, monkeypatch, tmp_path):
    """relayout(model, cache): the first call packs and writes the tile-pack file; a model whose row-major
    weights were never loaded (meta device) gets the same tiles from it and the same MLP output; a file
    whose block scales do not match the model is refused."""
    import importlib
    monkeypatch.setenv("SGLANG_FP8_HAND_GEMM", "1")
    from fp8_hand_b200 import fp8_hand_sm100, sglang_compat, tilepack
    importlib.reload(fp8_hand_sm100)
    try:
        H, inter = 512, 1024
        gu, gus = O.make_weight(2 * inter, H, seed=31)
        dn, dns = O.make_weight(H, inter, seed=32)

        def mlp_of(gw, dw, scale_mult=1.0):
            return sglang_compat.GatedMLP(sglang_compat.Fp8BlockLinear(gw, (gus * scale_mult).cuda()),
                                          sglang_compat.Fp8BlockLinear(dw, dns.cuda()))

        def meta(n, k):
            return torch.empty(n, k, dtype=torch.float8_e4m3fn, device="meta")

        cache = tmp_path / "mlp.bsfp8"
        a = mlp_of(gu.cuda(), dn.cuda())
        sglang_compat.post_load(a, cache=cache)
        assert set(tilepack.read_header(cache)["entries"]) == {"gate_up_proj", "down_proj"}
        b = mlp_of(meta(2 * inter, H), meta(H, inter))
        sglang_compat.post_load(b, cache=cache)
        for m in ("gate_up_proj", "down_proj"):
            assert torch.equal(getattr(a, m).weight.tiles, getattr(b, m).weight.tiles)
        x = O.make_activation(200, H, seed=33).cuda()
        assert torch.equal(a(x), b(x))
        with pytest.raises(tilepack.TilePackError):
            sglang_compat.post_load(mlp_of(meta(2 * inter, H), meta(H, inter), scale_mult=2.0), cache=cache)
    finally:
        monkeypatch.delenv("SGLANG_FP8_HAND_GEMM")
        importlib.reload(fp8_hand_sm100)


def test_rmsnorm_group_quant_strided_rows(cuda_lib):
    x = torch.randn(9, 384, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    w = torch.ones(256, dtype=torch.bfloat16)
    A_ref, As_ref, _ = O.rmsnorm_group_quant(x[:, :256].contiguous(), w, 1e-5)
    A, As = _ops().rmsnorm_group_quant(x.cuda()[:, :256], w.cuda(), 1e-5)
    assert torch.equal(A.cpu().view(torch.uint8), A_ref.view(torch.uint8)) and torch.equal(As.cpu(), As_ref)


@pytest.mark.parametrize("N,K", [(128, 128), (384, 640), (256, 5120)])
def test_pack_tiles_bit_exact(cuda_lib, N, K):
    g = torch.Generator().manual_seed(N * 7 + K)
    w = torch.randint(0, 256, (N, K), dtype=torch.uint8, generator=g)
    tiles = _ops().pack_tiles(w.cuda().view(torch.float8_e4m3fn))
    assert torch.equal(tiles.cpu(), O.relayout_tiles(w))


# --------------------------------------------------------------------------- GEMM
GEMM_CASES = [
    # (M, N, K)   decode (M <= 128) ...
    (1, 256, 512),
    (7, 384, 1024),
    (16, 1024, 5120),
    (33, 2048, 1024),
    (40, 1152, 1024),     # odd number of weight tiles
    (96, 768, 17408),     # few tiles, each split over many CTAs
    (5, 384, 17408),      # every tile spread over ~50 CTAs (many middle contributors)
    (3, 128, 256),        # fewer units than SMs
    (112, 1024, 5120),
    (128, 6144, 5120),    # config 1
    # ... prefill (M > 128)
    (129, 512, 1024),
    (200, 384, 640),      # odd number of 128-column blocks: half-empty last tile
    (257, 2048, 5120),
    (1024, 1024, 2048),   # 256-row tiles on CTA pairs from here on
    (600, 384, 640),      # last pair tile: peer rows all past M, half-empty last column tile
    (520, 2048, 1024),    # last pair tile: 8 valid rows
    (1040, 4864, 4096),   # 171 tiles on 148 SMs: stream-K (tiles split between neighbouring CTAs), ragged rows
]


@pytest.mark.parametrize("tiled", [True, False])
@pytest.mark.parametrize("M,N,K", GEMM_CASES)
def test_gemm_bf16_matches_oracle(cuda_lib, M, N, K, tiled):
    A, B, As, Bs, _ = O.make_gemm_case(M, N, K, seed=M * 31 + N + K, outlier_frac=0.05)
    ops = _ops()
    Bd = ops.pack_tiles(B.cuda()) if tiled else B.cuda()
    C = ops.gemm(*_dev(A), Bd, *_dev(As, Bs), b_tiled=tiled)
    torch.cuda.synchronize()
    ref = O.blockwise_matmul(A, B, As, Bs)
    assert C.dtype == torch.bfloat16 and tuple(C.shape) == (M, N)
    assert O.max_rel_error(C.cpu(), ref) <= GEMM_MAX_REL
    assert O.norm_rel_error(C.cpu(), ref) <= 4e-3


def test_decode_workspace_reuse_across_shapes(cuda_lib):
    """Decode calls of different widths share one cached workspace per stream: a narrow split-K call leaves
    partial tiles behind, and a wider call right after (more weight tiles, hence more arrival counters) must
    still see zeroed counters. Then the narrow shape again, and a fused call, on the same workspace; then a prefill
    GEMM that runs stream-K (171 tiles on 148 SMs) on the same workspace, its partial tiles where the decode
    partials were, and a decode call after it (checked on sampled rows where the full oracle would be slow)."""
    ops = _ops()
    shapes = [(16, 1024, 5120, False), (16, 40960, 5120, False), (16, 1024, 5120, False), (8, 8192, 2048, True),
              (3, 65536, 1024, False), (1040, 4864, 4096, False), (16, 40960, 5120, False)]
    for M, N, K, fused in shapes:
        A, B, As, Bs, _ = O.make_gemm_case(M, N, K, seed=N + M, outlier_frac=0.05)
        if fused:
            Q, Qs = ops.gemm_silu_quant(*_dev(A, B, As, Bs))
            _check_fused(Q, Qs, A, B, As, Bs)
        else:
            C = ops.gemm(*_dev(A, B, As, Bs))
            rows = torch.arange(M) if M <= 128 else torch.cat([torch.arange(0, M, 37), torch.tensor([M - 1])])
            ref = O.blockwise_matmul(A[rows], B, As[rows], Bs)
            assert O.max_rel_error(C.cpu()[rows], ref) <= GEMM_MAX_REL, (M, N, K)


@pytest.mark.parametrize("M,N,K", [(9, 768, 2048), (48, 768, 2048), (300, 768, 2048), (128, 256, 17408),
                                   (1040, 4864, 4096)])  # the last on stream-K
def test_gemm_fp32_out_matches_oracle_tightly(cuda_lib, M, N, K):
    A, B, As, Bs, _ = O.make_gemm_case(M, N, K, seed=N + K + M)
    C = _ops().gemm(*_dev(A, B, As, Bs), out_dtype=torch.float32)
    ref = O.blockwise_matmul(A, B, As, Bs)
    assert C.dtype == torch.float32
    # only fp32 summation order differs (tensor-core partials, split-K order)
    assert O.norm_rel_error(C.cpu(), ref) <= 1e-5
    assert O.max_rel_error(C.cpu(), ref) <= 1e-3


@pytest.mark.parametrize("M", [2, 64, 500, 1000])
def test_gemm_deterministic_and_linear(cuda_lib, M):
    """Two launches give identical bytes; doubling As (exact in fp32) doubles C exactly."""
    A, B, As, Bs, _ = O.make_gemm_case(M, 1024, 2048, seed=M)
    ops = _ops()
    Ad, Bd, Asd, Bsd = _dev(A, B, As, Bs)
    C1 = ops.gemm(Ad, Bd, Asd, Bsd, out_dtype=torch.float32)
    C2 = ops.gemm(Ad, Bd, Asd, Bsd, out_dtype=torch.float32)
    C3 = ops.gemm(Ad, Bd, Asd * 2, Bsd, out_dtype=torch.float32)
    assert torch.equal(C1, C2)
    assert torch.equal(C3, C1 * 2)


# --------------------------------------------------------------------------- fused gate_up
def _check_fused(Q, Qs, A, B, As, Bs):
    q_ref, s_ref, _ = O.fused_gate_up(A, B, As, Bs)
    Q, Qs = Q.cpu(), Qs.cpu()
    assert Q.dtype == torch.float8_e4m3fn and Qs.dtype == torch.float32
    assert tuple(Q.shape) == tuple(q_ref.shape) and tuple(Qs.shape) == tuple(s_ref.shape)
    rel = ((Qs - s_ref).abs() / s_ref).max().item()
    ulp = O.e4m3_ulp_distance(Q, q_ref)
    frac = (ulp > 0).float().mean().item()
    assert rel <= SCALE_REL, f"scale rel err {rel:.3g}"
    assert ulp.max().item() <= Q_ULP, f"max ulp {ulp.max().item()}"
    assert frac <= Q_FRAC, f"{frac:.3%} of elements differ"


FUSED_CASES = [(1, 512, 1024), (8, 2048, 5120), (14, 1024, 5120), (56, 512, 2048), (112, 2048, 5120),
               (128, 256, 512), (129, 512, 1024), (300, 1024, 5120), (1024, 512, 1024), (600, 512, 1024)]


@pytest.mark.parametrize("tiled", [True, False])
@pytest.mark.parametrize("M,N2,K", FUSED_CASES)
def test_fused_gate_up_matches_oracle(cuda_lib, M, N2, K, tiled):
    A, B, As, Bs, _ = O.make_gemm_case(M, N2, K, seed=M + N2 + K, outlier_frac=0.01)
    ops = _ops()
    Bd = ops.pack_tiles(B.cuda()) if tiled else B.cuda()
    Q, Qs = ops.gemm_silu_quant(*_dev(A), Bd, *_dev(As, Bs), b_tiled=tiled)
    _check_fused(Q, Qs, A, B, As, Bs)


def test_fused_gate_up_full_width_decode(cuda_lib):
    """Config 2's real weight (2 x 17408 rows, K = 5120) at M = 112, checked on a block subset."""
    M, inter, K = 112, 17408, 5120
    x = O.make_activation(M, K, seed=77)
    A, As = O.group_quant(x)
    Bg, Bsg = O.make_weight(inter, K, seed=78)
    Bu, Bsu = O.make_weight(inter, K, seed=79)
    B = torch.cat([Bg.view(torch.uint8), Bu.view(torch.uint8)]).view(torch.float8_e4m3fn)
    Bs = torch.cat([Bsg, Bsu])
    Q, Qs = _ops().gemm_silu_quant(*_dev(A, B, As, Bs))
    blocks = [0, 1, 67, 135]
    rows_g = torch.cat([torch.arange(b * 128, (b + 1) * 128) for b in blocks])
    sub_B = torch.cat([Bg.view(torch.uint8)[rows_g], Bu.view(torch.uint8)[rows_g]]).view(torch.float8_e4m3fn)
    sub_Bs = torch.cat([Bsg[blocks], Bsu[blocks]])
    cols = rows_g
    _check_fused(Q.cpu()[:, cols], Qs.cpu()[:, blocks], A, sub_B, As, sub_Bs)


# --------------------------------------------------------------------------- C-ABI contract
def test_abi_rejects_bad_arguments(cuda_lib):
    lib = cuda_lib
    A, B, As, Bs, _ = O.make_gemm_case(4, 256, 256, seed=1)
    Ad, Bd, Asd, Bsd = _dev(A, B, As, Bs)
    C = torch.empty(4, 256, dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # K not a multiple of 128
    assert lib.bs_fp8_gemm(Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), Asd.data_ptr(), Bsd.data_ptr(),
                           4, 256, 200, 256, 0, 0, None, 0, s) == 1
    # misaligned A
    assert lib.bs_fp8_gemm(Ad.data_ptr() + 1, Bd.data_ptr(), C.data_ptr(), Asd.data_ptr(), Bsd.data_ptr(),
                           4, 256, 256, 256, 0, 0, None, 0, s) == 2
    # decode shape without workspace
    assert lib.bs_fp8_gemm(Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), Asd.data_ptr(), Bsd.data_ptr(),
                           4, 256, 256, 256, 0, 0, None, 0, s) == 3
    # M == 0 is a no-op
    assert lib.bs_fp8_gemm(None, None, None, None, None, 0, 256, 256, 256, 0, 0, None, 0, s) == 0
    # fused with N2 not a multiple of 256
    Q = torch.empty(4, 64, dtype=torch.uint8, device="cuda")
    assert lib.bs_fp8_gemm_silu_quant(Ad.data_ptr(), Bd.data_ptr(), Q.data_ptr(), Asd.data_ptr(), Bsd.data_ptr(),
                                      Asd.data_ptr(), 4, 128, 256, 0, None, 0, s) == 1
    assert lib.bs_fp8_workspace_bytes(4, 256, 256, 0) > 0
    assert lib.bs_fp8_workspace_bytes(129, 256, 256, 0) == 0


def test_bounded_wait_reports_timeout(cuda_lib):
    """A wait that nothing satisfies gives up after its limit and leaves a status code; the
    context stays usable afterwards."""
    from fp8_hand_b200 import _native
    assert _native.status(clear=True) == 0
    rc = cuda_lib.bs_fp8_selftest_wait_timeout(ctypes.c_uint64(2_000_000), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert _native.status(clear=True) == 199
    assert _native.status(clear=True) == 0
    x = torch.ones(4, 128, dtype=torch.bfloat16, device="cuda")
    A, As = _ops().group_quant(x)
    assert torch.equal(As.cpu(), (torch.tensor(1.0) / torch.tensor(448.0)).expand(4, 1))
