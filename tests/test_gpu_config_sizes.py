"""GPU parity at the configured sizes, against the CPU oracle.

The kernels are persistent: at the configured sizes every CTA walks many output tiles, carrying TMEM
buffer and mbarrier phases from tile to tile, large activation panels take the grouped raster, and the
decode kernels split tiles across CTAs (stream-K). Small cases cannot reach those paths, so these tests
run the real shapes:

  * the fused gate_up + SiLU*up + quant kernel at M = 1024, 4096, 8192, K = 5120, N2 = 2 x 17408, with 1%
    of the activation rows scaled x50 (the prefill MLP configuration); the reference checks its fused kernel
    at (N2, K, M) = (34816, 5120, 1024) (logs/artifacts/20261031_hand/fused_test.py:39);
  * down_proj at M = 8192, K = 17408, N = 5120 (A panel 142.6 MB: the 2048-row raster groups);
  * the per-layer linears at M = 8192 (qkv, o, gate_up as a plain GEMM, down) and the reference's own
    M = 8192 verification shapes (logs/artifacts/20261031_hand/verify_hand.py:29-49);
  * the reference's persistent-walk cases (logs/artifacts/20261031_hand/sweep_hand.py:22-30), checked in full;
  * many-tile cases small enough for a full oracle comparison (512 plain tiles, 256 pair tiles);
  * the vocab-sized lm_head (N = 248320, K = 5120) at M = 1 and 112, in the row-major layout the drop-in
    path gives it and in tile-first layout (patches/apply_sglang_fp8_lm_head.py:38-49).

Weights and activations are made on the GPU (seeded), and the oracle runs on the bytes the kernel read.
Where a full comparison would take the CPU oracle minutes, a sample of rows (every M tile, both CTAs of a
pair tile, first and last rows, the x50 rows) times a sample of 128-column blocks (the first, the last and
blocks between) is compared. The bars are those of tests/test_gpu_kernels.py.
"""
import json

import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GEMM_MAX_REL = 1e-2
GEMM_NORM_REL = 4e-3
Q_ULP = 1
Q_FRAC = 1e-3
SCALE_REL = 1e-6
E4M3 = torch.float8_e4m3fn


def _ops():
    from fp8_hand_b200 import ops
    return ops


# --------------------------------------------------------------------------- seeded inputs on the GPU
def gpu_weight(N, K, seed, std=0.02, chunk=16384):
    """bf16 N(0, std) [N, K] quantised per 128x128 block (s = max(amax/448, 1e-12), q = e4m3(w/s)), made on
    the GPU in row chunks."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.empty(N, K, dtype=E4M3, device="cuda")
    s = torch.empty(N // 128, K // 128, dtype=torch.float32, device="cuda")
    for r0 in range(0, N, chunk):
        r1 = min(N, r0 + chunk)
        w = (torch.randn(r1 - r0, K, generator=g, device="cuda") * std).to(torch.bfloat16).float()
        sb = (w.abs().reshape((r1 - r0) // 128, 128, K // 128, 128).amax(dim=(1, 3)) / 448.0).clamp_min(1e-12)
        q[r0:r1] = (w / sb.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(E4M3)
        s[r0 // 128:r1 // 128] = sb
        del w
    return q, s


def gpu_activation(M, K, seed, outlier_frac=0.01):
    """bf16 N(0, 1) [M, K] with `outlier_frac` of the rows x50, and its per-token-group quant (the library's
    kernel, bit-exact with the oracle's quantiser: checked on the sampled rows). Returns (x, A, As, outlier rows)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, generator=g, device="cuda")
    n_out = int(round(outlier_frac * M))
    out_rows = torch.randperm(M, generator=g, device="cuda")[:n_out] if n_out else torch.empty(0, dtype=torch.long)
    if n_out:
        x[out_rows] *= 50.0
    x = x.to(torch.bfloat16)
    A, As = _ops().group_quant(x)
    return x, A, As, sorted(out_rows.tolist())


def sample_rows(M, tile_rows=256, per_tile=6, extra=(), seed=0):
    """Rows of every tile: its first row, the first and last rows of its second half (the peer CTA of a
    pair tile), its last row and two seeded rows; plus `extra` (x50 rows)."""
    g = torch.Generator().manual_seed(seed)
    rows = set()
    for t0 in range(0, M, tile_rows):
        t1 = min(M, t0 + tile_rows)
        for r in (t0, t0 + 127, t0 + 128, t1 - 1):
            if t0 <= r < t1:
                rows.add(r)
        for r in torch.randint(t0, t1, (max(0, per_tile - 4),), generator=g).tolist():
            rows.add(r)
    rows.update(r for r in extra if r < M)
    return sorted(rows)


def spread_blocks(nblk, count=8):
    """`count` 128-column blocks spread over [0, nblk): first two, last two and evenly spaced ones."""
    picks = {0, min(1, nblk - 1), max(0, nblk - 2), nblk - 1}
    for i in range(count):
        picks.add(i * (nblk - 1) // max(1, count - 1))
    return sorted(picks)


def _idx(blocks):
    return torch.cat([torch.arange(b * 128, (b + 1) * 128) for b in blocks])


# --------------------------------------------------------------------------- comparisons
def check_gemm(C, A, B, As, Bs, rows=None, blocks=None, label=""):
    """C (device, [M, N]) against the oracle on rows x 128-column blocks (all when None)."""
    M, N = C.shape
    rows_t = torch.arange(M) if rows is None else torch.tensor(rows)
    blocks = list(range(N // 128)) if blocks is None else blocks
    cols = _idx(blocks)
    rd, cd = rows_t.cuda(), cols.cuda()
    A_s = A.view(torch.uint8).index_select(0, rd).cpu().view(E4M3)
    As_s = As.index_select(0, rd).cpu()
    B_s = B.view(torch.uint8).index_select(0, cd).cpu().view(E4M3)
    Bs_s = Bs[torch.tensor(blocks).cuda()].cpu()
    got = C.index_select(0, rd).index_select(1, cd).cpu()
    ref = O.blockwise_matmul(A_s, B_s, As_s, Bs_s)
    mr, nr = O.max_rel_error(got, ref), O.norm_rel_error(got, ref)
    print(json.dumps({"check": "gemm", "case": label, "rows": len(rows_t), "cols": len(cols), "max_rel": mr,
                      "norm_rel": nr}))
    assert torch.isfinite(got.float()).all()
    assert mr <= GEMM_MAX_REL, f"{label}: max rel {mr:.3g}"
    assert nr <= GEMM_NORM_REL, f"{label}: norm rel {nr:.3g}"


def check_fused(Q, Qs, A, B, As, Bs, rows=None, gate_blocks=None, label=""):
    """Q e4m3 [M, I], Qs [M, I/128] (device) against the oracle's fused epilogue on rows x gate/up block pairs."""
    M, inter = Q.shape
    ib = inter // 128
    rows_t = torch.arange(M) if rows is None else torch.tensor(rows)
    gate_blocks = list(range(ib)) if gate_blocks is None else gate_blocks
    gcols = _idx(gate_blocks)
    rd = rows_t.cuda()
    A_s = A.view(torch.uint8).index_select(0, rd).cpu().view(E4M3)
    As_s = As.index_select(0, rd).cpu()
    wrows = torch.cat([gcols, gcols + inter]).cuda()
    B_s = B.view(torch.uint8).index_select(0, wrows).cpu().view(E4M3)
    Bs_s = Bs[torch.tensor(gate_blocks + [ib + j for j in gate_blocks]).cuda()].cpu()
    q_got = Q.view(torch.uint8).index_select(0, rd).index_select(1, gcols.cuda()).cpu().view(E4M3)
    s_got = Qs.index_select(0, rd).index_select(1, torch.tensor(gate_blocks).cuda()).cpu()
    q_ref, s_ref, _ = O.fused_gate_up(A_s, B_s, As_s, Bs_s)
    rel = ((s_got - s_ref).abs() / s_ref).max().item()
    ulp = O.e4m3_ulp_distance(q_got, q_ref)
    hist = torch.bincount(ulp.flatten().clamp_max(3), minlength=4).tolist()
    frac = (ulp > 0).float().mean().item()
    print(json.dumps({"check": "fused", "case": label, "rows": len(rows_t), "cols": len(gcols), "scale_rel": rel,
                      "ulp_hist_0_1_2_3plus": hist, "frac_differ": frac}))
    assert rel <= SCALE_REL, f"{label}: scale rel err {rel:.3g}"
    assert ulp.max().item() <= Q_ULP, f"{label}: max ulp {ulp.max().item()}"
    assert frac <= Q_FRAC, f"{label}: {frac:.3%} of elements differ"


def check_quant_rows(x, A, As, rows):
    """The library's activation quant on the sampled rows equals the oracle's quantiser bit for bit."""
    rd = torch.tensor(rows).cuda()
    qr, sr = O.group_quant(x.index_select(0, rd).cpu())
    assert torch.equal(A.view(torch.uint8).index_select(0, rd).cpu(), qr.view(torch.uint8))
    assert torch.equal(As.index_select(0, rd).cpu(), sr)


# --------------------------------------------------------------------------- prefill MLP, config sizes
@pytest.mark.parametrize("M", [1024, 4096, 8192])
def test_fused_gate_up_prefill_config(cuda_lib, M):
    """k_prefill<fused> at the prefill MLP sizes: every CTA pair walks tens of 256 x 256 tiles."""
    K, inter = 5120, 17408
    ops = _ops()
    B, Bs = gpu_weight(2 * inter, K, seed=101)
    x, A, As, out_rows = gpu_activation(M, K, seed=102 + M)
    tiles = ops.pack_tiles(B)
    Q, Qs = ops.gemm_silu_quant(A, tiles, As, Bs, b_tiled=True)
    torch.cuda.synchronize()
    rows = sample_rows(M, extra=out_rows[:16], seed=M)
    check_quant_rows(x, A, As, rows[:64])
    gblocks = spread_blocks(inter // 128, 8)
    check_fused(Q, Qs, A, B, As, Bs, rows=rows, gate_blocks=gblocks, label=f"fused M={M}")
    if M == 4096:
        # row-major weights take the same walk with per-row-block boxes
        Q2, Qs2 = ops.gemm_silu_quant(A, B, As, Bs, b_tiled=False)
        assert torch.equal(Q2.view(torch.uint8), Q.view(torch.uint8)) and torch.equal(Qs2, Qs)


def test_fused_gate_up_reference_check_shape(cuda_lib):
    """The reference's fused-kernel check shape (N2, K, M) = (34816, 5120, 1024), all 1024 rows."""
    K, inter, M = 5120, 17408, 1024
    ops = _ops()
    B, Bs = gpu_weight(2 * inter, K, seed=111)
    _, A, As, _ = gpu_activation(M, K, seed=112)
    Q, Qs = ops.gemm_silu_quant(A, ops.pack_tiles(B), As, Bs, b_tiled=True)
    check_fused(Q, Qs, A, B, As, Bs, rows=None, gate_blocks=spread_blocks(inter // 128, 12),
                label="fused reference shape M=1024")


def test_down_proj_prefill_config(cuda_lib):
    """down_proj at M = 8192 (K = 17408, N = 5120): the A panel exceeds L2, so the raster runs in groups."""
    M, K, N = 8192, 17408, 5120
    ops = _ops()
    B, Bs = gpu_weight(N, K, seed=121)
    _, A, As, out_rows = gpu_activation(M, K, seed=122)
    C = ops.gemm(A, ops.pack_tiles(B), As, Bs, b_tiled=True)
    torch.cuda.synchronize()
    rows = sample_rows(M, tile_rows=128, per_tile=4, extra=out_rows[:8], seed=5)
    check_gemm(C, A, B, As, Bs, rows=rows, blocks=spread_blocks(N // 128, 8), label="down_proj M=8192")


def test_down_proj_stream_k_config(cuda_lib):
    """down_proj at M = 1024 (K = 17408, N = 5120): 160 whole tiles would take two waves of the 148 SMs for 1.08
    waves of work, so the kernel runs stream-K (equal K-block ranges per CTA, a tile shared by two CTAs summed
    through the workspace). At M = 4096 (640 tiles, 86 % of five waves) it runs whole tiles."""
    M, K, N = 1024, 17408, 5120
    ops = _ops()
    from fp8_hand_b200 import select
    assert select(N, M, K=K)["split"] == "stream-k" and select(N, 4096, K=K)["split"] == "tile"
    B, Bs = gpu_weight(N, K, seed=141)
    _, A, As, out_rows = gpu_activation(M, K, seed=142)
    C = ops.gemm(A, ops.pack_tiles(B), As, Bs, b_tiled=True)
    C2 = ops.gemm(A, ops.pack_tiles(B), As, Bs, b_tiled=True)
    torch.cuda.synchronize()
    assert torch.equal(C, C2), "stream-K sums partials in a fixed order: two calls give the same bytes"
    rows = sample_rows(M, tile_rows=128, per_tile=4, extra=out_rows[:8], seed=9)
    check_gemm(C, A, B, As, Bs, rows=rows, blocks=spread_blocks(N // 128, 10), label=f"down_proj stream-K M={M}")


def test_mlp_prefill_chain_config(cuda_lib):
    """The whole MLP at M = 8192 through the drop-in API (group quant -> fused gate_up -> down_proj), the
    bench's workload, on sampled rows: down_proj's input is the fused kernel's own (Q, Qs)."""
    import importlib
    import os
    M, H, inter = 8192, 5120, 17408
    prev = os.environ.get("SGLANG_FP8_HAND_GEMM")
    os.environ["SGLANG_FP8_HAND_GEMM"] = "1"
    from fp8_hand_b200 import fp8_hand_sm100, sglang_compat
    importlib.reload(fp8_hand_sm100)
    try:
        gu, gus = gpu_weight(2 * inter, H, seed=131)
        dn, dns = gpu_weight(H, inter, seed=132)
        mlp = sglang_compat.GatedMLP(sglang_compat.Fp8BlockLinear(gu.clone(), gus),
                                     sglang_compat.Fp8BlockLinear(dn.clone(), dns))
        sglang_compat.post_load(mlp)
        x, A, As, out_rows = gpu_activation(M, H, seed=133)
        out = mlp(x)
        ops = _ops()
        Q, Qs = ops.gemm_silu_quant(A, mlp.gate_up_proj.weight.tiles, As, gus, b_tiled=True)
        rows = sample_rows(M, tile_rows=256, per_tile=4, extra=out_rows[:8], seed=7)
        # the fused stage on these rows, then down_proj on the kernel's own Q against the oracle
        check_fused(Q, Qs, A, gu, As, gus, rows=rows, gate_blocks=spread_blocks(inter // 128, 6),
                    label="MLP front half M=8192")
        check_gemm(out, Q, dn, Qs, dns, rows=rows, blocks=spread_blocks(H // 128, 6), label="MLP output M=8192")
    finally:
        if prev is None:
            os.environ.pop("SGLANG_FP8_HAND_GEMM", None)
        else:
            os.environ["SGLANG_FP8_HAND_GEMM"] = prev
        importlib.reload(fp8_hand_sm100)


# the linears of a decoder layer at M = 8192, and the reference's M = 8192 verification shapes
LAYER_LINEARS = [("qkv", 10240, 5120), ("o", 5120, 6144), ("gate_up", 34816, 5120), ("verify_16384", 16384, 5120),
                 ("verify_14336", 14336, 5120)]


@pytest.mark.parametrize("name,N,K", LAYER_LINEARS)
def test_layer_linears_m8192(cuda_lib, name, N, K):
    M = 8192
    ops = _ops()
    B, Bs = gpu_weight(N, K, seed=N + K)
    _, A, As, out_rows = gpu_activation(M, K, seed=N + 1)
    C = ops.gemm(A, ops.pack_tiles(B), As, Bs, b_tiled=True)
    rows = sample_rows(M, tile_rows=128, per_tile=4, extra=out_rows[:8], seed=N)
    check_gemm(C, A, B, As, Bs, rows=rows, blocks=spread_blocks(N // 128, 8), label=f"{name} M=8192")


# --------------------------------------------------------------------------- full comparisons of long walks
@pytest.mark.parametrize("N,K,M", [(5120, 6144, 128), (5120, 6144, 200), (14336, 5120, 257), (14336, 5120, 300),
                                   (1024, 5120, 8192)])
def test_reference_walk_shapes_full(cuda_lib, N, K, M):
    """The reference's persistent-walk correctness cases (partial last M tile, short last CTA), every output
    element against the oracle, in both weight layouts."""
    ops = _ops()
    B, Bs = gpu_weight(N, K, seed=N * 3 + M)
    _, A, As, _ = gpu_activation(M, K, seed=M + 7, outlier_frac=0.02)
    for tiled in (True, False):
        C = ops.gemm(A, ops.pack_tiles(B) if tiled else B, As, Bs, b_tiled=tiled)
        check_gemm(C, A, B, As, Bs, label=f"walk N={N} K={K} M={M} tiled={tiled}")


def test_many_tiles_full_plain(cuda_lib):
    """512 output tiles of 128 x 256 over at most 148 persistent CTAs (3-4 tiles each), full comparison."""
    M, N, K = 2048, 8192, 256
    ops = _ops()
    B, Bs = gpu_weight(N, K, seed=141)
    _, A, As, _ = gpu_activation(M, K, seed=142, outlier_frac=0.05)
    C = ops.gemm(A, ops.pack_tiles(B), As, Bs, b_tiled=True)
    check_gemm(C, A, B, As, Bs, label="plain 512 tiles")
    C32 = ops.gemm(A, ops.pack_tiles(B), As, Bs, b_tiled=True, out_dtype=torch.float32)
    ref = O.blockwise_matmul(A.cpu(), B.cpu(), As.cpu(), Bs.cpu())
    assert O.norm_rel_error(C32.cpu(), ref) <= 1e-5


def test_many_tiles_full_fused(cuda_lib):
    """256 pair tiles of 256 x (128 gate + 128 up) over 74 CTA pairs, full comparison."""
    M, N2, K = 2048, 8192, 256
    ops = _ops()
    B, Bs = gpu_weight(N2, K, seed=151)
    _, A, As, _ = gpu_activation(M, K, seed=152, outlier_frac=0.05)
    Q, Qs = ops.gemm_silu_quant(A, ops.pack_tiles(B), As, Bs, b_tiled=True)
    check_fused(Q, Qs, A, B, As, Bs, label="fused 256 pair tiles")


# --------------------------------------------------------------------------- lm_head
@pytest.fixture(scope="module")
def lm_head_weight():
    B, Bs = gpu_weight(248320, 5120, seed=161)
    yield B, Bs
    del B, Bs
    torch.cuda.empty_cache()


@pytest.mark.parametrize("tiled", [False, True])
@pytest.mark.parametrize("M", [1, 112])
def test_lm_head_decode(cuda_lib, lm_head_weight, M, tiled):
    """FP8 lm_head [248320 x 5120] at decode and verify sizes: 1940 weight tiles split over the SMs
    (stream-K), many tiles per CTA. Row-major weights are what the drop-in path gives lm_head."""
    B, Bs = lm_head_weight
    ops = _ops()
    _, A, As, _ = gpu_activation(M, 5120, seed=162 + M, outlier_frac=0.0)
    Bd = ops.pack_tiles(B) if tiled else B
    C = ops.gemm(A, Bd, As, Bs, b_tiled=tiled)
    check_gemm(C, A, B, As, Bs, blocks=spread_blocks(248320 // 128, 16), label=f"lm_head M={M} tiled={tiled}")
    del Bd
