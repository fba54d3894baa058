"""GPU, 2 ranks over NCCL: the tensor-parallel MLP against the single-GPU MLP on the same weights.

Runs as child processes, one per GPU, on a box with at least two GPUs (skipped otherwise). NVLS is
switched off for the test, and every collective has a short process-group timeout.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O

pytestmark = pytest.mark.gpu

H, INTER, M = 1024, 2048, 200
M_DECODE = 56


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    gu, gus = O.make_weight(2 * INTER, H, seed=11)
    dn, dns = O.make_weight(H, INTER, seed=12)
    x = O.make_activation(M, H, seed=13, outlier_frac=0.01)
    return gu, gus, dn, dns, x


def _worker(rank, world, port, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ucloud-ai-infra_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from fp8_hand_b200 import tp
        gu, gus, dn, dns, x = _inputs()
        shard = tp.make_shard(gu, gus, dn, dns, rank, world, device=dev, tiled=True)
        xd = x.to(dev)
        outs = (tp.TensorParallelMLP(shard)(xd),                                  # bf16 partials (config 4)
                tp.TensorParallelMLP(shard, partial_dtype=torch.float32)(xd),     # fp32 partials
                tp.TensorParallelMLP(shard, chunks=2)(xd))                        # overlapped row chunks
        # down_proj fused with the sum through NVSwitch multicast: prefill (200 rows) and decode (56 rows)
        try:
            mlp_mc = tp.TensorParallelMLP(shard, reduce="multimem")
            mc = (mlp_mc(xd).clone(), mlp_mc(xd[:M_DECODE].contiguous()).clone())
        except RuntimeError as e:  # no multicast mapping on this box: every rank raises the same
            mc = str(e)
        torch.cuda.synchronize()
        q.put((rank, tuple(o.cpu() for o in outs), mc if isinstance(mc, str) else tuple(o.cpu() for o in mc)))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_matches_single_gpu():
    from fp8_hand_b200 import ops
    gu, gus, dn, dns, x = _inputs()
    # single-GPU reference through the same kernels
    A, As = ops.group_quant(x.cuda())
    Q, Qs = ops.gemm_silu_quant(A, gu.cuda(), As, gus.cuda())
    single = ops.gemm(Q, dn.cuda(), Qs, dns.cuda(), out_dtype=torch.float32).to(torch.bfloat16).cpu()
    A, As = ops.group_quant(x[:M_DECODE].cuda())
    Q, Qs = ops.gemm_silu_quant(A, gu.cuda(), As, gus.cuda())
    single_dec = ops.gemm(Q, dn.cuda(), Qs, dns.cuda(), out_dtype=torch.float32).cpu()

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    outs = {r: o for r, o, _ in got}
    mcs = {r: m for r, _, m in got}
    for k in range(3):
        assert torch.equal(outs[0][k], outs[1][k])
    out_bf16, out_f32, out_chunked = outs[0]
    ref = single.float()
    # each rank's quant groups are exact slices of the single-GPU ones; with fp32 partials only the
    # fp32 sum order differs
    assert O.max_rel_error(out_f32, ref) <= 1e-2
    assert O.norm_rel_error(out_f32, ref) <= 4e-3
    # bf16 partials are rounded (half an ulp, 2^-8 of their magnitude) before the sum: absolute bound
    assert (out_bf16.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    assert O.norm_rel_error(out_bf16.float(), ref) <= 4e-3
    # row chunks (the 72-row tail runs the decode kernels, whose split-K sums in another order)
    assert (out_chunked.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    assert O.norm_rel_error(out_chunked.float(), ref) <= 4e-3
    # multicast reduction: bf16 partials added in bf16 by the switch, in no fixed order of ranks, so each
    # rank's copy is checked against the single-GPU result with the bf16-partial bound
    if isinstance(mcs[0], str):
        pytest.skip(f"NVSwitch multicast unavailable: {mcs[0]}")
    for r in range(world):
        mc_pre, mc_dec = mcs[r]
        for got_r, want in ((mc_pre, ref), (mc_dec, single_dec)):
            assert (got_r.float() - want).abs().max().item() <= 1e-2 * want.abs().max().item()
            assert O.norm_rel_error(got_r.float(), want) <= 4e-3
