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
        out = tp.TensorParallelMLP(shard)(x.to(dev))
        torch.cuda.synchronize()
        q.put((rank, out.cpu()))
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

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert torch.equal(outs[0], outs[1])
    # each rank's quant groups are exact slices of the single-GPU ones; only the fp32 sum order differs
    assert O.max_rel_error(outs[0], single.float()) <= 1e-2
    assert O.norm_rel_error(outs[0], single.float()) <= 4e-3
