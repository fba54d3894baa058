"""CPU, world_size 2 over gloo: the tensor-parallel MLP's sharding and its all_reduce.

The per-rank math is injected as the oracle (tests only) so the host logic of fp8_hand_b200.tp
(column-parallel gate_up, row-parallel down_proj, sum of partials) runs on CPU ranks and is
compared with the unsharded oracle MLP.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

H, INTER, M = 256, 512, 300  # M > 128 so that the row chunks are exercised


class OracleCompute:
    """Per-rank compute with the ops interface, backed by the CPU oracle (row-major weights)."""

    @staticmethod
    def group_quant(x):
        return O.group_quant(x)

    @staticmethod
    def gemm_silu_quant(A, B, As, Bs, b_tiled=False):
        assert not b_tiled
        q, s, _ = O.fused_gate_up(A, B, As, Bs)
        return q, s

    @staticmethod
    def gemm(A, B, As, Bs, b_tiled=False, out=None, out_dtype=torch.float32):
        assert not b_tiled
        C = O.blockwise_matmul(A, B, As, Bs)
        if out is None:
            return C.to(out_dtype)
        out.copy_(C)
        return out

    @staticmethod
    def pack_tiles(w):
        return O.relayout_tiles(w)


def _inputs():
    gu, gus = O.make_weight(2 * INTER, H, seed=1)
    dn, dns = O.make_weight(H, INTER, seed=2)
    x = O.make_activation(M, H, seed=3)
    return gu, gus, dn, dns, x


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fp8_hand_b200 import tp
        gu, gus, dn, dns, x = _inputs()
        shard = tp.make_shard(gu, gus, dn, dns, rank, world, tiled=False, compute=OracleCompute)
        out_bf16 = tp.TensorParallelMLP(shard, compute=OracleCompute)(x)  # bf16 partials (config 4)
        out_f32 = tp.TensorParallelMLP(shard, compute=OracleCompute, partial_dtype=torch.float32)(x)
        out_chunked = tp.TensorParallelMLP(shard, compute=OracleCompute, chunks=3)(x)
        q.put((rank, (out_bf16, out_f32, out_chunked)))
    finally:
        # rank 0 hosts the rendezvous store: no rank tears down before every rank is done with it
        dist.barrier()
        dist.destroy_process_group()


def test_shards_reassemble_the_weights():
    from fp8_hand_b200 import tp
    gu, gus, dn, dns, _ = _inputs()
    for world in (2, 4):
        parts = [tp.shard_gate_up(gu, gus, r, world) for r in range(world)]
        gate = torch.cat([p[0].view(torch.uint8)[: INTER // world] for p in parts])
        up = torch.cat([p[0].view(torch.uint8)[INTER // world:] for p in parts])
        assert torch.equal(torch.cat([gate, up]), gu.view(torch.uint8))
        assert torch.equal(torch.cat([p[1][: INTER // world // 128] for p in parts]), gus[: INTER // 128])
        cols = [tp.shard_down(dn, dns, r, world) for r in range(world)]
        assert torch.equal(torch.cat([c[0].view(torch.uint8) for c in cols], dim=1), dn.view(torch.uint8))
        assert torch.equal(torch.cat([c[1] for c in cols], dim=1), dns)
    with pytest.raises(ValueError):
        tp.shard_gate_up(gu, gus, 0, 3)


def test_rank_quant_groups_are_slices_of_the_full_output():
    """Each rank's fused output (Q_r, Qs_r) equals its column slice of the 1-GPU output."""
    from fp8_hand_b200 import tp
    gu, gus, _, _, x = _inputs()
    A, As = O.group_quant(x)
    q_full, s_full, _ = O.fused_gate_up(A, gu, As, gus)
    world = 2
    for r in range(world):
        w, s = tp.shard_gate_up(gu, gus, r, world)
        q, qs, _ = O.fused_gate_up(A, w, As, s)
        per = INTER // world
        assert torch.equal(q.view(torch.uint8), q_full.view(torch.uint8)[:, r * per:(r + 1) * per])
        assert torch.equal(qs, s_full[:, r * per // 128:(r + 1) * per // 128])


def test_tp2_gloo_matches_single_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gu, gus, dn, dns, x = _inputs()
    A, As = O.group_quant(x)
    Q, Qs, _ = O.fused_gate_up(A, gu, As, gus)
    ref = O.blockwise_matmul(Q, dn, Qs, dns)
    for k in range(3):
        assert torch.equal(outs[0][k], outs[1][k])
    out_bf16, out_f32, out_chunked = outs[0]
    # fp32 partials: only the summation order differs from one rank
    assert O.max_rel_error(out_f32.float(), ref) <= 1e-2
    # bf16 partials: each rank's partial is rounded to bf16 before the sum (half an ulp, 2^-8 of its
    # magnitude) and the sum again, so the bound is absolute, against the output's scale
    err = (out_bf16.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item()
    assert O.norm_rel_error(out_bf16.float(), ref) <= 4e-3
    # row chunks with their own collectives give the same result as one collective
    assert torch.equal(out_chunked, out_bf16)


def test_reduce_mode_contract():
    """The constructor's rules, on one CPU process (no process group): an unknown reduction is refused, the
    switch and multicast reductions add bf16 partials only, and without a process group every mode falls back to
    the single-rank path."""
    from fp8_hand_b200 import tp
    with pytest.raises(ValueError):
        tp.TensorParallelMLP(None, reduce="ring", compute=OracleCompute)
    for mode in ("switch", "multimem"):
        with pytest.raises(ValueError):
            tp.TensorParallelMLP(None, reduce=mode, partial_dtype=torch.float32, compute=OracleCompute)
        mlp = tp.TensorParallelMLP(None, reduce=mode, compute=OracleCompute)
        assert (mlp.world, mlp.rank, mlp.reduce) == (1, 0, "nccl")
