"""Tensor-parallel MLP over NCCL: one process per GPU inside one 8 x B200 box.

The reference runs on one GPU (scripts/run_sglang_48g.sh:117, `--tp-size 1`); this is the
B200-side extension for an 8-GPU box:

  gate_up  column-parallel, no collective. Rank r keeps gate rows [r*I/tp, (r+1)*I/tp) and the
           same up rows, packed as [gate_r; up_r], so the fused kernel's "up starts at N2/2"
           layout (patches/fp8_hand_sm89.py:450) holds per rank. I/tp is a multiple of 128, so
           no 128x128 scale block straddles two ranks.
  down     row-parallel over its K = I: rank r keeps columns [r*I/tp, (r+1)*I/tp) of W_down
           and the matching scale columns. The fused kernel's quant groups (128 wide) line up
           with those columns, so each rank's (Q_r, Qs_r) is exactly its slice of the 1-GPU
           (Q, Qs).
  reduce   all_reduce(sum) of the bf16 [M, H] partials (fp32 optional). With chunks > 1 the rows are
           processed in chunks and each chunk's all_reduce runs asynchronously while the next chunk
           computes; the library's persistent kernels then leave SMs free for NCCL when
           BS_FP8_SM_LIMIT caps their grid.
           reduce="multimem": no separate collective. The output is a symmetric-memory buffer with an
           NVSwitch multicast mapping, and the down_proj kernel adds each finished bf16 tile into every
           rank's copy (bs_fp8_gemm_reduce_multicast), so the reduction overlaps the GEMM tile by tile.
           A one-element NCCL all_reduce orders the zeroing of the copies before the GEMMs and the GEMMs
           before the result is read. `chunks` does not apply: the reduction already overlaps the GEMM.
           Two ranks only: the switch adds the ranks' bf16 partials into each copy in no fixed order, which
           for two partials (0 + a + b) always rounds the same way, but for three or more can round
           differently in different ranks' copies and leave the replicas unequal.
           reduce="switch": any number of ranks. Each rank's down_proj writes its partial into its own copy of
           a symmetric buffer (plain local stores), then one kernel (bs_fp8_tp_reduce_switch) has rank r read
           the r-th 1/tp of the rows reduced by the switch (multimem.ld_reduce, fp32 accumulation) and store
           the sums into every copy (multimem.st). Each GPU moves about (tp-1)/tp of the [M, H] buffer each way
           whatever tp is, against (tp-1) x the buffer into every GPU for "multimem"; the kernel's own
           cross-rank flags order the GEMMs before the reads and the stores before the return, so no NCCL call
           and no zeroing is needed, and every rank's copy holds the same bytes.

The per-rank math goes through `compute`, an object with group_quant / gemm_silu_quant / gemm:
the CUDA ops module by default. Tests on CPU ranks pass another implementation to check the
sharding and the collective without a GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

BLOCK = 128


@dataclass
class MLPShard:
    gate_up: torch.Tensor        # e4m3 [2 * I/tp, H] (or tile-first bytes)
    gate_up_scale: torch.Tensor  # fp32 [2 * I/tp / 128, H / 128]
    down: torch.Tensor           # e4m3 [H, I/tp]   (or tile-first bytes)
    down_scale: torch.Tensor     # fp32 [H / 128, I/tp / 128]
    tiled: bool = False


def shard_gate_up(w: torch.Tensor, s: torch.Tensor, rank: int, world: int) -> tuple[torch.Tensor, torch.Tensor]:
    """[gate; up] rows of the full gate_up weight -> this rank's [gate_r; up_r]."""
    n2, _ = w.shape
    inter = n2 // 2
    if inter % (BLOCK * world):
        raise ValueError(f"intermediate size {inter} is not a multiple of 128 * tp={world}")
    per = inter // world
    u8 = w.view(torch.uint8)
    rows = torch.cat([u8[rank * per:(rank + 1) * per], u8[inter + rank * per:inter + (rank + 1) * per]])
    pb = per // BLOCK
    ib = inter // BLOCK
    srows = torch.cat([s[rank * pb:(rank + 1) * pb], s[ib + rank * pb:ib + (rank + 1) * pb]])
    return rows.view(torch.float8_e4m3fn).contiguous(), srows.contiguous()


def shard_down(w: torch.Tensor, s: torch.Tensor, rank: int, world: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Columns [r*I/tp, (r+1)*I/tp) of W_down [H, I] and of its scales."""
    _, inter = w.shape
    if inter % (BLOCK * world):
        raise ValueError(f"intermediate size {inter} is not a multiple of 128 * tp={world}")
    per = inter // world
    pb = per // BLOCK
    cols = w.view(torch.uint8)[:, rank * per:(rank + 1) * per].contiguous().view(torch.float8_e4m3fn)
    return cols, s[:, rank * pb:(rank + 1) * pb].contiguous()


def make_shard(gate_up, gate_up_scale, down, down_scale, rank: int, world: int, device=None,
               tiled: bool = True, compute=None) -> MLPShard:
    gw, gs = shard_gate_up(gate_up, gate_up_scale, rank, world)
    dw, ds = shard_down(down, down_scale, rank, world)
    if device is not None:
        gw, gs, dw, ds = (t.to(device) for t in (gw, gs, dw, ds))
    if tiled:
        if compute is None:
            from . import ops as compute
        gw, dw = compute.pack_tiles(gw), compute.pack_tiles(dw)
    return MLPShard(gw, gs, dw, ds, tiled)


class TensorParallelMLP:
    """x [M, H] bf16 (replicated) -> quant -> fused gate_up_r -> down_r -> all_reduce -> [M, H]."""

    def __init__(self, shard: MLPShard, group=None, partial_dtype: torch.dtype = torch.bfloat16, compute=None,
                 chunks: int = 1, reduce: str = "nccl", return_buffer: bool = False):
        """reduce="multimem" and reduce="switch" return a copy of the shared output buffer unless
        return_buffer=True, in which case the caller gets the buffer's row view itself and must consume it before
        the next call overwrites it."""
        if compute is None:
            from . import ops as compute
        if reduce not in ("nccl", "multimem", "switch"):
            raise ValueError(f"reduce must be 'nccl', 'multimem' or 'switch', not {reduce!r}")
        if reduce in ("multimem", "switch") and partial_dtype != torch.bfloat16:
            raise ValueError("the switch reductions add bf16 partials")
        self.shard = shard
        self.group = group
        self.partial_dtype = partial_dtype
        self.compute = compute
        self.chunks = max(1, int(chunks))
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if reduce == "multimem" and self.world > 2:
            raise ValueError("reduce='multimem' needs exactly two ranks: with three or more the switch's bf16 "
                             "additions can round differently in different ranks' copies")
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.reduce = reduce if self.world > 1 else "nccl"
        self.return_buffer = return_buffer
        self._mc = None  # (output buffer [rows, n], symmetric-memory handle, multicast address of row 0)
        self._sw = None  # (data [rows, n], handle, data multicast address, flags, handle, flags multicast address)
        self._epoch = 0
        self._flag = None

    def _sync(self, device) -> None:
        """Orders every rank's earlier kernels on its stream before every rank's later ones."""
        if self._flag is None:
            self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        dist.all_reduce(self._flag, group=self.group)

    def multicast_out(self, m: int, n: int, device) -> tuple:
        """Rows [0, m) of this rank's copy of the bf16 output buffer in symmetric memory, with the multicast
        address of its row 0. One buffer serves every row count: rows are contiguous with stride n, so row 0's
        multicast address maps any leading row view. It is allocated (collectively: every rank calls this
        with the same m) on first use and when a larger m arrives, then at least doubling, so serving with
        varying batch sizes allocates O(log M) times and never keeps more than one buffer."""
        buf = self._mc
        if buf is None or m > buf[0].shape[0] or n != buf[0].shape[1]:
            import torch.distributed._symmetric_memory as symm_mem
            rows = m if buf is None or n != buf[0].shape[1] else max(m, 2 * buf[0].shape[0])
            self._mc = None
            out = symm_mem.empty(rows, n, dtype=torch.bfloat16, device=device)
            handle = symm_mem.rendezvous(out, self.group if self.group is not None else dist.group.WORLD)
            base = handle.multicast_ptr
            if not base:
                raise RuntimeError("the group has no NVSwitch multicast mapping (NVLS)")
            self._mc = (out, handle, base + (out.data_ptr() - handle.buffer_ptrs[handle.rank]))
        out, handle, mc = self._mc
        return out[:m], handle, mc

    def switch_buffers(self, m: int, n: int, device) -> tuple:
        """Rows [0, m) of this rank's copy of the symmetric bf16 partial/output buffer, its multicast address,
        and the flag buffer with its multicast address, for reduce="switch". Allocated collectively (every rank
        calls with the same m) on first use and when a larger m arrives, then at least doubling; the flags are
        zeroed and every rank has zeroed them before any rank's first reduction."""
        buf = self._sw
        if buf is None or m > buf[0].shape[0] or n != buf[0].shape[1]:
            import torch.distributed._symmetric_memory as symm_mem
            group = self.group if self.group is not None else dist.group.WORLD
            rows = m if buf is None or n != buf[0].shape[1] else max(m, 2 * buf[0].shape[0])
            self._sw = None
            data = symm_mem.empty(rows, n, dtype=torch.bfloat16, device=device)
            dh = symm_mem.rendezvous(data, group)
            flags = symm_mem.empty(self.compute.tp_flag_words(self.world), dtype=torch.int32, device=device)
            flags.zero_()
            fh = symm_mem.rendezvous(flags, group)
            if not dh.multicast_ptr or not fh.multicast_ptr:
                raise RuntimeError("the group has no NVSwitch multicast mapping (NVLS)")
            torch.cuda.synchronize(device)
            dist.barrier(group=group)
            self._sw = (data, dh, dh.multicast_ptr + (data.data_ptr() - dh.buffer_ptrs[dh.rank]),
                        flags, fh, fh.multicast_ptr + (flags.data_ptr() - fh.buffer_ptrs[fh.rank]))
            self._epoch = 0
        data, _, mc, flags, _, fmc = self._sw
        return data[:m], mc, flags, fmc

    def partial(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's [M, H] contribution (before the reduction)."""
        c, s = self.compute, self.shard
        A, As = c.group_quant(x)
        Q, Qs = c.gemm_silu_quant(A, s.gate_up, As, s.gate_up_scale, b_tiled=s.tiled)
        return c.gemm(Q, s.down, Qs, s.down_scale, b_tiled=s.tiled, out_dtype=self.partial_dtype)

    def _chunk_rows(self, m: int) -> list[tuple[int, int]]:
        step = -(-m // self.chunks)
        step = -(-step // BLOCK) * BLOCK  # whole 128-row tiles per chunk
        return [(r, min(r + step, m)) for r in range(0, m, step)]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.reduce == "switch":
            c, s = self.compute, self.shard
            data, mc, flags, fmc = self.switch_buffers(x.shape[0], s.down.shape[0] * (BLOCK if s.tiled else 1),
                                                       x.device)
            A, As = c.group_quant(x)
            Q, Qs = c.gemm_silu_quant(A, s.gate_up, As, s.gate_up_scale, b_tiled=s.tiled)
            c.gemm(Q, s.down, Qs, s.down_scale, b_tiled=s.tiled, out=data)
            self._epoch += 1
            c.tp_reduce_switch(data, mc, flags, fmc, self.rank, self.world, self._epoch)
            return data if self.return_buffer else data.clone()
        if self.reduce == "multimem":
            c, s = self.compute, self.shard
            out, _, mc = self.multicast_out(x.shape[0], s.down.shape[0] * (BLOCK if s.tiled else 1), x.device)
            out.zero_()
            self._sync(x.device)
            A, As = c.group_quant(x)
            Q, Qs = c.gemm_silu_quant(A, s.gate_up, As, s.gate_up_scale, b_tiled=s.tiled)
            c.gemm_reduce_multicast(Q, s.down, Qs, s.down_scale, out, mc, b_tiled=s.tiled)
            self._sync(x.device)
            return out if self.return_buffer else out.clone()
        if self.world == 1 or self.chunks == 1 or x.shape[0] <= BLOCK:
            part = self.partial(x)
            if self.world > 1:
                dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            return part.to(torch.bfloat16)
        # Chunked rows: chunk i's all_reduce overlaps chunk i+1's GEMMs. Every rank issues the same
        # collectives in the same order.
        c, s = self.compute, self.shard
        A, As = c.group_quant(x)
        out = torch.empty((x.shape[0], s.down.shape[0] * (BLOCK if s.tiled else 1)), dtype=self.partial_dtype,
                          device=x.device)
        works = []
        for r0, r1 in self._chunk_rows(x.shape[0]):
            Q, Qs = c.gemm_silu_quant(A[r0:r1], s.gate_up, As[r0:r1], s.gate_up_scale, b_tiled=s.tiled)
            c.gemm(Q, s.down, Qs, s.down_scale, b_tiled=s.tiled, out=out[r0:r1])
            works.append(dist.all_reduce(out[r0:r1], op=dist.ReduceOp.SUM, group=self.group, async_op=True))
        for w in works:
            w.wait()
        return out.to(torch.bfloat16)
