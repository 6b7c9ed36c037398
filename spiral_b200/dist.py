"""Multi-GPU partitioning of the quantized-weight path (one process per GPU).

Host-side plumbing only: the compute runs in libspiral_b200.so on each rank,
the collectives are torch.distributed (NCCL over NVLink on B200; gloo in the
CPU tests).  Two partitionings, as the reference's own multi-tile pattern
suggests (weights split by output column, input broadcast:
src/quants/tests/poc/calc.py:1-11, 154-215):

* dense MUL_MAT row-sharded by output feature: rank r owns weight rows
  ``row_range(N, world, r)`` and the bf16 outputs are all-gathered;
* MoE expert FFN expert-sharded: rank r owns experts ``expert_range``; tokens
  are sharded too, each token is sent (all-to-all) to every rank that owns one
  of its experts, the partial outputs come back (all-to-all) and the owner
  adds them in rank order (deterministic).

The expert compute is a callback so that the same dispatch/combine runs with
the CUDA library on GPUs and with a CPU reference in tests.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def row_range(n: int, world: int, rank: int, align: int = 16) -> tuple[int, int]:
    """Contiguous rows [n0, n1) of rank `rank`: near-equal shards whose
    boundaries are multiples of `align` (the GEMV tile height)."""
    units = (n + align - 1) // align
    u0, u1 = rank * units // world, (rank + 1) * units // world
    return min(n, u0 * align), min(n, u1 * align)


def expert_range(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Experts [e0, e1) owned by `rank` (contiguous, near-equal)."""
    return rank * n_experts // world, (rank + 1) * n_experts // world


def gather_rows(y_local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All-gather row-sharded outputs: y_local [M][n_r] of every rank (shards
    from row_range with equal sizes) -> [M][n_total] on every rank."""
    world = dist.get_world_size(group)
    M, n_r = y_local.shape
    if n_r * world != n_total:
        raise ValueError("gather_rows needs equal shards (n_total divisible by world * 16)")
    buf = torch.empty((world * M, n_r), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    return buf.view(world, M, n_r).permute(1, 0, 2).reshape(M, n_total)


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int], group) -> None:
    dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)


def moe_dispatch_combine(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, n_experts: int,
                         compute: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                         group=None) -> torch.Tensor:
    """Expert-parallel MoE over this rank's tokens.

    x [T_r][H] (any 2-byte dtype, H even), ids int32 [T_r][topk] (global expert ids),
    weights f32 [T_r][topk].  ``compute(x_recv, ids_recv, w_recv)`` returns the
    fp32 partial [R][H] of this rank's experts for the received tokens (ids of
    other ranks' experts are skipped by it).  Returns this rank's fp32 output
    [T_r][H]: the sum over owning ranks, in rank order, of their partials.
    """
    world = dist.get_world_size(group)
    dev = x.device
    T, H = x.shape
    topk = ids.shape[1]
    # rank owning each expert id (the inverse of expert_range); -1 for ids out of range
    e = ids.to(torch.int64)
    owner = torch.div((e + 1) * world + n_experts - 1, n_experts, rounding_mode="floor") - 1
    owner = torch.where((e >= 0) & (e < n_experts), owner, torch.full_like(owner, -1))
    # rank d of the send buffer holds, in token order, every token with an expert on d
    need = torch.zeros((world, T), dtype=torch.bool, device=dev)
    for d in range(world):
        need[d] = (owner == d).any(dim=1)
    send_tok = [torch.nonzero(need[d]).flatten() for d in range(world)]
    send_counts = torch.tensor([len(s) for s in send_tok], dtype=torch.int64, device=dev)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    order = torch.cat(send_tok) if T else torch.empty(0, dtype=torch.int64, device=dev)
    R = sum(rc)
    x_recv = torch.empty((R, H), dtype=x.dtype, device=dev)
    ids_recv = torch.empty((R, topk), dtype=ids.dtype, device=dev)
    w_recv = torch.empty((R, topk), dtype=weights.dtype, device=dev)
    # 2-byte rows travel as int32 pairs (a type both NCCL and gloo move)
    _a2a(x_recv.view(torch.int32), x[order].contiguous().view(torch.int32), rc, sc, group)
    _a2a(ids_recv, ids[order].contiguous(), rc, sc, group)
    _a2a(w_recv, weights[order].contiguous(), rc, sc, group)
    part_recv = compute(x_recv, ids_recv, w_recv) if R else torch.zeros((0, H), dtype=torch.float32, device=dev)
    part_back = torch.empty((sum(sc), H), dtype=torch.float32, device=dev)
    _a2a(part_back, part_recv.contiguous(), sc, rc, group)
    y = torch.zeros((T, H), dtype=torch.float32, device=dev)
    off = 0
    for d in range(world):  # rank order: deterministic
        n = sc[d]
        if n:
            y.index_add_(0, send_tok[d], part_back[off:off + n])
        off += n
    return y


class AllGatherExchange:
    """Exchange buffers for spiral_b200.mul_mat_allgather over a gathered
    width of n_total columns: one symmetric-memory allocation per rank
    (torch.distributed._symmetric_memory, peer-mapped over NVLink), zeroed,
    and the device array of every rank's pointer (``peers``).  Collective:
    every rank constructs it with the same n_total.  One exchange serves any
    number of calls (and outputs) of that width issued in the same order on
    every rank."""

    def __init__(self, n_total: int, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        from . import allgather_exchange_bytes

        nbytes = allgather_exchange_bytes(n_total)
        if nbytes <= 0:
            raise ValueError("n_total must be a positive multiple of 8")
        self.n_total = n_total
        self._group = group
        self._buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self._buf.zero_()
        self._hdl = symm_mem.rendezvous(self._buf, group=group if group is not None else dist.group.WORLD)
        self.peers = torch.tensor(list(self._hdl.buffer_ptrs), dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def reset(self) -> None:
        """Collective: zero every rank's exchange again, as after a gathered
        wait timed out (device status bit 8); calls after it start afresh."""
        from . import allgather_exchange_reset

        torch.cuda.synchronize(self._buf.device)  # no call of any rank still in flight
        dist.barrier(group=self._group)
        allgather_exchange_reset(self._buf, self.n_total)
        torch.cuda.synchronize(self._buf.device)
        dist.barrier(group=self._group)


class MoeExchange:
    """Exchange buffers for spiral_b200.moe_ffn_ep (expert-parallel MoE) for
    up to max_tokens tokens of width `hidden`: one symmetric-memory
    allocation per rank, zeroed, and the device array of every rank's
    pointer (``peers``).  Collective: every rank constructs it with the same
    arguments."""

    def __init__(self, hidden: int, max_tokens: int, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        from . import moe_ep_exchange_bytes

        nbytes = moe_ep_exchange_bytes(hidden, max_tokens)
        if nbytes <= 0:
            raise ValueError("hidden and max_tokens must be positive")
        self.hidden, self.max_tokens = hidden, max_tokens
        self._group = group
        self._buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self._buf.zero_()
        self._hdl = symm_mem.rendezvous(self._buf, group=group if group is not None else dist.group.WORLD)
        self.peers = torch.tensor(list(self._hdl.buffer_ptrs), dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def reset(self) -> None:
        """Collective: zero every rank's exchange again, as after a timed-out
        wait (device status bit 8)."""
        from . import moe_ep_exchange_reset

        torch.cuda.synchronize(self._buf.device)  # no call of any rank still in flight
        dist.barrier(group=self._group)
        moe_ep_exchange_reset(self._buf, self.hidden, self.max_tokens)
        torch.cuda.synchronize(self._buf.device)
        dist.barrier(group=self._group)
