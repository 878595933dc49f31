"""Column (N) sharding of the W4A16 GEMM across the GPUs of one node.

Output columns of y = x . W are independent, so rank r of P owns columns
[r*N/P, (r+1)*N/P): its slice of qweight is qweight[:, r*N/(8P):(r+1)*N/(8P)]
(packed words never straddle shards because N/P is a multiple of 8, in fact
of 32 for the TMA pitch rule), and scales/zeros[:, r*N/P:(r+1)*N/P].  x is
replicated.  The one exchange step is an all-gather of the [M, N/P] output
slices over NCCL (NVLink/NVSwitch), gathered as [P, M, N/P] and laid out as
[M, N].  Nothing else is partitioned.

Two forms of the exchange:
  * ``ColumnShardedW4A16``: local GEMM into [M, N/P], then an NCCL
    all-gather and a column permute (the plain tensor-parallel baseline);
  * ``PeerGatherW4A16``: the GEMM epilogue itself stores every finished tile
    into all ranks' [M, N] outputs over NVLink (peer-mapped symmetric memory,
    plain stores) and orders itself against the peers through signal pads,
    so the whole sharded call is one kernel launch per rank: the exchange
    overlaps the tiles still being computed and no gather or permute follows.

The reference has no multi-GPU path (every task is gpus = 1,
generate_tasks.py:149); this module is the benchmark's sharded configuration.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


def shard_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    if N % world:
        raise ValueError(f"N={N} is not divisible by world size {world}")
    n = N // world
    if n % 32:
        raise ValueError(f"shard width {n} must be a multiple of 32 columns")
    return rank * n, (rank + 1) * n


def shard_weights(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, world: int,
                  rank: int):
    """This rank's column shard (contiguous copies) of the packed weight,
    scales and zero points."""
    N = qweight.shape[1] * 8
    lo, hi = shard_bounds(N, world, rank)
    return (qweight[:, lo // 8:hi // 8].contiguous(), scales[:, lo:hi].contiguous(),
            zeros[:, lo:hi].contiguous())


def gather_columns(y_local: torch.Tensor, world: int, group: Optional[dist.ProcessGroup] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather [M, N/P] slices into y [M, N] (column block r from rank r)."""
    M, n = y_local.shape
    buf = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    if out is None:
        out = torch.empty((M, world * n), dtype=y_local.dtype, device=y_local.device)
    out.view(M, world, n).copy_(buf.view(world, M, n).permute(1, 0, 2))
    return out


class ColumnShardedW4A16(nn.Module):
    """Tensor-parallel W4A16 linear: local dequant-GEMM on this rank's column
    shard, then all-gather of the output columns."""

    def __init__(self, group_size: int = 128, process_group: Optional[dist.ProcessGroup] = None,
                 local_gemm: Optional[Callable] = None):
        super().__init__()
        self.group_size = group_size
        self.pg = process_group
        if local_gemm is None:
            from . import ops
            local_gemm = ops.w4a16_gemm
        self.local_gemm = local_gemm

    def forward(self, x: torch.Tensor, qweight_shard: torch.Tensor, scales_shard: torch.Tensor,
                zeros_shard: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(self.pg) if dist.is_initialized() else 1
        y_local = self.local_gemm(x, qweight_shard, scales_shard, zeros_shard, self.group_size)
        if world == 1:
            return y_local
        return gather_columns(y_local, world, self.pg)


class PeerBuffers:
    """Per-process cache of peer-mapped ("symmetric") CUDA buffers: an output
    buffer of at least the requested bytes and a zeroed signal pad, each
    rendezvoused with every rank of the group so that this process holds
    device addresses of all ranks' copies.  Allocation is collective: every
    rank must request the same sizes in the same order (true of a
    column-sharded layer, whose M and N agree across ranks).  NVLink multicast
    objects are not created (TORCH_SYMM_MEM_DISABLE_MULTICAST=1): the kernels
    use plain peer stores only."""

    PAD_WORDS = 64

    def __init__(self, device: torch.device, process_group: Optional[dist.ProcessGroup] = None):
        import os
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem
        self._symm = symm_mem
        self.device = device
        self.pg = process_group or dist.group.WORLD
        self.rank = dist.get_rank(self.pg)
        self.world = dist.get_world_size(self.pg)
        self._out = None
        self._out_handle = None
        pad = symm_mem.empty(self.PAD_WORDS, dtype=torch.int32, device=device)
        pad.zero_()
        self._pad = pad
        self._pad_handle = symm_mem.rendezvous(pad, self.pg)
        torch.cuda.synchronize(device)
        dist.barrier(group=self.pg)
        self.pad_ptrs = list(self._pad_handle.buffer_ptrs)

    def output(self, nbytes: int):
        """(local uint8 tensor of >= nbytes, every rank's address of it)."""
        if self._out is None or self._out.numel() < nbytes:
            torch.cuda.synchronize(self.device)  # no peer store into the old buffer is in flight
            dist.barrier(group=self.pg)
            self._out = None
            self._out_handle = None
            buf = self._symm.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
            self._out_handle = self._symm.rendezvous(buf, self.pg)
            self._out = buf
        return self._out, list(self._out_handle.buffer_ptrs)


class PeerGatherW4A16(nn.Module):
    """Tensor-parallel W4A16 linear whose all-gather is fused into the GEMM:
    one kernel per rank stores this rank's columns into every rank's y over
    NVLink, waiting before its first store until every peer has reached the
    same call (so no peer still reads its previous output) and completing only
    once all columns have landed.  Returns y [M, N] in x.dtype, a view of this
    module's peer-mapped buffer: it stays valid until the next forward call."""

    def __init__(self, group_size: int = 128, process_group: Optional[dist.ProcessGroup] = None):
        super().__init__()
        self.group_size = group_size
        self.pg = process_group
        self._bufs: Optional[PeerBuffers] = None

    def forward(self, x: torch.Tensor, qweight_shard: torch.Tensor, scales_shard: torch.Tensor,
                zeros_shard: torch.Tensor) -> torch.Tensor:
        from . import ops
        world = dist.get_world_size(self.pg)
        rank = dist.get_rank(self.pg)
        M = x.shape[0]
        n = qweight_shard.shape[1] * 8
        N = n * world
        if self._bufs is None:
            self._bufs = PeerBuffers(x.device, self.pg)
        buf, ptrs = self._bufs.output(M * N * x.element_size())
        y = buf[:M * N * x.element_size()].view(x.dtype).view(M, N)
        ops.w4a16_gemm_peers(x, qweight_shard, scales_shard, zeros_shard, self.group_size, ptrs, N, rank * n,
                             self._bufs.pad_ptrs, rank)
        return y


class PeerGatherMXFP8(nn.Module):
    """Column-sharded MXFP8 linear (B [N, K] split along N) whose all-gather is
    fused into the GEMM epilogue, like PeerGatherW4A16: one kernel per rank
    stores this rank's columns into every rank's y [M, N] fp16 over NVLink.
    Returns a view of this module's peer-mapped buffer, valid until the next
    forward call."""

    def __init__(self, process_group: Optional[dist.ProcessGroup] = None):
        super().__init__()
        self.pg = process_group
        self._bufs: Optional[PeerBuffers] = None

    def forward(self, a: torch.Tensor, scales_a: torch.Tensor, b_shard: torch.Tensor,
                scales_b_shard: torch.Tensor) -> torch.Tensor:
        from . import ops
        world = dist.get_world_size(self.pg)
        rank = dist.get_rank(self.pg)
        M = a.shape[0]
        n = b_shard.shape[0]
        N = n * world
        if self._bufs is None:
            self._bufs = PeerBuffers(a.device, self.pg)
        buf, ptrs = self._bufs.output(M * N * 2)
        y = buf[:M * N * 2].view(torch.float16).view(M, N)
        ops.mxfp8_gemm_peers(a, scales_a, b_shard, scales_b_shard, ptrs, N, rank * n, self._bufs.pad_ptrs, rank)
        return y


def _grouped_experts_at(xs: torch.Tensor, offsets: torch.Tensor, w) -> torch.Tensor:
    """Grouped gate/up (fused SiLU * mul) and down GEMMs over rows already
    grouped by local expert (expert e at [offsets[e], offsets[e+1]); rows past
    offsets[-1] are left untouched in the result)."""
    from . import ops
    gq, gs, gz, uq, us, uz, dq, ds, dz = w
    g = gq.shape[1] // gs.shape[1]
    gd = dq.shape[1] // ds.shape[1]
    h = ops.moe_grouped_gemm(xs, offsets, gq, gs, gz, g, up=(uq, us, uz))
    return ops.moe_grouped_gemm(h, offsets, dq, ds, dz, gd)


def _grouped_local_experts(rows: torch.Tensor, eid: torch.Tensor, n_local: int, w) -> torch.Tensor:
    """This rank's experts on the rows it received: stable regroup by local
    expert, fused gate/up/SiLU grouped GEMM, down grouped GEMM, un-permute."""
    from . import ops
    gq, gs, gz, uq, us, uz, dq, ds, dz = w
    order = torch.argsort(eid, stable=True)
    xs = rows[order].contiguous()
    counts = torch.bincount(eid, minlength=n_local)
    offsets = torch.zeros(n_local + 1, dtype=torch.int32, device=rows.device)
    offsets[1:] = torch.cumsum(counts, 0)
    g = gq.shape[1] // gs.shape[1]
    gd = dq.shape[1] // ds.shape[1]
    h = ops.moe_grouped_gemm(xs, offsets, gq, gs, gz, g, up=(uq, us, uz))
    ye = ops.moe_grouped_gemm(h, offsets, dq, ds, dz, gd)
    out = torch.empty_like(ye)
    out[order] = ye
    return out


class ExpertParallelMoE(nn.Module):
    """Expert-parallel quantised top-2 MoE: rank r of P holds experts
    [r*E/P, (r+1)*E/P) and its own T/P tokens (data parallel).  Per call:
      1. route the local tokens (top-2 over all E experts);
      2. all-to-all of per-destination row counts, then of the token rows
         (each (token, k) pair goes to the rank owning its expert);
      3. each rank runs its experts on the rows it received;
      4. reverse all-to-all of the expert outputs, then the gated combine of
         each token's two rows on its home rank.
    The reference MoE is dense and single-GPU (generate_tasks.py:368-378); this
    is the benchmark's expert-parallel configuration (one expert per GPU at 8).

    ``route``, ``expert`` and ``combine`` are injectable so the exchange logic
    runs on CPU ranks in tests; by default they are the library's CUDA ops,
    and the local experts run as the grouped W4A16 GEMMs (gate/up with the
    fused SiLU * mul, then down) over the received rows regrouped by expert,
    with ``local_weights`` = (gate_q, gate_s, gate_z, up_q, up_s, up_z,
    down_q, down_s, down_z) stacked over this rank's experts."""

    def __init__(self, n_experts: int, process_group: Optional[dist.ProcessGroup] = None,
                 route: Optional[Callable] = None, expert: Optional[Callable] = None,
                 combine: Optional[Callable] = None, padded: bool = True):
        super().__init__()
        self.E = n_experts
        self.padded = padded
        self.pg = process_group
        self._default_ops = route is None and combine is None
        if route is None or combine is None:
            from . import ops
            route = route or (lambda logits: ops.moe_route(logits)[:2])
            combine = combine or ops.moe_combine
        self.route = route
        self.expert = expert
        self.combine = combine

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor, local_weights) -> torch.Tensor:
        """x [T_local, D], router_logits [T_local, E]; local_weights is what
        ``expert(e_local, rows, local_weights)`` needs for this rank's experts."""
        if self.padded:
            return self._forward_padded(x, router_logits, local_weights)
        return self._forward_exact_splits(x, router_logits, local_weights)

    def _forward_padded(self, x, router_logits, local_weights):
        if x.is_cuda and self.expert is None and self._default_ops:
            return self._forward_padded_cuda(x, router_logits, local_weights)
        return self._forward_padded_torch(x, router_logits, local_weights)

    def _forward_padded_cuda(self, x, router_logits, local_weights):
        """The fixed-capacity exchange with the library's kernels for the
        bookkeeping: moe_route's expert-grouped permutation, ep_pack (send
        rows with their local expert ids, each token's two slots), one
        all-to-all, ep_regroup (stable order by local expert), ep_gather into
        the grouped GEMMs' rows and back, the return all-to-all, and the gated
        combine reading the returned rows in place."""
        from . import ops
        P = dist.get_world_size(self.pg)
        E, T, D = self.E, x.shape[0], x.shape[1]
        epr = E // P
        C = 2 * T
        _, gates, offsets, slot_token, token_slot = ops.moe_route(router_logits)
        send, pair_slot = ops.ep_pack(x, offsets, slot_token, token_slot, E, P, C)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.pg)
        loc, src, pos = ops.ep_regroup(recv, epr)
        rows = torch.empty((P * C, D), dtype=x.dtype, device=x.device)
        ops.ep_gather(recv, src, D, rows)
        y_sorted = _grouped_experts_at(rows, loc, local_weights)
        y_recv = torch.empty((P * C, D), dtype=x.dtype, device=x.device)
        ops.ep_gather(y_sorted, pos, D, y_recv)
        back = torch.empty_like(y_recv)
        dist.all_to_all_single(back, y_recv, group=self.pg)
        return self.combine(back, pair_slot, gates)

    def _forward_padded_torch(self, x, router_logits, local_weights):
        """Exchange with fixed-capacity all-to-alls: every (source, destination)
        pair gets C = 2 * T_local row slots (the most one rank can send to
        another), unused slots carry expert id -1.  All counts stay on the
        device: no host synchronisation, so the whole forward can be captured
        in a CUDA graph.  Row results equal the exact-split exchange's."""
        P = dist.get_world_size(self.pg)
        E, T, D = self.E, x.shape[0], x.shape[1]
        epr = E // P
        dev = x.device
        C = 2 * T
        topi, gates = self.route(router_logits)
        pair_e = topi.long().reshape(-1)  # pair j = (token j // 2, choice j % 2)
        pair_t = torch.arange(2 * T, device=dev) // 2
        order = torch.argsort(pair_e * (2 * T) + torch.arange(2 * T, device=dev))  # by expert, then pair
        dest = pair_e[order] // epr
        # counts by scatter-add (bincount reads its size back to the host)
        counts = torch.zeros(P, dtype=torch.int64, device=dev).scatter_add_(0, dest, torch.ones_like(dest))
        starts = torch.cumsum(counts, 0) - counts
        slot = dest * C + torch.arange(2 * T, device=dev) - starts[dest]
        # each row carries its local expert id (-1: empty slot) in an extra
        # column (small integers are exact in fp16 / bf16), so one all-to-all
        # moves rows and ids; 8 extra columns keep rows 16-byte pitched
        send = x.new_empty((P * C, D + 8))
        send[:, D] = -1
        send[slot, :D] = x[pair_t[order]]
        send[slot, D] = (pair_e[order] - dest * epr).to(x.dtype)
        recv2 = torch.empty_like(send)
        dist.all_to_all_single(recv2, send, group=self.pg)
        recv = recv2[:, :D]
        recv_eid = recv2[:, D].to(torch.int64)
        # this rank's experts over the received rows, regrouped by expert (empty slots last)
        key = torch.where(recv_eid >= 0, recv_eid, torch.full_like(recv_eid, epr))
        o2 = torch.argsort(key * (P * C) + torch.arange(P * C, device=dev))
        cnt = torch.zeros(epr + 1, dtype=torch.int64, device=dev).scatter_add_(0, key, torch.ones_like(key))[:epr]
        offsets = torch.zeros(epr + 1, dtype=torch.int32, device=dev)
        offsets[1:] = torch.cumsum(cnt, 0).to(torch.int32)
        rows = recv[o2].contiguous()
        if self.expert is None:
            y_sorted = _grouped_experts_at(rows, offsets, local_weights)
        else:
            y_sorted = torch.zeros_like(rows)
            offs = offsets.tolist()
            for el in range(epr):
                if offs[el + 1] > offs[el]:
                    y_sorted[offs[el]:offs[el + 1]] = self.expert(el, rows[offs[el]:offs[el + 1]].contiguous(),
                                                                  local_weights)
        y_recv = torch.empty((P * C, D), dtype=x.dtype, device=dev)
        y_recv[o2] = y_sorted
        back = torch.empty_like(y_recv)
        dist.all_to_all_single(back, y_recv, group=self.pg)
        ye = torch.empty((2 * T, D), dtype=x.dtype, device=dev)
        ye[order] = back[slot]
        token_slot = torch.arange(2 * T, device=dev, dtype=torch.int32).reshape(T, 2)
        return self.combine(ye, token_slot, gates)

    def _forward_exact_splits(self, x, router_logits, local_weights):
        """Exchange with all-to-alls of exactly the routed rows (split sizes
        read on the host each call)."""
        P = dist.get_world_size(self.pg)
        r = dist.get_rank(self.pg)
        E, T, D = self.E, x.shape[0], x.shape[1]
        epr = E // P
        topi, gates = self.route(router_logits)
        topi = topi.long()
        # (token, k) pairs sorted by destination rank, then expert, then token
        pair_e = topi.reshape(-1)
        pair_t = torch.arange(T, device=x.device).repeat_interleave(2)
        order = torch.argsort(pair_e * (T + 1) + pair_t, stable=True)
        dest = pair_e[order] // epr
        send_counts = torch.bincount(dest, minlength=P)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.pg)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        send_rows = x[pair_t[order]].contiguous()
        send_eid = pair_e[order].to(torch.int32).contiguous()
        recv_rows = x.new_empty((sum(rc), D))
        recv_eid = torch.empty((sum(rc),), dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_rows, send_rows, rc, sc, group=self.pg)
        dist.all_to_all_single(recv_eid, send_eid, rc, sc, group=self.pg)
        # local experts on their rows
        out = torch.empty_like(recv_rows)
        if self.expert is None:
            if recv_rows.shape[0]:
                out = _grouped_local_experts(recv_rows, (recv_eid - r * epr).long(), epr, local_weights)
        else:
            for el in range(epr):
                sel = torch.nonzero(recv_eid == r * epr + el).flatten()
                if sel.numel():
                    out[sel] = self.expert(el, recv_rows[sel].contiguous(), local_weights)
        # return trip, then undo the sort: row j of `back` is pair order[j]
        back = x.new_empty((sum(sc), D))
        dist.all_to_all_single(back, out, sc, rc, group=self.pg)
        ye = torch.empty((2 * T, D), dtype=x.dtype, device=x.device)
        ye[order] = back
        token_slot = torch.arange(2 * T, device=x.device, dtype=torch.int32).reshape(T, 2)
        return self.combine(ye, token_slot, gates)
