"""Multi-GPU partitioning of the paged decode (one process per GPU, torch.distributed).

Two ways the work splits across the GPUs of one box:

* by sequence (batch decode, varlen prefill): sequences are independent, so each rank
  runs the op on its own sequences with no data-path collective.  ``balance`` assigns
  sequences to ranks by longest-processing-time on their attended-key counts.
* by KV chunk (one very long context): each rank holds a page-aligned slice of every
  sequence's positions, runs the op on its slice with LSE output, and the partial
  outputs are exchanged over NCCL (all-gather of f32 O and LSE) and merged by the
  ``dvattn_lse_merge`` kernel -- the same log-sum-exp reduction the single-GPU split-KV
  uses (src/kernels/paged_kernel_v21.cuh:307-374), one level up.

The reference has no multi-GPU path; it would have to run one process per GPU because
its workspace is a process-wide static (src/kernels/paged_kernel_v21.cuh:397-408).
"""
from __future__ import annotations

import heapq
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .workloads import PagedCase


def balance(weights: Sequence[int], n: int) -> List[List[int]]:
    """Longest-processing-time assignment of items (by weight) to n bins; each bin's item
    list is sorted.  Deterministic (ties broken by index)."""
    heap = [(0, r) for r in range(n)]
    bins: List[List[int]] = [[] for _ in range(n)]
    for i in sorted(range(len(weights)), key=lambda i: (-weights[i], i)):
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + int(weights[i]), r))
    return [sorted(b) for b in bins]


def kv_chunk_bounds(total: int, block_size: int, n: int) -> List[Tuple[int, int]]:
    """Split logical positions [0, total) into n page-aligned, contiguous, near-equal chunks."""
    pages = -(-total // block_size)
    out = []
    for r in range(n):
        a = pages * r // n * block_size
        b = min(total, pages * (r + 1) // n * block_size)
        out.append((min(a, total), b))
    return out


def compact_pages(k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor):
    """A pool holding only the pages `block_tables` references, and the table renumbered
    into it.  Entries outside [0, NB) stay outside (-1), so they still read as zeros."""
    NB = k_cache.size(0)
    bt = block_tables.to(torch.int64)
    valid = (bt >= 0) & (bt < NB)
    used = torch.unique(bt[valid])
    lookup = torch.full((NB,), -1, dtype=torch.int64, device=bt.device)
    lookup[used] = torch.arange(used.numel(), device=bt.device)
    new_bt = torch.where(valid, lookup[bt.clamp(0, max(NB - 1, 0))], torch.full_like(bt, -1))
    idx = used.to(k_cache.device)
    return k_cache[idx].contiguous(), v_cache[idx].contiguous(), new_bt.to(torch.int32).contiguous()


def shard_batch(case: PagedCase, seqs: Sequence[int]) -> PagedCase:
    """The sequences `seqs` of a paged decode case as a case of their own, with a page pool
    holding only their pages (what the rank that owns them keeps in memory).  Turn lengths
    stay global (they place the turns in every sequence's logical positions)."""
    dev = case.queries.device
    idx = torch.as_tensor(list(seqs), dtype=torch.int64, device=dev)
    S = case.queries.size(2)
    kc, vc, bt = compact_pages(case.k_cache, case.v_cache, case.block_tables.index_select(0, idx))
    return PagedCase(queries=case.queries.index_select(0, idx).contiguous(),
                     locations=case.locations.index_select(1, idx).contiguous(),
                     cosines=case.cosines.index_select(1, idx).contiguous(),
                     sines=case.sines.index_select(1, idx).contiguous(),
                     fragment_lengths=case.fragment_lengths.clone(), k_cache=kc, v_cache=vc, block_tables=bt,
                     scale=case.scale,
                     turn_lens=None if case.turn_lens is None else case.turn_lens[list(seqs)],
                     meta=dict(case.meta, seqs=list(seqs), S=S))


def kv_chunk_shard(case: PagedCase, rank: int, world: int, local_pages: bool = False) -> PagedCase:
    """The slice of a single-turn paged case that rank `rank` of `world` attends over.
    Keys keep their rotation (it is relative to the turn start, which does not move);
    locations shift by the chunk start, so key l of the chunk is visible iff
    a + l <= loc.  local_pages=False shares the page pool (views); True gives the shard a
    pool of only the pages of its chunk (what the rank keeps in memory)."""
    F = case.locations.size(0)
    if F != 1:
        raise ValueError("kv_chunk_shard: KV-chunk sharding is defined for single-turn caches")
    BS = case.k_cache.size(1)
    L = int(case.fragment_lengths[0].item())
    a, b = kv_chunk_bounds(L, BS, world)[rank]
    dev = case.locations.device
    loc = case.locations.to(torch.int64) - a
    loc = torch.clamp(loc, min=-1).to(torch.int32)
    bt = case.block_tables[:, a // BS: max(a // BS + 1, -(-b // BS))].contiguous()
    kc, vc = case.k_cache, case.v_cache
    if local_pages:
        kc, vc, bt = compact_pages(kc, vc, bt)
    return PagedCase(queries=case.queries, locations=loc.contiguous(), cosines=case.cosines, sines=case.sines,
                     fragment_lengths=torch.tensor([b - a], dtype=torch.int32, device=dev), k_cache=kc,
                     v_cache=vc, block_tables=bt, scale=case.scale, turn_lens=case.turn_lens,
                     meta=dict(case.meta, chunk=(a, b)))


def _cuda_merge(part_out: torch.Tensor, part_lse: torch.Tensor, out: torch.Tensor, lse: Optional[torch.Tensor]):
    from .api import dvattn_lse_merge
    dvattn_lse_merge(part_out, part_lse, out, lse)
    return out


def allgather_merge(out_f32: torch.Tensor, lse: torch.Tensor, out: torch.Tensor, group=None,
                    merge: Optional[Callable] = None, lse_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Exchange this rank's partial (f32 output [..., Ev] + natural-log LSE [...]) with
    every rank of `group` and merge them into `out` on every rank.  `merge` defaults to
    the CUDA merge kernel; it is injectable so the exchange logic can run on CPU ranks."""
    world = dist.get_world_size(group)
    # gathered straight into the [parts, ...] layout the merge reads (no per-rank list, no stack)
    # (ranks concatenated along dim 0, which every backend accepts, then viewed as parts)
    o, l = out_f32.contiguous().reshape(-1), lse.contiguous().reshape(-1)
    po = torch.empty(world * o.numel(), dtype=o.dtype, device=o.device)
    pl = torch.empty(world * l.numel(), dtype=l.dtype, device=l.device)
    dist.all_gather_into_tensor(po, o, group=group)
    dist.all_gather_into_tensor(pl, l, group=group)
    po = po.view((world,) + tuple(out_f32.shape))
    pl = pl.view((world,) + tuple(lse.shape))
    return (merge or _cuda_merge)(po, pl, out, lse_out)


def packed_partials(out: torch.Tensor):
    """One f32 buffer holding a rank's partial outputs (shape of `out`) followed by its
    natural-log LSEs (shape out.shape[:-1]), so that allgather_merge_packed exchanges both
    in a single collective.  Returns (packed, out_f32 view, lse view); pass the views as the
    attention call's out_f32 / lse outputs."""
    Ev = out.size(-1)
    rows = out.numel() // Ev
    packed = torch.empty(rows * (Ev + 1), dtype=torch.float32, device=out.device)
    return packed, packed[: rows * Ev].view(out.shape), packed[rows * Ev:].view(out.shape[:-1])


class PeerExchange:
    """KV-sharded partials exchanged over peer memory: every rank holds one exchange region
    (two slots of packed f32 outputs + LSEs), the regions are mapped into every rank through
    CUDA IPC handles (exchanged once with all_gather_object), and one kernel per step
    signals, waits for every rank (bounded) and merges the partials read from the peers'
    memory (dvattn_lse_merge_peers).  Replaces the all-gather + merge pair of
    allgather_merge_packed; the step allocates nothing and can be captured in a CUDA graph.

    Use: o32, lse = ex.outputs(slot) as the attention call's out_f32 / lse_out, then
    ex.merge(slot, out); consecutive steps alternate slot 0 / 1."""

    def __init__(self, out: torch.Tensor, group=None):
        from . import capi
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PeerExchange: at most 8 ranks")
        self.shape = tuple(out.shape)
        self.Ev = out.size(-1)
        self.rows = out.numel() // self.Ev
        self.region = capi.PeerRegion(self.rows, self.Ev, out.device)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(self.region.handle), group=group)
        self.opened = []
        ptrs = []
        for j, h in enumerate(handles):
            if j == self.rank:
                ptrs.append(self.region.ptr)
            else:
                p = capi.open_peer_region(h, out.device)
                self.opened.append(p)
                ptrs.append(p)
        self.regions = ptrs
        self._slots = [self.region.slot(s) for s in (0, 1)]

    def outputs(self, slot: int):
        """(out_f32 [out.shape] f32, lse [out.shape[:-1]] f32) views of this rank's slot."""
        _, o32, lse = self._slots[slot]
        return o32.view(self.shape), lse.view(self.shape[:-1])

    def merge(self, slot: int, out: torch.Tensor, lse_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        from . import capi
        return capi.lse_merge_peers(self.regions, self.rank, slot, self.rows, self.Ev, out, lse_out)

    def status(self) -> int:
        """Error word of this rank's region: nonzero when a wait for another rank ran out."""
        return self.region.status()

    def close(self):
        """Unmap the peers' regions and free this rank's (after every rank is done)."""
        from . import capi
        torch.cuda.synchronize(self.region.device)
        dist.barrier(group=self.group)
        for p in self.opened:
            capi.lib().dvattn_peer_region_close(p)
        self.opened = []
        dist.barrier(group=self.group)
        self.region.free()


def gather_buffer(packed: torch.Tensor, group=None) -> torch.Tensor:
    """A receive buffer for allgather_merge_packed (allocated once and passed every step, so
    the step allocates nothing and can be captured in a CUDA graph)."""
    return torch.empty(dist.get_world_size(group) * packed.numel(), dtype=torch.float32, device=packed.device)


def allgather_merge_packed(packed: torch.Tensor, out: torch.Tensor, group=None, merge: Optional[Callable] = None,
                           lse_out: Optional[torch.Tensor] = None,
                           gathered: Optional[torch.Tensor] = None) -> torch.Tensor:
    """allgather_merge with one all-gather: `packed` is this rank's buffer from
    packed_partials.  The default merge reads the gathered parts in place
    (dvattn_lse_merge_packed); an injected `merge` gets the same (part_out, part_lse, out,
    lse_out) arguments as in allgather_merge.  `gathered` (from gather_buffer) is the
    receive buffer; without it one is allocated per call."""
    world = dist.get_world_size(group)
    Ev = out.size(-1)
    rows = out.numel() // Ev
    if packed.numel() != rows * (Ev + 1) or packed.dtype != torch.float32:
        raise ValueError("allgather_merge_packed: packed must be f32 with rows * (Ev + 1) elements")
    if packed.device != out.device:
        raise ValueError("allgather_merge_packed: packed and out must be on the same device")
    if gathered is None:
        g = torch.empty(world * packed.numel(), dtype=torch.float32, device=packed.device)
    else:
        if gathered.numel() != world * packed.numel() or gathered.dtype != torch.float32 or \
                gathered.device != packed.device or not gathered.is_contiguous():
            raise ValueError("allgather_merge_packed: gathered must be contiguous f32 [world * packed.numel()] "
                             "on packed's device")
        g = gathered
    dist.all_gather_into_tensor(g, packed.contiguous().reshape(-1), group=group)
    g = g.view(world, rows * (Ev + 1))
    if merge is None:
        from . import capi
        return capi.lse_merge_packed(g, out, lse_out)
    po = g[:, : rows * Ev].reshape((world,) + tuple(out.shape))
    pl = g[:, rows * Ev:].reshape((world,) + tuple(out.shape[:-1]))
    return merge(po, pl, out, lse_out)
