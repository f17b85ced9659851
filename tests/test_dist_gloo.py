"""Multi-GPU partitioning logic on CPU ranks (gloo, world size 2): KV-chunk sharding of a
long context, the all-gather + LSE-merge exchange, sequence balancing, and a rank that
fails between steps.  The attention of each shard runs through the CPU oracle and the
merge is injected (the product merge is the CUDA kernel, covered by the GPU tests)."""
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dvattn_b200 import dist as ddist
from dvattn_b200 import workloads as wl
from oracle import dvattn_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_merge(po, pl, out, lse_out):
    o, l = O.lse_merge(po, pl)
    out.copy_(o.to(out.dtype))
    if lse_out is not None:
        lse_out.copy_(l)
    return out


def _worker(rank, world, port, fn, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        fn(rank, world)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    return res


def _long_context_case():
    return wl.make_paged([[1000], [777]], Hq=16, Hkv=1, E=64, R=64, BS=16, dtype=torch.float32, seed=5)


def _kv_shard_and_merge(rank, world):
    c = _long_context_case()
    sh = ddist.kv_chunk_shard(c, rank, world)
    o32, lse = O.paged_sdpa_f32(sh.scale, sh.locations, sh.queries, sh.cosines, sh.sines, sh.fragment_lengths,
                                sh.k_cache, sh.v_cache, sh.block_tables)
    out = torch.empty_like(o32)
    lse_out = torch.empty_like(lse)
    ddist.allgather_merge(o32, lse, out, merge=_oracle_merge, lse_out=lse_out)
    ref, rlse = O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                                 c.k_cache, c.v_cache, c.block_tables)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(lse_out, rlse, rtol=1e-5, atol=1e-5)


def test_kv_chunk_sharding_and_merge_world2():
    res = _run(_kv_shard_and_merge)
    assert all(v == "ok" for v in res.values()), res


def _kv_shard_and_merge_packed(rank, world):
    c = _long_context_case()
    sh = ddist.kv_chunk_shard(c, rank, world)
    o32, lse = O.paged_sdpa_f32(sh.scale, sh.locations, sh.queries, sh.cosines, sh.sines, sh.fragment_lengths,
                                sh.k_cache, sh.v_cache, sh.block_tables)
    packed, po, pl = ddist.packed_partials(o32)
    po.copy_(o32)
    pl.copy_(lse)
    out = torch.empty_like(o32)
    lse_out = torch.empty_like(lse)
    ddist.allgather_merge_packed(packed, out, merge=_oracle_merge, lse_out=lse_out)
    ref, rlse = O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                                 c.k_cache, c.v_cache, c.block_tables)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(lse_out, rlse, rtol=1e-5, atol=1e-5)


def test_kv_chunk_sharding_and_packed_merge_world2():
    """One all-gather of the packed (outputs, LSEs) buffer per rank gives the unsharded result."""
    res = _run(_kv_shard_and_merge_packed)
    assert all(v == "ok" for v in res.values()), res


def _batch_shard(rank, world):
    tl = wl.config2_lengths(2, 12)
    weights = [sum(t) for t in tl]
    mine = ddist.balance(weights, world)[rank]
    c = wl.make_paged([tl[i] for i in mine], Hq=16, Hkv=1, E=64, R=32, BS=16, dtype=torch.float32, seed=rank)
    out, _ = O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths, c.k_cache,
                              c.v_cache, c.block_tables)
    # every rank did its share; no data-path collective, only a count check
    n = torch.tensor([len(mine)])
    dist.all_reduce(n)
    assert int(n) == 12 and torch.isfinite(out).all()


def test_batch_sharding_world2():
    res = _run(_batch_shard)
    assert all(v == "ok" for v in res.values()), res


def _failing_rank(rank, world):
    # rank 1 fails between steps (before its collective); rank 0 learns it from the
    # collective erroring out, not by hanging: gloo raises when the peer goes away
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
    except Exception:
        raise RuntimeError("peer failure observed") from None


def test_failing_rank_is_reported_not_hung():
    res = _run(_failing_rank)
    assert "injected failure" in res[1]
    assert res[0] != "ok" and "peer failure observed" in res[0]


def test_balance_is_lpt_and_deterministic():
    w = [5, 9, 1, 7, 3, 8]
    b = ddist.balance(w, 2)
    loads = [sum(w[i] for i in x) for x in b]
    assert sorted(sum(b, [])) == list(range(6))
    assert max(loads) - min(loads) <= max(w)
    assert b == ddist.balance(w, 2)


def test_kv_chunk_bounds_are_page_aligned_and_cover():
    for total, bs, n in [(131072, 64, 8), (1000, 16, 3), (5, 16, 4)]:
        cb = ddist.kv_chunk_bounds(total, bs, n)
        assert cb[0][0] == 0 and cb[-1][1] == total
        for (a, b), (c, d) in zip(cb, cb[1:]):
            assert b == c and a % bs == 0


def _kv_shard_local_pages(rank, world):
    c = _long_context_case()
    sh = ddist.kv_chunk_shard(c, rank, world, local_pages=True)
    # the rank keeps only its chunk's pages
    assert sh.k_cache.size(0) <= sh.block_tables.numel() < c.k_cache.size(0)
    o32, lse = O.paged_sdpa_f32(sh.scale, sh.locations, sh.queries, sh.cosines, sh.sines, sh.fragment_lengths,
                                sh.k_cache, sh.v_cache, sh.block_tables)
    packed, po, pl = ddist.packed_partials(o32)
    po.copy_(o32)
    pl.copy_(lse)
    gathered = ddist.gather_buffer(packed)
    out = torch.empty_like(o32)
    with pytest.raises(ValueError):
        ddist.allgather_merge_packed(packed, out, merge=_oracle_merge, gathered=gathered[1:])
    ddist.allgather_merge_packed(packed, out, merge=_oracle_merge, gathered=gathered)
    ref, _ = O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                              c.k_cache, c.v_cache, c.block_tables)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)


def test_kv_chunk_local_pages_and_gather_buffer_world2():
    """Each rank holds only its chunk's pages; the preallocated receive buffer is used."""
    res = _run(_kv_shard_local_pages)
    assert all(v == "ok" for v in res.values()), res


def test_shard_batch_matches_the_whole_batch():
    """A rank's sequences with a pool of only their pages give the rows of the whole batch."""
    c = wl.make_paged(wl.config2_lengths(2, 6), Hq=16, Hkv=2, E=64, R=32, BS=16, dtype=torch.float32, seed=7)
    ref, rlse = O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                                 c.k_cache, c.v_cache, c.block_tables)
    for seqs in ([0, 3], [5], [1, 2, 4]):
        sub = ddist.shard_batch(c, seqs)
        used = np.unique(c.block_tables[seqs].numpy())
        assert sub.k_cache.size(0) == int(((used >= 0) & (used < c.k_cache.size(0))).sum())
        out, lse = O.paged_sdpa_f32(sub.scale, sub.locations, sub.queries, sub.cosines, sub.sines,
                                    sub.fragment_lengths, sub.k_cache, sub.v_cache, sub.block_tables)
        torch.testing.assert_close(out, ref[seqs], rtol=0, atol=0)
        torch.testing.assert_close(lse, rlse[seqs], rtol=0, atol=0)
