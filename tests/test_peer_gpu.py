"""The peer-memory exchange of KV-sharded partials (dvattn_lse_merge_peers).

On one GPU the ranks are emulated inside one process: every "rank's" region is a local
allocation and the other ranks' signals are written by the test before the call, so only
one kernel ever waits (no two kernels that wait on each other share the GPU).  With two or
more GPUs, two processes (one per GPU, NCCL only for the handle exchange and the checks)
run the real exchange over NVLink.  Both are compared with the plain merge of the same
partials (dvattn_lse_merge), and a missing signal is checked to end in the error word and
NaN outputs rather than a hang."""
import os
import socket
import traceback

import pytest
import torch

from conftest import assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _flags(region):
    """int32 view of a region's control block (flags of rank j at word 16 + j)."""
    return capi.device_view(region.ptr, 64, region.device).view(torch.int32)


def _emulated(parts, rows, Ev, signal_upto, slot, calls_before, dtype=torch.bfloat16):
    regions = [capi.PeerRegion(rows, Ev, DEV) for _ in range(parts)]
    for r, reg in enumerate(regions):
        packed, o32, lse = reg.slot(slot)
        g = torch.Generator(device=DEV)
        g.manual_seed(100 + r)
        o32.copy_(torch.randn(rows * Ev, generator=g, device=DEV))
        lse.copy_(torch.randn(rows, generator=g, device=DEV) * 3)
        lse[r::7] = float("-inf")  # empty parts for some rows
    ctl = _flags(regions[0])
    ctl[0] = calls_before  # the call number this region has completed
    for j in range(signal_upto):
        ctl[16 + j] = calls_before + 1  # rank j has signalled this call
    out = torch.full((rows, Ev), float("nan"), dtype=dtype, device=DEV)
    lse_out = torch.full((rows,), float("nan"), device=DEV)
    capi.lse_merge_peers([r.ptr for r in regions], 0, slot, rows, Ev, out, lse_out)
    torch.cuda.synchronize()
    po = torch.stack([reg.slot(slot)[1].view(rows, Ev) for reg in regions])
    pl = torch.stack([reg.slot(slot)[2] for reg in regions])
    return regions, out, lse_out, po, pl


@pytest.mark.parametrize("parts,slot,calls_before", [(1, 0, 0), (3, 0, 0), (3, 1, 1), (8, 1, 5)])
def test_merge_peers_matches_plain_merge(parts, slot, calls_before):
    rows, Ev = 700, 128
    regions, out, lse_out, po, pl = _emulated(parts, rows, Ev, parts, slot, calls_before)
    ref = torch.empty_like(out)
    ref_lse = torch.empty_like(lse_out)
    capi.lse_merge(po.contiguous(), pl.contiguous(), ref, ref_lse)
    torch.cuda.synchronize()
    assert_out_close(out, ref.float(), torch.bfloat16, f"peer merge {parts} parts")
    fin = torch.isfinite(ref_lse)
    assert torch.equal(fin, torch.isfinite(lse_out))
    torch.testing.assert_close(lse_out[fin], ref_lse[fin], rtol=1e-5, atol=1e-5)
    assert regions[0].status() == 0
    # the call number advanced, and this rank signalled itself and the others
    ctl = _flags(regions[0]).cpu()
    assert int(ctl[0]) == calls_before + 1 and int(ctl[1]) == 0
    for j in range(1, parts):
        assert int(_flags(regions[j]).cpu()[16]) == calls_before + 1
    for r in regions:
        r.free()


def test_merge_peers_missing_signal_sets_error_and_nan():
    rows, Ev = 64, 128
    regions, out, lse_out, _, _ = _emulated(2, rows, Ev, 1, 0, 0)  # rank 1 never signals
    assert regions[0].status() != 0
    assert torch.isnan(out.float()).all() and torch.isnan(lse_out).all()
    for r in regions:
        r.free()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _two_gpu_worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from dvattn_b200 import dist as ddist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = f"cuda:{rank}"
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device(dev))
        full = wl.make_paged([[5000], [3001], [77]], Hq=32, Hkv=2, E=128, R=64, BS=16, dtype=torch.bfloat16,
                             seed=21).to(dev)
        ref = full.new_out()
        capi.paged_sdpa(*full.op_args(ref))
        sh = ddist.kv_chunk_shard(full, rank, world, local_pages=True)
        out = sh.new_out()
        ex = ddist.PeerExchange(out)
        for step in range(4):
            slot = step & 1
            o32, lse = ex.outputs(slot)
            capi.paged_sdpa(*sh.op_args(out), lse=lse, out_f32=o32)
            merged = torch.full_like(out, float("nan"))
            ex.merge(slot, merged)
            torch.cuda.synchronize()
            assert ex.status() == 0
            err = (merged.float() - ref.float()).abs()
            bound = 1.6e-2 * (ref.float().abs() + ref.float().abs().mean(dim=-1, keepdim=True))
            assert bool((err <= bound).all()), f"step {step}: max err {err.max().item()}"
        ex.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert all(v == "ok" for v in res.values()), res
