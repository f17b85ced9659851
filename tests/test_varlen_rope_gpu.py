"""GPU parity of dvattn_varlen_paged_sdpa, the standalone rope ops and the LSE merge."""
import numpy as np
import pytest
import torch

import fixtures
from conftest import assert_lse_close, assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
from oracle import dvattn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def run_varlen(c):
    g = c.to(DEV)
    T, Hq, _ = g.queries.shape
    out = torch.full((T, Hq, g.v_cache.size(3)), float("nan"), dtype=g.dtype, device=DEV)
    lse = torch.full((T, Hq), float("nan"), device=DEV)
    o32 = torch.full((T, Hq, g.v_cache.size(3)), float("nan"), device=DEV)
    capi.varlen_paged_sdpa(*g.capi_args(out), lse=lse, out_f32=o32)
    torch.cuda.synchronize()
    return out, lse, o32


def check_varlen(c, what):
    out, lse, o32 = run_varlen(c)
    ref32, rlse = O.varlen_paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                                          c.k_cache, c.v_cache, c.block_tables, c.cu_seqlens_q)
    assert_out_close(out, ref32.to(c.dtype), c.dtype, what)
    assert_out_close(o32, ref32, c.dtype, what + " f32")
    assert_lse_close(lse, rlse, what)


@pytest.mark.parametrize("name", fixtures.names("varlen_"))
def test_varlen_golden(name):
    t, m = fixtures.load(name)
    g = {k: v.to(DEV) for k, v in t.items()}
    out = torch.empty_like(g["out"])
    capi.varlen_paged_sdpa(out, m["scale"], g["locations"], g["queries"], g["cosines"], g["sines"],
                           g["fragment_lengths"], g["k_cache"], g["v_cache"], g["block_tables"], g["cu_seqlens_q"])
    torch.cuda.synchronize()
    assert_out_close(out, t["out"], t["out"].dtype, name)
    import dvattn_b200  # torch op path
    out2 = torch.empty_like(g["out"])
    torch.ops.libdvatt.dvattn_varlen_paged_sdpa(out2, m["scale"], g["locations"], g["queries"], g["cosines"],
                                                g["sines"], g["fragment_lengths"], g["k_cache"], g["v_cache"],
                                                g["block_tables"], g["cu_seqlens_q"], g["cu_seqlens_q"])
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_varlen_random(dtype):
    rs = np.random.RandomState(3)
    W = 6
    ql = rs.randint(1, 80, size=W)
    prior = rs.randint(0, 300, size=W)
    tl = [[int(a + b)] for a, b in zip(prior, ql)]
    c = wl.make_varlen(tl, ql.tolist(), Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=dtype, seed=3)
    check_varlen(c, f"varlen {dtype}")


def test_varlen_multiturn_and_skipped_turns():
    c = wl.make_varlen([[40, 0, 17], [0, 12, 9], [12, 3, 30]], [3, 9, 7], Hq=16, Hkv=1, E=128, R=64, BS=8,
                       dtype=torch.bfloat16, seed=4)
    check_varlen(c, "varlen turns")


def test_varlen_empty_sequences_in_batch():
    c = wl.make_varlen([[5], [9], [20]], [0, 9, 0], Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.float16, seed=6)
    check_varlen(c, "varlen empty seqs")


def test_config4_subset():
    tl, ql = wl.config4_lengths(4, 16)
    tl, ql = tl[:3], ql[:3]
    c = wl.make_varlen(tl, ql, Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=4)
    check_varlen(c, "config4 (3 sequences)")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_rope_ops(dtype):
    c = wl.make_paged([[20, 5], [7, 30]], Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=dtype, seed=2, S=3)
    g = c.to(DEV)
    out = torch.empty((2,) + tuple(g.queries.shape), dtype=dtype, device=DEV)
    capi.rope(out, g.queries, g.cosines, g.sines)
    torch.cuda.synchronize()
    ref = O.rope(c.queries, c.cosines, c.sines)
    assert_out_close(out, ref, dtype, "rope")
    import dvattn_b200
    out2 = dvattn_b200.dvattn_rope(g.queries, g.cosines, g.sines)
    assert torch.equal(out, out2)

    v = wl.make_varlen([[20], [9]], [4, 9], Hq=16, Hkv=1, E=128, R=32, BS=16, dtype=dtype, seed=2).to(DEV)
    vo = dvattn_b200.dvattn_varlen_rope(v.queries, v.cosines, v.sines)
    torch.cuda.synchronize()
    assert_out_close(vo, O.varlen_rope(v.queries.cpu(), v.cosines.cpu(), v.sines.cpu()), dtype, "varlen rope")


@pytest.mark.parametrize("name", fixtures.names("paged_"))
def test_rope_golden(name):
    t, _ = fixtures.load(name)
    g = {k: v.to(DEV) for k, v in t.items()}
    out = torch.empty_like(g["rotated"])
    capi.rope(out, g["queries"], g["cosines"], g["sines"])
    torch.cuda.synchronize()
    assert_out_close(out, t["rotated"], t["rotated"].dtype, name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_lse_merge_kernel(dtype):
    torch.manual_seed(0)
    P, rows, Ev = 4, 37, 256
    po = torch.randn(P, rows, Ev)
    pl = torch.randn(P, rows) * 3
    pl[1, :5] = float("-inf")
    pl[:, 7] = float("-inf")  # a row with no part
    ref, rl = O.lse_merge(po, pl)
    out = torch.empty(rows, Ev, dtype=dtype, device=DEV)
    lo = torch.empty(rows, device=DEV)
    capi.lse_merge(po.to(DEV), pl.to(DEV), out, lo)
    torch.cuda.synchronize()
    assert_out_close(out, ref.to(dtype), dtype, "merge")
    assert_lse_close(lo, rl, "merge")
    assert torch.all(out[7] == 0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_lse_merge_packed_kernel(dtype):
    """Packed parts (outputs then LSEs per part, as one all-gather lays them out) merge to
    the same result as the separate-buffer entry point, bit for bit."""
    torch.manual_seed(1)
    P, rows, Ev = 3, 29, 128
    po = torch.randn(P, rows, Ev)
    pl = torch.randn(P, rows) * 3
    pl[2, :4] = float("-inf")
    pl[:, 9] = float("-inf")
    packed = torch.cat([po.reshape(P, -1), pl], dim=1).contiguous().to(DEV)
    out = torch.empty(rows, Ev, dtype=dtype, device=DEV)
    lo = torch.empty(rows, device=DEV)
    capi.lse_merge_packed(packed, out, lo)
    out2 = torch.empty_like(out)
    lo2 = torch.empty_like(lo)
    capi.lse_merge(po.to(DEV), pl.to(DEV), out2, lo2)
    torch.cuda.synchronize()
    assert torch.equal(out, out2) and torch.equal(lo, lo2)
    assert torch.all(out[9] == 0)


def test_split_kv_across_parts_equals_whole():
    """A long sequence cut into page-aligned KV chunks, each run as its own paged call with
    LSE output, merges back to the unsplit result (the multi-GPU long-context path)."""
    from dvattn_b200 import dist
    c = wl.make_paged([[4096]] * 2, Hq=16, Hkv=1, E=128, R=128, BS=64, dtype=torch.float16, seed=17).to(DEV)
    whole = c.new_out()
    capi.paged_sdpa(*c.op_args(whole))
    parts_o, parts_l = [], []
    for r in range(4):
        sh = dist.kv_chunk_shard(c, r, 4)
        o = sh.new_out()
        l = torch.empty(o.shape[:3], device=DEV)
        o32 = torch.empty(o.shape, device=DEV)
        capi.paged_sdpa(*sh.op_args(o), lse=l, out_f32=o32)
        parts_o.append(o32)
        parts_l.append(l)
    merged = torch.empty_like(whole)
    capi.lse_merge(torch.stack(parts_o), torch.stack(parts_l), merged)
    torch.cuda.synchronize()
    assert_out_close(merged, whole.float(), torch.float16, "split-kv merge")


def test_packed_merge_of_real_shards_equals_unsharded():
    """Three KV-chunk shards of a real paged call write their partials through
    dist.packed_partials; the buffers laid end to end (as one all-gather produces them)
    merge with dvattn_lse_merge_packed to the unsharded call's output."""
    from dvattn_b200 import dist as ddist
    full = wl.make_paged([[3000], [1301], [64]], Hq=32, Hkv=2, E=128, R=64, BS=16, dtype=torch.bfloat16,
                         seed=31).to(DEV)
    ref = full.new_out()
    capi.paged_sdpa(*full.op_args(ref))
    parts = []
    for r in range(3):
        sh = ddist.kv_chunk_shard(full, r, 3, local_pages=True)
        out = sh.new_out()
        packed, o32, lse = ddist.packed_partials(out)
        capi.paged_sdpa(*sh.op_args(out), lse=lse, out_f32=o32)
        parts.append(packed)
    gathered = torch.stack(parts).contiguous()
    merged = torch.full_like(ref, float("nan"))
    capi.lse_merge_packed(gathered, merged)
    torch.cuda.synchronize()
    assert_out_close(merged, ref.float(), torch.bfloat16, "packed merge of 3 real shards")
