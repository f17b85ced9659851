"""GPU parity of the tensor-core varlen prefill (tcgen05 + TMEM) against the CPU oracle.

DVATTN_PREFILL=1 routes every supported varlen shape to the prefill kernel, however small,
so these cases exercise it; DVATTN_PREFILL=0 keeps them on the split-KV schedule, and the
two paths are compared with each other as well as with the oracle."""
import os

import numpy as np
import pytest
import torch

from conftest import assert_lse_close, assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
from oracle import dvattn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture
def prefill_mode():
    old = os.environ.get("DVATTN_PREFILL")

    def set_mode(v):
        os.environ["DVATTN_PREFILL"] = v

    set_mode("1")
    yield set_mode
    if old is None:
        os.environ.pop("DVATTN_PREFILL", None)
    else:
        os.environ["DVATTN_PREFILL"] = old


def run(c, cu=None):
    g = c.to(DEV)
    T, Hq, _ = g.queries.shape
    Ev = g.v_cache.size(3)
    out = torch.full((T, Hq, Ev), float("nan"), dtype=g.dtype, device=DEV)
    lse = torch.full((T, Hq), float("nan"), device=DEV)
    o32 = torch.full((T, Hq, Ev), float("nan"), device=DEV)
    args = list(g.capi_args(out))
    if cu is not None:
        args[-1] = cu.to(DEV)
    capi.varlen_paged_sdpa(*args, lse=lse, out_f32=o32)
    torch.cuda.synchronize()
    return out, lse, o32


def check(c, what, cu=None):
    out, lse, o32 = run(c, cu)
    ref32, rlse = O.varlen_paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                                          c.k_cache, c.v_cache, c.block_tables,
                                          c.cu_seqlens_q if cu is None else cu)
    assert_out_close(out, ref32.to(c.dtype), c.dtype, what)
    assert_out_close(o32, ref32, c.dtype, what + " f32")
    assert_lse_close(lse, rlse, what)
    return out, lse


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_random(prefill_mode, dtype):
    rs = np.random.RandomState(11)
    W = 5
    ql = rs.randint(1, 90, size=W)
    prior = rs.randint(0, 400, size=W)
    tl = [[int(a + b)] for a, b in zip(prior, ql)]
    c = wl.make_varlen(tl, ql.tolist(), Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=dtype, seed=11)
    check(c, f"prefill {dtype}")


@pytest.mark.parametrize("BS", [8, 32, 64, 128])
def test_prefill_page_sizes(prefill_mode, BS):
    c = wl.make_varlen([[300], [77], [140]], [40, 77, 19], Hq=16, Hkv=1, E=128, R=64, BS=BS,
                       dtype=torch.bfloat16, seed=BS)
    check(c, f"prefill BS={BS}")


@pytest.mark.parametrize("Hq,Hkv", [(8, 1), (12, 3), (32, 4)])
def test_prefill_gqa_below_16(prefill_mode, Hq, Hkv):
    c = wl.make_varlen([[130], [64]], [33, 64], Hq=Hq, Hkv=Hkv, E=128, R=16, BS=16, dtype=torch.float16, seed=Hq)
    check(c, f"prefill gqa {Hq}/{Hkv}")


def test_prefill_multiturn_and_skipped_turns(prefill_mode):
    c = wl.make_varlen([[40, 0, 17], [0, 12, 9], [200, 3, 130], [5, 260, 0]], [3, 9, 70, 0], Hq=16, Hkv=1,
                       E=128, R=64, BS=8, dtype=torch.bfloat16, seed=4)
    check(c, "prefill turns")


def test_prefill_empty_sequences(prefill_mode):
    c = wl.make_varlen([[5], [9], [20], [0], [33]], [0, 9, 0, 0, 17], Hq=16, Hkv=1, E=128, R=64, BS=16,
                       dtype=torch.float16, seed=6)
    check(c, "prefill empty seqs")


def test_prefill_invalid_pages_read_zero(prefill_mode):
    c = wl.make_varlen([[150], [90]], [30, 50], Hq=16, Hkv=1, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=8)
    bt = c.block_tables.clone()
    bt[0, 2] = -1
    bt[1, 0] = c.k_cache.size(0) + 5
    c.block_tables = bt
    check(c, "prefill invalid pages")


def test_prefill_tokens_past_last_sequence_go_to_sequence_0(prefill_mode):
    # the reference maps a token outside every [cu[w], cu[w+1]) to sequence 0
    c = wl.make_varlen([[120], [60], [90]], [20, 30, 25], Hq=16, Hkv=1, E=128, R=32, BS=16,
                       dtype=torch.bfloat16, seed=9)
    cu = c.cu_seqlens_q.clone()
    cu[-1] = cu[-1] - 9  # the last 9 tokens now belong to no sequence
    check(c, "prefill tail tokens", cu=cu)


def test_prefill_config4_subset(prefill_mode):
    tl, ql = wl.config4_lengths(4, 16)
    c = wl.make_varlen(tl[:3], ql[:3], Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=4)
    check(c, "prefill config4 (3 sequences)")


def test_prefill_matches_split_kv_path(prefill_mode):
    c = wl.make_varlen([[700], [257], [1000]], [300, 200, 64], Hq=32, Hkv=2, E=128, R=32, BS=16,
                       dtype=torch.bfloat16, seed=12)
    out1, lse1, o1 = run(c)
    prefill_mode("0")
    out0, lse0, o0 = run(c)
    torch.testing.assert_close(o1, o0, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(lse1, lse0, rtol=1e-4, atol=1e-4)


def test_prefill_repeatable(prefill_mode):
    c = wl.make_varlen([[500], [123]], [128, 123], Hq=16, Hkv=1, E=128, R=32, BS=32, dtype=torch.bfloat16, seed=13)
    a = run(c)
    b = run(c)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("mode", ["1", "0"])
def test_varlen_phases_equal_whole_call(prefill_mode, mode):
    prefill_mode(mode)
    c = wl.make_varlen([[400], [150]], [96, 150], Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=14)
    g = c.to(DEV)
    a = g.new_out()
    b = g.new_out()
    capi.VarlenCall(*g.capi_args(a))()
    call = capi.VarlenCall(*g.capi_args(b))
    for ph in (capi.DVATTN_PHASE_SCHEDULE, capi.DVATTN_PHASE_ATTEND, capi.DVATTN_PHASE_MERGE):
        call.phase(ph)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
