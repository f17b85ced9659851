"""GPU parity of the paged decode (dvattn_paged_sdpa) against the reference's outputs
(golden fixtures) and the CPU oracle, called through the C ABI (libdvattn_b200.so via
ctypes) unless a test says it exercises the torch op layer."""
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


def run_capi(case_tensors, scale, with_extra=True):
    (q, loc, cos, sin, L, kc, vc, bt) = case_tensors
    W, Hq, S, _ = q.shape
    out = torch.full((W, Hq, S, vc.size(3)), float("nan"), dtype=q.dtype, device=DEV)
    lse = torch.full((W, Hq, S), float("nan"), device=DEV) if with_extra else None
    o32 = torch.full((W, Hq, S, vc.size(3)), float("nan"), device=DEV) if with_extra else None
    capi.paged_sdpa(out, scale, loc, q, cos, sin, L, kc, vc, bt, lse=lse, out_f32=o32)
    torch.cuda.synchronize()
    return out, lse, o32


def case_tensors(c):
    c = c.to(DEV)
    return (c.queries, c.locations, c.cosines, c.sines, c.fragment_lengths, c.k_cache, c.v_cache, c.block_tables)


def check_vs_oracle(c, what):
    out, lse, o32 = run_capi(case_tensors(c), c.scale)
    ref32, rlse = O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                                   c.k_cache, c.v_cache, c.block_tables)
    assert_out_close(out, ref32.to(c.dtype), c.dtype, what + " out")
    assert_out_close(o32, ref32, c.dtype, what + " out_f32")
    assert_lse_close(lse, rlse, what + " lse")
    return out


@pytest.mark.parametrize("name", fixtures.names("paged_"))
def test_golden_capi(name):
    t, m = fixtures.load(name)
    args = tuple(t[k].to(DEV) for k in ("queries", "locations", "cosines", "sines", "fragment_lengths", "k_cache",
                                        "v_cache", "block_tables"))
    out, lse, o32 = run_capi(args, m["scale"])
    dt = t["out"].dtype
    assert_out_close(out, t["out"], dt, name)
    assert_out_close(o32, t["out_f32"], dt, name + " f32")
    assert_lse_close(lse, t["lse"], name)


@pytest.mark.parametrize("name", fixtures.names("paged_"))
def test_golden_torch_op(name):
    import dvattn_b200  # noqa: F401  (registers torch.ops.libdvatt)
    t, m = fixtures.load(name)
    g = {k: v.to(DEV) for k, v in t.items()}
    out = torch.empty_like(g["out"])
    torch.ops.libdvatt.dvattn_paged_sdpa(out, m["scale"], g["locations"], g["queries"], g["cosines"], g["sines"],
                                         g["fragment_lengths"], g["k_cache"], g["v_cache"], g["block_tables"])
    torch.cuda.synchronize()
    assert_out_close(out, t["out"], t["out"].dtype, name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("E", [64, 128, 256])
def test_dtypes_and_head_dims(dtype, E):
    c = wl.make_paged([[300, 45], [17, 900], [1, 1], [64, 0]], Hq=32, Hkv=2, E=E, R=32, BS=16, dtype=dtype, seed=E)
    check_vs_oracle(c, f"{dtype} E={E}")


@pytest.mark.parametrize("gqa", [1, 2, 4, 8, 16])
def test_gqa_ratios(gqa):
    c = wl.make_paged([[130], [47]], Hq=2 * gqa, Hkv=2, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=gqa)
    check_vs_oracle(c, f"gqa={gqa}")


@pytest.mark.parametrize("BS", [1, 3, 16, 64, 128, 256])
def test_page_sizes(BS):
    c = wl.make_paged([[513, 77], [1000, 3]], Hq=16, Hkv=1, E=128, R=64, BS=BS, dtype=torch.float16, seed=BS)
    check_vs_oracle(c, f"BS={BS}")


@pytest.mark.parametrize("R", [0, 2, 32, 64, 126, 128])
def test_rotary_dims(R):
    c = wl.make_paged([[200, 30]], Hq=16, Hkv=1, E=128, R=R, BS=16, dtype=torch.bfloat16, seed=R)
    check_vs_oracle(c, f"R={R}")


@pytest.mark.parametrize("S", [2, 5])
def test_multi_query(S):
    c = wl.make_paged([[90, 40], [7, 300]], Hq=32, Hkv=2, E=128, R=64, BS=16, dtype=torch.float16, seed=S, S=S)
    check_vs_oracle(c, f"S={S}")


def test_many_turns_and_empty_turns():
    rs = np.random.RandomState(7)
    tl = rs.randint(0, 90, size=(9, 7))
    tl[rs.rand(9, 7) < 0.3] = 0
    tl[:, 3] += 1
    c = wl.make_paged(tl.tolist(), Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=7)
    check_vs_oracle(c, "many turns")


def test_rows_without_keys_are_zero():
    c = wl.make_paged([[10, 5], [0, 0], [7, 0], [0, 3]], Hq=16, Hkv=1, E=128, R=64, BS=4, dtype=torch.bfloat16,
                      seed=3)
    out = check_vs_oracle(c, "empty rows")
    assert torch.all(out[1] == 0)


def test_partial_visibility_masks_in_turn():
    """loc inside a turn (not its last key) and loc past L: both follow `kp > loc`."""
    tl = [[50, 40], [60, 10]]
    loc = np.array([[[10], [59]], [[100], [-3]]])  # [F, W, S]
    c = wl.make_paged(tl, Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.float16, seed=5, loc_override=loc)
    check_vs_oracle(c, "partial loc")


def test_unused_block_table_entries_are_not_read():
    """Entries past each sequence's visible pages hold garbage (huge / negative ids): the
    kernel must never dereference them."""
    c = wl.make_paged([[33, 20], [500, 2], [1, 1]], Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=9,
                      fill=2 ** 30)
    check_vs_oracle(c, "garbage tables")
    c2 = wl.make_paged([[33, 20], [500, 2], [1, 1]], Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=9,
                       fill=-7)
    check_vs_oracle(c2, "negative tables")


def test_long_single_sequence_split_across_ctas():
    c = wl.make_paged([[65536]], Hq=16, Hkv=1, E=128, R=128, BS=64, dtype=torch.float16, seed=31)
    check_vs_oracle(c, "long context")


def test_many_short_sequences():
    rs = np.random.RandomState(8)
    tl = rs.randint(1, 40, size=(600, 1)).tolist()
    c = wl.make_paged(tl, Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=8)
    check_vs_oracle(c, "many short")


def test_config1_full():
    check_vs_oracle(wl.config1(), "config1")


def test_config2_full():
    check_vs_oracle(wl.config2(), "config2")


def test_config5_subset():
    c = wl.make_paged(wl.config5_lengths(5, 48), Hq=32, Hkv=2, E=256, R=64, BS=64, dtype=torch.float16, seed=5)
    check_vs_oracle(c, "config5 (48 sequences)")


def test_deterministic_and_workspace_reuse():
    c = wl.config2(W=8).to(DEV)
    out1 = c.new_out()
    out2 = c.new_out()
    call1 = capi.PagedCall(*c.op_args(out1))
    call2 = capi.PagedCall(*c.op_args(out2), workspace=call1.workspace)
    call1()
    call2()
    call1()
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)


def test_chained_call_reads_previous_output():
    """The second call's queries are the first call's output, with no other kernel between
    them: the second call must see the merged output, not what the buffer held before
    (the first kernel of a call may start early only when the previous call's outputs are
    none of its inputs)."""
    c = wl.config2(W=32).to(DEV)
    out1 = torch.full_like(c.new_out(), float("nan"))
    out2 = c.new_out()
    args1 = list(c.op_args(out1))
    args2 = list(c.op_args(out2))
    args2[3] = out1  # queries of the second call
    call1 = capi.PagedCall(*args1)
    call2 = capi.PagedCall(*args2)
    for _ in range(5):
        out1.fill_(float("nan"))
        call1()
        call2()
        torch.cuda.synchronize()
        ref = out1.clone()
        args3 = list(args2)
        args3[0] = torch.empty_like(out2)
        args3[3] = ref
        capi.PagedCall(*args3)()
        torch.cuda.synchronize()
        assert not torch.isnan(out2).any()
        assert torch.equal(out2, args3[0])


def test_torch_op_on_side_stream():
    import dvattn_b200
    c = wl.make_paged([[300, 45], [17, 900]], Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=1).to(DEV)
    ref = c.new_out()
    dvattn_b200.dvattn_paged_sdpa(c.queries, c.locations, c.cosines, c.sines, c.fragment_lengths, c.k_cache,
                                  c.v_cache, c.block_tables, c.scale, out=ref)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = dvattn_b200.dvattn_paged_sdpa(c.queries, c.locations, c.cosines, c.sines, c.fragment_lengths, c.k_cache,
                                            c.v_cache, c.block_tables, c.scale)
    s.synchronize()
    assert torch.equal(out, ref)


def test_torch_op_errors():
    import dvattn_b200  # noqa: F401
    c = wl.make_paged([[30]], Hq=32, Hkv=1, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=1).to(DEV)
    with pytest.raises(RuntimeError, match="unsupported"):
        torch.ops.libdvatt.dvattn_paged_sdpa(*c.op_args(c.new_out()))  # GQA 32
    c = wl.make_paged([[30]], Hq=16, Hkv=1, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=1).to(DEV)
    out = c.new_out().to(torch.float64)
    with pytest.raises(RuntimeError, match="dtype"):
        torch.ops.libdvatt.dvattn_paged_sdpa(*c.op_args(out))
    with pytest.raises(RuntimeError, match="contiguous"):
        strided = torch.empty(c.new_out().shape[:3] + (256,), dtype=torch.bfloat16, device=DEV)[..., ::2]
        torch.ops.libdvatt.dvattn_paged_sdpa(*c.op_args(strided))
    with pytest.raises(RuntimeError, match="wrong tensor ranks"):  # paged tensors given to the fragment op
        torch.ops.libdvatt.dvattn_sdpa(c.new_out(), 0.1, c.locations, c.queries, c.fragment_lengths, [c.k_cache],
                                       [c.v_cache])


@pytest.mark.parametrize("Hkv", [1, 2, 3, 4, 8, 16])
@pytest.mark.parametrize("BS", [8, 16, 64, 128])
def test_kv_head_counts_and_pages(Hkv, BS):
    """Covers the row kernel (Hkv in 1,2,4,8), the per-head TMA kernel (other Hkv) and the
    page-size windows of both."""
    c = wl.make_paged([[700, 90], [33, 400], [5, 0]], Hq=4 * Hkv, Hkv=Hkv, E=128, R=64, BS=BS,
                      dtype=torch.bfloat16, seed=Hkv * 100 + BS)
    check_vs_oracle(c, f"Hkv={Hkv} BS={BS}")


def test_config3_shape_subset():
    """Config 3 head layout (128/8, E=128, full rotary, page 64) on a shorter context."""
    c = wl.make_paged([[20000]] * 2, Hq=128, Hkv=8, E=128, R=128, BS=64, dtype=torch.float16, seed=3)
    check_vs_oracle(c, "config3 shape")


def test_error_flag_clear_after_calls():
    """The bounded waits never gave up: the workspace header's error word stays 0."""
    c = wl.config2(W=4).to(DEV)
    out = c.new_out()
    call = capi.PagedCall(*c.op_args(out))
    call()
    torch.cuda.synchronize()
    hdr = call.workspace[:16].cpu().view(torch.int32)
    assert int(hdr[3]) == 0  # {U (int64), n_eff, error}


_PDL_CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
c = wl.config2(W=8).to("cuda:0")
out = c.new_out()
call = capi.PagedCall(*c.op_args(out))
for _ in range(3):
    call()
torch.cuda.synchronize()
torch.save(out.cpu(), sys.argv[2])
"""


def test_pdl_switch_off_gives_identical_output(tmp_path):
    """DVATTN_PDL=0 (every call's first kernel an ordinary launch) changes only launch
    ordering: the output is bit-identical to the default launch."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    dst = str(tmp_path / "pdl_off.pt")
    env = dict(os.environ, DVATTN_PDL="0")
    r = subprocess.run([sys.executable, "-c", _PDL_CHILD, root, dst], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    c = wl.config2(W=8).to(DEV)
    out = c.new_out()
    call = capi.PagedCall(*c.op_args(out))
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), torch.load(dst))
