"""Bounded-wait aborts are reported to the caller.

Every wait inside the attention kernels gives up after ~2 s, sets an error word in the
call's workspace and ends the kernel.  dvattn_workspace_status reads that word back
(workspace == NULL: the allocation-free entry point's scratch); the paged decode's merge
kernel then writes NaN to every output of the call, the tensor-core prefill to the rows of
the items that gave up, and with DVATTN_CHECK_STATUS=1 the torch ops raise.

The failing case is made without faulting anything: DVATTN_TEST_STALL_TILE=<i> makes CTA 0
never issue the loads of its tile i, so the consumers' wait on that stage runs out with no
copy in flight.  Those runs happen in child processes (the hook is read once per process).
The reference surfaces kernel failures as a RuntimeError (src/binding.cu:200,
src/cuda_check.cuh:16-29).
"""
import os
import subprocess
import sys

import pytest
import torch

from dvattn_b200 import capi
from dvattn_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_status_zero_after_completed_calls():
    c = wl.config2(W=4).to(DEV)
    out = c.new_out()
    call = capi.PagedCall(*c.op_args(out))
    for _ in range(2):
        call()
        assert call.status() == 0
    v = wl.make_varlen([[300], [77]], [40, 77], Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16,
                       seed=2).to(DEV)
    vo = v.new_out()
    old = os.environ.get("DVATTN_PREFILL")
    os.environ["DVATTN_PREFILL"] = "1"
    try:
        vc = capi.VarlenCall(*v.capi_args(vo))
        vc()
        assert vc.status() == 0
    finally:
        if old is None:
            os.environ.pop("DVATTN_PREFILL", None)
        else:
            os.environ["DVATTN_PREFILL"] = old


def test_status_rejects_null_output_pointer():
    assert capi.lib().dvattn_workspace_status(None, None, None) == capi.DVATTN_ERR_INVALID_ARGUMENT


_CHILD = r"""
import ctypes, os, sys
import torch
sys.path.insert(0, sys.argv[1])
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
import dvattn_b200
what = sys.argv[2]
if what == "paged":
    c = wl.config2(W=4).to("cuda:0")
    out = c.new_out()
    lse = torch.zeros(out.shape[:-1], dtype=torch.float32, device="cuda:0")
    call = capi.PagedCall(*c.op_args(out), lse=lse)
    call()
    word = call.status()
    assert word != 0, "error word not set"
    assert torch.isnan(out.float()).all(), "outputs not marked invalid"
    assert torch.isnan(lse).all(), "lse not marked invalid"
    # the context is still usable: a plain copy and a second (stalled) call both return
    x = torch.arange(10, device="cuda:0").sum().item()
    assert x == 45
    print("paged", word)
elif what == "torch_op":
    c = wl.config2(W=4).to("cuda:0")
    try:
        dvattn_b200.dvattn_paged_sdpa(c.queries, c.locations, c.cosines, c.sines, c.fragment_lengths, c.k_cache,
                                      c.v_cache, c.block_tables, c.scale)
        torch.cuda.synchronize()
    except RuntimeError as e:
        assert "bounded wait" in str(e), str(e)
        print("torch_op raised")
    else:
        raise SystemExit("torch op did not raise")
elif what == "noalloc":
    c = wl.config2(W=4).to("cuda:0")
    out = c.new_out()
    a = capi.paged_args(*c.op_args(out))
    st = capi.lib().dvattn_paged_sdpa_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == 0, st
    word = capi.workspace_status(None)
    assert word != 0
    assert torch.isnan(out.float()).all()
    print("noalloc", word)
elif what == "prefill":
    os.environ["DVATTN_PREFILL"] = "1"
    v = wl.make_varlen([[300], [77]], [40, 77], Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16,
                       seed=2).to("cuda:0")
    vo = torch.zeros_like(v.new_out())
    vc = capi.VarlenCall(*v.capi_args(vo))
    vc()
    word = vc.status()
    assert word != 0
    nan_rows = torch.isnan(vo.float()).all(dim=-1)
    assert nan_rows.any(), "no row marked invalid"
    fin = torch.isfinite(vo.float()).all(dim=-1)
    assert bool((nan_rows | fin).all()), "rows partly written"
    print("prefill", word, int(nan_rows.sum()))
"""


@pytest.mark.parametrize("what", ["paged", "torch_op", "noalloc", "prefill"])
def test_stalled_wait_is_reported(what):
    env = dict(os.environ, DVATTN_TEST_STALL_TILE="0", DVATTN_CHECK_STATUS="1")
    r = subprocess.run([sys.executable, "-c", _CHILD, ROOT, what], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    assert r.stdout.strip(), r.stderr[-2000:]
