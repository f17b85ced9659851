"""The allocation-free paged decode entry point (dvattn_paged_sdpa_noalloc).

Some callers cannot hand the library a workspace: their memory pool owns the whole GPU
and forbids cudaMalloc after start-up, or they are plain C hosts without a device
allocator.  dvattn_paged_sdpa_noalloc serves them from a fixed scratch array inside the
library.  These tests call it through the C ABI and compare it with the regular
dvattn_paged_sdpa (caller-owned workspace) on two calls in a row, within the output
tolerance the other tests use.  The file sorts last so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import pytest
import torch

from conftest import assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _noalloc(case, out):
    a = capi.paged_args(*case.op_args(out))
    st = capi.lib().dvattn_paged_sdpa_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    return st


@pytest.mark.parametrize("make", [lambda: wl.config2(W=8, device=DEV),
                                  lambda: wl.make_paged([[300, 45], [17, 900], [0, 0]], Hq=32, Hkv=2, E=128, R=32,
                                                        BS=16, dtype=torch.float16, seed=4, device=DEV)])
def test_noalloc_matches_workspace_entry_point_twice(make):
    c = make()
    ref = c.new_out()
    capi.paged_sdpa(*c.op_args(ref))
    for _ in range(2):  # the second call reuses the scratch left by the first
        out = torch.full_like(ref, float("nan"))
        assert _noalloc(c, out) == capi.DVATTN_OK
        torch.cuda.synchronize()
        assert_out_close(out, ref.float(), c.dtype, "noalloc vs workspace entry point")


def test_noalloc_rejects_problems_beyond_the_scratch():
    """A batch whose workspace exceeds the fixed scratch is refused before anything is
    launched, so the argument struct may describe it without the tensors existing."""
    cap = capi.lib().dvattn_paged_sdpa_noalloc_max_workspace()
    assert cap == 32 << 20
    c = wl.make_paged([[20]], Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=1, device=DEV)
    a = capi.paged_args(*c.op_args(c.new_out()))
    a.W = 8_000_000  # prefix sums alone need 8 bytes per sequence row
    need = capi.lib().dvattn_paged_sdpa_workspace_size(ctypes.byref(a))
    assert need > cap
    assert capi.lib().dvattn_paged_sdpa_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == \
        capi.DVATTN_ERR_WORKSPACE


def test_noalloc_call_allocates_no_device_memory():
    """After the first call on the device (which looks up the scratch address), further
    calls change neither the torch allocator's statistics nor the device's free memory."""
    c = wl.config2(W=8, device=DEV)
    out = c.new_out()
    assert _noalloc(c, out) == capi.DVATTN_OK
    torch.cuda.synchronize()
    before_stats = torch.cuda.memory_stats(DEV)["allocated_bytes.all.current"]
    before_free = torch.cuda.mem_get_info(DEV)[0]
    for _ in range(3):
        assert _noalloc(c, out) == capi.DVATTN_OK
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats(DEV)["allocated_bytes.all.current"] == before_stats
    assert torch.cuda.mem_get_info(DEV)[0] == before_free
    assert capi.workspace_status(None) == 0
