"""Full-size parity: configs 2-5 of the benchmark whole, against the CPU oracle and, where
the reference's CUDA kernels accept the shape (E = Ev = 128, GQA 16:
src/kernels/paged_kernel_v21.cuh:413, varlen_paged_kernel_v21.cuh:410), against the
reference's own CUDA op built for sm_100a (oracle/_ref, run in a child process).  Also the
reference-generated varlen golden vectors through the tensor-core prefill kernel."""
import os
import subprocess
import sys
import tempfile

import pytest
import torch

import fixtures
from conftest import assert_lse_close, assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
from oracle import dvattn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "dvatt_ref.so")
needs_ref = pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref not built")


@pytest.fixture
def prefill_env():
    old = os.environ.get("DVATTN_PREFILL")

    def set_mode(v):
        if v is None:
            os.environ.pop("DVATTN_PREFILL", None)
        else:
            os.environ["DVATTN_PREFILL"] = v

    yield set_mode
    set_mode(old)


def reference_cuda(kind, args, out_shape, dtype):
    with tempfile.TemporaryDirectory() as d:
        src, dst = os.path.join(d, "in.pt"), os.path.join(d, "out.pt")
        torch.save(dict(kind=kind, args=tuple(a.cpu() if torch.is_tensor(a) else a for a in args),
                        out_shape=tuple(out_shape), dtype=dtype), src)
        subprocess.run([sys.executable, os.path.join(ROOT, "oracle", "run_ref.py"), src, dst], check=True,
                       timeout=900)
        return torch.load(dst)["out"]


def run_paged(c):
    g = c.to(DEV)
    out = torch.full_like(g.new_out(), float("nan"))
    lse = torch.full(out.shape[:-1], float("nan"), device=DEV)
    capi.paged_sdpa(*g.op_args(out), lse=lse)
    torch.cuda.synchronize()
    return out.cpu(), lse.cpu()


def run_varlen(c):
    g = c.to(DEV)
    out = torch.full_like(g.new_out(), float("nan"))
    lse = torch.full(out.shape[:-1], float("nan"), device=DEV)
    capi.varlen_paged_sdpa(*g.capi_args(out), lse=lse)
    torch.cuda.synchronize()
    return out.cpu(), lse.cpu()


def oracle_paged(c):
    return O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths, c.k_cache,
                            c.v_cache, c.block_tables)


def test_config3_whole_vs_oracle_and_reference_cuda():
    """Config 3 whole: 4 sequences x 131072 keys, 128/8 heads, fp16, full rotary, page 64."""
    c = wl.config3()
    out, lse = run_paged(c)
    ref, rlse = oracle_paged(c)
    assert_out_close(out, ref.to(c.dtype), c.dtype, "config3 whole vs oracle")
    assert_lse_close(lse, rlse, "config3 whole lse")
    if os.path.exists(REF_SO):
        rc = reference_cuda("paged", c.op_args(None)[1:], out.shape, c.dtype)
        assert_out_close(out, rc.float(), c.dtype, "config3 whole vs reference CUDA op")


def test_config5_whole_vs_oracle():
    """Config 5 whole: 256 sequences, E = 256, 1-4 turns (the reference's kernels reject E = 256)."""
    c = wl.config5()
    out, lse = run_paged(c)
    ref, rlse = oracle_paged(c)
    assert_out_close(out, ref.to(c.dtype), c.dtype, "config5 whole vs oracle")
    assert_lse_close(lse, rlse, "config5 whole lse")


@needs_ref
def test_config2_whole_vs_reference_cuda():
    c = wl.config2()
    out, _ = run_paged(c)
    rc = reference_cuda("paged", c.op_args(None)[1:], out.shape, c.dtype)
    assert_out_close(out, rc.float(), c.dtype, "config2 whole vs reference CUDA op")


@pytest.mark.parametrize("mode", [None, "1"])
def test_config4_whole_vs_oracle_and_reference_cuda(prefill_env, mode):
    """Config 4 whole: 16 sequences of chunked prefill; mode None = the default routing (the
    tensor-core prefill for a call this large), "1" = the prefill forced on."""
    prefill_env(mode)
    c = wl.config4()
    out, lse = run_varlen(c)
    ref, rlse = O.varlen_paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths,
                                        c.k_cache, c.v_cache, c.block_tables, c.cu_seqlens_q)
    assert_out_close(out, ref.to(c.dtype), c.dtype, "config4 whole vs oracle")
    assert_lse_close(lse, rlse, "config4 whole lse")
    if mode is None and os.path.exists(REF_SO):
        rc = reference_cuda("varlen", c.op_args(None)[1:], out.shape, c.dtype)
        assert_out_close(out, rc.float(), c.dtype, "config4 whole vs reference CUDA op")


def _prefill_eligible(t):
    """The shapes the tensor-core prefill takes (16-bit, E = Ev = 128, GQA <= 16, rotary dim
    a multiple of 16, page size a power of two in [8, 128])."""
    q, kc = t["queries"], t["k_cache"]
    Hq, Hkv, E = q.size(1), kc.size(2), q.size(2)
    R = 2 * t["cosines"].size(2)
    return (q.dtype in (torch.float16, torch.bfloat16) and E == 128 and t["v_cache"].size(3) == 128
            and Hq % Hkv == 0 and Hq // Hkv <= 16 and R % 16 == 0 and kc.size(1) in (8, 16, 32, 64, 128))


@pytest.mark.parametrize("name", [n for n in fixtures.names("varlen_")])
def test_varlen_golden_on_tensor_core_prefill(prefill_env, name):
    """The reference-generated varlen vectors through prefill_kernel (DVATTN_PREFILL=1)."""
    t, m = fixtures.load(name)
    if not _prefill_eligible(t):
        pytest.skip("shape outside the tensor-core prefill (goes to the split-KV path)")
    prefill_env("1")
    g = {k: v.to(DEV) for k, v in t.items()}
    out = torch.full_like(g["out"], float("nan"))
    capi.varlen_paged_sdpa(out, m["scale"], g["locations"], g["queries"], g["cosines"], g["sines"],
                           g["fragment_lengths"], g["k_cache"], g["v_cache"], g["block_tables"], g["cu_seqlens_q"])
    torch.cuda.synchronize()
    assert_out_close(out, t["out"], t["out"].dtype, name + " (tcgen05 prefill)")
