"""Parity against the reference's OWN CUDA op (its src/binding.cu built for sm_100a into
oracle/_ref by oracle/Makefile), run in a separate process on the same inputs.  The
reference kernels support E = Ev = 128 and GQA 16 only (paged_kernel_v21.cuh:413)."""
import os
import subprocess
import sys
import tempfile

import pytest
import torch

import fixtures
from conftest import assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "dvatt_ref.so")
pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref not built")]


def run_reference(kind, args, out_shape, dtype):
    with tempfile.TemporaryDirectory() as d:
        src, dst = os.path.join(d, "in.pt"), os.path.join(d, "out.pt")
        torch.save(dict(kind=kind, args=tuple(a.cpu() if torch.is_tensor(a) else a for a in args),
                        out_shape=tuple(out_shape), dtype=dtype), src)
        subprocess.run([sys.executable, os.path.join(ROOT, "oracle", "run_ref.py"), src, dst], check=True, timeout=600)
        return torch.load(dst)["out"]


def paged_cases():
    yield "paged_bf16_2turn", None
    yield "paged_f16_s2_fullrot", None
    yield "paged_f32_config1", None
    yield "config2", lambda: wl.config2(W=8)
    yield "multiturn_f16", lambda: wl.make_paged([[300, 45, 7], [17, 900, 0], [64, 64, 64]], Hq=32, Hkv=2, E=128,
                                                  R=64, BS=16, dtype=torch.float16, seed=9)


@pytest.mark.parametrize("name,make", list(paged_cases()))
def test_paged_matches_reference_cuda(name, make):
    if make is None:
        t, m = fixtures.load(name)
        c = wl.PagedCase(queries=t["queries"], locations=t["locations"], cosines=t["cosines"], sines=t["sines"],
                         fragment_lengths=t["fragment_lengths"], k_cache=t["k_cache"], v_cache=t["v_cache"],
                         block_tables=t["block_tables"], scale=m["scale"], turn_lens=None)
    else:
        c = make()
    ref = run_reference("paged", c.op_args(None)[1:], c.new_out().shape, c.dtype)
    g = c.to("cuda:0")
    out = g.new_out()
    capi.paged_sdpa(*g.op_args(out))
    torch.cuda.synchronize()
    assert_out_close(out, ref.float(), c.dtype, name + " vs reference CUDA op")


def test_varlen_matches_reference_cuda():
    tl, ql = wl.config4_lengths(4, 16)
    c = wl.make_varlen(tl[:2], ql[:2], Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=4)
    ref = run_reference("varlen", c.op_args(None)[1:], c.new_out().shape, c.dtype)
    g = c.to("cuda:0")
    out = g.new_out()
    capi.varlen_paged_sdpa(*g.capi_args(out))
    torch.cuda.synchronize()
    assert_out_close(out, ref.float(), c.dtype, "varlen vs reference CUDA op")
