"""GPU parity of the attention entry points that build the query rotation tables on the
device from the locations (dvattn_paged_sdpa_rope / dvattn_varlen_paged_sdpa_rope): the
rotation of turn f is the model's rotary embedding at the query's location there, as
DVAttnCache.update (python/dvattn/attention.py:161-191) builds the cos/sin it passes.
Checked against the oracle fed with host-built rotary tables of the same locations."""
import os

import numpy as np
import pytest
import torch

import dvattn_b200
from conftest import assert_lse_close, assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
from oracle import dvattn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BASE = 500000.0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_paged_rope_tables(dtype):
    c = wl.make_paged([[300, 40], [120, 9], [64, 77]], Hq=32, Hkv=2, E=128, R=64, BS=16, dtype=dtype, seed=21)
    cos, sin = O.rotary_tables(c.locations, 64, BASE, 1.0, dtype)  # [F, W, S, R]
    ref, rlse = O.paged_sdpa_f32(c.scale, c.locations, c.queries, cos, sin, c.fragment_lengths, c.k_cache, c.v_cache,
                                 c.block_tables)
    g = c.to(DEV)
    out = dvattn_b200.dvattn_paged_sdpa_rope(g.queries, g.locations, g.fragment_lengths, g.k_cache, g.v_cache,
                                             g.block_tables, c.scale, 64, BASE)
    torch.cuda.synchronize()
    assert_out_close(out, ref.to(dtype), dtype, "paged rope op")
    # the C ABI, with the device computing the inverse frequencies itself
    out2 = torch.empty_like(out)
    lse = torch.full(tuple(out.shape[:3]), float("nan"), device=DEV)
    capi.paged_sdpa_rope(out2, c.scale, g.locations, g.queries, g.fragment_lengths, g.k_cache, g.v_cache,
                         g.block_tables, 64, BASE, lse=lse)
    torch.cuda.synchronize()
    assert_out_close(out2, ref.to(dtype), dtype, "paged rope C ABI")
    assert_lse_close(lse, rlse, "paged rope C ABI")


def test_paged_rope_equals_views_tables():
    """Tables from dvattn_build_views (same device function) give the same bits."""
    F, W = 2, 3
    lens = np.array([200, 90], np.int32)
    order = np.array([[0, 1], [1, 0], [0, 1]], np.int32)
    loc, cos, sin = dvattn_b200.dvattn_build_views(torch.from_numpy(lens).to(DEV), torch.from_numpy(order).to(DEV),
                                                   1, 64, BASE, 1.0, torch.bfloat16)
    c = wl.make_paged([[200, 90]] * W, Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=22)
    g = c.to(DEV)
    a = dvattn_b200.dvattn_paged_sdpa(g.queries, loc, cos, sin, g.fragment_lengths, g.k_cache, g.v_cache,
                                      g.block_tables, c.scale)
    b = dvattn_b200.dvattn_paged_sdpa_rope(g.queries, loc, g.fragment_lengths, g.k_cache, g.v_cache, g.block_tables,
                                           c.scale, 64, BASE)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("mode", ["1", "0"])
def test_varlen_rope_tables(mode, monkeypatch):
    monkeypatch.setenv("DVATTN_PREFILL", mode)
    c = wl.make_varlen([[100, 400], [0, 150], [60, 33]], [96, 150, 20], Hq=32, Hkv=2, E=128, R=32, BS=16,
                       dtype=torch.bfloat16, seed=23)
    cos, sin = O.rotary_tables(c.locations, 32, BASE, 1.0, torch.bfloat16)  # [F, T, R]
    cos, sin = cos[..., :16].contiguous(), sin[..., :16].contiguous()
    ref, rlse = O.varlen_paged_sdpa_f32(c.scale, c.locations, c.queries, cos, sin, c.fragment_lengths, c.k_cache,
                                        c.v_cache, c.block_tables, c.cu_seqlens_q)
    g = c.to(DEV)
    out = dvattn_b200.dvattn_varlen_paged_sdpa_rope(g.queries, g.locations, g.fragment_lengths, g.k_cache, g.v_cache,
                                                    g.block_tables, g.cu_seqlens_q, c.scale, 32, BASE)
    torch.cuda.synchronize()
    assert_out_close(out, ref.to(torch.bfloat16), torch.bfloat16, "varlen rope op")
    out2 = torch.empty_like(out)
    lse = torch.full(tuple(out.shape[:2]), float("nan"), device=DEV)
    capi.varlen_paged_sdpa_rope(out2, c.scale, g.locations, g.queries, g.fragment_lengths, g.k_cache, g.v_cache,
                                g.block_tables, g.cu_seqlens_q, 32, BASE, lse=lse)
    torch.cuda.synchronize()
    assert_out_close(out2, ref.to(torch.bfloat16), torch.bfloat16, "varlen rope C ABI")
    assert_lse_close(lse, rlse, "varlen rope C ABI")


def test_rope_tables_reject_bad_rotary_dim():
    c = wl.make_paged([[40]], Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=24).to(DEV)
    with pytest.raises(RuntimeError):
        dvattn_b200.dvattn_paged_sdpa_rope(c.queries, c.locations, c.fragment_lengths, c.k_cache, c.v_cache,
                                           c.block_tables, c.scale, 63, BASE)
