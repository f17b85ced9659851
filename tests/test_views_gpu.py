"""GPU parity of dvattn_build_views (turn/view metadata built on the GPU) against the
oracle's restatement of DVAttnCache.update and the default rotary embedding."""
import numpy as np
import pytest
import torch

import dvattn_b200
from oracle import dvattn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_views_vs_oracle(dtype):
    rs = np.random.RandomState(3)
    F, W, n, R = 4, 6, 5, 64
    lens = rs.randint(5, 30000, size=F).astype(np.int32)
    order = np.stack([rs.permutation(F) for _ in range(W)]).astype(np.int32)
    loc, cos, sin = dvattn_b200.dvattn_build_views(torch.from_numpy(lens).to(DEV), torch.from_numpy(order).to(DEV),
                                                   n, R, 1000000.0, 1.0, dtype)
    torch.cuda.synchronize()
    eloc, ecos, esin = O.build_views(lens, order, n, R, 1000000.0, 1.0, dtype)
    assert torch.equal(loc.cpu(), eloc)
    # f32 transcendental results of the device and the host differ in the last bits; in
    # the model dtype they are equal except at rounding boundaries
    tol = {torch.float32: 2e-5, torch.bfloat16: 8e-3, torch.float16: 1e-3}[dtype]
    torch.testing.assert_close(cos.cpu(), ecos, rtol=0, atol=tol)
    torch.testing.assert_close(sin.cpu(), esin, rtol=0, atol=tol)
    assert torch.equal(cos[..., :R // 2], cos[..., R // 2:])


def test_views_feed_the_attention():
    """The built metadata drives dvattn_paged_sdpa the same as host-built metadata."""
    from dvattn_b200 import workloads as wl
    F, W, n = 2, 3, 1
    lens = np.array([40, 25], np.int32)
    order = np.array([[0, 1], [1, 0], [0, 1]], np.int32)
    loc, cos, sin = dvattn_b200.dvattn_build_views(torch.from_numpy(lens).to(DEV), torch.from_numpy(order).to(DEV),
                                                   n, 64, 10000.0)
    eloc, ecos, esin = O.build_views(lens, order, n, 64, 10000.0)
    c = wl.make_paged([[40, 25]] * W, Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.float32, seed=2)
    g = c.to(DEV)
    out = dvattn_b200.dvattn_paged_sdpa(g.queries, loc, cos, sin, g.fragment_lengths, g.k_cache, g.v_cache,
                                        g.block_tables, c.scale)
    torch.cuda.synchronize()
    ref, _ = O.paged_sdpa_f32(c.scale, eloc, c.queries, ecos, esin, c.fragment_lengths, c.k_cache, c.v_cache,
                              c.block_tables)
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-4, atol=1e-4)


import fixtures  # noqa: E402


@pytest.mark.parametrize("name", fixtures.names("views_"))
def test_views_golden(name):
    """Against HF's rotary module on the reference's locations (golden fixtures)."""
    t, m = fixtures.load(name)
    dt = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16}[str(m["dtype"])]
    loc, cos, sin = dvattn_b200.dvattn_build_views(t["seg_lengths"].to(DEV), t["seg_order"].to(DEV), int(m["n"]),
                                                   int(m["R"]), float(m["theta"]), 1.0, dt)
    torch.cuda.synchronize()
    assert torch.equal(loc.cpu(), t["locations"])
    tol = 2e-5 if dt == torch.float32 else 8e-3
    torch.testing.assert_close(cos.cpu(), t["cosines"], rtol=0, atol=tol)
    torch.testing.assert_close(sin.cpu(), t["sines"], rtol=0, atol=tol)


def test_views_capi_matches_op():
    """The C ABI entry point writes what the torch op writes (and with no inv_freq, the
    device computes 1/base^(2j/R) itself, equal to the host's within f32 rounding)."""
    from dvattn_b200 import capi
    rs = np.random.RandomState(8)
    F, W, n, R = 3, 4, 7, 128
    lens = torch.from_numpy(rs.randint(n, 5000, size=F).astype(np.int32)).to(DEV)
    order = torch.from_numpy(np.stack([rs.permutation(F) for _ in range(W)]).astype(np.int32)).to(DEV)
    loc, cos, sin = dvattn_b200.dvattn_build_views(lens, order, n, R, 500000.0, 1.0, torch.bfloat16)
    inv = (1.0 / (500000.0 ** (torch.arange(0, R, 2, dtype=torch.int64).float() / R))).to(DEV)
    for iv in (inv, None):
        l2, c2, s2 = torch.empty_like(loc), torch.empty_like(cos), torch.empty_like(sin)
        capi.build_views(l2, c2, s2, lens, order, 500000.0, 1.0, capi.DVATTN_BFLOAT16, inv_freq=iv)
        torch.cuda.synchronize()
        assert torch.equal(l2, loc)
        if iv is not None:
            assert torch.equal(c2, cos) and torch.equal(s2, sin)
        else:
            torch.testing.assert_close(c2, cos, rtol=0, atol=8e-3)
            torch.testing.assert_close(s2, sin, rtol=0, atol=8e-3)


@pytest.mark.parametrize("R", [0, 12, 24, 40])
def test_views_rotary_dims(R):
    """R/2 a multiple of 4 (R = 24, 40) takes the coalesced kernel, R = 12 the per-row one;
    R = 0 writes locations only."""
    rs = np.random.RandomState(R + 1)
    F, W, n = 3, 5, 9
    lens = rs.randint(n, 3000, size=F).astype(np.int32)
    order = np.stack([rs.permutation(F) for _ in range(W)]).astype(np.int32)
    loc, cos, sin = dvattn_b200.dvattn_build_views(torch.from_numpy(lens).to(DEV), torch.from_numpy(order).to(DEV),
                                                   n, R, 10000.0, 0.5, torch.float16)
    torch.cuda.synchronize()
    eloc, ecos, esin = O.build_views(lens, order, n, R, 10000.0, 0.5, torch.float16)
    assert torch.equal(loc.cpu(), eloc)
    if R:
        torch.testing.assert_close(cos.cpu(), ecos, rtol=0, atol=1e-3)
        torch.testing.assert_close(sin.cpu(), esin, rtol=0, atol=1e-3)
