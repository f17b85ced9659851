"""GPU parity of the contiguous-fragment ops dvattn_sdpa and dvattn_fused
(src/binding.cu:79-149, 356-372) against the reference's own outputs (golden fixtures) and
the CPU oracle (dvattn_sdpa_pt restated)."""
import numpy as np
import pytest
import torch

import fixtures
from conftest import assert_lse_close, assert_out_close
import dvattn_b200
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
from oracle import dvattn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def frags(t, m):
    F = int(m["F"])
    return [t["key_%d" % f].to(DEV) for f in range(F)], [t["value_%d" % f].to(DEV) for f in range(F)]


@pytest.mark.parametrize("name", fixtures.names("sdpa_"))
def test_sdpa_golden(name):
    t, m = fixtures.load(name)
    keys, vals = frags(t, m)
    rq, loc, fl = t["rotated"].to(DEV), t["locations"].to(DEV), t["fragment_lengths"].to(DEV)
    out = torch.empty_like(t["out"], device=DEV)
    torch.ops.libdvatt.dvattn_sdpa(out, m["scale"], loc, rq, fl, keys, vals)
    torch.cuda.synchronize()
    assert_out_close(out, t["out"], t["out"].dtype, name)
    # the Python wrapper with the reference's signature
    out2 = dvattn_b200.dvattn_sdpa(rq, loc, keys, vals, m["scale"], fragment_lengths=fl)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


@pytest.mark.parametrize("name", fixtures.names("sdpa_"))
def test_fused_golden(name):
    t, m = fixtures.load(name)
    if t["cosines"].shape[-1] == 0:
        pytest.skip("no rotation in this fixture")
    keys, vals = frags(t, m)
    q, cos, sin = t["queries"].to(DEV), t["cosines"].to(DEV), t["sines"].to(DEV)
    loc, fl = t["locations"].to(DEV), t["fragment_lengths"].to(DEV)
    rq = torch.empty_like(t["rotated"], device=DEV)
    out = torch.empty_like(t["out"], device=DEV)
    dvattn_b200.dvattn_fused(q, loc, keys, vals, m["scale"], fl, cos, sin, rotated_queries=rq, out=out)
    torch.cuda.synchronize()
    assert_out_close(rq, t["rotated"], t["rotated"].dtype, name + " rotated")
    assert_out_close(out, t["out"], t["out"].dtype, name)


CASES = {
    "bf16_e128": dict(lens=[300, 1200], W=4, Hq=32, Hkv=2, E=128, R=64, dtype=torch.bfloat16, seed=41),
    "f16_shared_s3": dict(lens=[700, 31, 95], W=3, Hq=16, Hkv=1, E=128, R=128, dtype=torch.float16, seed=42, S=3,
                          batch=1),
    "f32_e256": dict(lens=[130, 77], W=2, Hq=16, Hkv=2, E=256, R=64, dtype=torch.float32, seed=43),
    "bf16_e64_gqa8_3d": dict(lens=[500], W=1, Hq=16, Hkv=2, E=64, R=32, dtype=torch.bfloat16, seed=44, batch=None),
    "f16_long": dict(lens=[6000, 2500], W=2, Hq=16, Hkv=1, E=128, R=0, dtype=torch.float16, seed=45),
    "bf16_empty_and_skipped": dict(lens=[0, 90, 40], W=2, Hq=32, Hkv=2, E=128, R=64, dtype=torch.bfloat16, seed=46,
                                   skip_turns=(2,)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_sdpa_random(name):
    c = wl.make_sdpa(**CASES[name])
    g = c.to(DEV)
    W, Hq, S, E = c.queries.shape
    out = torch.full((W, Hq, S, E), float("nan"), dtype=c.dtype, device=DEV)
    lse = torch.full((W, Hq, S), float("nan"), device=DEV)
    o32 = torch.full((W, Hq, S, E), float("nan"), device=DEV)
    capi.sdpa(out, g.scale, g.locations, g.rotated, g.fragment_lengths, g.keys, g.values, lse=lse, out_f32=o32)
    torch.cuda.synchronize()
    ref, rlse = O.sdpa_pt(c.rotated, c.locations, c.keys, c.values, c.scale, return_lse=True)
    assert_out_close(out, ref.to(c.dtype), c.dtype, name)
    assert_out_close(o32, ref, c.dtype, name + " f32")
    assert_lse_close(lse, rlse, name)
    # the torch op gives the same bits as the C ABI
    out2 = torch.empty_like(out)
    torch.ops.libdvatt.dvattn_sdpa(out2, g.scale, g.locations, g.rotated, g.fragment_lengths, g.keys, g.values)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_sdpa_fully_masked_rows_are_zero():
    c = wl.make_sdpa([40, 25], W=2, Hq=16, Hkv=1, E=128, R=0, dtype=torch.bfloat16, seed=47)
    loc = c.locations.clone()
    loc[:, 1] = -1  # worker 1 sees nothing
    g = c.to(DEV)
    out = torch.full(tuple(c.queries.shape), float("nan"), dtype=c.dtype, device=DEV)
    lse = torch.full(tuple(c.queries.shape[:3]), float("nan"), device=DEV)
    capi.sdpa(out, g.scale, loc.to(DEV), g.rotated, g.fragment_lengths, g.keys, g.values, lse=lse)
    torch.cuda.synchronize()
    assert torch.equal(out[1].float().cpu(), torch.zeros_like(out[1].float().cpu()))
    assert torch.isinf(lse[1]).all() and (lse[1] < 0).all()
    ref = O.sdpa_pt(c.rotated[:, :1], c.locations[:, :1], [k[:1] for k in c.keys], [v[:1] for v in c.values],
                    c.scale)
    assert_out_close(out[:1], ref, c.dtype, "unmasked worker")


def test_sdpa_errors():
    c = wl.make_sdpa([10], W=1, Hq=16, Hkv=1, E=128, R=0, dtype=torch.bfloat16, seed=48).to(DEV)
    out = torch.empty(tuple(c.queries.shape), dtype=c.dtype, device=DEV)
    with pytest.raises(RuntimeError):  # one fragment per turn
        torch.ops.libdvatt.dvattn_sdpa(out, c.scale, c.locations, c.rotated, c.fragment_lengths, c.keys * 2,
                                       c.values)
    with pytest.raises(RuntimeError):  # unsupported dtype must raise, not pass silently
        torch.ops.libdvatt.dvattn_sdpa(out.to(torch.float64), c.scale, c.locations, c.rotated.double(),
                                       c.fragment_lengths, [k.double() for k in c.keys],
                                       [v.double() for v in c.values])


ROW_CASES = {
    "bf16_hkv1_e128": dict(lens=[333, 1290], W=3, Hq=16, Hkv=1, E=128, R=0, dtype=torch.bfloat16, seed=51),
    "f16_hkv2_e64_s2": dict(lens=[77, 501, 64], W=2, Hq=16, Hkv=2, E=64, R=0, dtype=torch.float16, seed=52, S=2),
    "bf16_hkv4_e128_shared": dict(lens=[129, 1000], W=5, Hq=64, Hkv=4, E=128, R=0, dtype=torch.bfloat16, seed=53,
                                  batch=1),
    "bf16_hkv8_e128": dict(lens=[45, 700], W=2, Hq=64, Hkv=8, E=128, R=0, dtype=torch.bfloat16, seed=54),
    "f16_hkv2_e256": dict(lens=[300, 17], W=2, Hq=32, Hkv=2, E=256, R=0, dtype=torch.float16, seed=55),
    "bf16_3d_frag": dict(lens=[250, 90], W=1, Hq=16, Hkv=2, E=128, R=0, dtype=torch.bfloat16, seed=56, batch=None),
    # more fragments than travel as a kernel parameter: tensor maps staged in the workspace
    "bf16_hkv2_6turns": dict(lens=[40, 300, 7, 129, 64, 513], W=3, Hq=32, Hkv=2, E=128, R=0, dtype=torch.bfloat16,
                             seed=58),
}


@pytest.mark.parametrize("name", sorted(ROW_CASES))
def test_sdpa_tma_row_path(name, monkeypatch):
    """16-bit fragments run on the TMA row kernel (one 5-D box per window); the cp.async
    kernel (DVATTN_SDPA_ROW=0) and the oracle give the same result."""
    c = wl.make_sdpa(**ROW_CASES[name])
    g = c.to(DEV)
    W, Hq, S, E = c.queries.shape
    res = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("DVATTN_SDPA_ROW", mode)
        out = torch.full((W, Hq, S, E), float("nan"), dtype=c.dtype, device=DEV)
        lse = torch.full((W, Hq, S), float("nan"), device=DEV)
        o32 = torch.full((W, Hq, S, E), float("nan"), device=DEV)
        capi.sdpa(out, g.scale, g.locations, g.rotated, g.fragment_lengths, g.keys, g.values, lse=lse, out_f32=o32)
        torch.cuda.synchronize()
        res[mode] = (out, lse, o32)
    ref, rlse = O.sdpa_pt(c.rotated, c.locations, c.keys, c.values, c.scale, return_lse=True)
    out, lse, o32 = res["1"]
    assert_out_close(out, ref.to(c.dtype), c.dtype, name)
    assert_out_close(o32, ref, c.dtype, name + " f32")
    assert_lse_close(lse, rlse, name)
    # the two kernels split the keys differently, so P is rounded to 16 bits at different
    # running maxima: agreement to the 16-bit rounding of P, not to the bit
    torch.testing.assert_close(o32, res["0"][2], rtol=0, atol=4e-3)
    torch.testing.assert_close(lse, res["0"][1], rtol=1e-5, atol=1e-5)


def test_sdpa_rows_past_fragment_length(monkeypatch):
    """Fragments with more rows than fragment_lengths (a preallocated buffer): only the
    first L_f rows exist for the op."""
    c = wl.make_sdpa([200, 150], W=2, Hq=32, Hkv=2, E=128, R=0, dtype=torch.bfloat16, seed=57)
    g = c.to(DEV)
    pad_k = [torch.cat((k, torch.randn_like(k[:, :, :37])), 2).contiguous() for k in g.keys]
    pad_v = [torch.cat((v, torch.randn_like(v[:, :, :37])), 2).contiguous() for v in g.values]
    out = torch.empty(tuple(c.queries.shape), dtype=c.dtype, device=DEV)
    capi.sdpa(out, g.scale, g.locations, g.rotated, g.fragment_lengths, pad_k, pad_v)
    torch.cuda.synchronize()
    ref = O.sdpa_pt(c.rotated, c.locations, c.keys, c.values, c.scale)
    assert_out_close(out, ref.to(c.dtype), c.dtype, "padded fragments")
