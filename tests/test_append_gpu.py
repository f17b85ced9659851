"""GPU parity of dvattn_paged_append (the paged KV append with fused K rotation) against
the reference's apply_rotary_pos_emb (golden fixtures) and the oracle's restatement of the
cache update (bit-exact: same f32 math and one rounding)."""
import numpy as np
import pytest
import torch

import fixtures
import dvattn_b200
from conftest import assert_lse_close, assert_out_close
from dvattn_b200 import capi
from dvattn_b200 import workloads as wl
from oracle import dvattn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("name", fixtures.names("append_"))
def test_append_golden_rotation(name):
    t, _ = fixtures.load(name)
    keys = t["keys"].to(DEV)
    W, Hkv, n, E = keys.shape
    BS = 16
    maxb = (n + BS - 1) // BS
    kc = torch.zeros((W * maxb, BS, Hkv, E), dtype=keys.dtype, device=DEV)
    vc = torch.zeros_like(kc)
    bt = torch.arange(W * maxb, dtype=torch.int32, device=DEV).reshape(W, maxb)
    pos = torch.zeros(W, dtype=torch.int32, device=DEV)
    dvattn_b200.dvattn_paged_append(kc, vc, keys, keys, t["cosines"].to(DEV), t["sines"].to(DEV), bt, pos)
    torch.cuda.synchronize()
    got = kc.reshape(W, maxb * BS, Hkv, E)[:, :n].permute(0, 2, 1, 3).cpu()
    assert torch.equal(got, t["rotated"]), name
    assert torch.equal(vc.reshape(W, maxb * BS, Hkv, E)[:, :n].permute(0, 2, 1, 3).cpu(), t["keys"])


# R = 24 (bf16) and R = 12 (f32) put a rotary half boundary inside a 16-byte chunk
@pytest.mark.parametrize("dtype,E,R", [(torch.bfloat16, 128, 64), (torch.float16, 256, 128), (torch.float32, 64, 0),
                                       (torch.bfloat16, 128, 24), (torch.float32, 64, 12), (torch.float32, 128, 32)])
@pytest.mark.parametrize("via", ["op", "capi"])
def test_append_random_vs_oracle(dtype, E, R, via):
    rs = np.random.RandomState(E + R)
    W, Hkv, n, BS, maxb = 5, 2, 37, 16, 12
    NB = W * maxb
    g = torch.Generator().manual_seed(7)
    kc = torch.randn((NB, BS, Hkv, E), generator=g).to(dtype)
    vc = torch.randn((NB, BS, Hkv, E), generator=g).to(dtype)
    keys = torch.randn((W, Hkv, n, E), generator=g).to(dtype)
    vals = torch.randn((W, Hkv, n, E), generator=g).to(dtype)
    cos, sin = wl.rope_angles(torch.from_numpy(rs.randint(0, 9000, (W, n))), R)
    bt = torch.from_numpy(rs.permutation(NB).reshape(W, maxb).astype(np.int32))
    bt[1, 3] = -1          # an invalid page: skipped
    bt[2, 5] = NB + 7      # a page outside the pool: skipped
    pos = torch.from_numpy(rs.randint(0, maxb * BS - n // 2, size=W).astype(np.int32))
    pos[4] = maxb * BS - 5  # runs past the block table: the tail is skipped
    counts = torch.from_numpy(np.array([n, 0, 11, n - 3, 20], np.int32))
    ek, ev = O.paged_append(kc, vc, keys, vals, cos, sin, bt, pos, counts)
    dk, dv = kc.to(DEV), vc.to(DEV)
    fn = dvattn_b200.dvattn_paged_append if via == "op" else capi.paged_append
    fn(dk, dv, keys.to(DEV), vals.to(DEV), cos.to(DEV), sin.to(DEV), bt.to(DEV), pos.to(DEV), counts.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(dk.cpu(), ek)
    assert torch.equal(dv.cpu(), ev)


def test_append_then_decode():
    """Prefill-style append of new tokens into turn 1 of each worker, then the paged decode
    over the updated cache, against the oracle on the oracle-updated cache."""
    c = wl.make_paged([[300, 40], [120, 9], [64, 77]], Hq=32, Hkv=2, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=5)
    W, Hkv, n, E = 3, 2, 8, 128
    g = torch.Generator().manual_seed(9)
    keys = torch.randn((W, Hkv, n, E), generator=g).to(torch.bfloat16)
    vals = torch.randn((W, Hkv, n, E), generator=g).to(torch.bfloat16)
    cos, sin = wl.rope_angles(torch.randint(0, 4000, (W, n), generator=g), 64)
    L = c.fragment_lengths.numpy()
    # new tokens overwrite the last n visible keys of turn 1 of each worker
    vis1 = np.minimum(L[1], c.locations[1, :, 0].numpy() + 1)
    pos = torch.from_numpy((L[0] + vis1 - n).astype(np.int32))
    ek, ev = O.paged_append(c.k_cache, c.v_cache, keys, vals, cos, sin, c.block_tables, pos)
    gc = c.to(DEV)
    dvattn_b200.dvattn_paged_append(gc.k_cache, gc.v_cache, keys.to(DEV), vals.to(DEV), cos.to(DEV), sin.to(DEV),
                                    gc.block_tables, pos.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(gc.k_cache.cpu(), ek) and torch.equal(gc.v_cache.cpu(), ev)
    out = dvattn_b200.dvattn_paged_sdpa(gc.queries, gc.locations, gc.cosines, gc.sines, gc.fragment_lengths,
                                        gc.k_cache, gc.v_cache, gc.block_tables, c.scale)
    torch.cuda.synchronize()
    ref, _ = O.paged_sdpa_f32(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths, ek, ev,
                              c.block_tables)
    assert_out_close(out, ref.to(out.dtype), out.dtype, "append then decode")
