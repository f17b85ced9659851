"""Generate the golden fixtures from the reference's OWN Python implementation.

Run in a container where the reference sources are mounted (default location below,
override with DVATTN_REFERENCE=<path>):  python tests/golden/make_golden.py

For each case it builds seeded inputs with dvattn_b200.workloads, then computes the
expected output with the reference's ``apply_rotary_pos_emb`` and ``dvattn_sdpa_pt``
(python/dvattn/attention.py:36-88), imported from the reference tree unmodified.  The
paged cache is turned into the per-turn fragments dvattn_sdpa_pt takes by reading
token l of turn f at logical position sum_{f'<f} L_f' + l through the block table
(src/kernels/paged_kernel_v21.cuh:101-115); unvisible tail positions are zero-filled
(they are masked).  The natural-log LSE is logsumexp(scale * qk) of the masked qk that
``return_intermediate_results=True`` returns.  The CUDA rope reads only the first R/2
entries of each cos/sin row; the generated rows have identical halves (HF convention),
so both readings agree.
"""
from __future__ import annotations

import importlib.metadata
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from dvattn_b200 import workloads as wl  # noqa: E402  (generators only; no native code)
import fixtures  # noqa: E402

# the reference checkout: DVATTN_REFERENCE, else a directory named "reference" beside the repo
REF = os.environ.get("DVATTN_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))


def load_reference():
    real = importlib.metadata.distribution

    def fake(name):
        if name == "dvattn":
            raise OSError("reference extension not installed; eager path only")
        return real(name)

    importlib.metadata.distribution = fake
    try:
        spec = importlib.util.spec_from_file_location("ref_attention", os.path.join(REF, "python/dvattn/attention.py"))
        mod = importlib.util.module_from_spec(spec)
        import warnings
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            spec.loader.exec_module(mod)
    finally:
        importlib.metadata.distribution = real
    return mod


def fragments(k_cache, v_cache, bt, L, nvis):
    """per-turn [W, Hkv, L_f, E] fragments; rows past nvis[f, w] are zero."""
    W = bt.shape[0]
    NB, BS, Hkv, E = k_cache.shape
    Ev = v_cache.shape[3]
    keys, vals = [], []
    off = 0
    for f in range(len(L)):
        Kf = torch.zeros(W, Hkv, int(L[f]), E, dtype=k_cache.dtype)
        Vf = torch.zeros(W, Hkv, int(L[f]), Ev, dtype=v_cache.dtype)
        for w in range(W):
            for l in range(int(nvis[f][w])):
                pos = off + l
                page = int(bt[w, pos // BS])
                Kf[w, :, l] = k_cache[page, pos % BS]
                Vf[w, :, l] = v_cache[page, pos % BS]
        keys.append(Kf)
        vals.append(Vf)
        off += int(L[f])
    return keys, vals


def golden_paged(ref, name, case: wl.PagedCase):
    q, loc, cos, sin = case.queries, case.locations, case.cosines, case.sines
    L = case.fragment_lengths.numpy()
    F = loc.shape[0]
    nvis = np.maximum(0, np.minimum(L[:, None], loc.numpy().max(axis=2) + 1))
    keys, vals = fragments(case.k_cache, case.v_cache, case.block_tables.numpy(), L, nvis)
    rq = torch.stack([ref.apply_rotary_pos_emb(q, cos[f], sin[f], unsqueeze_dim=1) for f in range(F)])
    res, qk, _ = ref.dvattn_sdpa_pt(rq, loc, keys, vals, case.scale, return_intermediate_results=True)
    lse = torch.logsumexp(case.scale * qk, dim=-1)
    assert torch.isfinite(res).all(), name
    fixtures.save(name, dict(queries=q, locations=loc, cosines=cos, sines=sin,
                             fragment_lengths=case.fragment_lengths, k_cache=case.k_cache, v_cache=case.v_cache,
                             block_tables=case.block_tables, out=res.to(q.dtype), out_f32=res, lse=lse,
                             rotated=rq),
                  dict(kind="paged", scale=case.scale))
    print("wrote", name, tuple(res.shape))


def golden_varlen(ref, name, case: wl.VarlenCase):
    q, loc, cos, sin = case.queries, case.locations, case.cosines, case.sines
    cu = case.cu_seqlens_q.numpy()
    L = case.fragment_lengths.numpy()
    F = loc.shape[0]
    T, Hq, E = q.shape
    Ev = case.v_cache.shape[3]
    out = torch.zeros(T, Hq, Ev)
    lse = torch.zeros(T, Hq)
    rq_all = torch.zeros(F, T, Hq, E, dtype=q.dtype)
    for w in range(len(cu) - 1):
        a, b = int(cu[w]), int(cu[w + 1])
        if a == b:
            continue
        qw = q[a:b].transpose(0, 1)[None]  # [1, Hq, Sw, E]
        locw = loc[:, a:b][:, None, :]  # [F, 1, Sw]
        full_c = torch.cat([cos[:, a:b], cos[:, a:b]], -1)  # [F, Sw, R]
        full_s = torch.cat([sin[:, a:b], sin[:, a:b]], -1)
        rq = torch.stack([ref.apply_rotary_pos_emb(qw, full_c[f][None], full_s[f][None], unsqueeze_dim=1)
                          for f in range(F)])  # [F, 1, Hq, Sw, E]
        rq_all[:, a:b] = rq[:, 0].transpose(1, 2)
        nvis = np.maximum(0, np.minimum(L[:, None], locw.numpy().max(axis=2) + 1))
        keys, vals = fragments(case.k_cache, case.v_cache, case.block_tables.numpy()[w:w + 1], L, nvis)
        res, qk, _ = ref.dvattn_sdpa_pt(rq, locw, keys, vals, case.scale, return_intermediate_results=True)
        out[a:b] = res[0].transpose(0, 1)
        lse[a:b] = torch.logsumexp(case.scale * qk, dim=-1)[0].transpose(0, 1)
    assert torch.isfinite(out).all(), name
    fixtures.save(name, dict(queries=q, locations=loc, cosines=cos, sines=sin,
                             fragment_lengths=case.fragment_lengths, k_cache=case.k_cache, v_cache=case.v_cache,
                             block_tables=case.block_tables, cu_seqlens_q=case.cu_seqlens_q, out=out.to(q.dtype),
                             out_f32=out, lse=lse, rotated=rq_all),
                  dict(kind="varlen", scale=case.scale))
    print("wrote", name, tuple(out.shape))


def golden_sdpa(ref, name, case: wl.SdpaCase):
    """Contiguous fragments: dvattn_sdpa_pt on the case's fragments directly, and the
    rotated queries of dvattn_fused with apply_rotary_pos_emb."""
    q, loc, cos, sin = case.queries, case.locations, case.cosines, case.sines
    F = loc.shape[0]
    if cos.shape[-1]:
        rq = torch.stack([ref.apply_rotary_pos_emb(q, cos[f], sin[f], unsqueeze_dim=1) for f in range(F)])
    else:
        rq = torch.stack([q.clone() for _ in range(F)])
    res, qk, _ = ref.dvattn_sdpa_pt(rq, loc, case.keys, case.values, case.scale, return_intermediate_results=True)
    lse = torch.logsumexp(case.scale * qk, dim=-1)
    assert torch.isfinite(res).all(), name
    t = dict(queries=q, rotated=rq, cosines=cos, sines=sin, locations=loc, fragment_lengths=case.fragment_lengths,
             out=res.to(q.dtype), out_f32=res, lse=lse)
    for f in range(F):
        t["key_%d" % f] = case.keys[f]
        t["value_%d" % f] = case.values[f]
    fixtures.save(name, t, dict(kind="sdpa", scale=case.scale, F=F))
    print("wrote", name, tuple(res.shape))


def main():
    ref = load_reference()
    bf, hf, f32 = torch.bfloat16, torch.float16, torch.float32
    only = sys.argv[1:]  # optional: kinds to (re)generate, e.g. "sdpa"
    if only and "paged" not in only and "varlen" not in only:
        return sdpa_only(ref)
    golden_paged(ref, "paged_f32_config1", wl.config1())
    golden_paged(ref, "paged_bf16_2turn", wl.make_paged([[37, 90], [150, 3], [64, 64]], Hq=32, Hkv=2, E=128, R=64,
                                                        BS=16, dtype=bf, seed=11))
    golden_paged(ref, "paged_f16_s2_fullrot", wl.make_paged([[77], [129]], Hq=16, Hkv=1, E=128, R=128, BS=16,
                                                            dtype=hf, seed=12, S=2))
    golden_paged(ref, "paged_f16_e256_4turn", wl.make_paged([[20, 33, 0, 0], [5, 1, 60, 14], [90, 0, 0, 0]], Hq=32,
                                                            Hkv=2, E=256, R=64, BS=64, dtype=hf, seed=13))
    golden_paged(ref, "paged_bf16_gqa8_norot", wl.make_paged([[45, 21], [13, 70]], Hq=16, Hkv=2, E=128, R=0, BS=8,
                                                             dtype=bf, seed=14))
    golden_paged(ref, "paged_f32_e64_3turn", wl.make_paged([[10, 0, 25], [33, 7, 1]], Hq=32, Hkv=2, E=64, R=32, BS=4,
                                                           dtype=f32, seed=15))
    golden_varlen(ref, "varlen_bf16", wl.make_varlen([[35], [1], [82]], [5, 1, 12], Hq=32, Hkv=2, E=128, R=32, BS=16,
                                                     dtype=bf, seed=21))
    golden_varlen(ref, "varlen_f16_2turn", wl.make_varlen([[40, 17], [0, 9], [12, 30]], [3, 9, 7], Hq=16, Hkv=1, E=128,
                                                          R=64, BS=16, dtype=hf, seed=22))
    golden_varlen(ref, "varlen_f32", wl.make_varlen([[6], [50]], [6, 2], Hq=16, Hkv=1, E=128, R=128, BS=16,
                                                    dtype=f32, seed=23))
    golden_sdpa(ref, "sdpa_bf16_w4", wl.make_sdpa([37, 90], W=4, Hq=32, Hkv=2, E=128, R=64, dtype=bf, seed=31))
    golden_sdpa(ref, "sdpa_f16_e256_shared_s2", wl.make_sdpa([20, 5, 61], W=3, Hq=16, Hkv=1, E=256, R=64, dtype=hf,
                                                              seed=32, S=2, batch=1))
    golden_sdpa(ref, "sdpa_f32_e64_3d", wl.make_sdpa([33, 12], W=1, Hq=16, Hkv=2, E=64, R=32, dtype=f32, seed=33,
                                                      batch=None))
    golden_sdpa(ref, "sdpa_bf16_gqa4_skip", wl.make_sdpa([50, 0, 70], W=2, Hq=16, Hkv=4, E=128, R=0, dtype=bf,
                                                          seed=34, skip_turns=(0,)))


def golden_append(ref, name, W, Hkv, n, E, R, dtype, seed):
    """K rotation of new tokens with the reference's apply_rotary_pos_emb (the keys the
    paged append writes)."""
    g = torch.Generator().manual_seed(seed)
    keys = torch.randn((W, Hkv, n, E), generator=g).to(dtype)
    pos = torch.randint(0, 8192, (W, n), generator=g)
    cos, sin = wl.rope_angles(pos, R)
    rk = ref.apply_rotary_pos_emb(keys, cos, sin) if R else keys.clone()
    fixtures.save(name, dict(keys=keys, cosines=cos, sines=sin, rotated=rk), dict(kind="append"))
    print("wrote", name, tuple(rk.shape))


def golden_views(name, lens, order, n, R, theta, dtype):
    """cos/sin of the turn/view locations from HF's LlamaRotaryEmbedding, the module the
    reference calls as model.rotary_emb (python/dvattn/attention.py:185), on the locations
    of DVAttnCache.update's walk (restated in oracle.build_views)."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    sys.path.insert(0, ROOT)
    from oracle import dvattn_oracle as O
    lens = np.asarray(lens, np.int32)
    order = np.asarray(order, np.int32)
    loc, _, _ = O.build_views(lens, order, n, R, theta, 1.0, dtype)
    cfg = LlamaConfig(hidden_size=R * 8, num_attention_heads=8, num_key_value_heads=2, rope_theta=theta,
                      max_position_embeddings=1 << 20)
    emb = LlamaRotaryEmbedding(cfg)
    F, W = loc.shape[:2]
    c, s_ = emb(torch.zeros(1, 1, R, dtype=dtype), loc.reshape(F * W, n).long())
    fixtures.save(name, dict(seg_lengths=torch.from_numpy(lens), seg_order=torch.from_numpy(order), locations=loc,
                             cosines=c.float().reshape(F, W, n, R), sines=s_.float().reshape(F, W, n, R)),
                  dict(kind="views", n=n, R=R, theta=theta, dtype=str(dtype).replace("torch.", "")))
    print("wrote", name)


def sdpa_only(ref):
    golden_views("views_bf16_theta1e6", [1200, 35, 77000], [[0, 1, 2], [2, 0, 1], [1, 2, 0], [0, 2, 1]], 5, 128,
                 1000000.0, torch.bfloat16)
    golden_views("views_f32_theta1e4", [64, 9], [[1, 0], [0, 1]], 3, 64, 10000.0, torch.float32)
    golden_append(ref, "append_bf16_r64", 3, 2, 17, 128, 64, torch.bfloat16, 51)
    golden_append(ref, "append_f16_r128", 2, 4, 9, 128, 128, torch.float16, 52)
    golden_append(ref, "append_f32_e64_r32", 2, 1, 5, 64, 32, torch.float32, 53)
    bf, hf, f32 = torch.bfloat16, torch.float16, torch.float32
    golden_sdpa(ref, "sdpa_bf16_w4", wl.make_sdpa([37, 90], W=4, Hq=32, Hkv=2, E=128, R=64, dtype=bf, seed=31))
    golden_sdpa(ref, "sdpa_f16_e256_shared_s2", wl.make_sdpa([20, 5, 61], W=3, Hq=16, Hkv=1, E=256, R=64, dtype=hf,
                                                              seed=32, S=2, batch=1))
    golden_sdpa(ref, "sdpa_f32_e64_3d", wl.make_sdpa([33, 12], W=1, Hq=16, Hkv=2, E=64, R=32, dtype=f32, seed=33,
                                                      batch=None))
    golden_sdpa(ref, "sdpa_bf16_gqa4_skip", wl.make_sdpa([50, 0, 70], W=2, Hq=16, Hkv=4, E=128, R=0, dtype=bf,
                                                          seed=34, skip_turns=(0,)))


if __name__ == "__main__":
    main()
