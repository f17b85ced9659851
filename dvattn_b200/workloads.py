"""Seeded synthetic inputs for the paged-decode and varlen-prefill ops.

There is no public dataset behind the reference's path; every benchmark config is
synthetic: q, k, v ~ N(0, 1) in the config dtype, cos/sin = cat(cos(theta*p), cos(theta*p))
with theta_i = 10000^(-2i/R) (HF duplicated halves), p = the query's position relative
to the start of each cache turn.  Structure (lengths, turn splits, page permutation) is
drawn with numpy's RandomState(seed) so it is identical on every machine; tensor values
use torch.Generator(seed) on the target device.

Layout conventions follow the reference schemas (src/binding.cu:151-203, 249-296): turn f
of every sequence occupies logical cache positions [sum_{f'<f} L_f', +L_f), L_f = the
longest turn f over the batch; pages that hold no visible key are not allocated and
their block-table entries are `fill` (0 by default).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

ESIZE = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}


def rope_angles(pos: torch.Tensor, R: int, base: float = 10000.0):
    """cos/sin of shape pos.shape + (R,) (duplicated halves), float32."""
    if R == 0:
        z = torch.zeros(pos.shape + (0,), dtype=torch.float32, device=pos.device)
        return z, z.clone()
    i = torch.arange(R // 2, dtype=torch.float64, device=pos.device)
    theta = base ** (-2.0 * i / R)
    ang = pos.to(torch.float64)[..., None] * theta
    c, s = torch.cos(ang).to(torch.float32), torch.sin(ang).to(torch.float32)
    return torch.cat([c, c], -1).contiguous(), torch.cat([s, s], -1).contiguous()


def _randn(shape, dtype, gen, device):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)


@dataclass
class PagedCase:
    """Inputs of one dvattn_paged_sdpa call (schema order) plus structure metadata."""
    queries: torch.Tensor
    locations: torch.Tensor
    cosines: torch.Tensor
    sines: torch.Tensor
    fragment_lengths: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_tables: torch.Tensor
    scale: float
    turn_lens: np.ndarray  # [W, F] visible keys per turn (S = 1 view)
    meta: Dict = field(default_factory=dict)

    @property
    def dtype(self):
        return self.queries.dtype

    def op_args(self, out):
        return (out, self.scale, self.locations, self.queries, self.cosines, self.sines, self.fragment_lengths,
                self.k_cache, self.v_cache, self.block_tables)

    def new_out(self):
        W, Hq, S, _ = self.queries.shape
        return torch.empty((W, Hq, S, self.v_cache.size(3)), dtype=self.dtype, device=self.queries.device)

    def to(self, device) -> "PagedCase":
        d = {k: getattr(self, k).to(device) for k in ("queries", "locations", "cosines", "sines", "fragment_lengths",
                                                       "k_cache", "v_cache", "block_tables")}
        return PagedCase(scale=self.scale, turn_lens=self.turn_lens, meta=dict(self.meta), **d)


def visible_keys(locations: np.ndarray, L: np.ndarray, cap: int) -> np.ndarray:
    """[F, W, S] number of visible keys of each turn for each query row."""
    off = np.concatenate([[0], np.cumsum(L)[:-1]]) if len(L) else np.zeros(0, np.int64)
    v = np.minimum(L[:, None, None], locations.astype(np.int64) + 1)
    v = np.minimum(v, cap - off[:, None, None])
    return np.maximum(v, 0)


def paged_bytes(case: PagedCase) -> int:
    """Algorithmic bytes of one call: attended K+V rows + q + out + cos/sin + tables + loc."""
    W, Hq, S, E = case.queries.shape
    Hkv, Ev = case.k_cache.size(2), case.v_cache.size(3)
    es = ESIZE[case.dtype]
    cap = case.block_tables.size(1) * case.k_cache.size(1)
    n = int(visible_keys(case.locations.cpu().numpy(), case.fragment_lengths.cpu().numpy(), cap).sum())
    kv = n * Hkv * (E + Ev) * es
    R = case.cosines.size(3)
    other = (W * Hq * S * E + W * Hq * S * Ev) * es + 2 * case.cosines.numel() // max(R, 1) * (R // 2) * 4 \
        + case.block_tables.numel() * 4 + case.locations.numel() * 4
    return kv + other


def paged_flops(case: PagedCase) -> int:
    W, Hq, S, E = case.queries.shape
    cap = case.block_tables.size(1) * case.k_cache.size(1)
    n = int(visible_keys(case.locations.cpu().numpy(), case.fragment_lengths.cpu().numpy(), cap).sum())
    return 2 * Hq * (E + case.v_cache.size(3)) * n


def make_paged(turn_lens: Sequence[Sequence[int]], Hq: int, Hkv: int, E: int, R: int, BS: int, dtype,
               seed: int = 0, S: int = 1, device="cpu", permute: bool = True, fill: int = 0,
               Ev: Optional[int] = None, extra_pages: int = 0, loc_override: Optional[np.ndarray] = None,
               rot_offsets: Optional[np.ndarray] = None) -> PagedCase:
    """Paged decode inputs.  turn_lens[w][f] = keys of turn f cached for sequence w.  Query s
    of S sees keys l <= len - S + s of the last non-empty turn and all earlier keys."""
    Ev = E if Ev is None else Ev
    tl = np.asarray(turn_lens, dtype=np.int64)
    W, F = tl.shape
    rs = np.random.RandomState(seed)
    L = tl.max(axis=0) if W else np.zeros(F, np.int64)
    off = np.concatenate([[0], np.cumsum(L)[:-1]]) if F else np.zeros(0, np.int64)
    total_logical = int(L.sum())
    maxb = max(1, -(-total_logical // BS))
    # pages that hold visible keys
    need = []
    for w in range(W):
        pages = set()
        for f in range(F):
            if tl[w, f] > 0:
                pages.update(range((off[f]) // BS, (off[f] + tl[w, f] - 1) // BS + 1))
        need.append(sorted(pages))
    npages = sum(len(p) for p in need) + extra_pages
    phys = rs.permutation(npages) if permute else np.arange(npages)
    bt = np.full((W, maxb), fill, dtype=np.int64)
    k = 0
    for w in range(W):
        for p in need[w]:
            bt[w, p] = phys[k]
            k += 1
    # locations: turn f fully visible except the S new queries of the last non-empty turn
    loc = np.zeros((F, W, S), np.int64)
    for w in range(W):
        nz = [f for f in range(F) if tl[w, f] > 0]
        last = nz[-1] if nz else -1
        for f in range(F):
            for s in range(S):
                loc[f, w, s] = (tl[w, f] - 1 - (S - 1 - s)) if f == last else tl[w, f] - 1
    if loc_override is not None:
        loc = np.asarray(loc_override, np.int64).reshape(F, W, S)
    # rotation offsets: query position relative to each turn's start
    if rot_offsets is None:
        pos = np.zeros((F, W, S), np.int64)
        for w in range(W):
            for f in range(F):
                for s in range(S):
                    pos[f, w, s] = int(tl[w, f:].sum()) - (S - 1 - s)
    else:
        pos = np.asarray(rot_offsets, np.int64).reshape(F, W, S)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    NB = max(npages, 1)
    q = _randn((W, Hq, S, E), dtype, gen, device)
    kc = _randn((NB, BS, Hkv, E), dtype, gen, device)
    vc = _randn((NB, BS, Hkv, Ev), dtype, gen, device)
    cos, sin = rope_angles(torch.from_numpy(pos).to(device), R)
    return PagedCase(
        queries=q, locations=torch.from_numpy(loc.astype(np.int32)).to(device), cosines=cos, sines=sin,
        fragment_lengths=torch.from_numpy(L.astype(np.int32)).to(device), k_cache=kc, v_cache=vc,
        block_tables=torch.from_numpy(bt.astype(np.int32)).to(device), scale=1.0 / math.sqrt(E), turn_lens=tl,
        meta=dict(W=W, F=F, S=S, Hq=Hq, Hkv=Hkv, E=E, Ev=Ev, R=R, BS=BS, seed=seed, npages=npages))


@dataclass
class VarlenCase:
    queries: torch.Tensor
    locations: torch.Tensor
    cosines: torch.Tensor
    sines: torch.Tensor
    fragment_lengths: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_tables: torch.Tensor
    cu_seqlens_q: torch.Tensor
    cu_seqlens_k: torch.Tensor
    scale: float
    meta: Dict = field(default_factory=dict)

    @property
    def dtype(self):
        return self.queries.dtype

    def op_args(self, out):
        return (out, self.scale, self.locations, self.queries, self.cosines, self.sines, self.fragment_lengths,
                self.k_cache, self.v_cache, self.block_tables, self.cu_seqlens_q, self.cu_seqlens_k)

    def capi_args(self, out):
        return (out, self.scale, self.locations, self.queries, self.cosines, self.sines, self.fragment_lengths,
                self.k_cache, self.v_cache, self.block_tables, self.cu_seqlens_q)

    def new_out(self):
        T, Hq, _ = self.queries.shape
        return torch.empty((T, Hq, self.v_cache.size(3)), dtype=self.dtype, device=self.queries.device)

    def to(self, device) -> "VarlenCase":
        d = {k: getattr(self, k).to(device) for k in ("queries", "locations", "cosines", "sines", "fragment_lengths",
                                                       "k_cache", "v_cache", "block_tables", "cu_seqlens_q",
                                                       "cu_seqlens_k")}
        return VarlenCase(scale=self.scale, meta=dict(self.meta), **d)


def make_varlen(turn_lens: Sequence[Sequence[int]], q_lens: Sequence[int], Hq: int, Hkv: int, E: int, R: int,
                BS: int, dtype, seed: int = 0, device="cpu", permute: bool = True, fill: int = 0,
                Ev: Optional[int] = None) -> VarlenCase:
    """Varlen prefill inputs.  turn_lens[w][f] = cached keys of turn f of sequence w,
    including the q_lens[w] new tokens, which are the last keys of the last turn (their K/V
    are already written, as in chunked prefill).  New token i of sequence w sees keys
    l <= len_last - q_w + i of the last turn and all keys of earlier turns (loc = -1 for an
    empty turn)."""
    Ev = E if Ev is None else Ev
    tl = np.asarray(turn_lens, dtype=np.int64)
    W, F = tl.shape
    ql = np.asarray(q_lens, dtype=np.int64)
    assert np.all(ql <= tl[:, -1])
    rs = np.random.RandomState(seed)
    L = tl.max(axis=0)
    off = np.concatenate([[0], np.cumsum(L)[:-1]])
    maxb = max(1, -(-int(L.sum()) // BS))
    need = []
    for w in range(W):
        pages = set()
        for f in range(F):
            if tl[w, f] > 0:
                pages.update(range(off[f] // BS, (off[f] + tl[w, f] - 1) // BS + 1))
        need.append(sorted(pages))
    npages = sum(len(p) for p in need)
    phys = rs.permutation(npages) if permute else np.arange(npages)
    bt = np.full((W, maxb), fill, dtype=np.int64)
    k = 0
    for w in range(W):
        for p in need[w]:
            bt[w, p] = phys[k]
            k += 1
    T = int(ql.sum())
    cu = np.concatenate([[0], np.cumsum(ql)]).astype(np.int64)
    loc = np.zeros((F, T), np.int64)
    pos = np.zeros((F, T), np.int64)
    for w in range(W):
        for i in range(ql[w]):
            t = cu[w] + i
            last_loc = tl[w, F - 1] - ql[w] + i
            for f in range(F):
                loc[f, t] = last_loc if f == F - 1 else tl[w, f] - 1
                pos[f, t] = int(tl[w, f:F - 1].sum()) + last_loc
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    NB = max(npages, 1)
    q = _randn((T, Hq, E), dtype, gen, device)
    kc = _randn((NB, BS, Hkv, E), dtype, gen, device)
    vc = _randn((NB, BS, Hkv, Ev), dtype, gen, device)
    cos, sin = rope_angles(torch.from_numpy(pos).to(device), R)
    cos, sin = cos[..., :R // 2].contiguous(), sin[..., :R // 2].contiguous()
    cu_t = torch.from_numpy(cu.astype(np.int32)).to(device)
    return VarlenCase(
        queries=q, locations=torch.from_numpy(loc.astype(np.int32)).to(device), cosines=cos, sines=sin,
        fragment_lengths=torch.from_numpy(L.astype(np.int32)).to(device), k_cache=kc, v_cache=vc,
        block_tables=torch.from_numpy(bt.astype(np.int32)).to(device), cu_seqlens_q=cu_t, cu_seqlens_k=cu_t.clone(),
        scale=1.0 / math.sqrt(E),
        meta=dict(W=W, F=F, T=T, Hq=Hq, Hkv=Hkv, E=E, Ev=Ev, R=R, BS=BS, seed=seed, q_lens=ql, turn_lens=tl))


@dataclass
class SdpaCase:
    """Inputs of one dvattn_sdpa / dvattn_fused call over contiguous per-turn fragments.
    ``queries`` [W,Hq,S,E] (unrotated, for dvattn_fused), ``rotated`` [F,W,Hq,S,E] (the
    dvattn_sdpa input, rotated from queries with cos/sin), keys/values F tensors
    [B,Hkv,L_f,E] (B = W, or 1 for fragments shared by all workers; ``batch=None`` gives
    3-D [Hkv,L_f,E] tensors, which the reference reads as B = 1 when W = 1)."""
    queries: torch.Tensor
    rotated: torch.Tensor
    cosines: torch.Tensor
    sines: torch.Tensor
    locations: torch.Tensor
    fragment_lengths: torch.Tensor
    keys: list
    values: list
    scale: float
    meta: dict

    @property
    def dtype(self):
        return self.queries.dtype

    def to(self, device) -> "SdpaCase":
        mv = lambda t: t.to(device)
        return SdpaCase(mv(self.queries), mv(self.rotated), mv(self.cosines), mv(self.sines), mv(self.locations),
                        mv(self.fragment_lengths), [mv(k) for k in self.keys], [mv(v) for v in self.values],
                        self.scale, dict(self.meta))


def make_sdpa(lens: Sequence[int], W: int, Hq: int, Hkv: int, E: int, R: int, dtype, seed: int = 0, S: int = 1,
              batch="w", device="cpu", skip_turns: Sequence[int] = ()) -> SdpaCase:
    """Contiguous-fragment inputs.  Turn f has L_f = lens[f] keys; the query (w, s) of turn
    f sees keys l <= loc[f,w,s] with loc ~ U[0, L_f) (-1 for turns listed in skip_turns and
    for empty fragments), and every query sees at least one key in some turn."""
    F = len(lens)
    rs = np.random.RandomState(seed)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    q = _randn((W, Hq, S, E), dtype, gen, device)
    loc = np.full((F, W, S), -1, np.int64)
    for f in range(F):
        if lens[f] > 0 and f not in skip_turns:
            loc[f] = rs.randint(0, lens[f], size=(W, S))
    live = [f for f in range(F) if lens[f] > 0 and f not in skip_turns]
    assert live, "at least one visible turn"
    dead = (loc.max(axis=0) < 0)
    loc[live[0]][dead] = lens[live[0]] - 1
    pos = rs.randint(0, 4096, size=(F, W, S))
    cos, sin = rope_angles(torch.from_numpy(pos).to(device), R)
    B = W if batch == "w" else 1
    keys, vals = [], []
    for f in range(F):
        shape = (B, Hkv, lens[f], E) if batch is not None else (Hkv, lens[f], E)
        keys.append(_randn(shape, dtype, gen, device))
        vals.append(_randn(shape, dtype, gen, device))
    # rotated queries as the reference's apply_rotary_pos_emb (first R entries rotated)
    rq = []
    for f in range(F):
        if R == 0:
            rq.append(q.clone())
            continue
        c = cos[f][:, None].to(torch.float32)   # [W,1,S,R]
        sn = sin[f][:, None].to(torch.float32)
        xr = q[..., :R].to(torch.float32)
        rot = torch.cat((-xr[..., R // 2:], xr[..., :R // 2]), -1)
        rq.append(torch.cat(((xr * c + rot * sn).to(dtype), q[..., R:]), -1))
    return SdpaCase(queries=q, rotated=torch.stack(rq).contiguous(), cosines=cos, sines=sin,
                    locations=torch.from_numpy(loc.astype(np.int32)).to(device),
                    fragment_lengths=torch.tensor(list(lens), dtype=torch.int32, device=device),
                    keys=keys, values=vals, scale=1.0 / math.sqrt(E),
                    meta=dict(F=F, W=W, Hq=Hq, Hkv=Hkv, E=E, R=R, S=S, batch=batch, seed=seed))


def varlen_flops(case: VarlenCase) -> int:
    Hq = case.queries.size(1)
    E, Ev = case.queries.size(2), case.v_cache.size(3)
    cap = case.block_tables.size(1) * case.k_cache.size(1)
    loc = case.locations.cpu().numpy()[:, :, None]
    n = int(visible_keys(loc, case.fragment_lengths.cpu().numpy(), cap).sum())
    return 2 * Hq * (E + Ev) * n


def varlen_bytes(case: VarlenCase) -> int:
    """Unique bytes: every cached K/V row of every sequence once + q + out + tables."""
    tl = case.meta["turn_lens"]
    Hkv, E, Ev = case.k_cache.size(2), case.queries.size(2), case.v_cache.size(3)
    es = ESIZE[case.dtype]
    kv = int(tl.sum()) * Hkv * (E + Ev) * es
    T, Hq, _ = case.queries.shape
    return kv + T * Hq * (E + Ev) * es + case.cosines.numel() * 8 + case.locations.numel() * 4 \
        + case.block_tables.numel() * 4


# ------------------------------------------------------------------------------------
# The benchmark configurations (BASELINE.json "configs", in order)
# ------------------------------------------------------------------------------------
def config1(device="cpu") -> PagedCase:
    """fp32 plumbing: W=1, 16/1 heads, E=128, R=64, L=1024 in 64 pages of 16 (identity
    block table), one turn, rotation offset 1024, seed 0."""
    return make_paged([[1024]], Hq=16, Hkv=1, E=128, R=64, BS=16, dtype=torch.float32, seed=0, device=device,
                      permute=False)


def config2_lengths(seed: int = 2, W: int = 32):
    rs = np.random.RandomState(seed)
    lens = rs.randint(512, 8193, size=W)
    split = np.array([rs.randint(1, n) for n in lens])
    return [[int(a), int(n - a)] for a, n in zip(split, lens)]


def config2(device="cpu", seed: int = 2, W: int = 32) -> PagedCase:
    """bf16 batched paged decode: W=32, 64/4 heads, E=128, R=64, len ~ U[512, 8192], page 16,
    two turns split at U[1, len-1], random page permutation."""
    return make_paged(config2_lengths(seed, W), Hq=64, Hkv=4, E=128, R=64, BS=16, dtype=torch.bfloat16, seed=seed,
                      device=device)


def config2_sdpa(device="cpu", seed: int = 2, W: int = 32) -> SdpaCase:
    """Config 2's shape on the contiguous-fragment op: per turn one K and one V fragment
    [W, 4, L_f, 128] bf16 with L_f the longest turn of the batch; worker w sees its own
    len_{w,f} keys (loc = len - 1); queries per turn [2, 32, 64, 1, 128]."""
    tl = np.asarray(config2_lengths(seed, W), dtype=np.int64)  # [W, F]
    F = tl.shape[1]
    Lf = tl.max(axis=0)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    Hq, Hkv, E = 64, 4, 128
    q = _randn((W, Hq, 1, E), torch.bfloat16, gen, device)
    rq = _randn((F, W, Hq, 1, E), torch.bfloat16, gen, device)
    keys = [_randn((W, Hkv, int(Lf[f]), E), torch.bfloat16, gen, device) for f in range(F)]
    vals = [_randn((W, Hkv, int(Lf[f]), E), torch.bfloat16, gen, device) for f in range(F)]
    loc = torch.from_numpy(np.ascontiguousarray(tl.T - 1, dtype=np.int32)).reshape(F, W, 1).contiguous().to(device)
    z = torch.zeros((F, W, 1, 0), dtype=torch.float32, device=device)
    return SdpaCase(queries=q, rotated=rq, cosines=z, sines=z.clone(), locations=loc,
                    fragment_lengths=torch.from_numpy(Lf.astype(np.int32)).to(device), keys=keys, values=vals,
                    scale=1.0 / math.sqrt(E), meta=dict(F=F, W=W, Hq=Hq, Hkv=Hkv, E=E, R=0, S=1, batch="w", seed=seed,
                                                        turn_lens=tl))


def sdpa_bytes(case: SdpaCase) -> int:
    """Algorithmic bytes of one dvattn_sdpa call: attended K+V rows of each worker + the
    per-turn queries + out + locations (padding past a worker's location is not counted)."""
    F, W, Hq, S, E = case.rotated.shape
    es = ESIZE[case.dtype]
    loc = case.locations.cpu().numpy().astype(np.int64)
    L = case.fragment_lengths.cpu().numpy().astype(np.int64)
    rows = np.array([k.size(-2) for k in case.keys], dtype=np.int64)
    Hkv = case.keys[0].size(-3)
    n = np.clip(np.minimum(loc.max(axis=2) + 1, np.minimum(L, rows)[:, None]), 0, None).sum()
    return int(n) * Hkv * 2 * E * es + case.rotated.numel() * es + W * Hq * S * E * es + case.locations.numel() * 4


def config3(device="cpu", seed: int = 3, L: int = 131072, W: int = 4) -> PagedCase:
    """fp16 long context: W=4, 128/8 heads, E=128, R=128 (full rotary), L=131072, page 64, one turn."""
    return make_paged([[L]] * W, Hq=128, Hkv=8, E=128, R=128, BS=64, dtype=torch.float16, seed=seed, device=device)


def config4_lengths(seed: int = 4, W: int = 16):
    rs = np.random.RandomState(seed)
    q = rs.randint(1, 2049, size=W)
    p = rs.randint(0, 16385, size=W)
    return [[int(a + b)] for a, b in zip(p, q)], [int(x) for x in q]


def config4(device="cpu", seed: int = 4, W: int = 16) -> VarlenCase:
    """bf16 varlen chunked prefill: 16 sequences, q ~ U[1,2048] new tokens after p ~ U[0,16384]
    cached ones, causal, 32/2 heads, E=128, R=32, page 16."""
    tl, ql = config4_lengths(seed, W)
    return make_varlen(tl, ql, Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=seed, device=device)


def config5_lengths(seed: int = 5, W: int = 256):
    rs = np.random.RandomState(seed)
    lens = np.clip(np.round(rs.lognormal(7.6, 0.8, size=W)), 16, 32768).astype(np.int64)
    out = []
    for n in lens:
        k = rs.randint(1, 5)
        cuts = np.sort(rs.choice(np.arange(1, n), size=k - 1, replace=False)) if k > 1 else np.array([], np.int64)
        parts = np.diff(np.concatenate([[0], cuts, [n]])).tolist()
        out.append([int(x) for x in parts] + [0] * (4 - k))
    return out


def config5(device="cpu", seed: int = 5, W: int = 256) -> PagedCase:
    """fp16 serving mix: W=256, 32/2 heads, E=256, R=64, len ~ lognormal(7.6, 0.8) clipped to
    [16, 32768], page 64, 1-4 turns per sequence (missing turns: length 0, loc = -1)."""
    return make_paged(config5_lengths(seed, W), Hq=32, Hkv=2, E=256, R=64, BS=64, dtype=torch.float16, seed=seed,
                      device=device)


CONFIGS = {1: config1, 2: config2, 3: config3, 4: config4, 5: config5}
