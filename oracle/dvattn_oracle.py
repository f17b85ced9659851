"""CPU oracle for the DVAttn paged/varlen attention forward.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this module; only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm use it, as
the checker and as the timed CPU port of the reference's pure-PyTorch path.

It restates, in torch-on-CPU (f32 math), the reference algorithm:

* ``rotate_half`` / ``apply_rotary_pos_emb``  -- python/dvattn/attention.py:75-88
* ``sdpa_pt``                                  -- python/dvattn/attention.py:36-65
  (GQA by repeat_interleave, f32 q.k, mask kp > loc, one softmax over the concatenated
  turns, @ V), extended to return the natural-log LSE of scale*q.k.
* ``paged_sdpa``   -- the `dvattn_paged_sdpa` op (src/binding.cu:151-203): q rotated per
  turn from the first R/2 entries of each cos/sin row (src/rope.cuh:24-45), rounded to the
  dtype, key l of turn f read at logical position sum_{f'<f} L_f' + l through the block
  table (src/kernels/paged_kernel_v21.cuh:101-115), rows that see no key -> 0
  (paged_kernel_v21.cuh:330-345, 366-373).
* ``varlen_paged_sdpa`` -- `dvattn_varlen_paged_sdpa` (src/binding.cu:249-296): token ->
  sequence by cu_seqlens_q (varlen_paged_kernel_v21.cuh:40-47), negative loc skips a turn
  (:76-80).
* ``rope`` / ``varlen_rope`` -- the standalone rotation ops (src/rope.cuh:2-114).

Two implementations of the attention are kept: ``sdpa_pt`` follows the reference line
by line (used on small cases, pinned to the reference's own outputs by
tests/golden/), and ``paged_sdpa``/``varlen_paged_sdpa`` compute the same mathematics per
(row, KV head) so that full-size configs fit in host memory; tests check the two agree.
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import numpy as np
import torch


# ---------------------------------------------------------------------------------
# python/dvattn/attention.py:75-88
# ---------------------------------------------------------------------------------
def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary_pos_emb(x, cos, sin, unsqueeze_dim=1):
    cos = cos.unsqueeze(unsqueeze_dim)
    sin = sin.unsqueeze(unsqueeze_dim)
    rotary_dim = cos.shape[-1]
    x_rot, x_pass = x[..., :rotary_dim], x[..., rotary_dim:]
    x_rot_emb = (x_rot * cos) + (rotate_half(x_rot) * sin)
    return torch.cat((x_rot_emb, x_pass), dim=-1).to(x.dtype)


def half_to_full(cs: torch.Tensor, R: int) -> torch.Tensor:
    """The CUDA rope reads only the first R/2 entries of a cos/sin row (src/rope.cuh:24-45,
    100-116); duplicating them gives the row apply_rotary_pos_emb expects."""
    h = cs[..., : R // 2]
    return torch.cat([h, h], -1)


# ---------------------------------------------------------------------------------
# python/dvattn/attention.py:36-65 (+ LSE)
# ---------------------------------------------------------------------------------
def sdpa_pt(queries, locations, keys, values, scale, return_lse=False):
    """queries [F,W,Hq,S,E] (already rotated), locations [F,W,S], keys[f] [W|1,Hkv,L_f,E]."""
    qk = []
    vals = []
    for f in range(len(keys)):
        key = keys[f].repeat_interleave(queries.size(-3) // keys[f].size(-3), -3)
        val = values[f].repeat_interleave(queries.size(-3) // values[f].size(-3), -3)
        kp = torch.arange(0, key.size(-2), dtype=torch.int32, device=key.device)
        qp = locations[f]
        kp = kp[None, None, None, :]
        qp = qp[:, None, :, None]
        mask = kp > qp
        att = queries[f].to(torch.float32) @ key.transpose(-1, -2).to(torch.float32)
        att.masked_fill_(mask, float("-inf"))
        qk.append(att)
        vals.append(val)
    qk = torch.concat(qk, dim=-1)
    vals = torch.concat(vals, dim=-2).to(torch.float32)
    att = torch.softmax(scale * qk, dim=-1)
    result = att @ vals
    if return_lse:
        return result, torch.logsumexp(scale * qk, dim=-1)
    return result.to(queries.dtype)


# ---------------------------------------------------------------------------------
# paged layout helpers
# ---------------------------------------------------------------------------------
def turn_offsets(L: np.ndarray) -> np.ndarray:
    return np.concatenate([[0], np.cumsum(L)[:-1]]).astype(np.int64) if len(L) else np.zeros(0, np.int64)


def effective_locations(loc: np.ndarray, L: np.ndarray, cap: int) -> np.ndarray:
    """Locations with the block-table bound applied: positions at or past max_blocks *
    block_size are never visible (loc is clipped to cap - off_f - 1)."""
    off = turn_offsets(L)
    shape = (-1,) + (1,) * (loc.ndim - 1)
    return np.minimum(loc.astype(np.int64), (cap - off - 1).reshape(shape))


def gather_turn(k_cache, v_cache, bt_row: np.ndarray, off: int, n: int, BS: int, NB: int):
    """Rows [off, off+n) of one sequence's logical cache -> K [Hkv, n, E], V [Hkv, n, Ev].
    Pages outside [0, NB) read as zeros."""
    pos = np.arange(off, off + n, dtype=np.int64)
    page = bt_row[pos // BS].astype(np.int64)
    ok = (page >= 0) & (page < NB)
    page_c = np.where(ok, page, 0)
    idx_p = torch.from_numpy(page_c)
    idx_s = torch.from_numpy(pos % BS)
    K = k_cache[idx_p, idx_s]  # [n, Hkv, E]
    V = v_cache[idx_p, idx_s]
    if not ok.all():
        m = torch.from_numpy(~ok)
        K = K.clone()
        V = V.clone()
        K[m] = 0
        V[m] = 0
    return K.transpose(0, 1), V.transpose(0, 1)


def _attend_rows(qrot: List[torch.Tensor], locs: np.ndarray, Ks, Vs, scale: float):
    """One KV head, G query heads, Srow query rows.
    qrot[f] [G, Srow, E] (dtype), locs [F, Srow], Ks[f] [n_f, E], Vs[f] [n_f, Ev]
    -> out [G, Srow, Ev] f32, lse [G, Srow] (natural log); rows without keys -> 0 / -inf."""
    scores = []
    for f in range(len(Ks)):
        n = Ks[f].size(0)
        s = qrot[f].to(torch.float32) @ Ks[f].to(torch.float32).T  # [G, Srow, n]
        kp = torch.arange(n)[None, None, :]
        qp = torch.from_numpy(locs[f].astype(np.int64))[None, :, None]
        s = s.masked_fill(kp > qp, float("-inf"))
        scores.append(s)
    G, Srow = qrot[0].shape[:2]
    Ev = Vs[0].size(-1) if Vs else 0
    if not scores or sum(x.size(-1) for x in scores) == 0:
        return torch.zeros(G, Srow, Ev), torch.full((G, Srow), float("-inf"))
    s = torch.cat(scores, -1) * scale
    V = torch.cat([v.to(torch.float32) for v in Vs], 0)
    lse = torch.logsumexp(s, -1)
    p = torch.softmax(s, -1)
    out = p @ V
    dead = torch.isinf(lse)
    out[dead] = 0.0
    return out, lse


def rotate_turn(q: torch.Tensor, cos_row: torch.Tensor, sin_row: torch.Tensor, R: int, unsqueeze_dim: int):
    """q [..., E] (dtype) rotated with the first R/2 entries of the cos/sin rows, which
    broadcast against q after ``unsqueeze(unsqueeze_dim)``."""
    if R == 0:
        return q.clone()
    return apply_rotary_pos_emb(q, half_to_full(cos_row, R), half_to_full(sin_row, R), unsqueeze_dim=unsqueeze_dim)


def paged_sdpa(scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
               out_dtype=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """dvattn_paged_sdpa on CPU -> (out [W,Hq,S,Ev] in the dtype, lse [W,Hq,S] f32).
    Also returns nothing else; the f32 output is available via ``paged_sdpa_f32``."""
    out32, lse = paged_sdpa_f32(scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache,
                                block_tables)
    dt = out_dtype or queries.dtype
    return out32.to(dt), lse


def paged_sdpa_f32(scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables):
    queries, cosines, sines = queries.cpu(), cosines.cpu(), sines.cpu()
    k_cache, v_cache = k_cache.cpu(), v_cache.cpu()
    loc = locations.cpu().numpy().astype(np.int64)
    L = fragment_lengths.cpu().numpy().astype(np.int64)
    bt = block_tables.cpu().numpy()
    W, Hq, S, E = queries.shape
    NB, BS, Hkv, _ = k_cache.shape
    Ev = v_cache.size(3)
    F = loc.shape[0]
    R = cosines.size(3)
    G = Hq // Hkv
    cap = bt.shape[1] * BS
    locs = effective_locations(loc, L, cap)
    off = turn_offsets(L)
    out = torch.zeros(W, Hq, S, Ev)
    lse = torch.full((W, Hq, S), float("-inf"))
    for w in range(W):
        nvis = [int(max(0, min(L[f], locs[f, w].max() + 1))) for f in range(F)]
        qrot = [rotate_turn(queries[w], cosines[f, w], sines[f, w], R, 0) for f in range(F)]  # [Hq, S, E]
        for h in range(Hkv):
            Ks, Vs = [], []
            for f in range(F):
                K, V = gather_turn(k_cache, v_cache, bt[w], int(off[f]), nvis[f], BS, NB)
                Ks.append(K[h])
                Vs.append(V[h])
            o, l = _attend_rows([qr[h * G:(h + 1) * G] for qr in qrot], locs[:, w], Ks, Vs, scale)
            out[w, h * G:(h + 1) * G] = o
            lse[w, h * G:(h + 1) * G] = l
    return out, lse


def varlen_paged_sdpa(scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
                      cu_seqlens_q, out_dtype=None):
    out32, lse = varlen_paged_sdpa_f32(scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache,
                                       block_tables, cu_seqlens_q)
    return out32.to(out_dtype or queries.dtype), lse


def varlen_paged_sdpa_f32(scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache,
                          block_tables, cu_seqlens_q):
    """dvattn_varlen_paged_sdpa on CPU -> (out [T,Hq,Ev] f32, lse [T,Hq])."""
    queries, cosines, sines = queries.cpu(), cosines.cpu(), sines.cpu()
    k_cache, v_cache = k_cache.cpu(), v_cache.cpu()
    loc = locations.cpu().numpy().astype(np.int64)  # [F, T]
    L = fragment_lengths.cpu().numpy().astype(np.int64)
    bt = block_tables.cpu().numpy()
    cu = cu_seqlens_q.cpu().numpy().astype(np.int64)
    T, Hq, E = queries.shape
    NB, BS, Hkv, _ = k_cache.shape
    Ev = v_cache.size(3)
    F = loc.shape[0]
    R = 2 * cosines.size(2)
    G = Hq // Hkv
    cap = bt.shape[1] * BS
    locs = effective_locations(loc, L, cap)
    off = turn_offsets(L)
    W = len(cu) - 1
    # token -> sequence: the first w with t < cu[w+1], else 0
    seq = np.zeros(T, np.int64)
    for t in range(T):
        hit = np.nonzero(t < cu[1:])[0]
        seq[t] = hit[0] if len(hit) else 0
    out = torch.zeros(T, Hq, Ev)
    lse = torch.full((T, Hq), float("-inf"))
    for w in sorted(set(seq.tolist())):
        toks = np.nonzero(seq == w)[0]
        nvis = [int(max(0, min(L[f], locs[f, toks].max() + 1))) for f in range(F)]
        qrot = [rotate_turn(queries[toks], cosines[f, toks], sines[f, toks], R, 1).transpose(0, 1)
                for f in range(F)]  # [Hq, n_tok, E]
        for h in range(Hkv):
            Ks, Vs = [], []
            for f in range(F):
                K, V = gather_turn(k_cache, v_cache, bt[w], int(off[f]), nvis[f], BS, NB)
                Ks.append(K[h])
                Vs.append(V[h])
            o, l = _attend_rows([qr[h * G:(h + 1) * G] for qr in qrot], locs[:, toks], Ks, Vs, scale)
            out[toks, h * G:(h + 1) * G] = o.transpose(0, 1)
            lse[toks, h * G:(h + 1) * G] = l.transpose(0, 1)
    return out, lse


def rope(queries, cosines, sines):
    """dvattn_rope: [W,Hq,S,E] x [F,W,S,R] -> [F,W,Hq,S,E] (src/rope.cuh:2-52)."""
    queries, cosines, sines = queries.cpu(), cosines.cpu(), sines.cpu()
    R = cosines.size(3)
    return torch.stack([rotate_turn(queries, cosines[f], sines[f], R, 1) for f in range(cosines.size(0))])


def varlen_rope(queries, cosines, sines):
    """dvattn_varlen_rope: [T,H,E] x [F,T,R/2] -> [F,T,H,E] (src/rope.cuh:54-101)."""
    queries, cosines, sines = queries.cpu(), cosines.cpu(), sines.cpu()
    R = 2 * cosines.size(2)
    return torch.stack([rotate_turn(queries, cosines[f], sines[f], R, 1) for f in range(cosines.size(0))])


def lse_merge(part_out: torch.Tensor, part_lse: torch.Tensor):
    """Merge [P, rows, Ev] f32 partials with natural-log LSEs [P, rows] (empty = -inf)."""
    mx = part_lse.max(0).values
    mx_safe = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
    wgt = torch.exp(part_lse - mx_safe)
    den = wgt.sum(0)
    out = (wgt[..., None] * part_out).sum(0) / torch.where(den > 0, den, torch.ones_like(den))[..., None]
    lse = torch.where(den > 0, mx_safe + torch.log(den), torch.full_like(den, float("-inf")))
    return out, lse


# ---------------------------------------------------------------------------------
# the reference algorithm verbatim on a paged case (small sizes): gather pages into
# per-turn fragments and call sdpa_pt, the way a caller of the reference's eager path
# would.  Used to pin the fast restatement above.
# ---------------------------------------------------------------------------------
def paged_via_sdpa_pt(scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
                      trim: bool = False):
    """trim=True cuts each turn's fragment after the last key any row of the batch can see
    (the keys cut are masked for every row, so the result is the same); with one sequence
    per call this is the sequence's own visible length, as a caller with per-sequence
    fragments would pass them."""
    loc = locations.cpu()
    L = fragment_lengths.cpu().numpy().astype(np.int64)
    bt = block_tables.cpu().numpy()
    W, Hq, S, E = queries.shape
    NB, BS, Hkv, _ = k_cache.shape
    F = loc.size(0)
    R = cosines.size(3)
    off = turn_offsets(L)
    vis_max = np.maximum(0, np.minimum(L[:, None], loc.numpy().max(axis=2) + 1))  # [F, W]
    keys, values = [], []
    for f in range(F):
        Lf = int(vis_max[f].max()) if (trim and W) else int(L[f])
        Kf = torch.zeros(W, Hkv, Lf, E, dtype=k_cache.dtype)
        Vf = torch.zeros(W, Hkv, Lf, v_cache.size(3), dtype=v_cache.dtype)
        for w in range(W):
            n = int(vis_max[f, w])
            K, V = gather_turn(k_cache.cpu(), v_cache.cpu(), bt[w], int(off[f]), n, BS, NB)
            Kf[w, :, :n] = K
            Vf[w, :, :n] = V
        keys.append(Kf)
        values.append(Vf)
    rq = torch.stack([apply_rotary_pos_emb(queries.cpu(), half_to_full(cosines[f].cpu(), R),
                                           half_to_full(sines[f].cpu(), R), unsqueeze_dim=1) for f in range(F)])
    out, lse = sdpa_pt(rq, loc, keys, values, scale, return_lse=True)
    return out, lse


# ---------------------------------------------------------------------------------
# paged KV append with K rotation: apply_rotary_pos_emb on the new keys
# (python/dvattn/attention.py:302-304) + the cache update of the last counts[w] tokens
# (attention.py:131-149), written through the block table
# ---------------------------------------------------------------------------------
def paged_append(k_cache, v_cache, keys, values, cosines, sines, block_tables, positions, counts=None):
    """Returns updated copies of k_cache / v_cache (CPU)."""
    k_cache, v_cache = k_cache.clone().cpu(), v_cache.clone().cpu()
    keys, values = keys.cpu(), values.cpu()
    W, Hkv, n, E = keys.shape
    R = cosines.size(2)
    if R:
        rk = apply_rotary_pos_emb(keys, cosines.cpu(), sines.cpu(), unsqueeze_dim=1)
    else:
        rk = keys
    bt = block_tables.cpu().numpy()
    pos = positions.cpu().numpy()
    cnt = counts.cpu().numpy() if counts is not None else np.full(W, n)
    NB, BS = k_cache.shape[:2]
    for w in range(W):
        c = int(max(0, min(n, cnt[w])))
        for i in range(c):
            t = n - c + i
            lp = int(pos[w]) + i
            if lp < 0 or lp >= bt.shape[1] * BS:
                continue
            page = int(bt[w, lp // BS])
            if page < 0 or page >= NB:
                continue
            k_cache[page, lp % BS] = rk[w, :, t]
            v_cache[page, lp % BS] = values[w, :, t]
    return k_cache, v_cache


# ---------------------------------------------------------------------------------
# turn/view metadata: DVAttnCache.update at layer 0 (python/dvattn/attention.py:161-191)
# and the model's default rotary embedding of the locations (HF rotary: inv_freq =
# 1 / base^(arange(0, R, 2) / R) in f32, freqs = inv_freq * pos, emb = cat(freqs, freqs),
# cos/sin times attention_scaling, returned in the model dtype, widened to f32)
# ---------------------------------------------------------------------------------
def build_views(seg_lengths, seg_order, n, R, rope_base, attention_scaling=1.0, dtype=torch.float32):
    lens = [int(x) for x in seg_lengths]
    order = np.asarray(seg_order)
    F, W = len(lens), order.shape[0]
    loc = torch.zeros((F, W, n), dtype=torch.int32)
    for w in range(W):
        # worker w's list, then the backward walk of the reference
        lst = sorted(range(F), key=lambda f: order[w, f])
        pos = 0
        for f in reversed(lst):
            pos += lens[f]
            loc[f, w] = torch.arange(pos - n, pos, dtype=torch.int32)
    if R == 0:
        z = torch.zeros((F, W, n, 0))
        return loc, z, z.clone()
    cos, sin = rotary_tables(loc, R, rope_base, attention_scaling, dtype)
    return loc, cos, sin


def rotary_tables(loc, R, rope_base, attention_scaling=1.0, dtype=torch.float32):
    """The model's default rotary embedding at positions `loc` (any shape): cos/sin
    [..., R] f32 with equal halves, computed as HF's rotary module does (inv_freq =
    1 / base^(arange(0, R, 2) / R) in f32, freqs = pos * inv_freq, cat(freqs, freqs),
    times attention_scaling, in the model dtype, widened to f32)."""
    inv_freq = 1.0 / (rope_base ** (torch.arange(0, R, 2, dtype=torch.int64).float() / R))
    freqs = torch.as_tensor(loc).float()[..., None] * inv_freq
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = (emb.cos() * attention_scaling).to(dtype).to(torch.float32)
    sin = (emb.sin() * attention_scaling).to(dtype).to(torch.float32)
    return cos, sin
