"""Python wrappers in the style of python/dvattn/attention.py (``dvattn_fused``,
``dvattn_sdpa``, ``dvattn_rope``, ``rotate_half``, ``apply_rotary_pos_emb`` keep the
reference names and arguments, attention.py:17-88); the paged ops, which the reference
only exposes as ``torch.ops.libdvatt.*``, get thin wrappers that allocate ``out`` when it
is not given.
"""
from __future__ import annotations

from typing import Optional

import torch

_ops = torch.ops.libdvatt


def dvattn_fused(queries: torch.Tensor, locations: torch.Tensor, keys: list, values: list, scale: float,
                 fragment_lengths, cosines: torch.Tensor, sines: torch.Tensor, *, rotated_queries, out):
    """Rope + attention over contiguous per-turn fragments (attention.py:17-21): queries
    [W,Hq,S,E] are rotated into ``rotated_queries`` [F,W,Hq,S,E], then attend."""
    _ops.dvattn_fused(out, rotated_queries, scale, locations, queries.contiguous(), fragment_lengths, keys, values,
                      cosines, sines)
    return out


def dvattn_sdpa(queries: torch.Tensor, locations: torch.Tensor, keys: list, values: list, scale: float,
                fragment_lengths=None, out=None) -> torch.Tensor:
    """Attention over contiguous per-turn fragments (attention.py:24-34): queries
    [F,W,Hq,S,E] (rotated), keys/values F tensors [Hkv,L_f,E] or [B,Hkv,L_f,E] (B = 1 or W),
    locations [F,W,S] -> out [W,Hq,S,Ev]."""
    if out is None:
        out = torch.empty((queries.size(1), queries.size(2), queries.size(3), values[0].size(-1)),
                          dtype=queries.dtype, device=queries.device)
    if fragment_lengths is None:
        fragment_lengths = torch.tensor([k.size(-2) for k in keys], dtype=torch.int32, device=queries.device)
    keys = [k.contiguous() for k in keys]
    values = [v.contiguous() for v in values]
    _ops.dvattn_sdpa(out, scale, locations, queries.contiguous(), fragment_lengths, keys, values)
    return out


def dvattn_paged_sdpa(queries: torch.Tensor, locations: torch.Tensor, cosines: torch.Tensor, sines: torch.Tensor,
                      fragment_lengths: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      block_tables: torch.Tensor, scale: float, out: Optional[torch.Tensor] = None,
                      lse: Optional[torch.Tensor] = None, out_f32: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Paged multi-turn decode.  queries [W,Hq,S,E] (unrotated), cos/sin [F,W,S,R] f32,
    locations [F,W,S] i32, fragment_lengths [F] i32, k/v cache [NB,BS,Hkv,E], block_tables
    [W,max_blocks] i32 -> out [W,Hq,S,Ev].  ``lse`` ([W,Hq,S] f32, natural log) and
    ``out_f32`` are optional extra outputs."""
    if out is None:
        out = torch.empty(queries.shape[:3] + (v_cache.size(3),), dtype=queries.dtype, device=queries.device)
    if lse is None and out_f32 is None:
        _ops.dvattn_paged_sdpa(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache,
                               block_tables)
    else:
        _ops.dvattn_paged_sdpa_ex(out, lse, out_f32, scale, locations, queries, cosines, sines, fragment_lengths,
                                  k_cache, v_cache, block_tables)
    return out


def dvattn_varlen_paged_sdpa(queries: torch.Tensor, locations: torch.Tensor, cosines: torch.Tensor,
                             sines: torch.Tensor, fragment_lengths: torch.Tensor, k_cache: torch.Tensor,
                             v_cache: torch.Tensor, block_tables: torch.Tensor, cu_seqlens_q: torch.Tensor,
                             cu_seqlens_k: Optional[torch.Tensor], scale: float, out: Optional[torch.Tensor] = None,
                             lse: Optional[torch.Tensor] = None,
                             out_f32: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Varlen chunked prefill.  queries [T,Hq,E], cos/sin [F,T,R/2] f32, locations [F,T]
    i32 (negative = turn skipped), cu_seqlens_q [W+1] i32 -> out [T,Hq,Ev]."""
    if out is None:
        out = torch.empty((queries.size(0), queries.size(1), v_cache.size(3)), dtype=queries.dtype,
                          device=queries.device)
    if cu_seqlens_k is None:
        cu_seqlens_k = cu_seqlens_q
    if lse is None and out_f32 is None:
        _ops.dvattn_varlen_paged_sdpa(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache,
                                      v_cache, block_tables, cu_seqlens_q, cu_seqlens_k)
    else:
        _ops.dvattn_varlen_paged_sdpa_ex(out, lse, out_f32, scale, locations, queries, cosines, sines,
                                         fragment_lengths, k_cache, v_cache, block_tables, cu_seqlens_q,
                                         cu_seqlens_k)
    return out


_ROUND = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def dvattn_build_views(seg_lengths: torch.Tensor, seg_order: torch.Tensor, n: int, R: int, rope_base: float,
                       attention_scaling: float = 1.0, dtype=torch.float32):
    """Turn/view metadata on the GPU (DVAttnCache.update, attention.py:161-191): for F
    segments with lengths seg_lengths [F] i32 and each worker's segment order seg_order
    [W, F] i32 (index of segment f in worker w's list), the locations [F, W, n] of the n new
    tokens and their cos/sin [F, W, n, R] f32 from the model's rotary embedding (base
    ``rope_base``, scaled, rounded through ``dtype`` as the model returns them)."""
    F, W = seg_lengths.size(0), seg_order.size(0)
    dev = seg_lengths.device
    loc = torch.empty((F, W, n), dtype=torch.int32, device=dev)
    cos = torch.empty((F, W, n, R), dtype=torch.float32, device=dev)
    sin = torch.empty((F, W, n, R), dtype=torch.float32, device=dev)
    inv_freq = _inv_freq(R, rope_base, dev)
    _ops.dvattn_build_views(loc, cos, sin, seg_lengths, seg_order, inv_freq, rope_base, attention_scaling,
                            _ROUND[dtype])
    return loc, cos, sin


def _inv_freq(R: int, rope_base: float, device) -> Optional[torch.Tensor]:
    """The inverse frequencies exactly as the model's rotary module computes them (host)."""
    if not R:
        return None
    return (1.0 / (rope_base ** (torch.arange(0, R, 2, dtype=torch.int64).float() / R))).to(device)


def dvattn_paged_sdpa_rope(queries: torch.Tensor, locations: torch.Tensor, fragment_lengths: torch.Tensor,
                           k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor, scale: float,
                           rotary_dim: int, rope_base: float, attention_scaling: float = 1.0,
                           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dvattn_paged_sdpa with the query rotation of turn f taken as the model's rotary
    embedding at the query's own location loc[f, w, s] (what DVAttnCache.update passes,
    attention.py:161-191), built on the device: no cosines/sines tensors."""
    if out is None:
        W, Hq, S, _ = queries.shape
        out = torch.empty((W, Hq, S, v_cache.size(3)), dtype=queries.dtype, device=queries.device)
    _ops.dvattn_paged_sdpa_rope(out, scale, locations, queries, fragment_lengths, k_cache, v_cache, block_tables,
                                rotary_dim, rope_base, attention_scaling, _inv_freq(rotary_dim, rope_base, out.device))
    return out


def dvattn_varlen_paged_sdpa_rope(queries: torch.Tensor, locations: torch.Tensor, fragment_lengths: torch.Tensor,
                                  k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                                  cu_seqlens_q: torch.Tensor, scale: float, rotary_dim: int, rope_base: float,
                                  attention_scaling: float = 1.0, cu_seqlens_k: Optional[torch.Tensor] = None,
                                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dvattn_varlen_paged_sdpa with the rotation tables built on the device from the
    locations (token t of turn f rotated by the rotary embedding at loc[f, t])."""
    if out is None:
        T, Hq, _ = queries.shape
        out = torch.empty((T, Hq, v_cache.size(3)), dtype=queries.dtype, device=queries.device)
    _ops.dvattn_varlen_paged_sdpa_rope(out, scale, locations, queries, fragment_lengths, k_cache, v_cache,
                                       block_tables, cu_seqlens_q,
                                       cu_seqlens_k if cu_seqlens_k is not None else cu_seqlens_q, rotary_dim,
                                       rope_base, attention_scaling, _inv_freq(rotary_dim, rope_base, out.device))
    return out


def dvattn_paged_append(k_cache: torch.Tensor, v_cache: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                        cosines: torch.Tensor, sines: torch.Tensor, block_tables: torch.Tensor,
                        positions: torch.Tensor, counts: Optional[torch.Tensor] = None) -> None:
    """Append new tokens to the paged cache with the keys rotated as apply_rotary_pos_emb
    (attention.py:302-304): keys/values [W,Hkv,n,E|Ev] (unrotated), cos/sin [W,n,R] f32
    (full width), positions [W] i32 = logical position of worker w's first new token,
    counts [W] i32 = how many of the n tokens are new (the last ones; left padding)."""
    _ops.dvattn_paged_append(k_cache, v_cache, keys, values, cosines, sines, block_tables, positions, counts)


def dvattn_rope(queries: torch.Tensor, cosines: torch.Tensor, sines: torch.Tensor, out=None) -> torch.Tensor:
    """Same signature as python/dvattn/attention.py:68-72: out [F,W,Hq,S,E]."""
    if out is None:
        out = torch.empty((cosines.size(0),) + tuple(queries.shape), dtype=queries.dtype, device=queries.device)
    _ops.dvattn_rope(out, queries, cosines, sines)
    return out


def dvattn_varlen_rope(queries: torch.Tensor, cosines: torch.Tensor, sines: torch.Tensor, out=None) -> torch.Tensor:
    """out [F,T,H,E] from queries [T,H,E] and cos/sin [F,T,R/2]."""
    if out is None:
        out = torch.empty((cosines.size(0),) + tuple(queries.shape), dtype=queries.dtype, device=queries.device)
    _ops.dvattn_varlen_rope(out, queries, cosines, sines)
    return out


def dvattn_lse_merge(part_out: torch.Tensor, part_lse: torch.Tensor, out: torch.Tensor,
                     lse_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Merge [parts, ..., Ev] f32 partials with their natural-log LSEs [parts, ...] into out."""
    _ops.dvattn_lse_merge(out, lse_out, part_out, part_lse)
    return out


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Rotates half the hidden dims of the input (python/dvattn/attention.py:75-79)."""
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary_pos_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, unsqueeze_dim: int = 1) -> torch.Tensor:
    """Partial rotary embedding with rotary_dim = cos.shape[-1] (python/dvattn/attention.py:82-88).
    Used on the key side by callers; the attention ops rotate queries themselves."""
    cos = cos.unsqueeze(unsqueeze_dim)
    sin = sin.unsqueeze(unsqueeze_dim)
    rotary_dim = cos.shape[-1]
    x_rot, x_pass = x[..., :rotary_dim], x[..., rotary_dim:]
    x_rot_emb = (x_rot * cos) + (rotate_half(x_rot) * sin)
    return torch.cat((x_rot_emb, x_pass), dim=-1).to(x.dtype)
