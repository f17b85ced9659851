"""dvattn_b200 -- B200-native (sm_100a) DVAttn attention forward.

Importing the package loads ``dvatt.abi3.so``, which registers the reference's
``torch.ops.libdvatt`` schemas (``dvattn_paged_sdpa``, ``dvattn_varlen_paged_sdpa``,
``dvattn_rope``, ``dvattn_varlen_rope``, ``dvattn_sdpa``, ``dvattn_fused``) plus the B200
additions (``dvattn_paged_sdpa_ex``, ``dvattn_varlen_paged_sdpa_ex``, ``dvattn_lse_merge``,
``dvattn_paged_append``, ``dvattn_build_views`` and the ``*_rope`` attention variants).  There is no CPU fallback: if the native libraries are missing,
the import fails.
"""
from __future__ import annotations

import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
TORCH_OPS_LIB = os.path.join(_HERE, "dvatt.abi3.so")
CAPI_LIB = os.path.join(_HERE, "libdvattn_b200.so")


def _load() -> None:
    if not os.path.exists(TORCH_OPS_LIB) or not os.path.exists(CAPI_LIB):
        raise ImportError(
            "dvattn_b200: native libraries not built (expected %s and %s); run `python dvattn_b200/_build.py`"
            % (CAPI_LIB, TORCH_OPS_LIB))
    torch.ops.load_library(TORCH_OPS_LIB)


_load()

from .api import (  # noqa: E402
    apply_rotary_pos_emb,
    dvattn_build_views,
    dvattn_fused,
    dvattn_lse_merge,
    dvattn_paged_append,
    dvattn_paged_sdpa,
    dvattn_paged_sdpa_rope,
    dvattn_rope,
    dvattn_sdpa,
    dvattn_varlen_paged_sdpa,
    dvattn_varlen_paged_sdpa_rope,
    dvattn_varlen_rope,
    rotate_half,
)

__all__ = [
    "apply_rotary_pos_emb",
    "dvattn_build_views",
    "dvattn_fused",
    "dvattn_lse_merge",
    "dvattn_paged_append",
    "dvattn_paged_sdpa",
    "dvattn_paged_sdpa_rope",
    "dvattn_rope",
    "dvattn_sdpa",
    "dvattn_varlen_paged_sdpa",
    "dvattn_varlen_paged_sdpa_rope",
    "dvattn_varlen_rope",
    "rotate_half",
]
