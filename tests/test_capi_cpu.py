"""The C-ABI library loads and exports every entry point include/dvattn_b200.h declares;
argument validation answers without touching a GPU; the torch op layer registers the
reference's schemas.  CPU only (no kernel is launched)."""
import ctypes
import os
import re

import pytest
import torch

import dvattn_b200
from dvattn_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dvattn_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_]+\**\s+\**(dvattn_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_expected_functions():
    assert header_functions() == sorted(capi.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = capi.lib()
    for name in header_functions():
        assert hasattr(lib, name), name
    assert lib.dvattn_abi_version() == 1


def test_status_strings():
    lib = capi.lib()
    for st in range(5):
        assert lib.dvattn_status_string(st)
    assert b"unknown" in lib.dvattn_status_string(99)


def _args(**kw):
    a = capi.PagedArgs()
    base = dict(dtype=capi.DVATTN_BFLOAT16, F=1, W=2, Hq=32, Hkv=2, E=128, Ev=128, S=1, R=64, block_size=16,
                max_blocks_per_seq=4, num_blocks=8, scale=0.1)
    base.update(kw)
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,status", [
    (dict(dtype=7), capi.DVATTN_ERR_UNSUPPORTED),
    (dict(E=96, Ev=96), capi.DVATTN_ERR_UNSUPPORTED),
    (dict(Ev=64), capi.DVATTN_ERR_UNSUPPORTED),
    (dict(Hq=64, Hkv=2), capi.DVATTN_ERR_UNSUPPORTED),   # GQA 32
    (dict(Hq=33), capi.DVATTN_ERR_INVALID_ARGUMENT),     # Hq % Hkv
    (dict(R=130), capi.DVATTN_ERR_INVALID_ARGUMENT),
    (dict(R=63), capi.DVATTN_ERR_INVALID_ARGUMENT),
    (dict(block_size=0), capi.DVATTN_ERR_INVALID_ARGUMENT),
    (dict(Hkv=0), capi.DVATTN_ERR_INVALID_ARGUMENT),
])
def test_validation_without_gpu(kw, status):
    a = _args(**kw)
    assert capi.lib().dvattn_paged_sdpa(ctypes.byref(a), None, 0, None) == status
    assert capi.lib().dvattn_paged_sdpa_workspace_size(ctypes.byref(a)) == 0


def test_null_args_and_empty_problem():
    lib = capi.lib()
    assert lib.dvattn_paged_sdpa(None, None, 0, None) == capi.DVATTN_ERR_INVALID_ARGUMENT
    # W * S == 0: nothing to do, success without a launch (reference: problem_size == 0)
    a = _args(W=0)
    assert lib.dvattn_paged_sdpa(ctypes.byref(a), None, 0, None) == capi.DVATTN_OK
    # missing pointers with work to do
    a = _args()
    assert lib.dvattn_paged_sdpa(ctypes.byref(a), None, 0, None) == capi.DVATTN_ERR_INVALID_ARGUMENT


def test_rope_and_merge_validation_without_gpu():
    lib = capi.lib()
    assert lib.dvattn_rope(capi.DVATTN_FLOAT16, 1, 1, 1, 1, 64, 65, None, None, None, None, None) == \
        capi.DVATTN_ERR_INVALID_ARGUMENT
    assert lib.dvattn_rope(capi.DVATTN_FLOAT16, 0, 1, 1, 1, 64, 32, None, None, None, None, None) == capi.DVATTN_OK
    assert lib.dvattn_varlen_rope(capi.DVATTN_FLOAT16, 1, 0, 1, 64, 32, None, None, None, None, None) == capi.DVATTN_OK
    assert lib.dvattn_lse_merge(capi.DVATTN_FLOAT32, 2, 0, 128, None, None, None, None, None) == capi.DVATTN_OK
    assert lib.dvattn_lse_merge(capi.DVATTN_FLOAT32, 2, 4, 0, None, None, None, None, None) == \
        capi.DVATTN_ERR_INVALID_ARGUMENT
    assert lib.dvattn_lse_merge_packed(capi.DVATTN_FLOAT32, 2, 0, 128, None, None, None, None) == capi.DVATTN_OK
    assert lib.dvattn_lse_merge_packed(capi.DVATTN_FLOAT32, 2, 4, 128, None, None, None, None) == \
        capi.DVATTN_ERR_INVALID_ARGUMENT


# the schemas of the reference extension (src/binding.cu:410-420)
REFERENCE_SCHEMAS = {
    "dvattn_sdpa": "libdvatt::dvattn_sdpa(Tensor(a!) output, float scale, Tensor locations, Tensor queries, "
                   "Tensor fragment_lengths, Tensor[] key_fragments, Tensor[] value_fragments) -> ()",
    "dvattn_paged_sdpa": "libdvatt::dvattn_paged_sdpa(Tensor(a!) output, float scale, Tensor locations, "
                         "Tensor queries, Tensor cosines, Tensor sines, Tensor fragment_lengths, Tensor k_cache, "
                         "Tensor v_cache, Tensor block_tables) -> ()",
    "dvattn_rope": "libdvatt::dvattn_rope(Tensor(a!) output, Tensor queries, Tensor cosines, Tensor sines) -> ()",
    "dvattn_fused": "libdvatt::dvattn_fused(Tensor(a!) output, Tensor(b!) rq, float scale, Tensor locations, "
                    "Tensor queries, Tensor fragment_lengths, Tensor[] key_fragments, Tensor[] value_fragments, "
                    "Tensor cosines, Tensor sines) -> ()",
    "dvattn_varlen_rope": "libdvatt::dvattn_varlen_rope(Tensor(a!) output, Tensor queries, Tensor cosines, "
                          "Tensor sines) -> ()",
    "dvattn_varlen_paged_sdpa": "libdvatt::dvattn_varlen_paged_sdpa(Tensor(a!) output, float scale, "
                                "Tensor locations, Tensor queries, Tensor cosines, Tensor sines, "
                                "Tensor fragment_lengths, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
                                "Tensor cu_seqlens_q, Tensor cu_seqlens_k) -> ()",
}


@pytest.mark.parametrize("name", sorted(REFERENCE_SCHEMAS))
def test_reference_schemas_registered(name):
    op = getattr(torch.ops.libdvatt, name)
    assert str(op.default._schema) == REFERENCE_SCHEMAS[name]
    assert torch.Tag.needs_fixed_stride_order in op.default.tags


def test_unknown_dtype_raises():
    """The reference silently does nothing for an unknown dtype; this build raises."""
    out = torch.empty(1, 16, 1, 128, dtype=torch.float64)
    with pytest.raises(Exception):
        torch.ops.libdvatt.dvattn_paged_sdpa(out, 0.1, torch.zeros(1, 1, 1, dtype=torch.int32),
                                             torch.empty(1, 16, 1, 128, dtype=torch.float64),
                                             torch.empty(1, 1, 1, 64), torch.empty(1, 1, 1, 64),
                                             torch.ones(1, dtype=torch.int32), torch.empty(1, 16, 1, 128),
                                             torch.empty(1, 16, 1, 128), torch.zeros(1, 1, dtype=torch.int32))


def test_peer_exchange_validation_without_gpu():
    lib = capi.lib()
    assert lib.dvattn_peer_region_bytes(512, 128) == 256 + 2 * ((512 * 129 * 4 + 255) // 256 * 256)
    assert lib.dvattn_peer_region_bytes(512, 6) == 0  # Ev must be a multiple of 4
    assert lib.dvattn_peer_slot_offset(512, 128, 0) == 256
    assert lib.dvattn_peer_slot_offset(512, 128, 2) == 0
    regions = (ctypes.c_void_p * 2)(None, None)
    for world, rank, slot in ((0, 0, 0), (9, 0, 0), (2, 2, 0), (2, 0, 2)):
        assert lib.dvattn_lse_merge_peers(capi.DVATTN_BFLOAT16, world, rank, slot, 16, 128, regions, 1, None,
                                          None) == capi.DVATTN_ERR_INVALID_ARGUMENT
    # null or misaligned region pointers are refused before any launch
    assert lib.dvattn_lse_merge_peers(capi.DVATTN_BFLOAT16, 2, 0, 0, 16, 128, regions, 1, None,
                                      None) == capi.DVATTN_ERR_INVALID_ARGUMENT
    assert lib.dvattn_peer_region_alloc(16, None, None) == capi.DVATTN_ERR_INVALID_ARGUMENT
    assert lib.dvattn_workspace_status(None, None, None) == capi.DVATTN_ERR_INVALID_ARGUMENT
