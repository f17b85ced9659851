"""ctypes binding of the C ABI (include/dvattn_b200.h) of libdvattn_b200.so.

This is what a non-torch host (an engine written in C, Go, Java ...) sees: plain
structs of pointers and sizes.  The helpers below fill those structs from torch
tensors (device pointers + shapes) and call the library on the current torch stream;
tests and the benchmark use them to exercise the boundary itself rather than the
torch op layer.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

from . import CAPI_LIB

DVATTN_OK = 0
DVATTN_ERR_INVALID_ARGUMENT = 1
DVATTN_ERR_UNSUPPORTED = 2
DVATTN_ERR_WORKSPACE = 3
DVATTN_ERR_CUDA = 4

DVATTN_PHASE_ALL = 0
DVATTN_PHASE_SCHEDULE = 1
DVATTN_PHASE_ATTEND = 2
DVATTN_PHASE_MERGE = 3

DVATTN_FLOAT32 = 0
DVATTN_FLOAT16 = 1
DVATTN_BFLOAT16 = 2

_DTYPE = {torch.float32: DVATTN_FLOAT32, torch.float16: DVATTN_FLOAT16, torch.bfloat16: DVATTN_BFLOAT16}

# Every function the header declares (checked against the header by the tests).
EXPORTS = [
    "dvattn_abi_version",
    "dvattn_status_string",
    "dvattn_paged_sdpa_workspace_size",
    "dvattn_paged_sdpa",
    "dvattn_paged_sdpa_phase",
    "dvattn_varlen_paged_sdpa_phase",
    "dvattn_paged_sdpa_noalloc_max_workspace",
    "dvattn_paged_sdpa_noalloc",
    "dvattn_workspace_status",
    "dvattn_varlen_paged_sdpa_workspace_size",
    "dvattn_varlen_paged_sdpa",
    "dvattn_rope",
    "dvattn_varlen_rope",
    "dvattn_lse_merge",
    "dvattn_lse_merge_packed",
    "dvattn_peer_region_bytes",
    "dvattn_peer_slot_offset",
    "dvattn_peer_region_alloc",
    "dvattn_peer_region_open",
    "dvattn_peer_region_close",
    "dvattn_peer_region_free",
    "dvattn_lse_merge_peers",
    "dvattn_sdpa_workspace_size",
    "dvattn_sdpa",
    "dvattn_paged_append",
    "dvattn_build_views",
    "dvattn_paged_sdpa_rope_workspace_size",
    "dvattn_paged_sdpa_rope",
    "dvattn_varlen_paged_sdpa_rope_workspace_size",
    "dvattn_varlen_paged_sdpa_rope",
]

_vp = ctypes.c_void_p
_i = ctypes.c_int


class PagedArgs(ctypes.Structure):
    _fields_ = [("dtype", _i), ("F", _i), ("W", _i), ("Hq", _i), ("Hkv", _i), ("E", _i), ("Ev", _i), ("S", _i),
                ("R", _i), ("block_size", _i), ("max_blocks_per_seq", _i), ("num_blocks", ctypes.c_longlong),
                ("scale", ctypes.c_float), ("out", _vp), ("queries", _vp), ("cosines", _vp), ("sines", _vp),
                ("locations", _vp), ("fragment_lengths", _vp), ("k_cache", _vp), ("v_cache", _vp),
                ("block_tables", _vp), ("lse_out", _vp), ("out_f32", _vp)]


class VarlenArgs(ctypes.Structure):
    _fields_ = [("dtype", _i), ("F", _i), ("W", _i), ("Hq", _i), ("Hkv", _i), ("E", _i), ("Ev", _i), ("T", _i),
                ("R", _i), ("block_size", _i), ("max_blocks_per_seq", _i), ("num_blocks", ctypes.c_longlong),
                ("scale", ctypes.c_float), ("out", _vp), ("queries", _vp), ("cosines", _vp), ("sines", _vp),
                ("locations", _vp), ("fragment_lengths", _vp), ("k_cache", _vp), ("v_cache", _vp),
                ("block_tables", _vp), ("cu_seqlens_q", _vp), ("cu_seqlens_k", _vp), ("lse_out", _vp),
                ("out_f32", _vp)]


class SdpaArgs(ctypes.Structure):
    _fields_ = [("dtype", _i), ("F", _i), ("W", _i), ("Hq", _i), ("Hkv", _i), ("E", _i), ("Ev", _i), ("S", _i),
                ("scale", ctypes.c_float), ("out", _vp), ("queries", _vp), ("locations", _vp),
                ("fragment_lengths", _vp), ("key_fragments", ctypes.POINTER(_vp)),
                ("value_fragments", ctypes.POINTER(_vp)), ("fragment_rows", ctypes.POINTER(_i)),
                ("fragment_batch", ctypes.POINTER(_i)), ("lse_out", _vp), ("out_f32", _vp)]


class AppendArgs(ctypes.Structure):
    _fields_ = [("dtype", _i), ("W", _i), ("Hkv", _i), ("E", _i), ("Ev", _i), ("n", _i), ("R", _i),
                ("block_size", _i), ("max_blocks_per_seq", _i), ("num_blocks", ctypes.c_longlong),
                ("k_cache", _vp), ("v_cache", _vp), ("keys", _vp), ("values", _vp), ("cosines", _vp),
                ("sines", _vp), ("block_tables", _vp), ("positions", _vp), ("counts", _vp)]


class ViewsArgs(ctypes.Structure):
    _fields_ = [("F", _i), ("W", _i), ("n", _i), ("R", _i), ("rope_base", ctypes.c_float),
                ("attention_scaling", ctypes.c_float), ("round_dtype", _i), ("seg_lengths", _vp),
                ("seg_order", _vp), ("inv_freq", _vp), ("locations", _vp), ("cosines", _vp), ("sines", _vp)]


class RotaryArgs(ctypes.Structure):
    _fields_ = [("rope_base", ctypes.c_float), ("attention_scaling", ctypes.c_float), ("round_dtype", _i),
                ("inv_freq", _vp)]


_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load libdvattn_b200.so and declare the signatures (no GPU needed to load)."""
    global _lib
    if _lib is None:
        if not os.path.exists(CAPI_LIB):
            raise ImportError("libdvattn_b200.so is not built")
        L = ctypes.CDLL(CAPI_LIB)
        L.dvattn_abi_version.restype = _i
        L.dvattn_status_string.restype = ctypes.c_char_p
        L.dvattn_status_string.argtypes = [_i]
        L.dvattn_paged_sdpa_workspace_size.restype = ctypes.c_size_t
        L.dvattn_paged_sdpa_workspace_size.argtypes = [ctypes.POINTER(PagedArgs)]
        L.dvattn_paged_sdpa.restype = _i
        L.dvattn_paged_sdpa.argtypes = [ctypes.POINTER(PagedArgs), _vp, ctypes.c_size_t, _vp]
        L.dvattn_paged_sdpa_phase.restype = _i
        L.dvattn_paged_sdpa_phase.argtypes = [ctypes.POINTER(PagedArgs), _vp, ctypes.c_size_t, _i, _vp]
        L.dvattn_sdpa_workspace_size.restype = ctypes.c_size_t
        L.dvattn_sdpa_workspace_size.argtypes = [ctypes.POINTER(SdpaArgs)]
        L.dvattn_sdpa.restype = _i
        L.dvattn_sdpa.argtypes = [ctypes.POINTER(SdpaArgs), _vp, ctypes.c_size_t, _vp]
        L.dvattn_varlen_paged_sdpa_phase.restype = _i
        L.dvattn_varlen_paged_sdpa_phase.argtypes = [ctypes.POINTER(VarlenArgs), _vp, ctypes.c_size_t, _i, _vp]
        L.dvattn_paged_sdpa_noalloc_max_workspace.restype = ctypes.c_size_t
        L.dvattn_paged_sdpa_noalloc_max_workspace.argtypes = []
        L.dvattn_paged_sdpa_noalloc.restype = _i
        L.dvattn_paged_sdpa_noalloc.argtypes = [ctypes.POINTER(PagedArgs), _vp]
        L.dvattn_workspace_status.restype = _i
        L.dvattn_workspace_status.argtypes = [_vp, _vp, ctypes.POINTER(_i)]
        L.dvattn_varlen_paged_sdpa_workspace_size.restype = ctypes.c_size_t
        L.dvattn_varlen_paged_sdpa_workspace_size.argtypes = [ctypes.POINTER(VarlenArgs)]
        L.dvattn_varlen_paged_sdpa.restype = _i
        L.dvattn_varlen_paged_sdpa.argtypes = [ctypes.POINTER(VarlenArgs), _vp, ctypes.c_size_t, _vp]
        L.dvattn_rope.restype = _i
        L.dvattn_rope.argtypes = [_i] * 7 + [_vp] * 5
        L.dvattn_varlen_rope.restype = _i
        L.dvattn_varlen_rope.argtypes = [_i] * 6 + [_vp] * 5
        L.dvattn_lse_merge.restype = _i
        L.dvattn_lse_merge.argtypes = [_i, _i, ctypes.c_longlong, _i, _vp, _vp, _vp, _vp, _vp]
        L.dvattn_lse_merge_packed.restype = _i
        L.dvattn_lse_merge_packed.argtypes = [_i, _i, ctypes.c_longlong, _i, _vp, _vp, _vp, _vp]
        L.dvattn_peer_region_bytes.restype = ctypes.c_size_t
        L.dvattn_peer_region_bytes.argtypes = [ctypes.c_longlong, _i]
        L.dvattn_peer_slot_offset.restype = ctypes.c_size_t
        L.dvattn_peer_slot_offset.argtypes = [ctypes.c_longlong, _i, _i]
        L.dvattn_peer_region_alloc.restype = _i
        L.dvattn_peer_region_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]
        L.dvattn_peer_region_open.restype = _i
        L.dvattn_peer_region_open.argtypes = [_vp, ctypes.POINTER(_vp)]
        L.dvattn_peer_region_close.restype = _i
        L.dvattn_peer_region_close.argtypes = [_vp]
        L.dvattn_peer_region_free.restype = _i
        L.dvattn_peer_region_free.argtypes = [_vp]
        L.dvattn_lse_merge_peers.restype = _i
        L.dvattn_lse_merge_peers.argtypes = [_i, _i, _i, _i, ctypes.c_longlong, _i, ctypes.POINTER(_vp), _vp, _vp, _vp]
        L.dvattn_paged_append.restype = _i
        L.dvattn_paged_append.argtypes = [ctypes.POINTER(AppendArgs), _vp]
        L.dvattn_paged_sdpa_rope_workspace_size.restype = ctypes.c_size_t
        L.dvattn_paged_sdpa_rope_workspace_size.argtypes = [ctypes.POINTER(PagedArgs), ctypes.POINTER(RotaryArgs)]
        L.dvattn_paged_sdpa_rope.restype = _i
        L.dvattn_paged_sdpa_rope.argtypes = [ctypes.POINTER(PagedArgs), ctypes.POINTER(RotaryArgs), _vp, ctypes.c_size_t,
                                             _vp]
        L.dvattn_varlen_paged_sdpa_rope_workspace_size.restype = ctypes.c_size_t
        L.dvattn_varlen_paged_sdpa_rope_workspace_size.argtypes = [ctypes.POINTER(VarlenArgs), ctypes.POINTER(RotaryArgs)]
        L.dvattn_varlen_paged_sdpa_rope.restype = _i
        L.dvattn_varlen_paged_sdpa_rope.argtypes = [ctypes.POINTER(VarlenArgs), ctypes.POINTER(RotaryArgs), _vp,
                                                    ctypes.c_size_t, _vp]
        L.dvattn_build_views.restype = _i
        L.dvattn_build_views.argtypes = [ctypes.POINTER(ViewsArgs), _vp]
        _lib = L
    return _lib


class DvattnError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {lib().dvattn_status_string(status).decode()} (status {status})")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def paged_args(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
               lse=None, out_f32=None) -> PagedArgs:
    a = PagedArgs()
    a.dtype = _DTYPE.get(out.dtype, -1)
    a.F = locations.size(0)
    a.W, a.Hq, a.S, a.Ev = out.shape
    a.Hkv = k_cache.size(2)
    a.E = queries.size(3)
    a.R = cosines.size(3)
    a.block_size = k_cache.size(1)
    a.max_blocks_per_seq = block_tables.size(1)
    a.num_blocks = k_cache.size(0)
    a.scale = scale
    a.out, a.queries, a.cosines, a.sines = out.data_ptr(), queries.data_ptr(), cosines.data_ptr(), sines.data_ptr()
    a.locations, a.fragment_lengths = locations.data_ptr(), fragment_lengths.data_ptr()
    a.k_cache, a.v_cache, a.block_tables = k_cache.data_ptr(), v_cache.data_ptr(), block_tables.data_ptr()
    a.lse_out, a.out_f32 = _ptr(lse), _ptr(out_f32)
    return a


def varlen_args(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
                cu_seqlens_q, lse=None, out_f32=None) -> VarlenArgs:
    a = VarlenArgs()
    a.dtype = _DTYPE.get(out.dtype, -1)
    a.F = locations.size(0)
    a.W = cu_seqlens_q.numel() - 1
    a.T, a.Hq, a.E = queries.shape
    a.Hkv = k_cache.size(2)
    a.Ev = v_cache.size(3)
    a.R = 2 * cosines.size(2)
    a.block_size = k_cache.size(1)
    a.max_blocks_per_seq = block_tables.size(1)
    a.num_blocks = k_cache.size(0)
    a.scale = scale
    a.out, a.queries, a.cosines, a.sines = out.data_ptr(), queries.data_ptr(), cosines.data_ptr(), sines.data_ptr()
    a.locations, a.fragment_lengths = locations.data_ptr(), fragment_lengths.data_ptr()
    a.k_cache, a.v_cache, a.block_tables = k_cache.data_ptr(), v_cache.data_ptr(), block_tables.data_ptr()
    a.cu_seqlens_q = cu_seqlens_q.data_ptr()
    a.cu_seqlens_k = None
    a.lse_out, a.out_f32 = _ptr(lse), _ptr(out_f32)
    return a


class PagedCall:
    """A prepared paged-decode call through the C ABI: argument struct + workspace,
    reusable across launches (workspace reuse is stream-ordered)."""

    def __init__(self, *tensors, lse=None, out_f32=None, workspace: Optional[torch.Tensor] = None):
        self.args = paged_args(*tensors, lse=lse, out_f32=out_f32)
        self._keep = (tensors, lse, out_f32)
        n = lib().dvattn_paged_sdpa_workspace_size(ctypes.byref(self.args))
        if n == 0 and self.args.W * self.args.S > 0 and self.args.Hq > 0:
            raise DvattnError(lib().dvattn_paged_sdpa(ctypes.byref(self.args), None, 0, None), "workspace size")
        self.ws_bytes = n
        if workspace is None:
            workspace = torch.empty(max(n, 256), dtype=torch.uint8, device=tensors[0].device)
        self.workspace = workspace

    def __call__(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        st = lib().dvattn_paged_sdpa(ctypes.byref(self.args), self.workspace.data_ptr(), self.workspace.numel(),
                                     _stream(stream))
        if st != DVATTN_OK:
            raise DvattnError(st, "dvattn_paged_sdpa")

    def status(self, stream: Optional[torch.cuda.Stream] = None) -> int:
        """Error word of the last launch on this call's workspace (0 = completed)."""
        return workspace_status(self.workspace, stream)

    def phase(self, phase: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        st = lib().dvattn_paged_sdpa_phase(ctypes.byref(self.args), self.workspace.data_ptr(),
                                           self.workspace.numel(), phase, _stream(stream))
        if st != DVATTN_OK:
            raise DvattnError(st, "dvattn_paged_sdpa_phase")


class VarlenCall:
    def __init__(self, *tensors, lse=None, out_f32=None, workspace: Optional[torch.Tensor] = None):
        self.args = varlen_args(*tensors, lse=lse, out_f32=out_f32)
        self._keep = (tensors, lse, out_f32)
        n = lib().dvattn_varlen_paged_sdpa_workspace_size(ctypes.byref(self.args))
        if n == 0 and self.args.T > 0 and self.args.Hq > 0:
            raise DvattnError(lib().dvattn_varlen_paged_sdpa(ctypes.byref(self.args), None, 0, None), "workspace size")
        self.ws_bytes = n
        if workspace is None:
            workspace = torch.empty(max(n, 256), dtype=torch.uint8, device=tensors[0].device)
        self.workspace = workspace

    def __call__(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        st = lib().dvattn_varlen_paged_sdpa(ctypes.byref(self.args), self.workspace.data_ptr(),
                                            self.workspace.numel(), _stream(stream))
        if st != DVATTN_OK:
            raise DvattnError(st, "dvattn_varlen_paged_sdpa")

    def status(self, stream: Optional[torch.cuda.Stream] = None) -> int:
        """Error word of the last launch on this call's workspace (0 = completed)."""
        return workspace_status(self.workspace, stream)

    def phase(self, phase: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        st = lib().dvattn_varlen_paged_sdpa_phase(ctypes.byref(self.args), self.workspace.data_ptr(),
                                                  self.workspace.numel(), phase, _stream(stream))
        if st != DVATTN_OK:
            raise DvattnError(st, "dvattn_varlen_paged_sdpa_phase")


def workspace_status(workspace: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None) -> int:
    """dvattn_workspace_status: the error word of the last attention call on `workspace`
    (None: the last dvattn_paged_sdpa_noalloc call on the current device).  0 = completed;
    nonzero = a bounded wait in a kernel gave up and that call's outputs are invalid.
    Waits for the stream."""
    word = _i(0)
    st = lib().dvattn_workspace_status(_ptr(workspace), _stream(stream), ctypes.byref(word))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_workspace_status")
    return word.value


def paged_sdpa(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
               lse=None, out_f32=None):
    PagedCall(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
              lse=lse, out_f32=out_f32)()
    return out


def varlen_paged_sdpa(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache,
                      block_tables, cu_seqlens_q, lse=None, out_f32=None):
    VarlenCall(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
               cu_seqlens_q, lse=lse, out_f32=out_f32)()
    return out


def rope(out, queries, cosines, sines):
    F, W, Hq, S, E = out.shape
    st = lib().dvattn_rope(_DTYPE.get(out.dtype, -1), F, W, Hq, S, E, cosines.size(3), out.data_ptr(),
                           queries.data_ptr(), cosines.data_ptr(), sines.data_ptr(), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_rope")
    return out


def varlen_rope(out, queries, cosines, sines):
    F, T, H, E = out.shape
    st = lib().dvattn_varlen_rope(_DTYPE.get(out.dtype, -1), F, T, H, E, 2 * cosines.size(2), out.data_ptr(),
                                  queries.data_ptr(), cosines.data_ptr(), sines.data_ptr(), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_varlen_rope")
    return out


def lse_merge(part_out, part_lse, out, lse_out=None):
    parts = part_out.size(0)
    Ev = part_out.size(-1)
    rows = out.numel() // Ev
    st = lib().dvattn_lse_merge(_DTYPE.get(out.dtype, -1), parts, rows, Ev, part_out.data_ptr(), part_lse.data_ptr(),
                                out.data_ptr(), _ptr(lse_out), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_lse_merge")
    return out


def lse_merge_packed(packed, out, lse_out=None):
    """dvattn_lse_merge_packed: packed f32 [parts, rows * (Ev + 1)] (each part's outputs, then
    its LSEs) -> out [..., Ev]."""
    Ev = out.size(-1)
    rows = out.numel() // Ev
    parts = packed.size(0)
    if packed.dtype != torch.float32 or not packed.is_contiguous() or packed.numel() != parts * rows * (Ev + 1):
        raise ValueError("lse_merge_packed: packed must be contiguous f32 [parts, rows * (Ev + 1)]")
    st = lib().dvattn_lse_merge_packed(_DTYPE.get(out.dtype, -1), parts, rows, Ev, packed.data_ptr(), out.data_ptr(),
                                       _ptr(lse_out), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_lse_merge_packed")
    return out


class _DeviceArray:
    """__cuda_array_interface__ of device memory this library allocated, so that torch can
    view it without a copy (the view does not own the memory)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3}


def device_view(ptr: int, numel: int, device) -> torch.Tensor:
    """A float32 torch tensor over `numel` floats of device memory at `ptr` (no copy)."""
    return torch.as_tensor(_DeviceArray(ptr, (numel,)), device=device)


class PeerRegion:
    """One rank's exchange region for dvattn_lse_merge_peers (allocated by the library with
    cudaMalloc; its CUDA IPC handle lets the other ranks map it)."""

    HANDLE_BYTES = 64

    def __init__(self, rows: int, Ev: int, device):
        self.rows, self.Ev = int(rows), int(Ev)
        self.nbytes = lib().dvattn_peer_region_bytes(self.rows, self.Ev)
        if self.nbytes == 0:
            raise DvattnError(DVATTN_ERR_INVALID_ARGUMENT, "dvattn_peer_region_bytes")
        self.device = torch.device(device)
        ptr = _vp()
        self.handle = (ctypes.c_char * self.HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            st = lib().dvattn_peer_region_alloc(self.nbytes, ctypes.byref(ptr), self.handle)
        if st != DVATTN_OK:
            raise DvattnError(st, "dvattn_peer_region_alloc")
        self.ptr = ptr.value

    def slot(self, s: int):
        """(packed f32 [rows * (Ev + 1)], out_f32 view [rows * Ev], lse view [rows]) of slot s."""
        off = lib().dvattn_peer_slot_offset(self.rows, self.Ev, s)
        packed = device_view(self.ptr + off, self.rows * (self.Ev + 1), self.device)
        return packed, packed[: self.rows * self.Ev], packed[self.rows * self.Ev:]

    def status(self) -> int:
        word = _i(0)
        st = lib().dvattn_workspace_status(self.ptr, _stream(None), ctypes.byref(word))
        if st != DVATTN_OK:
            raise DvattnError(st, "dvattn_workspace_status")
        return word.value

    def free(self):
        if self.ptr:
            with torch.cuda.device(self.device):
                lib().dvattn_peer_region_free(self.ptr)
            self.ptr = None


def open_peer_region(handle: bytes, device) -> int:
    """Map another rank's region (its IPC handle) into this process; returns the pointer."""
    ptr = _vp()
    buf = (ctypes.c_char * PeerRegion.HANDLE_BYTES).from_buffer_copy(handle)
    with torch.cuda.device(torch.device(device)):
        st = lib().dvattn_peer_region_open(buf, ctypes.byref(ptr))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_peer_region_open")
    return ptr.value


def lse_merge_peers(regions, rank: int, slot: int, rows: int, Ev: int, out, lse_out=None):
    """dvattn_lse_merge_peers on the current stream; regions = device pointers of every
    rank's region as mapped in this process."""
    arr = (_vp * len(regions))(*regions)
    st = lib().dvattn_lse_merge_peers(_DTYPE.get(out.dtype, -1), len(regions), rank, slot, rows, Ev, arr,
                                      out.data_ptr(), _ptr(lse_out), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_lse_merge_peers")
    return out


class SdpaCall:
    """A prepared dvattn_sdpa call through the C ABI: queries [F,W,Hq,S,E] (rotated),
    keys/values lists of F tensors [Hkv,L,E] or [B,Hkv,L,E] (B = 1 or W); argument struct,
    fragment pointer arrays and workspace kept across launches."""

    def __init__(self, out, scale, locations, queries, fragment_lengths, keys, values, lse=None, out_f32=None,
                 workspace: Optional[torch.Tensor] = None):
        W, Hq, S, Ev = out.shape
        F, E = locations.size(0), queries.size(4)
        batched = keys[0].dim() == 4
        fo = 1 if batched else 0
        self._kp = (_vp * F)(*[k.data_ptr() for k in keys])
        self._vp = (_vp * F)(*[v.data_ptr() for v in values])
        self._rows = (_i * F)(*[k.size(fo + 1) for k in keys])
        self._batch = (_i * F)(*[(k.size(0) if batched else 1) for k in keys])
        self._keep = (out, locations, queries, fragment_lengths, keys, values, lse, out_f32)
        self.args = SdpaArgs(_DTYPE.get(out.dtype, -1), F, W, Hq, keys[0].size(fo), E, Ev, S, float(scale),
                             out.data_ptr(), queries.data_ptr(), locations.data_ptr(), fragment_lengths.data_ptr(),
                             self._kp, self._vp, self._rows, self._batch, _ptr(lse), _ptr(out_f32))
        n = lib().dvattn_sdpa_workspace_size(ctypes.byref(self.args))
        if n == 0 and W * S > 0 and Hq > 0:
            raise DvattnError(lib().dvattn_sdpa(ctypes.byref(self.args), None, 0, None), "dvattn_sdpa workspace size")
        if workspace is None:
            workspace = torch.empty(max(n, 256), dtype=torch.uint8, device=out.device)
        self.workspace = workspace

    def __call__(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        st = lib().dvattn_sdpa(ctypes.byref(self.args), self.workspace.data_ptr(), self.workspace.numel(),
                               _stream(stream))
        if st != DVATTN_OK:
            raise DvattnError(st, "dvattn_sdpa")


def sdpa(out, scale, locations, queries, fragment_lengths, keys, values, lse=None, out_f32=None):
    """dvattn_sdpa through the C ABI (one prepared call)."""
    SdpaCall(out, scale, locations, queries, fragment_lengths, keys, values, lse=lse, out_f32=out_f32)()
    return out


def paged_append(k_cache, v_cache, keys, values, cosines, sines, block_tables, positions, counts=None):
    """dvattn_paged_append through the C ABI: keys/values [W,Hkv,n,E|Ev] (keys unrotated),
    cosines/sines [W,n,R] f32, positions [W] i32, counts [W] i32 or None."""
    W, Hkv, n, E = keys.shape
    NB, BS = k_cache.shape[:2]
    a = AppendArgs(_DTYPE.get(k_cache.dtype, -1), W, Hkv, E, values.size(3), n, cosines.size(2), BS,
                   block_tables.size(1), NB, k_cache.data_ptr(), v_cache.data_ptr(), keys.data_ptr(),
                   values.data_ptr(), _ptr(cosines), _ptr(sines), block_tables.data_ptr(), positions.data_ptr(),
                   _ptr(counts))
    st = lib().dvattn_paged_append(ctypes.byref(a), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_paged_append")


def build_views(locations, cosines, sines, seg_lengths, seg_order, rope_base, attention_scaling=1.0,
                round_dtype=DVATTN_FLOAT32, inv_freq=None):
    """dvattn_build_views through the C ABI: locations [F,W,n] i32, cosines/sines [F,W,n,R] f32
    (written), seg_lengths [F] i32, seg_order [W,F] i32, inv_freq [R/2] f32 or None."""
    F, W, n = locations.shape
    a = ViewsArgs(F, W, n, cosines.size(3), float(rope_base), float(attention_scaling), round_dtype,
                  seg_lengths.data_ptr(), seg_order.data_ptr(), _ptr(inv_freq), locations.data_ptr(),
                  _ptr(cosines), _ptr(sines))
    st = lib().dvattn_build_views(ctypes.byref(a), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_build_views")


def paged_sdpa_rope(out, scale, locations, queries, fragment_lengths, k_cache, v_cache, block_tables, rotary_dim,
                    rope_base, attention_scaling=1.0, inv_freq=None, lse=None, out_f32=None):
    """dvattn_paged_sdpa_rope through the C ABI (rotation tables built on the device from
    the locations; cos/sin rounded through the output dtype)."""
    dummy = torch.empty((locations.size(0), out.size(0), out.size(2), rotary_dim), device=out.device)
    a = paged_args(out, scale, locations, queries, dummy, dummy, fragment_lengths, k_cache, v_cache, block_tables,
                   lse=lse, out_f32=out_f32)
    a.cosines = None
    a.sines = None
    r = RotaryArgs(float(rope_base), float(attention_scaling), _DTYPE.get(out.dtype, -1), _ptr(inv_freq))
    n = lib().dvattn_paged_sdpa_rope_workspace_size(ctypes.byref(a), ctypes.byref(r))
    ws = torch.empty(max(n, 256), dtype=torch.uint8, device=out.device)
    st = lib().dvattn_paged_sdpa_rope(ctypes.byref(a), ctypes.byref(r), ws.data_ptr(), ws.numel(), _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_paged_sdpa_rope")
    return out


def varlen_paged_sdpa_rope(out, scale, locations, queries, fragment_lengths, k_cache, v_cache, block_tables,
                           cu_seqlens_q, rotary_dim, rope_base, attention_scaling=1.0, inv_freq=None, lse=None,
                           out_f32=None):
    """dvattn_varlen_paged_sdpa_rope through the C ABI."""
    dummy = torch.empty((locations.size(0), queries.size(0), rotary_dim // 2), device=out.device)
    a = varlen_args(out, scale, locations, queries, dummy, dummy, fragment_lengths, k_cache, v_cache, block_tables,
                    cu_seqlens_q, lse=lse, out_f32=out_f32)
    a.cosines = None
    a.sines = None
    r = RotaryArgs(float(rope_base), float(attention_scaling), _DTYPE.get(out.dtype, -1), _ptr(inv_freq))
    n = lib().dvattn_varlen_paged_sdpa_rope_workspace_size(ctypes.byref(a), ctypes.byref(r))
    ws = torch.empty(max(n, 256), dtype=torch.uint8, device=out.device)
    st = lib().dvattn_varlen_paged_sdpa_rope(ctypes.byref(a), ctypes.byref(r), ws.data_ptr(), ws.numel(),
                                             _stream(None))
    if st != DVATTN_OK:
        raise DvattnError(st, "dvattn_varlen_paged_sdpa_rope")
    return out
