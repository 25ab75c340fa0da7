"""ctypes binding of libvqb200.so (the C ABI declared in include/vqb.h).

The shared library is the product: this module only loads it, mirrors the C
structs and turns a non-OK `vqb_status` into the exception class the
reference raises for the same condition (ValueError for shape/format errors,
NotImplementedError for unsupported geometry, RuntimeError for a sharded
codebook or a CUDA failure; vq_switch.py:3106-3128, :5285-5296).  There is no
CPU fallback: if the library cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import threading

PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG / "libvqb200.so"

VQB_OK = 0
VQB_BAD_SHAPE = 1
VQB_BAD_WPR = 2
VQB_UNSUPPORTED_GEOMETRY = 3
VQB_CODEBOOK_SHARDED = 4
VQB_CUDA_ERROR = 5
VQB_TIMEOUT = 6
VQB_BAD_ROUTING = 7
VQB_WORKSPACE_TOO_SMALL = 8
VQB_BAD_ALIGNMENT = 9
VQB_NULL_POINTER = 10

VQB_F16, VQB_BF16, VQB_F32 = 0, 1, 2
PATH_AUTO, PATH_DECODE, PATH_PREFILL = 0, 1, 2


class LinearDesc(ctypes.Structure):
    _fields_ = [
        ("num_experts", ctypes.c_int32),
        ("out_features", ctypes.c_int32),
        ("in_features", ctypes.c_int32),
        ("dim", ctypes.c_int32),
        ("num_codes", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("pack_bits", ctypes.c_int32),
        ("code_bytes", ctypes.c_int32),
        ("expected_num_codes", ctypes.c_int32),
        ("codes_last_dim", ctypes.c_int32),
        ("codes", ctypes.c_void_p),
        ("codebook", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("row_table", ctypes.c_void_p),
        ("num_rows", ctypes.c_int32),
        ("codebook_halves", ctypes.c_void_p),
    ]


class MoeBlockDesc(ctypes.Structure):
    _fields_ = [("gate", LinearDesc), ("up", LinearDesc), ("down", LinearDesc), ("top_k", ctypes.c_int32)]


class DenseMlpDesc(ctypes.Structure):
    _fields_ = [("gate", LinearDesc), ("up", LinearDesc), ("down", LinearDesc)]


class MoeBlockOptions(ctypes.Structure):
    _fields_ = [("wait_limit_us", ctypes.c_int32), ("stall_cta", ctypes.c_int32)]


class Options(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_int32),
        ("k_split", ctypes.c_int32),
        ("max_fused_pairs", ctypes.c_int32),
        ("decode_variant", ctypes.c_int32),
        ("stage_codebook", ctypes.c_int32),
        ("pairs_per_chunk", ctypes.c_int32),
        ("reuse", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class EpLayout(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("world", "rank", "tokens", "top_k", "hidden", "experts_per_rank")]


class EpOptions(ctypes.Structure):
    _fields_ = [("phases", ctypes.c_int32), ("wait_limit_us", ctypes.c_int32)]


VQB_EP_MAX_WORLD = 8
VQB_EP_STATUS_OFFSET = 272
VQB_EP_IPC_HANDLE_BYTES = 64


class VQBError(RuntimeError):
    """A non-OK status that maps to no narrower Python exception."""


_lock = threading.Lock()
_lib = None


def _bind(L):
    P, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    L.vqb_version.restype = ctypes.c_char_p
    L.vqb_status_string.restype = ctypes.c_char_p
    L.vqb_status_string.argtypes = [i32]
    L.vqb_unpack.restype = i32
    L.vqb_unpack.argtypes = [P, i64, i64, i32, i32, P, P]
    L.vqb_switch_workspace_size.restype = sz
    L.vqb_switch_workspace_size.argtypes = [P, i32, i32, P]
    L.vqb_switch_forward.restype = i32
    L.vqb_switch_forward.argtypes = [P, P, i32, i32, P, i32, P, i32, P, sz, P, P]
    L.vqb_dense_workspace_size.restype = sz
    L.vqb_dense_workspace_size.argtypes = [P, i64, P]
    L.vqb_dense_forward.restype = i32
    L.vqb_dense_forward.argtypes = [P, P, i32, i64, P, i32, P, sz, P, P]
    L.vqb_switch_forward_static.restype = i32
    L.vqb_switch_forward_static.argtypes = [P, P, i32, i32, P, i32, P, i32, P, P]
    L.vqb_swiglu.restype = i32
    L.vqb_swiglu.argtypes = [P, P, P, i64, i32, P]
    L.vqb_moe_combine.restype = i32
    L.vqb_moe_combine.argtypes = [P, P, P, i32, i32, i32, i32, P]
    L.vqb_launch_count.restype = ctypes.c_uint64
    L.vqb_launch_count.argtypes = []
    L.vqb_time_next_kernel.restype = i32
    L.vqb_time_next_kernel.argtypes = [P, P]
    L.vqb_switch_path.restype = i32
    L.vqb_switch_path.argtypes = [P, i32, i32, P]
    L.vqb_moe_combine_partial.restype = i32
    L.vqb_moe_combine_partial.argtypes = [P, P, P, P, i32, i32, i32, i32, P]
    L.vqb_moe_route.restype = i32
    L.vqb_moe_route.argtypes = [P, i32, i32, i32, P, P, P]
    L.vqb_codebook_halves.restype = i32
    L.vqb_codebook_halves.argtypes = [P, i32, P, P]
    L.vqb_moe_block_supported.restype = i32
    L.vqb_moe_block_supported.argtypes = [P, i32, i32]
    L.vqb_moe_block_workspace_size.restype = sz
    L.vqb_moe_block_workspace_size.argtypes = [P, i32]
    L.vqb_moe_block_forward.restype = i32
    L.vqb_moe_block_forward.argtypes = [P, P, P, i32, i32, P, P, P, P, sz, P, P]
    L.vqb_dense_mlp_supported.restype = i32
    L.vqb_dense_mlp_supported.argtypes = [P, i32, i32]
    L.vqb_dense_mlp_workspace_size.restype = sz
    L.vqb_dense_mlp_workspace_size.argtypes = [P, i32]
    L.vqb_dense_mlp_forward.restype = i32
    L.vqb_dense_mlp_forward.argtypes = [P, P, i32, i32, P, P, sz, P, P]
    L.vqb_ep_region_bytes.restype = sz
    L.vqb_ep_region_bytes.argtypes = [P, P]
    L.vqb_ep_region_alloc.restype = i32
    L.vqb_ep_region_alloc.argtypes = [P, P]
    L.vqb_ep_region_free.restype = i32
    L.vqb_ep_region_free.argtypes = [P]
    L.vqb_ep_ipc_handle.restype = i32
    L.vqb_ep_ipc_handle.argtypes = [P, P]
    L.vqb_ep_ipc_open.restype = i32
    L.vqb_ep_ipc_open.argtypes = [P, P]
    L.vqb_ep_ipc_close.restype = i32
    L.vqb_ep_ipc_close.argtypes = [P]
    L.vqb_ep_dispatch.restype = i32
    L.vqb_ep_dispatch.argtypes = [P, P, P, i32, i32, P, P, P, P]
    L.vqb_ep_combine.restype = i32
    L.vqb_ep_combine.argtypes = [P, P, P, i32, P, P]
    L.vqb_ep_reduce.restype = i32
    L.vqb_ep_reduce.argtypes = [P, P, P, i32, i32, P]
    return L


def lib():
    """Load (building first if the toolchain is here and the .so is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists() or os.environ.get("VQB_REBUILD") == "1":
                from . import build as _build
                _build.build()
            try:
                _lib = _bind(ctypes.CDLL(str(LIB_PATH)))
            except OSError as e:  # no silent fallback: the native path is the product
                raise RuntimeError(f"libvqb200.so could not be loaded from {LIB_PATH}: {e}") from e
    return _lib


def status_string(st: int) -> str:
    return lib().vqb_status_string(int(st)).decode()


def check(st: int, what: str = "") -> None:
    if st == VQB_OK:
        return
    msg = f"{what}: {status_string(st)} (vqb_status {st})" if what else status_string(st)
    if st in (VQB_BAD_SHAPE, VQB_BAD_WPR, VQB_BAD_ALIGNMENT, VQB_NULL_POINTER,
              VQB_WORKSPACE_TOO_SMALL, VQB_BAD_ROUTING):
        raise ValueError(msg)
    if st == VQB_UNSUPPORTED_GEOMETRY:
        raise NotImplementedError(msg)
    raise VQBError(msg)


def version() -> str:
    return lib().vqb_version().decode()


def exported_symbols():
    """Names of every function include/vqb.h declares (for the load test)."""
    return ["vqb_version", "vqb_status_string", "vqb_unpack", "vqb_switch_workspace_size",
            "vqb_switch_forward", "vqb_dense_workspace_size", "vqb_dense_forward", "vqb_switch_forward_static",
            "vqb_launch_count", "vqb_time_next_kernel", "vqb_swiglu", "vqb_moe_combine", "vqb_switch_path",
            "vqb_moe_combine_partial", "vqb_moe_route", "vqb_codebook_halves", "vqb_moe_block_supported",
            "vqb_moe_block_workspace_size", "vqb_moe_block_forward", "vqb_dense_mlp_supported",
            "vqb_dense_mlp_workspace_size", "vqb_dense_mlp_forward", "vqb_ep_region_bytes", "vqb_ep_region_alloc", "vqb_ep_region_free",
            "vqb_ep_ipc_handle", "vqb_ep_ipc_open", "vqb_ep_ipc_close", "vqb_ep_dispatch", "vqb_ep_combine",
            "vqb_ep_reduce"]


def launch_count() -> int:
    """Kernels libvqb200.so has launched in this process (graph replays excluded)."""
    return int(lib().vqb_launch_count())


def time_next_kernel(start_event, stop_event) -> None:
    """Record two torch.cuda.Event objects around the dominant kernel of this
    thread's next projection call (on the call's stream), then disarm."""
    check(lib().vqb_time_next_kernel(ctypes.c_void_p(start_event.cuda_event), ctypes.c_void_p(stop_event.cuda_event)),
          "vqb_time_next_kernel")


class CodebookHalves:
    """The [2][K][4] dimension halves of a d8 codebook (vqb_codebook_halves),
    built once and rebuilt only when the codebook tensor is replaced or
    modified in place (its data pointer, shape or version counter changes).
    Never built while a CUDA graph is being captured: the call then passes
    NULL and the library derives the halves inside the call."""

    def __init__(self):
        self._key = None
        self._t = None

    def pointer(self, codebook):
        import torch
        if codebook.dim() != 2 or int(codebook.shape[1]) != 8 or not codebook.is_cuda \
                or codebook.dtype != torch.float16 or not codebook.is_contiguous():
            return None
        key = (codebook.data_ptr(), tuple(codebook.shape), codebook._version, codebook.device)
        if key != self._key:
            if torch.cuda.is_current_stream_capturing():
                return None
            K = int(codebook.shape[0])
            t = torch.empty((2, K, 4), dtype=torch.float16, device=codebook.device)
            stream = ctypes.c_void_p(torch.cuda.current_stream(codebook.device).cuda_stream)
            check(lib().vqb_codebook_halves(ctypes.c_void_p(codebook.data_ptr()), K, ctypes.c_void_p(t.data_ptr()),
                                            stream), "vqb_codebook_halves")
            self._t, self._key = t, key
        return self._t.data_ptr()
