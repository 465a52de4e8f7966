"""ctypes binding of libegnn_b200.so (the C ABI in include/egnn_b200.h).

The library is loaded from the package directory.  There is no fallback: if
the shared object is missing or fails to load, every call raises
``NativeLibraryError``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

# The in-tree build; PYMOLECULAR_B200_LIB points at another build of the same
# library (same C ABI) instead.
LIB_PATH = Path(os.environ.get("PYMOLECULAR_B200_LIB") or Path(__file__).resolve().parent / "libegnn_b200.so")

EGNN_OK = 0
EGNN_ERR_INVALID_ARG = 1
EGNN_ERR_INDEX = 2
EGNN_ERR_CUDA = 3
EGNN_ERR_UNSUPPORTED = 4
EGNN_ERR_WORKSPACE = 5

FLAG_RESIDUAL = 1
FLAG_ATTENTION = 2
FLAG_NORMALIZE = 4
FLAG_TANH = 8
FLAG_COORDS_SUM = 16

PREC_FP32 = 0
PREC_BF16 = 1

WS_FWD = 0
WS_BWD = 1

LINEAR_BWD_STATIC_SCRATCH_BYTES = 4 << 20   # EGNN_LINEAR_BWD_STATIC_SCRATCH_BYTES

VP = C.c_void_p


class NativeLibraryError(RuntimeError):
    """libegnn_b200.so is missing or could not be loaded."""


class EgnnError(RuntimeError):
    """A C ABI call returned a non-zero egnn_status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class LayerDesc(C.Structure):
    _fields_ = [("n_nodes", C.c_int64), ("n_edges", C.c_int64), ("hidden", C.c_int32),
                ("edge_attr_dim", C.c_int32), ("flags", C.c_int32), ("precision", C.c_int32),
                ("in_dim", C.c_int32), ("out_dim", C.c_int32)]   # 0: hidden


class Graph(C.Structure):
    _fields_ = [("row_ptr", VP), ("col_idx", VP), ("row_idx", VP), ("edge_id", VP),
                ("src_ptr", VP), ("src_edge", VP)]


_PARAM_FIELDS = ["edge_w1", "edge_b1", "edge_w2", "edge_b2", "node_w1", "node_b1", "node_w2",
                 "node_b2", "coord_w1", "coord_b1", "coord_w2", "att_w", "att_b"]


GRAPH_RADIUS = 0
GRAPH_KNN = 1


class SpatialDesc(C.Structure):
    _fields_ = [("n_nodes", C.c_int64), ("n_graphs", C.c_int64), ("x", VP), ("graph_ptr", VP),
                ("mode", C.c_int32), ("max_nbrs", C.c_int32), ("cutoff", C.c_float)]


class LayerParams(C.Structure):
    _fields_ = [(f, VP) for f in _PARAM_FIELDS]


class LayerGrads(C.Structure):
    _fields_ = [(f, VP) for f in _PARAM_FIELDS]


# name -> (restype, argtypes)
_SIGNATURES = {
    "egnn_csr_workspace_size": (C.c_size_t, [C.c_int64, C.c_int64]),
    "egnn_csr_build": (C.c_int, [C.c_int64, C.c_int64, VP, VP, VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "egnn_csr_build_async": (C.c_int, [C.c_int64, C.c_int64, VP, VP, VP, VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "egnn_csr_transpose": (C.c_int, [C.c_int64, C.c_int64, VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "egnn_graph_check": (C.c_int, [C.c_int64, C.c_int64, C.POINTER(Graph), VP, C.c_size_t, VP]),
    "egnn_fc_graph_workspace_size": (C.c_size_t, [C.c_int64]),
    "egnn_fc_graph": (C.c_int, [C.c_int64, C.c_int64, VP, C.c_int64, VP, VP, VP, VP, C.c_size_t, VP]),
    "egnn_spatial_workspace_size": (C.c_size_t, [C.c_int64]),
    "egnn_spatial_count": (C.c_int, [C.POINTER(SpatialDesc), VP, VP, C.c_size_t, VP]),
    "egnn_spatial_fill": (C.c_int, [C.POINTER(SpatialDesc), VP, VP, VP, VP, C.c_size_t, VP]),
    "egnn_morton_workspace_size": (C.c_size_t, [C.c_int64]),
    "egnn_morton_order": (C.c_int, [C.c_int64, VP, C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_int,
                                    VP, VP, VP, C.c_size_t, VP]),
    "egnn_saved_size": (C.c_size_t, [C.POINTER(LayerDesc)]),
    "egnn_workspace_size": (C.c_size_t, [C.POINTER(LayerDesc), C.c_int, C.c_int]),
    "egnn_layer_fwd": (C.c_int, [C.POINTER(LayerDesc), C.POINTER(Graph), C.POINTER(LayerParams),
                                 VP, VP, VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "egnn_layer_bwd": (C.c_int, [C.POINTER(LayerDesc), C.POINTER(Graph), C.POINTER(LayerParams),
                                 VP, VP, VP, VP, VP, VP, VP, VP, C.POINTER(LayerGrads), VP,
                                 C.c_size_t, VP]),
    "egnn_graph_mse_workspace_size": (C.c_size_t, [C.c_int64]),
    "egnn_graph_mse_fwd": (C.c_int, [C.c_int64, C.c_int64, VP, C.c_int64, VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "egnn_graph_mse_bwd": (C.c_int, [C.c_int64, C.c_int64, VP, VP, VP, VP, VP, C.c_int64, VP]),
    "egnn_linear_fwd": (C.c_int, [C.c_int64, C.c_int32, C.c_int32, VP, VP, VP, VP, VP]),
    "egnn_linear_workspace_size": (C.c_size_t, [C.c_int64, C.c_int32, C.c_int32]),
    "egnn_linear_bwd": (C.c_int, [C.c_int64, C.c_int32, C.c_int32, VP, VP, VP, VP, VP, VP, VP,
                                  C.c_size_t, VP]),
    "egnn_linear_bwd_static": (C.c_int, [C.c_int64, C.c_int32, C.c_int32, VP, VP, VP, VP, VP, VP, VP]),
    "egnn_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
    "egnn_version": (C.c_char_p, []),
    "egnn_device_status": (C.c_int, [VP]),
    "egnn_launch_count": (C.c_uint64, []),
    "egnn_launch_count_reset": (None, []),
    "egnn_kernel_timing": (None, [C.c_int]),
    "egnn_kernel_time": (C.c_int, [C.c_char_p, C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (loads it on first use)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeLibraryError(
                    f"{LIB_PATH} not found; build it with `python -m pymolecular_b200.build`")
            try:
                handle = C.CDLL(str(LIB_PATH))
            except OSError as exc:  # pragma: no cover - environment specific
                raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def kernel_time(name: str):
    """(total ms, launches) of a timed kernel since egnn_kernel_timing(1)."""
    ms = C.c_double(0.0)
    n = C.c_int64(0)
    check(lib().egnn_kernel_time(name.encode(), C.byref(ms), C.byref(n)), "egnn_kernel_time")
    return ms.value, n.value


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().egnn_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status != EGNN_OK:
        raise EgnnError(status, f"{what}: {last_error()}" if what else last_error())


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
