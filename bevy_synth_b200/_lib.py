"""ctypes binding of libsparseconv.so (the C ABI in include/sparseconv.h).

The library is built in-tree (``bevy_synth_b200/libsparseconv.so``) by
``bevy_synth_b200.build``.  There is no fallback: if the library is missing
or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsparseconv.so")

SC_OK = 0
SC_ERR_INVALID = -1
SC_ERR_CUDA = -2
SC_ERR_UNSUPPORTED = -3
SC_ERR_CAPACITY = -4
SC_ERR_RANGE = -5
SC_ERR_DEVICE = -6

DTYPE_F32 = 0
DTYPE_BF16 = 1

# Every symbol include/sparseconv.h declares (checked by tests/test_abi.py).
EXPORTED = (
    "sc_version", "sc_last_error", "sc_device_fault", "sc_kernel_rows", "sc_kernel_offsets",
    "sc_neighbor_workspace_bytes", "sc_neighbor_map", "sc_neighbor_map_query", "sc_neighbor_status",
    "sc_neighbor_map_noalloc", "sc_neighbor_schedule_scratch_bytes", "sc_neighbor_schedule",
    "sc_subm_conv_forward", "sc_conv_uses_tensor_cores", "sc_layer_norm_act", "sc_bf16_round",
    "sc_cast", "sc_subdivide_scratch_bytes", "sc_subdivide", "sc_subdivide_async", "sc_linear_forward", "sc_gather_rows", "sc_subdiv_head",
    "sc_patchify3d_scratch_bytes", "sc_patchify3d_forward", "sc_neighbor_schedule_grouped_scratch_bytes",
    "sc_neighbor_schedule_grouped", "sc_set_wait_limit_ns", "sc_neighbor_tile_sources_bytes",
    "sc_neighbor_tile_sources",
)


class SparseConvError(RuntimeError):
    """An error returned through the C ABI (the reference returns Err(String))."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class ScConvConfig(ctypes.Structure):
    _fields_ = [
        ("in_channels", ctypes.c_int64), ("out_channels", ctypes.c_int64),
        ("kernel_d", ctypes.c_int64), ("kernel_h", ctypes.c_int64), ("kernel_w", ctypes.c_int64),
        ("in_channels_per_group", ctypes.c_int64), ("out_channels_per_group", ctypes.c_int64),
        ("groups", ctypes.c_int64),
        ("axis_order", ctypes.c_int32 * 3), ("axis_sign", ctypes.c_int32 * 3),
    ]


class ScPatchify3dConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in ("in_channels", "out_channels", "frames", "height", "width",
                                              "tubelet_size", "patch_h", "patch_w")]


class ScEpilogue(ctypes.Structure):
    _fields_ = [
        ("d_residual", ctypes.c_void_p),
        ("d_residual_offset", ctypes.c_void_p),
        ("residual_repeat", ctypes.c_int32),
        ("layer_norm", ctypes.c_int32),
        ("ln_width", ctypes.c_int32),
        ("ln_eps", ctypes.c_float),
        ("d_ln_gamma", ctypes.c_void_p),
        ("d_ln_beta", ctypes.c_void_p),
        ("silu", ctypes.c_int32),
        ("d_out2", ctypes.c_void_p),
        ("d_out_row_map", ctypes.c_void_p),
        ("out_row_map_cols", ctypes.c_int32),
        ("d_row_order", ctypes.c_void_p),
        ("d_neighbor_rows_ordered", ctypes.c_void_p),
        ("d_tile_sources", ctypes.c_void_p),
        ("tile_sources_max", ctypes.c_int32),
    ]


_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SIGS = {
    "sc_version": ([], ctypes.c_int),
    "sc_last_error": ([ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "sc_device_fault": ([ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
    "sc_set_wait_limit_ns": ([ctypes.c_uint64], ctypes.c_int),
    "sc_neighbor_tile_sources_bytes": ([_I64, _I64, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "sc_neighbor_tile_sources": ([_P, _P, _I64, _I64, _P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32), _P],
                                 ctypes.c_int),
    "sc_kernel_rows": ([_P, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "sc_kernel_offsets": ([_P, _P], ctypes.c_int),
    "sc_neighbor_workspace_bytes": ([_I64, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "sc_neighbor_map": ([_P, _P, _I64, _P, ctypes.c_size_t, _P, _P], ctypes.c_int),
    "sc_neighbor_map_query": ([_P, _P, _I64, _P, _I64, _P, ctypes.c_size_t, _P, _P], ctypes.c_int),
    "sc_neighbor_status": ([_P, ctypes.POINTER(ctypes.c_int32), _P], ctypes.c_int),
    "sc_neighbor_map_noalloc": ([_P, _P, _I64, _P, _P], ctypes.c_int),
    "sc_neighbor_schedule_scratch_bytes": ([_I64, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "sc_neighbor_schedule": ([_P, _P, _I64, _P, ctypes.c_size_t, _P, _P, _P], ctypes.c_int),
    "sc_subm_conv_forward": ([_P, ctypes.c_int, _P, _I64, _P, _I64, _P, _P, _P, _P, _P], ctypes.c_int),
    "sc_conv_uses_tensor_cores": ([_P, ctypes.c_int, ctypes.POINTER(ctypes.c_int32)], ctypes.c_int),
    "sc_layer_norm_act": ([ctypes.c_int, _P, _I64, _I64, _P, _P, ctypes.c_float, ctypes.c_int32,
                           ctypes.c_int32, _P, _P], ctypes.c_int),
    "sc_bf16_round": ([_P, _I64, _P, _P], ctypes.c_int),
    "sc_cast": ([ctypes.c_int, ctypes.c_int, _P, _I64, _P, _P], ctypes.c_int),
    "sc_gather_rows": ([_P, _I64, _I64, _P, _I64, _P, _P], ctypes.c_int),
    "sc_subdiv_head": ([ctypes.c_int, _P, _I64, _I64, _P, _P, ctypes.c_float, _P, ctypes.c_int, _P, _P, _P],
                       ctypes.c_int),
    "sc_patchify3d_scratch_bytes": ([_P, _I64, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "sc_patchify3d_forward": ([_P, ctypes.c_int, _P, _I64, _P, _I64, _P, _P, _P, ctypes.c_size_t, _P, _P],
                              ctypes.c_int),
    "sc_neighbor_schedule_grouped_scratch_bytes": ([_I64, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "sc_neighbor_schedule_grouped": ([_P, _P, _I64, _P, _P, ctypes.c_size_t, _P, _P, _P], ctypes.c_int),
    "sc_subdivide_scratch_bytes": ([_I64, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "sc_subdivide": ([_P, _P, _I64, _I64, _P, _P, _P, _P, ctypes.POINTER(ctypes.c_int64), _P], ctypes.c_int),
    "sc_subdivide_async": ([_P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "sc_linear_forward": ([ctypes.c_int, _P, _I64, _I64, _P, _I64, _P, _P, ctypes.c_int32, _P, _P], ctypes.c_int),
}


def lib() -> ctypes.CDLL:
    """Load libsparseconv.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SparseConvError(SC_ERR_UNSUPPORTED,
                                  f"libsparseconv.so not built at {LIB_PATH}; run bevy_synth_b200.build")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().sc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != SC_OK:
        raise SparseConvError(rc, last_error())


FAULT_WAIT_TIMEOUT = 1 << 0
FAULT_BAD_NEIGHBOR = 1 << 1
FAULT_TMEM = 1 << 2


def set_wait_limit_ns(ns: int) -> None:
    """Time limit of the kernels' bounded waits on the current device (0 = the 2 s default)."""
    check(lib().sc_set_wait_limit_ns(int(ns)))


def device_fault() -> int:
    v = ctypes.c_uint32(0)
    check(lib().sc_device_fault(ctypes.byref(v)))
    return v.value
