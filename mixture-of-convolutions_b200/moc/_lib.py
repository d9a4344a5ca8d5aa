"""ctypes binding of the C ABI in ``include/moc_b200.h`` (``libmoc_b200.so``).

The shared library is built in-tree by ``csrc/Makefile`` (``python -m moc.build``).
There is no fallback: if the library is missing or fails to load, every kernel
launch raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_NAME = "libmoc_b200.so"
_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), _LIB_NAME)

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
INDEX_CODES = {torch.int32: 0, torch.int64: 1}

MOC_OK = 0
MOC_ERR_CUDA = 6


class MocProblem(ctypes.Structure):
    """Mirror of ``struct moc_problem``."""

    _fields_ = [
        ("batch", ctypes.c_int64),
        ("seq_len", ctypes.c_int64),
        ("n_tokens", ctypes.c_int64),
        ("dim", ctypes.c_int64),
        ("n_bases", ctypes.c_int32),
        ("kernel_size", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32),
        ("alpha_dtype", ctypes.c_int32),
        ("basis_dtype", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("cu_seqlens", ctypes.c_void_p),
        ("cu_seqlens_dtype", ctypes.c_int32),
        ("n_seqs", ctypes.c_int64),
        ("chunk_indices", ctypes.c_void_p),
        ("chunk_indices_dtype", ctypes.c_int32),
        ("n_chunks", ctypes.c_int64),
        ("chunk_size", ctypes.c_int32),
        ("halo", ctypes.c_void_p),
        ("halo_strides", ctypes.c_int64 * 3),
    ]


class MocDecodeModule(ctypes.Structure):
    """Mirror of ``struct moc_decode_module``."""

    _fields_ = [
        ("dim", ctypes.c_int64),
        ("n_bases", ctypes.c_int32),
        ("kernel_size", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("router_act", ctypes.c_int32),
        ("weight", ctypes.c_void_p),
        ("basis", ctypes.c_void_p),
        ("x", ctypes.c_void_p),
        ("cache", ctypes.c_void_p),
        ("alpha", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
    ]


DECODE_MAX_MODULES = 4


class MocProjModule(ctypes.Structure):
    """Mirror of ``struct moc_proj_module``."""

    _fields_ = [
        ("dim", ctypes.c_int64),
        ("row_offset", ctypes.c_int64),
        ("n_bases", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("alpha", ctypes.c_void_p),
        ("basis", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
    ]


PROJ_MAX_MODULES = 4


class MocProjProblem(ctypes.Structure):
    """Mirror of ``struct moc_proj_problem``."""

    _fields_ = [
        ("batch", ctypes.c_int64),
        ("seq_len", ctypes.c_int64),
        ("in_dim", ctypes.c_int64),
        ("dim", ctypes.c_int64),
        ("n_bases", ctypes.c_int32),
        ("kernel_size", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("h", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("alpha", ctypes.c_void_p),
        ("basis", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
    ]

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t
_PROB = ctypes.POINTER(MocProblem)

# name -> (restype, argtypes); the complete exported surface of include/moc_b200.h
SIGNATURES = {
    "moc_version": (ctypes.c_char_p, []),
    "moc_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "moc_last_cuda_error": (ctypes.c_char_p, []),
    "moc_set_kernel_path": (ctypes.c_int, [ctypes.c_int]),
    "moc_launch_count": (ctypes.c_uint64, []),
    "moc_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "moc_wait_timeout_probe": (ctypes.c_int, [ctypes.c_uint32, _P]),
    "moc_cluster_wait_timeout_probe": (ctypes.c_int, [ctypes.c_uint32, _P]),
    "moc_forward": (ctypes.c_int, [_PROB, _P, _P, _P, _P, _P]),
    "moc_backward_workspace_bytes": (_SZ, [_PROB]),
    "moc_backward": (ctypes.c_int, [_PROB, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "moc_step": (
        ctypes.c_int,
        [_I64, _I64, _I32, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, ctypes.POINTER(_I64), _P, _P],
    ),
    "moc_router_forward": (ctypes.c_int, [_I64, _I64, _I32, _I32, _I32, _P, _P, _P, _P]),
    "moc_router_backward_workspace_bytes": (_SZ, [_I64, _I64, _I32, _I32]),
    "moc_router_backward": (
        ctypes.c_int,
        [_I64, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _P, _P, _P, _SZ, _P],
    ),
    "moc_router_backward_noalloc": (
        ctypes.c_int,
        [_I64, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _I32, _P, _P, _P],
    ),
    "moc_prepare_chunk_indices": (ctypes.c_int, [_P, _I32, _I64, _I32, _P, _I64, _P]),
    "moc_decode_step_multi": (ctypes.c_int, [_I32, ctypes.POINTER(MocDecodeModule), _I64, _I64, _P, _P]),
    "moc_proj_forward": (ctypes.c_int, [ctypes.POINTER(MocProjProblem), _P]),
    "moc_proj_forward_multi": (ctypes.c_int, [_I32, ctypes.POINTER(MocProjModule), _I64, _I64, _I64, _I32, _P, _P,
                                              _I64, _P]),
    "moc_proj_forward_save": (ctypes.c_int, [ctypes.POINTER(MocProjProblem), _P, _P]),
    "moc_proj_forward_multi_save": (ctypes.c_int, [_I32, ctypes.POINTER(MocProjModule), ctypes.POINTER(_P), _I64,
                                                   _I64, _I64, _I32, _P, _P, _I64, _P]),
    "moc_comm_create": (ctypes.c_int, [_I32, _I32, _I64, ctypes.POINTER(_P), _P]),
    "moc_comm_connect": (ctypes.c_int, [_P, _P]),
    "moc_comm_allreduce": (ctypes.c_int, [_P, _I32, ctypes.POINTER(_P), ctypes.POINTER(_I64), ctypes.POINTER(_I32), _P]),
    "moc_comm_destroy": (ctypes.c_int, [_P]),
    "moc_comm_set_poll_limit": (ctypes.c_int, [_P, ctypes.c_uint32]),
    "moc_comm_status": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "moc_comm_reset": (ctypes.c_int, [_P, _P]),
    "moc_comm_wait_timeout_probe": (ctypes.c_int, [ctypes.c_uint32, _P]),
}

COMM_MAX_RANKS = 8
COMM_MAX_SEGMENTS = 4
IPC_HANDLE_BYTES = 64

_lib = None
_lock = threading.Lock()


def library_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library, with every prototype declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(
                f"moc CUDA library not found at {_LIB_PATH}; build it with "
                "`python -m moc.build` (or `make -C csrc`)"
            )
        lib = ctypes.CDLL(_LIB_PATH)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc == MOC_OK:
        return
    lib = load()
    msg = lib.moc_error_string(rc).decode()
    if rc == MOC_ERR_CUDA:
        msg += f" [{lib.moc_last_cuda_error().decode()}]"
    raise RuntimeError(f"{what} failed: {msg} (code {rc})")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype for the moc kernels: {t.dtype}") from None


def index_code(t: torch.Tensor) -> int:
    try:
        return INDEX_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported index dtype: {t.dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(load().moc_launch_count())


def device_status(clear: bool = False) -> int:
    """OR of the MOC_STATUS_* bits the staging kernels recorded (synchronous read)."""
    v = ctypes.c_int(0)
    check(load().moc_device_status(ctypes.byref(v), int(clear)), "moc_device_status")
    return v.value


def set_kernel_path(path: int) -> None:
    """0 = automatic (tensor-core kernels where supported), 1 = generic CUDA-core kernels,
    2 = automatic with the warp-level convolution backward for every shape."""
    check(load().moc_set_kernel_path(path), "moc_set_kernel_path")
