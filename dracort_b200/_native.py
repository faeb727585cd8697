"""ctypes binding of libdraco_gguf.so (the C ABI in include/draco_gguf.h).

The library is loaded lazily on first use and never replaced by a Python
implementation: if it cannot be loaded, every call raises KernelError.  Status
codes are mapped onto the reference's exception classes
(draco/exceptions.py): type/shape errors -> DracoFormatError (as
draco/format/gguf.py:284-296 raises), argument/alignment errors -> ValueError,
CUDA failures and device-side timeouts -> KernelError.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

from dracort_b200.exceptions import DracoFormatError, KernelError

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libdraco_gguf.so"

DRACO_OK = 0
DRACO_ERR_TYPE = 1
DRACO_ERR_SHAPE = 2
DRACO_ERR_ALIGN = 3
DRACO_ERR_CUDA = 4
DRACO_ERR_TIMEOUT = 5
DRACO_ERR_ARG = 6
DRACO_ERR_WORKSPACE = 7
DRACO_ERR_PEER = 8

LAYOUT_GGUF = 0
LAYOUT_GGUF_DLAST = 1
LAYOUT_TILED = 2

GEMV_MAX_PROBLEMS = 8
GEMV_MAX_BATCH = 32
GEMV_ACCUMULATE = 1  # draco_gemv_problem.flags: y += result
TP_MAX_WORLD = 8
IPC_HANDLE_BYTES = 64

#: every symbol include/draco_gguf.h declares
EXPORTED_SYMBOLS = (
    "draco_version",
    "draco_last_error_string",
    "draco_gguf_block_geometry",
    "draco_gguf_packed_bytes",
    "draco_gguf_tiled_bytes",
    "draco_gguf_dequant",
    "draco_gguf_dequant_bf16",
    "draco_gguf_repack",
    "draco_gguf_gemv_workspace_bytes",
    "draco_gguf_gemv_launch_count",
    "draco_rope_kv_append",
    "draco_attention_cached",
    "draco_attention_workspace_bytes",
    "draco_attention_decode",
    "draco_gguf_gemv_grouped",
    "draco_gguf_gemv",
    "draco_gguf_gemv_grouped_ex",
    "draco_rmsnorm",
    "draco_gguf_gemv_grouped_noalloc",
    "draco_gguf_gemv_noalloc_status",
    "draco_gguf_gemm",
    "draco_gguf_gemm_rows",
    "draco_swiglu_bf16_rows",
    "draco_swiglu_bf16",
    "draco_swiglu_f32",
    "draco_tp_buffer_alloc",
    "draco_tp_buffer_free",
    "draco_ipc_get_handle",
    "draco_ipc_open",
    "draco_ipc_close",
    "draco_gguf_gemv_grouped_tp",
    "draco_tp_finish",
)

DTYPE_F32 = 0
DTYPE_BF16 = 1
GEMM_MAX_PROBLEMS = 16


class GemvProblem(ctypes.Structure):
    """Mirror of ``draco_gemv_problem``."""

    _fields_ = [
        ("qtype", ctypes.c_int),
        ("flags", ctypes.c_int),
        ("w", ctypes.c_void_p),
        ("x", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("n_rows", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("ldx", ctypes.c_int64),
        ("ldy", ctypes.c_int64),
    ]


class GemvInput(ctypes.Structure):
    """Mirror of ``draco_gemv_input``."""

    _fields_ = [
        ("mode", ctypes.c_int),
        ("eps", ctypes.c_float),
        ("aux", ctypes.c_void_p),
        ("ldaux", ctypes.c_int64),
    ]


INPUT_PLAIN = 0
INPUT_RMSNORM = 1
INPUT_SWIGLU = 2


class GemmProblem(ctypes.Structure):
    """Mirror of ``draco_gemm_problem``."""

    _fields_ = [
        ("qtype", ctypes.c_int),
        ("ydtype", ctypes.c_int),
        ("w", ctypes.c_void_p),
        ("x", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("m", ctypes.c_int64),
        ("n_rows", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("ldx", ctypes.c_int64),
        ("ldy", ctypes.c_int64),
    ]


class TpExchange(ctypes.Structure):
    """Mirror of ``draco_tp_exchange``."""

    _fields_ = [
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("buffers", ctypes.c_void_p * 8),
        ("flags_off", ctypes.c_int64),
        ("counter_off", ctypes.c_int64),
        ("y_off", ctypes.c_int64 * 8),
        ("parity_stride", ctypes.c_int64 * 8),
    ]


_lock = threading.Lock()
_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the shared library; raise KernelError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise KernelError(
                f"libdraco_gguf.so not found at {_LIB_PATH}; build it with "
                f"`python -m dracort_b200.build` (nvcc, sm_100a)"
            )
        try:
            lib = ctypes.CDLL(str(_LIB_PATH))
        except OSError as e:  # pragma: no cover - depends on the host
            raise KernelError(f"cannot load {_LIB_PATH}: {e}") from e
        vp, i64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        lib.draco_version.restype = ctypes.c_char_p
        lib.draco_version.argtypes = []
        lib.draco_last_error_string.restype = ctypes.c_char_p
        lib.draco_last_error_string.argtypes = []
        lib.draco_gguf_block_geometry.restype = c_int
        lib.draco_gguf_block_geometry.argtypes = [c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]
        lib.draco_gguf_packed_bytes.restype = i64
        lib.draco_gguf_packed_bytes.argtypes = [c_int, i64, i64]
        lib.draco_gguf_tiled_bytes.restype = i64
        lib.draco_gguf_tiled_bytes.argtypes = [c_int, i64, i64]
        for name in ("draco_gguf_dequant", "draco_gguf_dequant_bf16"):
            f = getattr(lib, name)
            f.restype = c_int
            f.argtypes = [c_int, c_int, vp, vp, i64, i64, vp]
        lib.draco_gguf_repack.restype = c_int
        lib.draco_gguf_repack.argtypes = [c_int, c_int, vp, vp, i64, i64, vp]
        lib.draco_gguf_gemv_workspace_bytes.restype = ctypes.c_size_t
        lib.draco_gguf_gemv_workspace_bytes.argtypes = [ctypes.POINTER(GemvProblem), c_int, c_int]
        lib.draco_rope_kv_append.restype = c_int
        lib.draco_rope_kv_append.argtypes = [vp] * 9 + [c_int] * 6 + [vp]
        lib.draco_attention_cached.restype = c_int
        lib.draco_attention_cached.argtypes = [vp] * 5 + [c_int, vp] + [c_int] * 6 + [vp, ctypes.c_size_t, vp]
        lib.draco_attention_decode.restype = c_int
        lib.draco_attention_decode.argtypes = [vp] * 9 + [c_int, vp] + [c_int] * 6 + [vp, ctypes.c_size_t, vp]
        lib.draco_attention_workspace_bytes.restype = ctypes.c_size_t
        lib.draco_attention_workspace_bytes.argtypes = [c_int] * 4
        lib.draco_gguf_gemv_launch_count.restype = c_int
        lib.draco_gguf_gemv_launch_count.argtypes = [ctypes.POINTER(GemvProblem), c_int, c_int]
        lib.draco_gguf_gemv_grouped.restype = c_int
        lib.draco_gguf_gemv_grouped.argtypes = [ctypes.POINTER(GemvProblem), c_int, c_int, vp, ctypes.c_size_t, vp]
        lib.draco_gguf_gemv_grouped_ex.restype = c_int
        lib.draco_gguf_gemv_grouped_ex.argtypes = [ctypes.POINTER(GemvProblem), ctypes.POINTER(GemvInput), c_int, c_int,
                                                   vp, ctypes.c_size_t, vp]
        lib.draco_rmsnorm.restype = c_int
        lib.draco_rmsnorm.argtypes = [vp, vp, vp, i64, i64, ctypes.c_float, c_int, vp]
        lib.draco_gguf_gemv_grouped_noalloc.restype = c_int
        lib.draco_gguf_gemv_grouped_noalloc.argtypes = [ctypes.POINTER(GemvProblem), c_int, c_int, vp]
        lib.draco_gguf_gemv_noalloc_status.restype = c_int
        lib.draco_gguf_gemv_noalloc_status.argtypes = [ctypes.POINTER(c_int), vp]
        lib.draco_gguf_gemm.restype = c_int
        lib.draco_gguf_gemm.argtypes = [ctypes.POINTER(GemmProblem), c_int, vp, vp]
        lib.draco_gguf_gemm_rows.restype = c_int
        lib.draco_gguf_gemm_rows.argtypes = [ctypes.POINTER(GemmProblem), c_int, vp, vp, vp]
        lib.draco_swiglu_bf16_rows.restype = c_int
        lib.draco_swiglu_bf16_rows.argtypes = [vp, vp, vp, c_int, i64, i64, vp, vp]
        lib.draco_swiglu_bf16.restype = c_int
        lib.draco_swiglu_bf16.argtypes = [vp, vp, vp, i64, vp]
        lib.draco_swiglu_f32.restype = c_int
        lib.draco_swiglu_f32.argtypes = [vp, vp, vp, i64, vp]
        lib.draco_tp_buffer_alloc.restype = c_int
        lib.draco_tp_buffer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        lib.draco_tp_buffer_free.restype = c_int
        lib.draco_tp_buffer_free.argtypes = [vp]
        lib.draco_ipc_get_handle.restype = c_int
        lib.draco_ipc_get_handle.argtypes = [vp, vp]
        lib.draco_ipc_open.restype = c_int
        lib.draco_ipc_open.argtypes = [vp, ctypes.POINTER(vp)]
        lib.draco_ipc_close.restype = c_int
        lib.draco_ipc_close.argtypes = [vp]
        lib.draco_gguf_gemv_grouped_tp.restype = c_int
        lib.draco_gguf_gemv_grouped_tp.argtypes = [ctypes.POINTER(GemvProblem), c_int, c_int,
                                                   ctypes.POINTER(TpExchange), vp, ctypes.c_size_t, vp]
        lib.draco_tp_finish.restype = c_int
        lib.draco_tp_finish.argtypes = [ctypes.POINTER(TpExchange), c_int, i64, i64, c_int, vp, i64, i64, c_int,
                                        vp, vp, vp]
        lib.draco_gguf_gemv.restype = c_int
        lib.draco_gguf_gemv.argtypes = [c_int, vp, vp, vp, vp, c_int, i64, i64, vp, ctypes.c_size_t, vp]
        _lib = lib
        return lib


def last_error() -> str:
    return load().draco_last_error_string().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    """Raise the reference-style exception for a non-zero status."""
    if rc == DRACO_OK:
        return
    msg = last_error() or what
    if rc in (DRACO_ERR_TYPE, DRACO_ERR_SHAPE):
        raise DracoFormatError(msg)
    if rc in (DRACO_ERR_ALIGN, DRACO_ERR_ARG, DRACO_ERR_WORKSPACE):
        raise ValueError(msg)
    raise KernelError(f"{msg} (status {rc})")


def version() -> str:
    return load().draco_version().decode()
