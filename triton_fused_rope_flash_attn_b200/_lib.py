"""ctypes binding of the C ABI declared in ``include/frsa.h``.

The library is built in-tree (``_lib/libfrsa.so``). There is no fallback: if it
is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH

FRSA_DTYPE_BF16 = 0
FRSA_DTYPE_F16 = 1
FRSA_DTYPE_F32 = 2
FRSA_FLAG_NO_ROPE = 1

EXPORTED_SYMBOLS = (
    "frsa_fwd",
    "frsa_qkv_rope",
    "frsa_qkv_rope_bwd",
    "frsa_convert_in",
    "frsa_convert_out",
    "frsa_bwd",
    "frsa_bwd_workspace_bytes",
    "frsa_strerror",
    "frsa_query_status",
    "frsa_abi_version",
    "frsa_last_error_detail",
    "frsa_bwd_noalloc",
    "frsa_bwd_noalloc_max_elements",
)


class FrsaAttnArgs(ctypes.Structure):
    """Mirror of ``frsa_attn_args`` (include/frsa.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("d_o", ctypes.c_void_p),
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("delta", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("cosp", ctypes.c_void_p),
        ("sinp", ctypes.c_void_p),
        ("B", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("D", ctypes.c_int64),
        ("n_pos", ctypes.c_int64),
        ("has_cls", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32),
        ("compute_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q_strides", ctypes.c_int64 * 3),
        ("k_strides", ctypes.c_int64 * 3),
        ("v_strides", ctypes.c_int64 * 3),
        ("flags", ctypes.c_int32),
    ]


class FrsaQkvArgs(ctypes.Structure):
    """Mirror of ``frsa_qkv_args`` (include/frsa.h)."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("w", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("cosp", ctypes.c_void_p),
        ("sinp", ctypes.c_void_p),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("B", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("C", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("n_pos", ctypes.c_int64),
        ("has_cls", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class FrsaQkvBwdArgs(ctypes.Structure):
    """Mirror of ``frsa_qkv_bwd_args`` (include/frsa.h)."""

    _fields_ = [
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("cosp", ctypes.c_void_p),
        ("sinp", ctypes.c_void_p),
        ("dqkv", ctypes.c_void_p),
        ("B", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("C", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("n_pos", ctypes.c_int64),
        ("has_cls", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class FrsaConvertArgs(ctypes.Structure):
    """Mirror of ``frsa_convert_args`` (include/frsa.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("q_out", ctypes.c_void_p),
        ("k_out", ctypes.c_void_p),
        ("v_out", ctypes.c_void_p),
        ("cosp", ctypes.c_void_p),
        ("sinp", ctypes.c_void_p),
        ("B", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("D", ctypes.c_int64),
        ("n_pos", ctypes.c_int64),
        ("has_cls", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class FrsaError(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, code: int, where: str):
        self.code = code
        detail = load().frsa_last_error_detail().decode() if code == 6 else ""
        super().__init__(f"{where}: {strerror(code)} (code {code})" +
                         (f" [{detail}]" if detail else ""))


_LIB = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the C-ABI library."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(
            f"libfrsa.so not found at {p}; build it with "
            "`python -m triton_fused_rope_flash_attn_b200.build`")
    lib = ctypes.CDLL(p)
    lib.frsa_fwd.argtypes = [ctypes.POINTER(FrsaAttnArgs), ctypes.c_void_p]
    lib.frsa_fwd.restype = ctypes.c_int
    lib.frsa_bwd.argtypes = [ctypes.POINTER(FrsaAttnArgs), ctypes.c_void_p]
    lib.frsa_bwd.restype = ctypes.c_int
    lib.frsa_bwd_workspace_bytes.argtypes = [ctypes.POINTER(FrsaAttnArgs)]
    lib.frsa_bwd_workspace_bytes.restype = ctypes.c_size_t
    lib.frsa_strerror.argtypes = [ctypes.c_int]
    lib.frsa_strerror.restype = ctypes.c_char_p
    lib.frsa_query_status.argtypes = []
    lib.frsa_query_status.restype = ctypes.c_int
    lib.frsa_qkv_rope.argtypes = [ctypes.POINTER(FrsaQkvArgs), ctypes.c_void_p]
    lib.frsa_qkv_rope.restype = ctypes.c_int
    lib.frsa_qkv_rope_bwd.argtypes = [ctypes.POINTER(FrsaQkvBwdArgs), ctypes.c_void_p]
    lib.frsa_qkv_rope_bwd.restype = ctypes.c_int
    for name in ("frsa_convert_in", "frsa_convert_out"):
        getattr(lib, name).argtypes = [ctypes.POINTER(FrsaConvertArgs), ctypes.c_void_p]
        getattr(lib, name).restype = ctypes.c_int
    lib.frsa_bwd_noalloc.argtypes = [ctypes.POINTER(FrsaAttnArgs), ctypes.c_void_p]
    lib.frsa_bwd_noalloc.restype = ctypes.c_int
    lib.frsa_bwd_noalloc_max_elements.argtypes = []
    lib.frsa_bwd_noalloc_max_elements.restype = ctypes.c_size_t
    lib.frsa_last_error_detail.argtypes = []
    lib.frsa_last_error_detail.restype = ctypes.c_char_p
    lib.frsa_abi_version.argtypes = []
    lib.frsa_abi_version.restype = ctypes.c_int
    if path is None:
        _LIB = lib
    return lib


def strerror(code: int) -> str:
    return load().frsa_strerror(int(code)).decode()


def check(code: int, where: str) -> None:
    if code != 0:
        raise FrsaError(code, where)
