"""ctypes binding of the C ABI in ``include/dbk.h`` (``_lib/libdbk.so``).

The library is built in-tree by :mod:`decodebench_b200.build_native`. Loading
fails loudly: there is no CPU or PyTorch fallback for the fused kernels.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libdbk.so"

DBK_F16, DBK_BF16 = 0, 1
DBK_ESHAPE = -2
DBK_OP_RMSNORM_GEMV, DBK_OP_GATEUP_SWIGLU, DBK_OP_GEMV = 0, 1, 2

# Every symbol include/dbk.h declares: name -> (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_I64 = ctypes.c_int64
SIGNATURES = {
    "dbk_abi_version": (_I, []),
    "dbk_status_string": (ctypes.c_char_p, [_I]),
    "dbk_take_device_error": (_I, []),
    "dbk_set_spin_limit": (_I, [ctypes.c_uint32]),
    "dbk_test_bounded_wait": (_I, [_I, _P]),
    "dbk_workspace_bytes": (_SZ, [_I, _I64, _I64, _I64]),
    "dbk_flashdecode_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "dbk_rmsnorm_gemv": (_I, [_P, _P, _P, _P, _I, _I, _I, _F, _I, _P, _SZ, _P]),
    "dbk_gateup_swiglu": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P, _SZ, _P]),
    "dbk_gemv": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P]),
    "dbk_mlp_block": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P, _SZ, _P]),
    "dbk_mlp_block_workspace_bytes": (_SZ, []),
    "dbk_oproj_mlp_block": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I,
                                 _P, _SZ, _P]),
    "dbk_flashdecode": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I,
                             _P, _SZ, _P]),
    "dbk_flashdecode_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I,
                                     _P]),
    "dbk_comm_buffer_bytes": (_SZ, [_SZ, _I]),
    "dbk_comm_alloc": (_I, [_SZ, _I, ctypes.POINTER(_P), _P]),
    "dbk_comm_open": (_I, [_I, _I, _P, _P, ctypes.POINTER(_P)]),
    "dbk_comm_close": (_I, [_P]),
    "dbk_comm_free": (_I, [_P]),
    "dbk_allgather": (_I, [_P, _P, _P, _I, _SZ, _SZ, _SZ, _SZ, _P]),
    "dbk_rmsnorm_gemv_allgather": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P]),
    "dbk_gateup_swiglu_allgather": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P]),
    "dbk_gemv_allgather": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "dbk_copy": (_I, [_P, _P, _SZ, _P]),
    "dbk_gemv_fp8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "dbk_rmsnorm_gemv_fp8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P]),
    "dbk_gateup_swiglu_fp8": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P]),
    "dbk_qkv_rope_append": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                                 _F, _I, _P]),
}

DBK_COMM_RECORD_BYTES = 128

_lib = None


class DbkError(RuntimeError):
    """A dbk_* entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed with status {status}: {status_string(status)}")


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the kernel library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"decodebench_b200 kernel library not found at {p}; build it with "
            "`python -m decodebench_b200.build_native` (no CPU fallback exists)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.dbk_abi_version() != 1:
        raise RuntimeError("decodebench_b200: kernel library ABI version mismatch")
    if path is None:
        _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().dbk_status_string(status).decode()


def check(fn: str, status: int) -> None:
    if status != 0:
        raise DbkError(fn, status)
